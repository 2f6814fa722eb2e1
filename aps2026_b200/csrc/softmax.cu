// Causal, sliding-window, scaled softmax over a [heads, T, T] score tensor.
//
// Reference: the softmax inside k_attention_tree_gqa4 (src/tensor.cu:2526
// scale, :2549-2585 max / exp / denominator / divide; window :2435-2439);
// same math in k_attention_grouped_gqa4 (:2371-2385). The reference has no
// standalone softmax kernel (softmax_last_dim, include/tensor.h:152, is
// declared but never defined).
//
// One CTA (or, for rows of <= 256 keys, one warp) per query row, grid-stride
// over heads * T rows. The row's in-window chunk of scores is read with
// 128-bit loads straight into registers -- chunks wholly outside
// [i + 1 - window, i] are never read -- scaled, reduced to the max,
// exponentiated, summed, divided, and the full row (zeros outside the
// window) written with 128-bit stores.
// B2_FLAG_EXACT_ORDER: the reference's exponential ((float)exp((double)d),
// bit for bit, through the table-driven exp_ref of fastexp.cuh), the
// exponentials staged in shared memory and summed by one thread in ascending
// key order, and Markstein division with one correctly rounded reciprocal
// per row -- bit-identical to the reference, and issue-bound on the
// exponential. Default: CUDA's expf, a tree-order denominator and a
// multiplication by the row's rounded reciprocal (within the tolerance of
// that mode), with the next row's chunks loaded during this row's
// reductions; at T = 2048 it streams at ~80% of the HBM copy rate.
// Algorithmic bytes: 4 * (window cells) read + 4 * T written per row.
#include "common.cuh"
#include "fastexp.cuh"

namespace b2 {
namespace {

constexpr int kSmThreads = 256;
constexpr int kSmWarps = kSmThreads / 32;

struct SoftmaxArgs {
    const float* scores;
    float* probs;
    std::size_t rows;  // heads * T
    std::size_t T, ld, window;
    float scale;
};

// e / d rounded to nearest, for 0 <= e <= 1 and a row denominator d >= 1,
// given y = RN(1/d) (one correctly rounded reciprocal per row): with
// q = RN(e * y) within one ulp of e / d and the residual r = e - d q exact
// (a fused multiply-add), RN(q + r y) is the correctly rounded quotient
// (Markstein's theorem, P. Markstein, IBM J. Res. Dev. 34(1), 1990). Three
// FMA-pipe operations instead of a full division per element; arguments
// below 2^-96, whose residual could leave the normal range, divide directly.
// In the default (tree-order) mode the quotient is RN(e * y) instead, within
// 1.5 ulp of e / d.
template <bool EXACT>
__device__ __forceinline__ float div_by_row(float e, float d, float y) {
    if (!EXACT) return __fmul_rn(e, y);  // (y is NaN when d is)
    if (e < 0x1p-96f) return __fdiv_rn(e, d);  // (0 / NaN must stay NaN)
    const float q = __fmul_rn(e, y);
    const float r = __fmaf_rn(-d, q, e);
    return __fmaf_rn(r, y, q);
}

// The part of one row a thread holds: V chunks of 4 keys, chunk k at keys
// 4 c_k .. 4 c_k + 3 with c_k = first + k * stride. Chunks with no key in
// the window [begin, i] are never read; inside read chunks, keys outside the
// window hold -inf, whose exponential is +0 (no per-element masks in the
// exponential or sum).
// The raw chunks of one row a thread holds, as loaded (chunk k at keys
// 4 c_k .. 4 c_k + 3, c_k = first + k * stride; chunks with no key in the
// window [begin, i] are not read). (Column indices are 32-bit: T * 4 bytes
// fits the shared-memory row limit.)
template <int V>
struct RowChunks {
    float4 s[V];
    unsigned any = 0, full = 0;  // bit k: chunk k holds some / only window keys

    __device__ __forceinline__ void fetch(const float4* src, unsigned first, unsigned stride, unsigned T4,
                                          unsigned begin, unsigned i) {
        any = full = 0;
#pragma unroll
        for (int k = 0; k < V; ++k) {
            const unsigned c = first + static_cast<unsigned>(k) * stride, j0 = 4 * c;
            const bool a_k = c < T4 && j0 <= i && j0 + 3 >= begin;
            const bool f_k = a_k && j0 >= begin && j0 + 3 <= i;
            any |= static_cast<unsigned>(a_k) << k;
            full |= static_cast<unsigned>(f_k) << k;
            s[k] = a_k ? ld_stream(src + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
};

// The part of one row a thread holds, scaled: keys outside the window inside
// read chunks hold -inf, whose exponential is +0 (no per-element masks in
// the exponential or sum).
template <int V, bool EXACT>
struct RowPart {
    float v[V][4];
    unsigned any = 0, full = 0;

    // Scales fetched chunks; returns the thread's max score.
    __device__ __forceinline__ float take(const RowChunks<V>& r, unsigned first, unsigned stride, unsigned begin,
                                          unsigned i, float scale) {
        any = r.any;
        full = r.full;
        float mx = -3.402823466e+38F;
#pragma unroll
        for (int k = 0; k < V; ++k) {
            const unsigned j0 = 4 * (first + static_cast<unsigned>(k) * stride);
            const bool a_k = (any >> k) & 1u;
            v[k][0] = __fmul_rn(r.s[k].x, scale);
            v[k][1] = __fmul_rn(r.s[k].y, scale);
            v[k][2] = __fmul_rn(r.s[k].z, scale);
            v[k][3] = __fmul_rn(r.s[k].w, scale);
            if (!((full >> k) & 1u)) {
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    if (!(a_k && j0 + e >= begin && j0 + e <= i)) v[k][e] = -__int_as_float(0x7f800000);
            }
            mx = fmaxf(mx, fmaxf(fmaxf(v[k][0], v[k][1]), fmaxf(v[k][2], v[k][3])));
        }
        return mx;
    }
    // Loads and scales the chunks; returns the thread's max score.
    __device__ __forceinline__ float load(const float4* src, unsigned first, unsigned stride, unsigned T4,
                                          unsigned begin, unsigned i, float scale) {
        RowChunks<V> r;
        r.fetch(src, first, stride, T4, begin, i);
        return take(r, first, stride, begin, i, scale);
    }
    // v <- exp(v - m) (zeros in unread chunks); returns the thread's sum.
    __device__ __forceinline__ float exp_sum(float m, const double* tab) {
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < V; ++k) {
            if ((any >> k) & 1u) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    v[k][e] = exp_mode<EXACT>(__fsub_rn(v[k][e], m), tab);
                    sum = __fadd_rn(sum, v[k][e]);
                }
            } else {
                v[k][0] = v[k][1] = v[k][2] = v[k][3] = 0.0f;
            }
        }
        return sum;
    }
    // dst chunk c_k <- v / d (zeros outside the window).
    __device__ __forceinline__ void store(float4* dst, unsigned first, unsigned stride, unsigned T4,
                                          unsigned begin, unsigned i, float d, float y) const {
#pragma unroll
        for (int k = 0; k < V; ++k) {
            const unsigned c = first + static_cast<unsigned>(k) * stride, j0 = 4 * c;
            if (c >= T4) continue;
            float pv[4] = {0.f, 0.f, 0.f, 0.f};
            if ((full >> k) & 1u) {
#pragma unroll
                for (int e = 0; e < 4; ++e) pv[e] = div_by_row<EXACT>(v[k][e], d, y);
            } else if ((any >> k) & 1u) {
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    if (j0 + e >= begin && j0 + e <= i) pv[e] = div_by_row<EXACT>(v[k][e], d, y);
            }
            st_plain(dst + c, make_float4(pv[0], pv[1], pv[2], pv[3]));
        }
    }
};

// One CTA of THREADS threads per query row, V float4 per thread; block
// reductions through shared memory.
template <int THREADS, int V, bool EXACT>
__global__ void __launch_bounds__(THREADS)
causal_softmax_block(SoftmaxArgs a) {
    pdl_begin();
    constexpr int WARPS = THREADS / 32;
    __shared__ float red[2][WARPS];
    __shared__ float denom_s;
    __shared__ double tab[64];
    extern __shared__ __align__(16) float staged[];  // EXACT: T floats
    load_exp2_table(tab);
    __syncthreads();
    const unsigned T4 = static_cast<unsigned>(a.T / 4);
    auto window_of = [&](std::size_t row, unsigned* i, unsigned* begin) {
        *i = static_cast<unsigned>(row % a.T);
        *begin = *i + 1 > a.window ? static_cast<unsigned>(*i + 1 - a.window) : 0u;
    };
    // Tree order: the next row's chunks are loaded while this row is reduced
    // and written (+2.6% at T = 2048). Exact order loads each row in turn:
    // the look-ahead's registers cost it more than they hide.
    RowChunks<V> next;
    if (!EXACT && blockIdx.x < a.rows) {
        unsigned i0, b0;
        window_of(blockIdx.x, &i0, &b0);
        next.fetch(reinterpret_cast<const float4*>(a.scores + blockIdx.x * a.ld), threadIdx.x, THREADS, T4, b0, i0);
    }
    for (std::size_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
        unsigned i, begin;
        window_of(row, &i, &begin);
        float4* dst = reinterpret_cast<float4*>(a.probs + row * a.ld);
        if (EXACT)
            next.fetch(reinterpret_cast<const float4*>(a.scores + row * a.ld), threadIdx.x, THREADS, T4, begin, i);
        RowPart<V, EXACT> part;
        const float mine = part.take(next, threadIdx.x, THREADS, begin, i, a.scale);
        if (!EXACT && row + gridDim.x < a.rows) {
            unsigned in, bn;
            window_of(row + gridDim.x, &in, &bn);
            next.fetch(reinterpret_cast<const float4*>(a.scores + (row + gridDim.x) * a.ld), threadIdx.x, THREADS,
                       T4, bn, in);
        }
        const float m = block_max<WARPS>(mine, red[0]);
        const float local_sum = part.exp_sum(m, tab);
        float denom;
        if (EXACT) {
#pragma unroll
            for (int k = 0; k < V; ++k) {
                const std::size_t c = threadIdx.x + static_cast<std::size_t>(k) * THREADS;
                if (c < T4)
                    reinterpret_cast<float4*>(staged)[c] =
                        make_float4(part.v[k][0], part.v[k][1], part.v[k][2], part.v[k][3]);
            }
            __syncthreads();
            if (threadIdx.x == 0) {
                float d = 0.0f;
                for (std::size_t j = begin; j <= i; ++j) d = __fadd_rn(d, staged[j]);
                denom_s = d;
            }
            __syncthreads();
            denom = denom_s;
        } else {
            denom = block_sum<WARPS>(local_sum, red[1]);
        }
        part.store(dst, threadIdx.x, THREADS, T4, begin, i, denom, __frcp_rn(denom));
        if (EXACT) __syncthreads();  // staged[] / denom_s reused by the next row
    }
}


// One warp per query row: the row's in-window 128-bit chunks go straight to
// registers (lane l holds chunks l, l+32, ..., V per lane), max and sum are
// warp shuffles -- no block barrier per row -- and 4 warps per CTA keep ~20
// rows in flight per SM. EXACT stages the exponentials in the warp's slice of
// shared memory and lane 0 sums them in ascending key order.
constexpr int kWarpRowThreads = 128;
constexpr int kWarpRowWarps = kWarpRowThreads / 32;

template <int V, bool EXACT>
__global__ void __launch_bounds__(kWarpRowThreads)
causal_softmax_warp(SoftmaxArgs a) {
    pdl_begin();
    __shared__ double tab[64];
    extern __shared__ __align__(16) float staged[];  // EXACT: kWarpRowWarps x T floats
    load_exp2_table(tab);
    __syncthreads();
    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float* mine = staged + static_cast<std::size_t>(warp) * a.T;
    const unsigned T4 = static_cast<unsigned>(a.T / 4);
    for (std::size_t row = static_cast<std::size_t>(blockIdx.x) * kWarpRowWarps + warp; row < a.rows;
         row += static_cast<std::size_t>(gridDim.x) * kWarpRowWarps) {
        const unsigned i = static_cast<unsigned>(row % a.T);
        const unsigned begin = i + 1 > a.window ? static_cast<unsigned>(i + 1 - a.window) : 0u;
        const float4* src = reinterpret_cast<const float4*>(a.scores + row * a.ld);
        float4* dst = reinterpret_cast<float4*>(a.probs + row * a.ld);
        RowPart<V, EXACT> part;
        const float m = warp_max(part.load(src, lane, 32, T4, begin, i, a.scale));
        const float local_sum = part.exp_sum(m, tab);
        float denom;
        if (EXACT) {
#pragma unroll
            for (int k = 0; k < V; ++k) {
                const std::size_t c = lane + 32 * static_cast<std::size_t>(k);
                if (c < T4)
                    reinterpret_cast<float4*>(mine)[c] =
                        make_float4(part.v[k][0], part.v[k][1], part.v[k][2], part.v[k][3]);
            }
            __syncwarp();
            float d = 0.0f;
            if (lane == 0)
                for (std::size_t j = begin; j <= i; ++j) d = __fadd_rn(d, mine[j]);
            denom = __shfl_sync(0xffffffffu, d, 0);
        } else {
            denom = warp_sum(local_sum);
        }
        part.store(dst, lane, 32, T4, begin, i, denom, __frcp_rn(denom));
        if (EXACT) __syncwarp();  // the warp's staging slice is reused by its next row
    }
}

// Any T / ld / alignment: scaled scores staged in shared memory (T floats).
template <bool EXACT>
__global__ void __launch_bounds__(kSmThreads)
causal_softmax_smem(SoftmaxArgs a) {
    pdl_begin();
    __shared__ float red[2][kSmWarps];
    __shared__ float denom_s;
    __shared__ double tab[64];
    extern __shared__ __align__(16) float staged[];
    load_exp2_table(tab);
    __syncthreads();
    for (std::size_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
        const std::size_t i = row % a.T;
        const std::size_t begin = i + 1 > a.window ? i + 1 - a.window : 0;
        const float* src = a.scores + row * a.ld;
        float* dst = a.probs + row * a.ld;
        float local_max = -3.402823466e+38F;
        for (std::size_t j = begin + threadIdx.x; j <= i; j += kSmThreads) {
            const float x = __fmul_rn(src[j], a.scale);
            staged[j] = x;
            local_max = fmaxf(local_max, x);
        }
        const float m = block_max<kSmWarps>(local_max, red[0]);
        float local_sum = 0.0f;
        for (std::size_t j = begin + threadIdx.x; j <= i; j += kSmThreads) {
            const float ex = exp_mode<EXACT>(__fsub_rn(staged[j], m), tab);
            staged[j] = ex;
            local_sum = __fadd_rn(local_sum, ex);
        }
        float denom;
        if (EXACT) {
            __syncthreads();
            if (threadIdx.x == 0) {
                float d = 0.0f;
                for (std::size_t j = begin; j <= i; ++j) d = __fadd_rn(d, staged[j]);
                denom_s = d;
            }
            __syncthreads();
            denom = denom_s;
        } else {
            denom = block_sum<kSmWarps>(local_sum, red[1]);
        }
        const float rden = __frcp_rn(denom);
        for (std::size_t j = threadIdx.x; j < a.T; j += kSmThreads)
            dst[j] = (j >= begin && j <= i) ? div_by_row<EXACT>(staged[j], denom, rden) : 0.0f;
        __syncthreads();
    }
}

template <int THREADS, int V, bool EXACT>
int launch_block(const SoftmaxArgs& a, cudaStream_t s) {
    const std::size_t smem = EXACT ? a.T * sizeof(float) : 0;
    auto kernel = causal_softmax_block<THREADS, V, EXACT>;
    if (allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem) != cudaSuccess)
        return launch_result("causal softmax: shared memory attribute");
    const unsigned grid = wave_grid(reinterpret_cast<const void*>(kernel), THREADS, smem, a.rows);
    launch_pdl(kernel, grid, THREADS, smem, s, a);
    return B2_OK;
}

template <int V, bool EXACT>
int launch_warp(const SoftmaxArgs& a, cudaStream_t s) {
    const std::size_t smem = EXACT ? kWarpRowWarps * a.T * sizeof(float) : 0;
    auto kernel = causal_softmax_warp<V, EXACT>;
    if (allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem) != cudaSuccess)
        return launch_result("causal softmax: shared memory attribute");
    const std::size_t blocks = (a.rows + kWarpRowWarps - 1) / kWarpRowWarps;
    const unsigned grid = wave_grid(reinterpret_cast<const void*>(kernel), kWarpRowThreads, smem, blocks);
    launch_pdl(kernel, grid, kWarpRowThreads, smem, s, a);
    return B2_OK;
}

template <bool EXACT>
int launch_smem(const SoftmaxArgs& a, cudaStream_t s) {
    const std::size_t smem = a.T * sizeof(float);
    auto kernel = causal_softmax_smem<EXACT>;
    if (allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem) != cudaSuccess)
        return launch_result("causal softmax: shared memory attribute");
    const unsigned grid = wave_grid(reinterpret_cast<const void*>(kernel), kSmThreads, smem, a.rows);
    launch_pdl(kernel, grid, kSmThreads, smem, s, a);
    return B2_OK;
}

// Short rows (T <= 256) take a warp each; longer rows a CTA each. Measured
// at T = 2048 on B200: 128 threads x 4 float4 per thread beats 256 x 2,
// 512 x 1 and a warp per row (16 float4 per lane: too many registers).
template <bool EXACT>
int dispatch(const SoftmaxArgs& a, bool vec, cudaStream_t s) {
    const std::size_t T4 = a.T / 4;
    if (vec) {
        if (T4 <= 32) return launch_warp<1, EXACT>(a, s);
        if (T4 <= 64) return launch_warp<2, EXACT>(a, s);
        if (T4 <= 512) return launch_block<128, 4, EXACT>(a, s);
        if (T4 <= 1024) return launch_block<256, 4, EXACT>(a, s);
        if (T4 <= 2048) return launch_block<256, 8, EXACT>(a, s);
    }
    return launch_smem<EXACT>(a, s);
}

}  // namespace
}  // namespace b2

extern "C" int b2_causal_softmax(const float* scores, float* probs, size_t heads, size_t T,
                                 size_t ld, float scale, size_t window, uint32_t flags,
                                 b2_stream_t stream) {
    using namespace b2;
    if (heads == 0 || T == 0) return B2_OK;
    if (!scores || !probs) return invalid("b2_causal_softmax: null pointer");
    if (ld < T) return invalid("b2_causal_softmax: ld < T");
    if (window == 0) return invalid("b2_causal_softmax: window == 0");
    if (T * sizeof(float) > 220 * 1024)
        return set_error(B2_ERR_UNSUPPORTED, "b2_causal_softmax: T too large");
    SoftmaxArgs a{scores, probs, heads * T, T, ld, window, scale};
    const bool vec = (T % 4) == 0 && (ld % 4) == 0 && aligned16(scores) && aligned16(probs);
    const int rc = (flags & B2_FLAG_EXACT_ORDER) ? dispatch<true>(a, vec, as_stream(stream))
                                                 : dispatch<false>(a, vec, as_stream(stream));
    if (rc != B2_OK) return rc;
    return launch_result("b2_causal_softmax");
}
