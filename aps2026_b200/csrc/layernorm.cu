// LayerNorm family: plain LN, residual add + LN, and MoE un-permute +
// carried residual add + LN, each one pass over the row.
//
// Reference: k_layer_norm / k_add_layer_norm (src/tensor.cu:2130-2178) with
// ln_stage / ln_moments / ln_write (:2017-2128). There a whole 256-thread
// CTA waits while thread 0 sums the row twice serially from shared memory.
//
// Here (default, tree order) the row lives in registers: THREADS x V float4
// (at h = 4096: 256 x 4 for plain LN, 512 x 2 for the two- and three-input
// forms), loaded with 128-bit streaming loads, mean and variance come from
// two register passes with warp shuffles and one shared slot per warp, and
// the output is written straight from registers -- the row crosses HBM
// exactly once in each direction. CTAs loop over rows (grid = one resident
// wave of the device). Rows too long for registers are staged in shared
// memory by bulk (TMA) copies.
//
// With B2_FLAG_EXACT_ORDER the moments are formed in ascending order exactly
// as ln_serial_sum / ln_serial_var do (var += t * t as a fused
// multiply-add), so the output is bit-identical to the reference: for plain
// LN over many rows by the 32-row batched kernel (one warp runs 32 rows'
// chains side by side), otherwise by one thread per row over the row staged
// in shared memory, with 128-thread CTAs keeping more rows resident per SM
// to overlap those serial chains.
//
// Output: y = fma((x - mean) * inv, gamma, beta), inv = 1 / sqrtf(var / h +
// eps), the reference's ln_write arithmetic (:2043-2047).
#include "rowload.cuh"

namespace b2 {
namespace {

enum LnMode { kLN = 0, kAddLN = 1, kCombineAddLN = 2 };

struct LnArgs {
    const float* x;             // kLN: input; kAddLN: in/out residual stream
    const float* res;           // kAddLN: residual; kCombineAddLN: carry
    const float* gamma;
    const float* beta;
    float* y;                   // normalised output
    float* x_out;               // kAddLN: x (in place); kCombineAddLN: sum
    const float* expert_out;    // kCombineAddLN
    const std::uint8_t* routes;
    const std::uint32_t* route_positions;
    std::size_t expert_rows;
    std::size_t rows;
    std::size_t h;
    float eps;
};

__device__ __forceinline__ float sum4(const float4& v) {
    return __fadd_rn(__fadd_rn(v.x, v.y), __fadd_rn(v.z, v.w));
}

__device__ __forceinline__ float sqdev4(const float4& v, float m) {
    const float a = __fsub_rn(v.x, m), b = __fsub_rn(v.y, m);
    const float c = __fsub_rn(v.z, m), d = __fsub_rn(v.w, m);
    return __fadd_rn(__fmaf_rn(a, a, __fmul_rn(b, b)), __fmaf_rn(c, c, __fmul_rn(d, d)));
}

__device__ __forceinline__ float ln_out(float s, float mean, float inv, float w, float b) {
    return __fmaf_rn(__fmul_rn(__fsub_rn(s, mean), inv), w, b);
}

__device__ __forceinline__ float4 ln_out4(const float4& s, float mean, float inv,
                                          const float4& w, const float4& b) {
    return make_float4(ln_out(s.x, mean, inv, w.x, b.x), ln_out(s.y, mean, inv, w.y, b.y),
                       ln_out(s.z, mean, inv, w.z, b.z), ln_out(s.w, mean, inv, w.w, b.w));
}

__device__ __forceinline__ float inv_std(float var_sum, float h, float eps) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(var_sum, h), eps)));
}

// Serial ascending moments over a shared-memory row (ln_serial_sum /
// ln_serial_var / ln_moments, src/tensor.cu:2063-2128), float4 reads for
// latency, the additions in index order.
__device__ __forceinline__ void serial_moments(const float* s, std::size_t h, float eps,
                                               float* mean_out, float* inv_out) {
    float sum = 0.0f;
    std::size_t j = 0;
    if ((h & 15u) == 0) {
        const float4* s4 = reinterpret_cast<const float4*>(s);
        for (std::size_t v = 0; v < h / 4; v += 4) {
            const float4 a = s4[v], b = s4[v + 1], c = s4[v + 2], d = s4[v + 3];
            sum = __fadd_rn(sum, a.x); sum = __fadd_rn(sum, a.y);
            sum = __fadd_rn(sum, a.z); sum = __fadd_rn(sum, a.w);
            sum = __fadd_rn(sum, b.x); sum = __fadd_rn(sum, b.y);
            sum = __fadd_rn(sum, b.z); sum = __fadd_rn(sum, b.w);
            sum = __fadd_rn(sum, c.x); sum = __fadd_rn(sum, c.y);
            sum = __fadd_rn(sum, c.z); sum = __fadd_rn(sum, c.w);
            sum = __fadd_rn(sum, d.x); sum = __fadd_rn(sum, d.y);
            sum = __fadd_rn(sum, d.z); sum = __fadd_rn(sum, d.w);
        }
        j = h;
    }
    for (; j < h; ++j) sum = __fadd_rn(sum, s[j]);
    const float m = __fdiv_rn(sum, static_cast<float>(h));
    float var = 0.0f;
    j = 0;
    if ((h & 15u) == 0) {
        const float4* s4 = reinterpret_cast<const float4*>(s);
        for (std::size_t v = 0; v < h / 4; v += 4) {
            const float4 q[4] = {s4[v], s4[v + 1], s4[v + 2], s4[v + 3]};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                float t;
                t = __fsub_rn(q[u].x, m); var = __fmaf_rn(t, t, var);
                t = __fsub_rn(q[u].y, m); var = __fmaf_rn(t, t, var);
                t = __fsub_rn(q[u].z, m); var = __fmaf_rn(t, t, var);
                t = __fsub_rn(q[u].w, m); var = __fmaf_rn(t, t, var);
            }
        }
        j = h;
    }
    for (; j < h; ++j) {
        const float t = __fsub_rn(s[j], m);
        var = __fmaf_rn(t, t, var);
    }
    *mean_out = m;
    *inv_out = inv_std(var, static_cast<float>(h), eps);
}

// Produces float4 chunk j of row r of the value to normalise, and writes it
// back to x_out where the mode keeps the sum.
template <int MODE>
__device__ __forceinline__ float4 load_chunk(const LnArgs& a, std::size_t r, std::size_t h4,
                                             std::size_t j, const CombineRows& cr) {
    const std::size_t o = r * h4 + j;
    if (MODE == kLN) return ld_stream(reinterpret_cast<const float4*>(a.x) + o);
    if (MODE == kAddLN)
        return add4(ld_plain(reinterpret_cast<const float4*>(a.x) + o),
                    ld_stream(reinterpret_cast<const float4*>(a.res) + o));
    const float4* e = reinterpret_cast<const float4*>(a.expert_out);
    const float4 lo = cr.lo < a.expert_rows ? ld_stream(e + cr.lo * h4 + j) : zero4();
    const float4 hi = cr.hi < a.expert_rows ? ld_stream(e + cr.hi * h4 + j) : zero4();
    return add4(combine4(lo, hi), ld_stream(reinterpret_cast<const float4*>(a.res) + o));
}

// Register-resident rows: h / 4 <= THREADS * V.
template <int MODE, int THREADS, int V, bool EXACT>
__global__ void __launch_bounds__(THREADS)
ln_rows_reg(LnArgs a) {
    pdl_begin();
    constexpr int WARPS = THREADS / 32;
    __shared__ float red[2][WARPS];
    __shared__ float stats[2];
    extern __shared__ __align__(16) float staged[];  // EXACT only: h floats
    const std::size_t h4 = a.h / 4;
    const float hf = static_cast<float>(a.h);
    const float4* g4 = reinterpret_cast<const float4*>(a.gamma);
    const float4* b4 = reinterpret_cast<const float4*>(a.beta);

    for (std::size_t r = blockIdx.x; r < a.rows; r += gridDim.x) {
        CombineRows cr{0, 0};
        if (MODE == kCombineAddLN) cr = combine_rows(a.routes, a.route_positions, r, a.expert_rows);
        float4 v[V];
#pragma unroll
        for (int k = 0; k < V; ++k) {
            const std::size_t j = threadIdx.x + static_cast<std::size_t>(k) * THREADS;
            v[k] = j < h4 ? load_chunk<MODE>(a, r, h4, j, cr) : zero4();
        }
        if (MODE != kLN) {
#pragma unroll
            for (int k = 0; k < V; ++k) {
                const std::size_t j = threadIdx.x + static_cast<std::size_t>(k) * THREADS;
                if (j < h4) st_plain(reinterpret_cast<float4*>(a.x_out) + r * h4 + j, v[k]);
            }
        }
        float mean, inv;
        if (EXACT) {
            float4* s4 = reinterpret_cast<float4*>(staged);
#pragma unroll
            for (int k = 0; k < V; ++k) {
                const std::size_t j = threadIdx.x + static_cast<std::size_t>(k) * THREADS;
                if (j < h4) s4[j] = v[k];
            }
            __syncthreads();
            if (threadIdx.x == 0) serial_moments(staged, a.h, a.eps, &stats[0], &stats[1]);
            __syncthreads();
            mean = stats[0];
            inv = stats[1];
        } else {
            float part = 0.0f;
#pragma unroll
            for (int k = 0; k < V; ++k) part = __fadd_rn(part, sum4(v[k]));
            mean = __fdiv_rn(block_sum<WARPS>(part, red[0]), hf);
            float part2 = 0.0f;
#pragma unroll
            for (int k = 0; k < V; ++k) {
                const std::size_t j = threadIdx.x + static_cast<std::size_t>(k) * THREADS;
                if (j < h4) part2 = __fadd_rn(part2, sqdev4(v[k], mean));
            }
            inv = inv_std(block_sum<WARPS>(part2, red[1]), hf, a.eps);
        }
#pragma unroll
        for (int k = 0; k < V; ++k) {
            const std::size_t j = threadIdx.x + static_cast<std::size_t>(k) * THREADS;
            if (j < h4)
                st_plain(reinterpret_cast<float4*>(a.y) + r * h4 + j,
                         ln_out4(v[k], mean, inv, __ldg(g4 + j), __ldg(b4 + j)));
        }
    }
}

// Any h / alignment: the row is staged in shared memory (h floats).
template <int MODE, bool EXACT>
__global__ void __launch_bounds__(256)
ln_rows_smem(LnArgs a) {
    pdl_begin();
    constexpr int THREADS = 256, WARPS = 8;
    __shared__ float red[2][WARPS];
    __shared__ float stats[2];
    extern __shared__ __align__(16) float staged[];
    const std::size_t h = a.h;
    const float hf = static_cast<float>(h);
    for (std::size_t r = blockIdx.x; r < a.rows; r += gridDim.x) {
        const std::size_t base = r * h;
        CombineRows cr{0, 0};
        if (MODE == kCombineAddLN) cr = combine_rows(a.routes, a.route_positions, r, a.expert_rows);
        for (std::size_t j = threadIdx.x; j < h; j += THREADS) {
            float s;
            if (MODE == kLN) {
                s = a.x[base + j];
            } else if (MODE == kAddLN) {
                s = __fadd_rn(a.x[base + j], a.res[base + j]);
            } else {
                const float lo = cr.lo < a.expert_rows ? a.expert_out[cr.lo * h + j] : 0.0f;
                const float hi = cr.hi < a.expert_rows ? a.expert_out[cr.hi * h + j] : 0.0f;
                s = __fadd_rn(combine_one(lo, hi), a.res[base + j]);
            }
            if (MODE != kLN) a.x_out[base + j] = s;
            staged[j] = s;
        }
        __syncthreads();
        float mean, inv;
        if (EXACT) {
            if (threadIdx.x == 0) serial_moments(staged, h, a.eps, &stats[0], &stats[1]);
            __syncthreads();
            mean = stats[0];
            inv = stats[1];
        } else {
            float part = 0.0f;
            for (std::size_t j = threadIdx.x; j < h; j += THREADS) part = __fadd_rn(part, staged[j]);
            mean = __fdiv_rn(block_sum<WARPS>(part, red[0]), hf);
            float part2 = 0.0f;
            for (std::size_t j = threadIdx.x; j < h; j += THREADS) {
                const float t = __fsub_rn(staged[j], mean);
                part2 = __fmaf_rn(t, t, part2);
            }
            inv = inv_std(block_sum<WARPS>(part2, red[1]), hf, a.eps);
        }
        for (std::size_t j = threadIdx.x; j < h; j += THREADS)
            a.y[base + j] = ln_out(staged[j], mean, inv, a.gamma[j], a.beta[j]);
        __syncthreads();  // staged[] is rewritten by the next row
    }
}

// Rows too long for registers, h % 4 == 0 and 16-byte aligned: each row's
// inputs (x; x and the residual; or the two expert rows and the carry) are
// staged in shared memory by 1-D bulk (TMA) copies issued by one thread and
// completing on an mbarrier, then reduced and written like ln_rows_smem.
// Copies of an expert row outside expert_out are not issued (the row reads
// as zeros, as in the register path). A wait that does not complete stops the
// CTA and reports B2_CHECK_WAIT.
template <int MODE, bool EXACT>
__global__ void __launch_bounds__(256)
ln_rows_bulk(LnArgs a) {
    pdl_begin();
    constexpr int THREADS = 256, WARPS = 8;
    __shared__ float red[2][WARPS];
    __shared__ float stats[2];
    __shared__ __align__(8) std::uint64_t bar;
    extern __shared__ __align__(128) float in[];  // NIN rows of h floats; in[0..h) becomes the sum
    const std::size_t h = a.h;
    const unsigned bytes = static_cast<unsigned>(h * sizeof(float));
    const float hf = static_cast<float>(h);
    if (threadIdx.x == 0) mbar_init(&bar, 1);
    __syncthreads();
    unsigned parity = 0;
    for (std::size_t r = blockIdx.x; r < a.rows; r += gridDim.x, parity ^= 1u) {
        CombineRows cr{0, 0};
        if (MODE == kCombineAddLN) cr = combine_rows(a.routes, a.route_positions, r, a.expert_rows);
        const bool lo_ok = MODE == kCombineAddLN && cr.lo < a.expert_rows;
        const bool hi_ok = MODE == kCombineAddLN && cr.hi < a.expert_rows;
        if (threadIdx.x == 0) {
            fence_proxy_async_smem();  // the previous row's shared accesses come first
            if (MODE == kLN) {
                mbar_expect_tx(&bar, bytes);
                bulk_g2s(in, a.x + r * h, bytes, &bar);
            } else if (MODE == kAddLN) {
                mbar_expect_tx(&bar, 2 * bytes);
                bulk_g2s(in, a.x + r * h, bytes, &bar);
                bulk_g2s(in + h, a.res + r * h, bytes, &bar);
            } else {
                mbar_expect_tx(&bar, (1u + lo_ok + hi_ok) * bytes);
                bulk_g2s(in, a.res + r * h, bytes, &bar);
                if (lo_ok) bulk_g2s(in + h, a.expert_out + cr.lo * h, bytes, &bar);
                if (hi_ok) bulk_g2s(in + 2 * h, a.expert_out + cr.hi * h, bytes, &bar);
            }
        }
        if (__syncthreads_or(!mbar_wait(&bar, parity))) {  // a copy never landed: stop, report
            if (threadIdx.x == 0) {
                flag_check(B2_CHECK_WAIT);
                mbar_wait(&bar, parity);  // one more bounded wait for the copies in flight
            }
            return;
        }
        float4* s4 = reinterpret_cast<float4*>(in);
        const std::size_t h4 = h / 4;
        if (MODE != kLN) {
            for (std::size_t j = threadIdx.x; j < h4; j += THREADS) {
                float4 v;
                if (MODE == kAddLN) {
                    v = add4(s4[j], s4[h4 + j]);
                } else {
                    const float4 lo = lo_ok ? s4[h4 + j] : zero4(), hi = hi_ok ? s4[2 * h4 + j] : zero4();
                    v = add4(combine4(lo, hi), s4[j]);
                }
                s4[j] = v;
                st_plain(reinterpret_cast<float4*>(a.x_out) + r * h4 + j, v);
            }
            __syncthreads();
        }
        float mean, inv;
        if (EXACT) {
            if (threadIdx.x == 0) serial_moments(in, h, a.eps, &stats[0], &stats[1]);
            __syncthreads();
            mean = stats[0];
            inv = stats[1];
        } else {
            float part = 0.0f;
            for (std::size_t j = threadIdx.x; j < h4; j += THREADS) part = __fadd_rn(part, sum4(s4[j]));
            mean = __fdiv_rn(block_sum<WARPS>(part, red[0]), hf);
            float part2 = 0.0f;
            for (std::size_t j = threadIdx.x; j < h4; j += THREADS) part2 = __fadd_rn(part2, sqdev4(s4[j], mean));
            inv = inv_std(block_sum<WARPS>(part2, red[1]), hf, a.eps);
        }
        const float4* g4 = reinterpret_cast<const float4*>(a.gamma);
        const float4* b4 = reinterpret_cast<const float4*>(a.beta);
        for (std::size_t j = threadIdx.x; j < h4; j += THREADS)
            st_plain(reinterpret_cast<float4*>(a.y) + r * h4 + j,
                     ln_out4(s4[j], mean, inv, __ldg(g4 + j), __ldg(b4 + j)));
        __syncthreads();  // in[] is refilled for the next row
    }
}

// Reference-order (B2_FLAG_EXACT_ORDER) LayerNorm of many rows (plain
// LayerNorm; the fused-add forms keep the per-row kernel, which measured
// faster with their second and third input streams). The serial sums are 2h
// dependent additions per row; issued one row per thread they leave 31 of a
// warp's lanes idle. Here a CTA takes 32 rows at a time and warp 0 runs the
// 32 rows' chains side by side, lane r summing row r's staged chunk in
// ascending order, while the other 15 warps stage the next chunk
// (kExactChunk floats of each row) into the other shared buffer with
// coalesced 128-bit loads, 8 in flight per thread. Pass A forms the sums,
// pass B the squared deviations (re-reading the 32 rows, which one CTA per
// SM keeps within L2), pass C writes y with every thread. Same operations in
// the same order as serial_moments, so the output is bit-identical to the
// reference.
constexpr int kExactRows = 32;
constexpr int kExactChunk = 512;
constexpr int kExactPitch = kExactChunk + 4;  // floats; spreads the lanes' rows over the banks
constexpr int kExactThreads = 512;

__global__ void __launch_bounds__(kExactThreads, 1)
ln_exact_batch(LnArgs a) {
    pdl_begin();
    constexpr int THREADS = kExactThreads, LOADERS = THREADS - 32, U = 8;
    extern __shared__ __align__(16) float stage_buf[];  // [2][kExactRows][kExactPitch]
    __shared__ float mean_s[kExactRows], inv_s[kExactRows];
    const unsigned tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const std::size_t h = a.h, h4 = h / 4;
    const int chunks = static_cast<int>((h + kExactChunk - 1) / kExactChunk);
    const float hf = static_cast<float>(h);
    const float4* x4 = reinterpret_cast<const float4*>(a.x);
    for (std::size_t b0 = static_cast<std::size_t>(blockIdx.x) * kExactRows; b0 < a.rows;
         b0 += static_cast<std::size_t>(gridDim.x) * kExactRows) {
        const int nr = static_cast<int>(a.rows - b0 < kExactRows ? a.rows - b0 : kExactRows);
        // copies chunk c of the batch's rows into buffer c & 1; each thread
        // issues U loads before it stores any, so a chunk costs a few memory
        // latencies, not one per item
        auto stage = [&](int c, unsigned first, unsigned stride) {
            const std::size_t c4 = static_cast<std::size_t>(c) * (kExactChunk / 4);
            const unsigned len4 = static_cast<unsigned>(min(static_cast<std::size_t>(kExactChunk / 4), h4 - c4));
            const unsigned total = static_cast<unsigned>(nr) * len4;
            float4* buf = reinterpret_cast<float4*>(stage_buf + (c & 1) * kExactRows * kExactPitch);
            for (unsigned it0 = first; it0 < total; it0 += stride * U) {
                float4 v[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const unsigned it = it0 + u * stride;
                    if (it < total) v[u] = ld_plain(x4 + (b0 + it / len4) * h4 + c4 + it % len4);
                }
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const unsigned it = it0 + u * stride;
                    if (it < total) buf[(it / len4) * (kExactPitch / 4) + it % len4] = v[u];
                }
            }
        };
        // lane r runs f over row r's elements of chunk c, in ascending order
        auto chain = [&](int c, auto f) {
            const std::size_t c4 = static_cast<std::size_t>(c) * (kExactChunk / 4);
            const unsigned len4 = static_cast<unsigned>(min(static_cast<std::size_t>(kExactChunk / 4), h4 - c4));
            const float4* row = reinterpret_cast<const float4*>(stage_buf + (c & 1) * kExactRows * kExactPitch +
                                                                  lane * kExactPitch);
#pragma unroll 4
            for (unsigned i = 0; i < len4; ++i) {
                const float4 v = row[i];
                f(v.x);
                f(v.y);
                f(v.z);
                f(v.w);
            }
        };
        float acc = 0.0f, mean = 0.0f;
        for (int pass = 0; pass < 2; ++pass) {
            stage(0, tid, THREADS);
            __syncthreads();
            for (int c = 0; c < chunks; ++c) {
                if (warp != 0) {
                    if (c + 1 < chunks) stage(c + 1, tid - 32, LOADERS);
                } else if (lane < static_cast<unsigned>(nr)) {
                    if (pass == 0)
                        chain(c, [&](float x) { acc = __fadd_rn(acc, x); });
                    else
                        chain(c, [&](float x) {
                            const float t = __fsub_rn(x, mean);
                            acc = __fmaf_rn(t, t, acc);
                        });
                }
                __syncthreads();
            }
            if (pass == 0) {
                mean = __fdiv_rn(acc, hf);
                acc = 0.0f;
            }
        }
        if (warp == 0 && lane < static_cast<unsigned>(nr)) {
            mean_s[lane] = mean;
            inv_s[lane] = inv_std(acc, hf, a.eps);
        }
        __syncthreads();
        // ---- pass C: y for the batch, all threads, coalesced ----
        const float4* g4 = reinterpret_cast<const float4*>(a.gamma);
        const float4* be4 = reinterpret_cast<const float4*>(a.beta);
        const std::size_t total = static_cast<std::size_t>(nr) * h4;
        for (std::size_t it0 = tid; it0 < total; it0 += THREADS * U) {
            float4 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {  // all loads first
                const std::size_t it = it0 + static_cast<std::size_t>(u) * THREADS;
                if (it < total) v[u] = ld_plain(x4 + b0 * h4 + it);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const std::size_t it = it0 + static_cast<std::size_t>(u) * THREADS;
                if (it >= total) continue;
                const std::size_t r = it / h4, j = it % h4;
                st_plain(reinterpret_cast<float4*>(a.y) + b0 * h4 + it,
                         ln_out4(v[u], mean_s[r], inv_s[r], __ldg(g4 + j), __ldg(be4 + j)));
            }
        }
        __syncthreads();  // mean_s / inv_s and the buffers are reused by the next batch
    }
}

constexpr std::size_t kMaxSmemRow = 220 * 1024;  // + static reduction slots <= 227 KB

template <int MODE, int THREADS, int V, bool EXACT>
int launch_reg(const LnArgs& a, cudaStream_t s) {
    const std::size_t smem = EXACT ? a.h * sizeof(float) : 0;
    auto kernel = ln_rows_reg<MODE, THREADS, V, EXACT>;
    if (allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem) != cudaSuccess)
        return launch_result("layer norm: shared memory attribute");
    const unsigned grid = wave_grid(reinterpret_cast<const void*>(kernel), THREADS, smem, a.rows);
    launch_pdl(kernel, grid, THREADS, smem, s, a);
    return B2_OK;
}

int launch_exact_batch(const LnArgs& a, cudaStream_t s) {
    const std::size_t smem = 2 * kExactRows * kExactPitch * sizeof(float);
    if (allow_dynamic_smem(reinterpret_cast<const void*>(ln_exact_batch), smem) != cudaSuccess)
        return launch_result("layer norm: shared memory attribute");
    const std::size_t batches = (a.rows + kExactRows - 1) / kExactRows;
    const unsigned grid = static_cast<unsigned>(batches < static_cast<std::size_t>(sm_count()) ? batches : sm_count());
    launch_pdl(ln_exact_batch, grid, kExactThreads, smem, s, a);
    return B2_OK;
}

template <int MODE, bool EXACT>
int launch_bulk(const LnArgs& a, cudaStream_t s) {
    constexpr int NIN = MODE == kLN ? 1 : (MODE == kAddLN ? 2 : 3);
    const std::size_t smem = NIN * a.h * sizeof(float);
    auto kernel = ln_rows_bulk<MODE, EXACT>;
    if (allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem) != cudaSuccess)
        return launch_result("layer norm: shared memory attribute");
    const unsigned grid = wave_grid(reinterpret_cast<const void*>(kernel), 256, smem, a.rows);
    launch_pdl(kernel, grid, 256, smem, s, a);
    return B2_OK;
}

template <int MODE, bool EXACT>
int launch_smem(const LnArgs& a, cudaStream_t s) {
    const std::size_t smem = a.h * sizeof(float);
    auto kernel = ln_rows_smem<MODE, EXACT>;
    if (allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem) != cudaSuccess)
        return launch_result("layer norm: shared memory attribute");
    const unsigned grid = wave_grid(reinterpret_cast<const void*>(kernel), 256, smem, a.rows);
    launch_pdl(kernel, grid, 256, smem, s, a);
    return B2_OK;
}

// Picks, for plain LayerNorm in reference order over at least 32 rows per
// SM, the 32-row batched kernel; otherwise the register-resident variant
// whose THREADS * V covers h / 4, else bulk-copy staging (aligned rows,
// h % 4 == 0), else the scalar shared-memory one.
template <int MODE>
int dispatch(const LnArgs& a, bool exact, bool vec_ok, cudaStream_t s, const char* what) {
    if (a.h * sizeof(float) > kMaxSmemRow && exact)
        return set_error(B2_ERR_UNSUPPORTED, std::string(what) + ": h too large");
    int rc = B2_OK;
    const std::size_t h4 = a.h / 4;
    if (MODE == kLN && vec_ok && exact && a.rows >= static_cast<std::size_t>(kExactRows) * sm_count()) {
        rc = launch_exact_batch(a, s);  // enough rows for a 32-row batch on every SM
    } else if (vec_ok && !exact && h4 <= 256 * 8) {
        if (h4 <= 256) rc = launch_reg<MODE, 256, 1, false>(a, s);
        else if (h4 <= 512) rc = launch_reg<MODE, 256, 2, false>(a, s);
        // (at h = 4096 the two- and three-input forms run at 99% of the HBM
        // copy rate as 512 x 2 against 94-96% as 256 x 4; plain LN is 10%
        // slower as 512 x 2)
        else if (h4 <= 1024) rc = MODE != kLN ? launch_reg<MODE, 512, 2, false>(a, s)
                                              : launch_reg<MODE, 256, 4, false>(a, s);
        else rc = launch_reg<MODE, 256, 8, false>(a, s);
    } else if (vec_ok && exact && h4 <= 128 * 8) {
        if (h4 <= 128) rc = launch_reg<MODE, 128, 1, true>(a, s);
        else if (h4 <= 256) rc = launch_reg<MODE, 128, 2, true>(a, s);
        else if (h4 <= 512) rc = launch_reg<MODE, 128, 4, true>(a, s);
        else rc = launch_reg<MODE, 128, 8, true>(a, s);
    } else if (vec_ok && (MODE == kLN ? 1 : MODE == kAddLN ? 2 : 3) * a.h * sizeof(float) <= kMaxSmemRow) {
        rc = exact ? launch_bulk<MODE, true>(a, s) : launch_bulk<MODE, false>(a, s);
    } else {
        if (a.h * sizeof(float) > kMaxSmemRow)
            return set_error(B2_ERR_UNSUPPORTED, std::string(what) + ": h too large");
        rc = exact ? launch_smem<MODE, true>(a, s) : launch_smem<MODE, false>(a, s);
    }
    if (rc != B2_OK) return rc;
    return launch_result(what);
}

bool all_aligned(std::initializer_list<const void*> ps) {
    for (const void* p : ps)
        if (p && !aligned16(p)) return false;
    return true;
}

}  // namespace
}  // namespace b2

B2_DEFINE_CHECK_TAKER(layernorm)

extern "C" {

int b2_layer_norm(const float* x, const float* gamma, const float* beta, float* y,
                  size_t rows, size_t h, float eps, uint32_t flags, b2_stream_t stream) {
    using namespace b2;
    if (rows == 0) return B2_OK;
    if (!x || !gamma || !beta || !y) return invalid("layer norm: null pointer");
    if (h == 0) return invalid("layer norm shape");
    LnArgs a{};
    a.x = x; a.gamma = gamma; a.beta = beta; a.y = y;
    a.rows = rows; a.h = h; a.eps = eps;
    const bool vec = (h & 3u) == 0 && all_aligned({x, gamma, beta, y});
    return dispatch<kLN>(a, (flags & B2_FLAG_EXACT_ORDER) != 0, vec, as_stream(stream),
                         "b2_layer_norm");
}

int b2_add_layer_norm(float* x, const float* residual, const float* gamma, const float* beta,
                      float* y, size_t rows, size_t h, float eps, uint32_t flags,
                      b2_stream_t stream) {
    using namespace b2;
    if (rows == 0) return B2_OK;
    if (!x || !residual || !gamma || !beta || !y) return invalid("add layer norm: null pointer");
    if (h == 0) return invalid("add layer norm shape");
    LnArgs a{};
    a.x = x; a.res = residual; a.gamma = gamma; a.beta = beta; a.y = y; a.x_out = x;
    a.rows = rows; a.h = h; a.eps = eps;
    const bool vec = (h & 3u) == 0 && all_aligned({x, residual, gamma, beta, y});
    return dispatch<kAddLN>(a, (flags & B2_FLAG_EXACT_ORDER) != 0, vec, as_stream(stream),
                            "b2_add_layer_norm");
}

int b2_moe_combine_add_layer_norm(const float* expert_out, size_t expert_rows,
                                  const uint8_t* routes, const uint32_t* route_positions,
                                  const float* carry, const float* gamma, const float* beta,
                                  float* x_out, float* y, size_t rows, size_t h, float eps,
                                  uint32_t flags, b2_stream_t stream) {
    using namespace b2;
    if (rows == 0) return B2_OK;
    if (!expert_out || !routes || !route_positions || !carry || !gamma || !beta || !x_out || !y)
        return invalid("combine add layer norm: null pointer");
    if (h == 0) return invalid("combine add layer norm shape");
    LnArgs a{};
    a.res = carry; a.gamma = gamma; a.beta = beta; a.y = y; a.x_out = x_out;
    a.expert_out = expert_out; a.routes = routes; a.route_positions = route_positions;
    a.expert_rows = expert_rows; a.rows = rows; a.h = h; a.eps = eps;
    const bool vec = (h & 3u) == 0 && all_aligned({expert_out, carry, gamma, beta, x_out, y});
    return dispatch<kCombineAddLN>(a, (flags & B2_FLAG_EXACT_ORDER) != 0, vec,
                                   as_stream(stream), "b2_moe_combine_add_layer_norm");
}

}  // extern "C"
