// Causal, sliding-window, scaled softmax over a [heads, T, T] score tensor.
//
// Reference: the softmax inside k_attention_tree_gqa4 (src/tensor.cu:2526
// scale, :2549-2585 max / exp / denominator / divide; window :2435-2439);
// same math in k_attention_grouped_gqa4 (:2371-2385). The reference has no
// standalone softmax kernel (softmax_last_dim, include/tensor.h:152, is
// declared but never defined).
//
// One CTA per query row (grid-stride over heads * T rows). The row's
// in-window chunk of scores is read with 128-bit loads straight into
// registers -- chunks wholly outside [i + 1 - window, i] are never read --
// scaled, reduced to the max, exponentiated as the reference does --
// (float)exp((double)d), bit for bit, through the table-driven exp_ref of
// fastexp.cuh -- summed, divided, and the full row (zeros outside
// the window) written with 128-bit stores. Default: tree-order denominator.
// B2_FLAG_EXACT_ORDER: the exponentials are staged in shared memory and one
// thread sums them in ascending key order, as the reference does, making the
// output bit-identical.
// HBM bound: 4 * (window cells) read + 4 * T written per row.
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

template <int V, bool EXACT>
__global__ void __launch_bounds__(kSmThreads)
causal_softmax_reg(SoftmaxArgs a) {
    __shared__ float red[2][kSmWarps];
    __shared__ float denom_s;
    __shared__ double tab[64];
    extern __shared__ __align__(16) float staged[];  // EXACT: T floats
    load_exp2_table(tab);
    __syncthreads();
    const std::size_t T4 = a.T / 4;
    for (std::size_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
        const std::size_t i = row % a.T;
        const std::size_t begin = i + 1 > a.window ? i + 1 - a.window : 0;
        const float4* src = reinterpret_cast<const float4*>(a.scores + row * a.ld);
        float4* dst = reinterpret_cast<float4*>(a.probs + row * a.ld);
        float v[V][4];
        unsigned valid = 0;  // bit 4k+e: element e of chunk k is inside the window
        float local_max = -3.402823466e+38F;
#pragma unroll
        for (int k = 0; k < V; ++k) {
            const std::size_t c = threadIdx.x + static_cast<std::size_t>(k) * kSmThreads;
            const std::size_t j0 = 4 * c;
            const bool any = c < T4 && j0 <= i && j0 + 3 >= begin;
            float4 s = any ? ld_stream(src + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            const float sv[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const std::size_t j = j0 + e;
                v[k][e] = __fmul_rn(sv[e], a.scale);
                if (any && j >= begin && j <= i) {
                    valid |= 1u << (4 * k + e);
                    local_max = fmaxf(local_max, v[k][e]);
                }
            }
        }
        const float m = block_max<kSmWarps>(local_max, red[0]);
        float local_sum = 0.0f;
#pragma unroll
        for (int k = 0; k < V; ++k)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float ex = (valid >> (4 * k + e)) & 1u ? exp_ref(__fsub_rn(v[k][e], m), tab) : 0.0f;
                v[k][e] = ex;
                local_sum = __fadd_rn(local_sum, ex);
            }
        float denom;
        if (EXACT) {
#pragma unroll
            for (int k = 0; k < V; ++k) {
                const std::size_t c = threadIdx.x + static_cast<std::size_t>(k) * kSmThreads;
                if (c < T4)
                    reinterpret_cast<float4*>(staged)[c] = make_float4(v[k][0], v[k][1], v[k][2], v[k][3]);
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
            denom = block_sum<kSmWarps>(local_sum, red[1]);
        }
#pragma unroll
        for (int k = 0; k < V; ++k) {
            const std::size_t c = threadIdx.x + static_cast<std::size_t>(k) * kSmThreads;
            if (c < T4) {
                float pv[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                    pv[e] = (valid >> (4 * k + e)) & 1u ? __fdiv_rn(v[k][e], denom) : 0.0f;
                st_plain(dst + c, make_float4(pv[0], pv[1], pv[2], pv[3]));
            }
        }
        if (EXACT) __syncthreads();  // staged[] / denom_s reused by the next row
    }
}

// Any T / ld / alignment: scaled scores staged in shared memory (T floats).
template <bool EXACT>
__global__ void __launch_bounds__(kSmThreads)
causal_softmax_smem(SoftmaxArgs a) {
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
            const float ex = exp_ref(__fsub_rn(staged[j], m), tab);
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
        for (std::size_t j = threadIdx.x; j < a.T; j += kSmThreads)
            dst[j] = (j >= begin && j <= i) ? __fdiv_rn(staged[j], denom) : 0.0f;
        __syncthreads();
    }
}

template <int V, bool EXACT>
int launch_reg(const SoftmaxArgs& a, cudaStream_t s) {
    const std::size_t smem = EXACT ? a.T * sizeof(float) : 0;
    auto kernel = causal_softmax_reg<V, EXACT>;
    if (allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem) != cudaSuccess)
        return launch_result("causal softmax: shared memory attribute");
    const unsigned grid = wave_grid(reinterpret_cast<const void*>(kernel), kSmThreads, smem, a.rows);
    kernel<<<grid, kSmThreads, smem, s>>>(a);
    return B2_OK;
}

template <bool EXACT>
int launch_smem(const SoftmaxArgs& a, cudaStream_t s) {
    const std::size_t smem = a.T * sizeof(float);
    auto kernel = causal_softmax_smem<EXACT>;
    if (allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem) != cudaSuccess)
        return launch_result("causal softmax: shared memory attribute");
    const unsigned grid = wave_grid(reinterpret_cast<const void*>(kernel), kSmThreads, smem, a.rows);
    kernel<<<grid, kSmThreads, smem, s>>>(a);
    return B2_OK;
}

template <bool EXACT>
int dispatch(const SoftmaxArgs& a, bool vec, cudaStream_t s) {
    const std::size_t T4 = a.T / 4;
    if (vec && T4 <= 8 * kSmThreads) {
        if (T4 <= kSmThreads) return launch_reg<1, EXACT>(a, s);
        if (T4 <= 2 * kSmThreads) return launch_reg<2, EXACT>(a, s);
        if (T4 <= 4 * kSmThreads) return launch_reg<4, EXACT>(a, s);
        return launch_reg<8, EXACT>(a, s);
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
