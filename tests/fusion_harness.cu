// TEST HARNESS ONLY (compiled by tests/test_fusion_gpu.py): a plain GEMM
// C[M, N] = A[M, K] . B[N, K]^T standing in for a caller's projection
// kernel, with the fusion hooks of include/aps2026_b200_fusion.cuh:
//   prologue  A[r, k] = b2_fusion::layer_norm_value(X[r, k], mean[r], inv[r],
//             gamma[k], beta[k]) formed while loading, from the statistics of
//             b2_layer_norm_stats;
//   epilogue  output columns j and j + half of each head rotated by
//             b2_fusion::rope_rotate with the b2_rope_table entries of the
//             row's position, before the store.
// One thread per (row, head, j < half) keeps the RoPE pair in registers, as
// the reference's 8x8 tile does for its columns 64 apart. The dot products
// are ascending-k FMA chains in both the fused and the unfused launch, so
// the comparison isolates the hooks.
#include <cstddef>
#include <cstdint>

#include <cuda_runtime.h>

#include "aps2026_b200_fusion.cuh"

namespace {

struct Args {
    const float* a;  // A, or X when the prologue applies
    const float* b;
    float* c;
    std::size_t m, n, k, head_dim;
    const float* mean;
    const float* inv;
    const float* gamma;
    const float* beta;
    const float* cos_t;
    const float* sin_t;
    const std::uint32_t* row_pos;
    int prologue, epilogue;
};

__global__ void gemm_pairs(Args p) {
    const std::size_t half = p.head_dim / 2;
    const std::size_t pairs = p.n / 2;  // (head, j < half) per row
    const std::size_t id = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (id >= p.m * pairs) return;
    const std::size_t r = id / pairs, pr = id % pairs;
    const std::size_t head = pr / half, j = pr % half;
    const std::size_t c0 = head * p.head_dim + j, c1 = c0 + half;
    float acc0 = 0.0f, acc1 = 0.0f;
    for (std::size_t kk = 0; kk < p.k; ++kk) {
        float av = p.a[r * p.k + kk];
        if (p.prologue) av = b2_fusion::layer_norm_value(av, p.mean[r], p.inv[r], p.gamma[kk], p.beta[kk]);
        acc0 = __fmaf_rn(av, p.b[c0 * p.k + kk], acc0);
        acc1 = __fmaf_rn(av, p.b[c1 * p.k + kk], acc1);
    }
    if (p.epilogue) {
        const std::size_t t = static_cast<std::size_t>(p.row_pos[r]) * half + j;
        b2_fusion::rope_rotate(acc0, acc1, p.cos_t[t], p.sin_t[t]);
    }
    p.c[r * p.n + c0] = acc0;
    p.c[r * p.n + c1] = acc1;
}

// The prologue alone: out[r, k] = layer_norm_value(X[r, k], ...).
__global__ void prologue_rows(const float* x, const float* mean, const float* inv, const float* gamma,
                              const float* beta, float* out, std::size_t m, std::size_t k) {
    const std::size_t id = static_cast<std::size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (id >= m * k) return;
    const std::size_t r = id / k, kk = id % k;
    out[id] = b2_fusion::layer_norm_value(x[id], mean[r], inv[r], gamma[kk], beta[kk]);
}

}  // namespace

extern "C" int harness_gemm(const float* a, const float* b, float* c, std::size_t m, std::size_t n, std::size_t k,
                            std::size_t head_dim, const float* mean, const float* inv, const float* gamma,
                            const float* beta, const float* cos_t, const float* sin_t, const std::uint32_t* row_pos,
                            int prologue, int epilogue, void* stream) {
    Args p{a, b, c, m, n, k, head_dim, mean, inv, gamma, beta, cos_t, sin_t, row_pos, prologue, epilogue};
    const std::size_t threads = m * (n / 2);
    gemm_pairs<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
    return static_cast<int>(cudaGetLastError());
}

extern "C" int harness_prologue(const float* x, const float* mean, const float* inv, const float* gamma,
                                const float* beta, float* out, std::size_t m, std::size_t k, void* stream) {
    const std::size_t n = m * k;
    prologue_rows<<<static_cast<unsigned>((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, mean, inv, gamma, beta, out, m, k);
    return static_cast<int>(cudaGetLastError());
}
