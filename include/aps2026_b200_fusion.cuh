/*
 * aps2026_b200_fusion.cuh -- device-side fusion hooks for a caller's own GEMM
 * kernels (CUDA C++, header only, sm_100a).
 *
 * The non-GEMM ops of the prefill path sit between GEMMs, so two of them can
 * move into the GEMMs around them and save a round trip of the activations
 * through HBM:
 *
 *   - RoPE as the q/k projection's epilogue. Output columns j and j + half of
 *     one head (half = head_dim / 2) form a rotation pair; a GEMM tile that
 *     keeps both in one thread's registers -- the reference's 8x8 q/k tile
 *     does, its columns tx*4+i and 64+tx*4+i being 64 apart
 *     (ezzy0654/aps2026 docs/2026-08-26-optimization.md:217-219, tile at
 *     src/tensor.cu:713-831) -- rotates them with rope_rotate before the
 *     store, and the separate RoPE pass (20 KB per row per layer at 16 + 4
 *     heads of 128) disappears.
 *   - LayerNorm as the next GEMM's prologue. With each row's mean and 1/std
 *     from b2_layer_norm_stats, the GEMM forms its A operand element by
 *     element with layer_norm_value while loading x, and the normalised
 *     rows are never written.
 *
 * Both functions are the arithmetic of the library's own kernels (b2_rope,
 * b2_layer_norm and its fused forms call them), so an epilogue or prologue
 * built on them gives bit for bit what the separate launches give, and the
 * reference's kernels give with B2_FLAG_EXACT_ORDER statistics
 * (tests/test_fusion_gpu.py checks both through a test GEMM).
 */
#ifndef APS2026_B200_FUSION_CUH
#define APS2026_B200_FUSION_CUH

namespace b2_fusion {

/*
 * Rotate-half RoPE of one pair: x0 = column j, x1 = column j + half of one
 * head, c / s = the cos / sin table entries [pos * half + j] of b2_rope_table.
 *   x0' = x0 * c - x1 * s,   x1' = x1 * c + x0 * s
 * with the multiply-adds fused as nvcc fuses the reference's k_rope
 * expressions (src/tensor.cu:2180-2197): fma(x0, c, -(x1 * s)) and
 * fma(x0, s, x1 * c).
 */
__device__ __forceinline__ void rope_rotate(float& x0, float& x1, float c, float s) {
    const float a = __fmaf_rn(x0, c, -__fmul_rn(x1, s));
    const float b = __fmaf_rn(x0, s, __fmul_rn(x1, c));
    x0 = a;
    x1 = b;
}

/*
 * LayerNorm output of one element: ((x - mean) * inv) * gamma + beta, the
 * last operation fused, as the reference's ln_write (src/tensor.cu:2043-2047).
 */
__device__ __forceinline__ float layer_norm_value(float x, float mean, float inv, float gamma, float beta) {
    return __fmaf_rn(__fmul_rn(__fsub_rn(x, mean), inv), gamma, beta);
}

}  // namespace b2_fusion

#endif /* APS2026_B200_FUSION_CUH */
