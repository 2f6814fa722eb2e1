// Row-source helpers shared by the LayerNorm family and the MoE un-permute:
// how one 128-bit chunk of "the row to normalise" is produced.
#pragma once

#include "common.cuh"

namespace b2 {

// The two source rows of token t's MoE output, in the order the reference
// accumulates them: the assignment of the LOWER expert id first
// (k_moe_combine, src/tensor.cu:1975-1986). A position outside
// [0, expert_rows) is reported and replaced by `expert_rows` (= "no row").
struct CombineRows {
    std::size_t lo, hi;
};

__device__ __forceinline__ CombineRows combine_rows(const std::uint8_t* routes,
                                                    const std::uint32_t* route_positions,
                                                    std::size_t t, std::size_t expert_rows) {
    const std::uint8_t e0 = __ldg(routes + 2 * t), e1 = __ldg(routes + 2 * t + 1);
    const std::size_t p0 = __ldg(route_positions + 2 * t);
    const std::size_t p1 = __ldg(route_positions + 2 * t + 1);
    CombineRows r;
    r.lo = e0 < e1 ? p0 : p1;
    r.hi = e0 < e1 ? p1 : p0;
    if (r.lo >= expert_rows || r.hi >= expert_rows) {
        if (threadIdx.x == 0) flag_check(B2_CHECK_COMBINE);
        if (r.lo >= expert_rows) r.lo = expert_rows;
        if (r.hi >= expert_rows) r.hi = expert_rows;
    }
    return r;
}

// value = 0; value += 0.5 * lo; value += 0.5 * hi -- each += a fused
// multiply-add, as nvcc compiles the reference's accumulation.
__device__ __forceinline__ float combine_one(float lo, float hi) {
    return __fmaf_rn(0.5f, hi, __fmaf_rn(0.5f, lo, 0.0f));
}

__device__ __forceinline__ float4 combine4(const float4& lo, const float4& hi) {
    return make_float4(combine_one(lo.x, hi.x), combine_one(lo.y, hi.y),
                       combine_one(lo.z, hi.z), combine_one(lo.w, hi.w));
}

__device__ __forceinline__ float4 add4(const float4& a, const float4& b) {
    return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z),
                       __fadd_rn(a.w, b.w));
}

__device__ __forceinline__ float4 zero4() { return make_float4(0.f, 0.f, 0.f, 0.f); }

}  // namespace b2
