// Row gather: out[i, :] = x[rows[i], :] (embedding lookup, last-row pick,
// node -> token expansion).
//
// Reference: tensor_ops::gather_rows_gpu (src/tensor.cu:3379-3387,
// :3419-3426) launching k_gather_rows (:2635-2642), which moves one float
// per thread with two integer divisions per element. Here one CTA copies a
// whole row with 128-bit loads/stores, all of a thread's loads issued before
// its stores; CTAs loop over rows (grid = one resident wave) so the index is
// read once per row. HBM bound: 2 * h * 4 bytes + 4 index bytes per row.
#include "common.cuh"

namespace b2 {
namespace {

constexpr int kGatherThreads = 256;
constexpr int kGatherUnroll = 4;  // float4 per thread in flight per step

__global__ void __launch_bounds__(kGatherThreads)
gather_rows_vec(const float4* __restrict__ x, std::size_t x_rows, std::size_t h4,
                const std::uint32_t* __restrict__ rows, std::size_t count,
                float4* __restrict__ out) {
    pdl_begin();
    for (std::size_t i = blockIdx.x; i < count; i += gridDim.x) {
        const std::uint32_t src = __ldg(rows + i);
        float4* dst = out + i * h4;
        if (src >= x_rows) {
            if (threadIdx.x == 0) flag_check(B2_CHECK_GATHER);
            for (std::size_t j = threadIdx.x; j < h4; j += kGatherThreads)
                dst[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            continue;
        }
        const float4* s = x + static_cast<std::size_t>(src) * h4;
        for (std::size_t j0 = threadIdx.x; j0 < h4; j0 += kGatherThreads * kGatherUnroll) {
            float4 v[kGatherUnroll];
#pragma unroll
            for (int u = 0; u < kGatherUnroll; ++u) {
                const std::size_t j = j0 + static_cast<std::size_t>(u) * kGatherThreads;
                if (j < h4) v[u] = ld_stream(s + j);
            }
#pragma unroll
            for (int u = 0; u < kGatherUnroll; ++u) {
                const std::size_t j = j0 + static_cast<std::size_t>(u) * kGatherThreads;
                if (j < h4) st_plain(dst + j, v[u]);
            }
        }
    }
}

// Any h or alignment: same structure, 4-byte elements.
__global__ void __launch_bounds__(kGatherThreads)
gather_rows_scalar(const float* __restrict__ x, std::size_t x_rows, std::size_t h,
                   const std::uint32_t* __restrict__ rows, std::size_t count,
                   float* __restrict__ out) {
    pdl_begin();
    for (std::size_t i = blockIdx.x; i < count; i += gridDim.x) {
        const std::uint32_t src = __ldg(rows + i);
        float* dst = out + i * h;
        if (src >= x_rows) {
            if (threadIdx.x == 0) flag_check(B2_CHECK_GATHER);
            for (std::size_t j = threadIdx.x; j < h; j += kGatherThreads) dst[j] = 0.0f;
            continue;
        }
        const float* s = x + static_cast<std::size_t>(src) * h;
        for (std::size_t j = threadIdx.x; j < h; j += kGatherThreads) dst[j] = __ldg(s + j);
    }
}

}  // namespace
}  // namespace b2

B2_DEFINE_CHECK_TAKER(gather)

extern "C" int b2_gather_rows(const float* x, size_t x_rows, size_t h,
                              const uint32_t* rows, size_t count, float* out,
                              b2_stream_t stream) {
    using namespace b2;
    if (count == 0) return B2_OK;
    if (!x || !rows || !out) return invalid("b2_gather_rows: null pointer");
    if (h == 0) return invalid("b2_gather_rows: h == 0");
    cudaStream_t s = as_stream(stream);
    if ((h & 3u) == 0 && aligned16(x) && aligned16(out)) {
        const unsigned grid = wave_grid(reinterpret_cast<const void*>(gather_rows_vec),
                                        kGatherThreads, 0, count);
        launch_pdl(gather_rows_vec, grid, kGatherThreads, 0, s, 
            reinterpret_cast<const float4*>(x), x_rows, h / 4, rows, count,
            reinterpret_cast<float4*>(out));
    } else {
        const unsigned grid = wave_grid(reinterpret_cast<const void*>(gather_rows_scalar),
                                        kGatherThreads, 0, count);
        launch_pdl(gather_rows_scalar, grid, kGatherThreads, 0, s, x, x_rows, h, rows, count, out);
    }
    return launch_result("b2_gather_rows");
}

extern "C" int b2_moe_gather_compact(const float* x, size_t x_rows, size_t h,
                                     const uint32_t* assignment_rows, size_t assignments,
                                     float* compact, b2_stream_t stream) {
    return b2_gather_rows(x, x_rows, h, assignment_rows, assignments, compact, stream);
}
