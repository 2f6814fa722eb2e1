// Row gather: out[i, :] = x[rows[i], :] (embedding lookup, last-row pick,
// node -> token expansion).
//
// Reference: tensor_ops::gather_rows_gpu (src/tensor.cu:3379-3387,
// :3419-3426) launching k_gather_rows (:2635-2642), which moves one float
// per thread with two integer divisions per element. Here one CTA copies a
// whole row with 128-bit loads/stores, all of a thread's loads issued before
// its stores; CTAs loop over rows (grid = one resident wave) so the index is
// read once per row. HBM bound: 2 * h * 4 bytes + 4 index bytes per row.
//
// Rows of aligned, 16-byte-multiple length go through the bulk-copy (TMA)
// engine instead (gather_rows_bulk): a one-warp CTA keeps a ring of
// kBulkStages row chunks in shared memory, each loaded by one
// cp.async.bulk completing on its own mbarrier and written out by one bulk
// store, so a CTA has up to kBulkStages * kBulkChunk bytes in flight with
// no register staging and three CTAs fit an SM.
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

constexpr int kBulkStages = 4;
constexpr std::size_t kBulkMinRowBytes = 4096;  // shorter rows: the register-staged kernel
constexpr unsigned kBulkChunk = 16384;  // bytes per stage; a row of 4096 floats is one chunk

// Unit u = chunk (u % chunks_per_row) of output row u / chunks_per_row. The
// CTA's units are blockIdx.x + k * gridDim.x, k = 0 .. n-1; unit k sits in
// slot k % kBulkStages, whose barrier completes phase k / kBulkStages.
// Lane 0 issues every copy; all lanes wait and write the zeros of an
// out-of-range row. Each wait is bounded; on a timeout the CTA reports
// B2_CHECK_WAIT, waits (again bounded) for the loads it issued, drains its
// stores and stops.
__global__ void __launch_bounds__(32)
gather_rows_bulk(const float* __restrict__ x, std::size_t x_rows, std::size_t h,
                 const std::uint32_t* __restrict__ rows, std::size_t count, float* __restrict__ out) {
    pdl_begin();
    extern __shared__ __align__(128) unsigned char stage[];  // [kBulkStages][kBulkChunk]
    __shared__ __align__(8) std::uint64_t bar[kBulkStages];
    const unsigned lane = threadIdx.x;
    const std::size_t row_bytes = h * sizeof(float);
    const std::size_t cpr = (row_bytes + kBulkChunk - 1) / kBulkChunk;  // chunks per row
    const std::size_t units = count * cpr;
    if (blockIdx.x >= units) return;
    const std::size_t n = (units - 1 - blockIdx.x) / gridDim.x + 1;
    if (lane == 0)
        for (int i = 0; i < kBulkStages; ++i) mbar_init(&bar[i], 1);
    __syncwarp();
    // row, source row, byte offset and size of the CTA's k-th unit
    struct Unit {
        std::size_t row, off;
        std::uint32_t src;
        unsigned bytes;
    };
    auto unit = [&](std::size_t k) {
        const std::size_t u = blockIdx.x + k * gridDim.x;
        Unit t;
        t.row = u / cpr;
        t.off = (u % cpr) * kBulkChunk;
        t.bytes = static_cast<unsigned>(row_bytes - t.off < kBulkChunk ? row_bytes - t.off : kBulkChunk);
        t.src = __ldg(rows + t.row);
        return t;
    };
    auto issue = [&](std::size_t k) {  // lane 0
        const Unit t = unit(k);
        std::uint64_t* b = &bar[k % kBulkStages];
        if (t.src >= x_rows) {
            mbar_arrive(b);  // nothing to load; the consumer writes zeros
            return;
        }
        mbar_expect_tx(b, t.bytes);
        bulk_g2s(stage + (k % kBulkStages) * kBulkChunk,
                 reinterpret_cast<const unsigned char*>(x) + t.src * row_bytes + t.off, t.bytes, b);
    };
    if (lane == 0)
        for (std::size_t k = 0; k < n && k < static_cast<std::size_t>(kBulkStages); ++k) issue(k);
    for (std::size_t k = 0; k < n; ++k) {
        const unsigned parity = static_cast<unsigned>((k / kBulkStages) & 1u);
        if (!__all_sync(0xffffffffu, mbar_wait(&bar[k % kBulkStages], parity))) {
            if (lane == 0) {
                flag_check(B2_CHECK_WAIT);
                // the loads issued so far (units up to k + kBulkStages - 2, or the
                // first kBulkStages when k == 0) may still land: one bounded wait
                // each on their barriers, the only completion signal a global ->
                // shared bulk copy has, then the stores' bulk group. A wait that
                // gives up again means the copy engine has stopped; an unbounded
                // wait would hang the GPU, so the warp returns and B2_CHECK_WAIT
                // tells the host that the context is no longer usable.
                const std::size_t issued = k == 0 ? kBulkStages : k + kBulkStages - 1;
                for (std::size_t j = k; j < n && j < issued; ++j)
                    mbar_wait(&bar[j % kBulkStages], static_cast<unsigned>((j / kBulkStages) & 1u));
                bulk_wait<0>();
            }
            __syncwarp();
            return;
        }
        const Unit t = unit(k);
        unsigned char* dst = reinterpret_cast<unsigned char*>(out) + t.row * row_bytes + t.off;
        if (t.src >= x_rows) {
            if (lane == 0 && t.off == 0) flag_check(B2_CHECK_GATHER);
            for (unsigned j = lane * 16u; j < t.bytes; j += 32u * 16u)
                *reinterpret_cast<float4*>(dst + j) = make_float4(0.f, 0.f, 0.f, 0.f);
        } else if (lane == 0) {
            bulk_s2g(dst, stage + (k % kBulkStages) * kBulkChunk, t.bytes);
        }
        if (lane == 0) {
            bulk_commit();  // (an empty group for a zero-filled unit)
            // refill the previous unit's slot once its store has read it
            if (k >= 1 && k - 1 + kBulkStages < n) {
                bulk_wait_read<1>();
                issue(k - 1 + kBulkStages);
            }
        }
        __syncwarp();
    }
    if (lane == 0) bulk_wait<0>();
    __syncwarp();
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
    if ((h & 3u) == 0 && aligned16(x) && aligned16(out) && h * sizeof(float) >= kBulkMinRowBytes) {
        constexpr std::size_t smem = kBulkStages * kBulkChunk;
        if (allow_dynamic_smem(reinterpret_cast<const void*>(gather_rows_bulk), smem) != cudaSuccess)
            return launch_result("b2_gather_rows: shared memory attribute");
        const std::size_t units = count * ((h * sizeof(float) + kBulkChunk - 1) / kBulkChunk);
        const unsigned grid = wave_grid(reinterpret_cast<const void*>(gather_rows_bulk), 32, smem, units);
        launch_pdl(gather_rows_bulk, grid, 32, smem, s, x, x_rows, h, rows, count, out);
    } else if ((h & 3u) == 0 && aligned16(x) && aligned16(out)) {
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
