// Rotary position embedding on Q and K in one launch, plus the host builder
// of the cos/sin table.
//
// Reference: rope_table (src/tensor.cu:2695-2737, host) and k_rope
// (:2180-2197), launched once for Q and once for K by apply_rope_gpu /
// apply_rope_tree_gpu (:3297-3314, :3342-3359) with one scalar pair per
// thread and three 64-bit divisions per pair.
//
// Here a CTA owns whole rows: its threads cover the (q_heads + kv_heads) x
// head_dim/8 float4 pairs of a row -- the first and second halves of a head
// are rotated together from two 128-bit loads. The
// cos/sin rows (head_dim/2 floats each, 1 MB for 4096 positions) stay in L2.
// HBM bound: 2 * (q_heads + kv_heads) * head_dim * 4 bytes per row.
#include <cmath>
#include <vector>

#include "common.cuh"

namespace b2 {
namespace {

// Rows per thread per step. One: measured at config 5 (131,072 rows, 16 + 4
// heads of 128) 400 us against 456 us for two and 569 us for four -- with
// one row per step, consecutive CTAs stream consecutive rows.
constexpr int kRopeRowsPerStep = 1;

// out0 = x0 * c - x1 * s, out1 = x1 * c + x0 * s, fused the way nvcc fuses
// the reference's expressions in k_rope -- the public epilogue hook of
// aps2026_b200_fusion.cuh, so a GEMM epilogue built on it rotates exactly
// as this kernel does.
__device__ __forceinline__ void rotate(float& x0, float& x1, float c, float s) {
    b2_fusion::rope_rotate(x0, x1, c, s);
}

struct RopeArgs {
    float* q;
    float* k;
    const std::uint32_t* row_pos;
    const float* cos_t;
    const float* sin_t;
    std::size_t rows, q_heads, kv_heads, head_dim, table_rows;
};

// Vector path: head_dim % 8 == 0 and 16-byte aligned operands.
__global__ void __launch_bounds__(1024)
rope_vec(RopeArgs a) {
    pdl_begin();
    const unsigned half4 = static_cast<unsigned>(a.head_dim / 8);  // float4 per half head
    const unsigned per_row = static_cast<unsigned>(a.q_heads + a.kv_heads) * half4;
    const unsigned q_items = static_cast<unsigned>(a.q_heads) * half4;
    const std::size_t q_row4 = a.q_heads * a.head_dim / 4, k_row4 = a.kv_heads * a.head_dim / 4;
    const std::size_t half_t4 = a.head_dim / 8;  // table row in float4
    float4* q4 = reinterpret_cast<float4*>(a.q);
    float4* k4 = reinterpret_cast<float4*>(a.k);
    const float4* c4 = reinterpret_cast<const float4*>(a.cos_t);
    const float4* s4 = reinterpret_cast<const float4*>(a.sin_t);

    for (std::size_t r0 = static_cast<std::size_t>(blockIdx.x) * kRopeRowsPerStep; r0 < a.rows;
         r0 += static_cast<std::size_t>(gridDim.x) * kRopeRowsPerStep) {
        for (unsigned it = threadIdx.x; it < per_row; it += blockDim.x) {
            const bool is_q = it < q_items;
            const unsigned local = is_q ? it : it - q_items;
            const unsigned head = local / half4, g = local % half4;
            float4* base = is_q ? q4 : k4;
            const std::size_t row4 = is_q ? q_row4 : k_row4;
            const std::size_t off = static_cast<std::size_t>(head) * 2 * half4 + g;
            float4 x0[kRopeRowsPerStep], x1[kRopeRowsPerStep], c[kRopeRowsPerStep], s[kRopeRowsPerStep];
            bool ok[kRopeRowsPerStep];
#pragma unroll
            for (int u = 0; u < kRopeRowsPerStep; ++u) {
                const std::size_t r = r0 + u;
                ok[u] = false;
                if (r < a.rows) {
                    const std::uint32_t pos = __ldg(a.row_pos + r);
                    if (pos < a.table_rows) {
                        ok[u] = true;
                        float4* p = base + r * row4 + off;
                        x0[u] = ld_plain(p);
                        x1[u] = ld_plain(p + half4);
                        c[u] = __ldg(c4 + static_cast<std::size_t>(pos) * half_t4 + g);
                        s[u] = __ldg(s4 + static_cast<std::size_t>(pos) * half_t4 + g);
                    } else if (it == 0) {
                        flag_check(B2_CHECK_ROPE);
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < kRopeRowsPerStep; ++u) {
                if (!ok[u]) continue;
                rotate(x0[u].x, x1[u].x, c[u].x, s[u].x);
                rotate(x0[u].y, x1[u].y, c[u].y, s[u].y);
                rotate(x0[u].z, x1[u].z, c[u].z, s[u].z);
                rotate(x0[u].w, x1[u].w, c[u].w, s[u].w);
                float4* p = base + (r0 + u) * row4 + off;
                st_plain(p, x0[u]);
                st_plain(p + half4, x1[u]);
            }
        }
    }
}

// Any even head_dim / alignment: one pair per thread, rows strided by CTA.
__global__ void __launch_bounds__(256)
rope_scalar(RopeArgs a) {
    pdl_begin();
    const std::size_t half = a.head_dim / 2;
    const std::size_t per_row = (a.q_heads + a.kv_heads) * half;
    const std::size_t q_items = a.q_heads * half;
    for (std::size_t r = blockIdx.x; r < a.rows; r += gridDim.x) {
        const std::uint32_t pos = __ldg(a.row_pos + r);
        if (pos >= a.table_rows) {
            if (threadIdx.x == 0) flag_check(B2_CHECK_ROPE);
            continue;
        }
        for (std::size_t it = threadIdx.x; it < per_row; it += blockDim.x) {
            const bool is_q = it < q_items;
            const std::size_t local = is_q ? it : it - q_items;
            const std::size_t head = local / half, j = local % half;
            float* x = is_q ? a.q + (r * a.q_heads + head) * a.head_dim
                            : a.k + (r * a.kv_heads + head) * a.head_dim;
            float x0 = x[j], x1 = x[j + half];
            rotate(x0, x1, __ldg(a.cos_t + pos * half + j), __ldg(a.sin_t + pos * half + j));
            x[j] = x0;
            x[j + half] = x1;
        }
    }
}

}  // namespace
}  // namespace b2

B2_DEFINE_CHECK_TAKER(rope)

extern "C" {

int b2_rope_table(size_t max_seq, size_t head_dim, float theta, float* cos_host,
                  float* sin_host) {
    if (!cos_host || !sin_host) return b2::invalid("b2_rope_table: null pointer");
    if (head_dim == 0 || (head_dim & 1u)) return b2::invalid("b2_rope_table: head_dim must be even");
    const std::size_t half = head_dim / 2;
    // Same float expressions as the reference's host table (powf, then cosf
    // and sinf of p * inv), so every entry is the same float.
    std::vector<float> inv(half);
    for (std::size_t j = 0; j < half; ++j)
        inv[j] = std::pow(theta, -2.0f * static_cast<float>(j) / static_cast<float>(head_dim));
    for (std::size_t p = 0; p < max_seq; ++p)
        for (std::size_t j = 0; j < half; ++j) {
            const float angle = static_cast<float>(p) * inv[j];
            cos_host[p * half + j] = std::cos(angle);
            sin_host[p * half + j] = std::sin(angle);
        }
    return B2_OK;
}

int b2_rope(float* q, float* k, const uint32_t* row_pos, size_t rows, size_t q_heads,
            size_t kv_heads, size_t head_dim, const float* cos_table, const float* sin_table,
            size_t table_rows, b2_stream_t stream) {
    using namespace b2;
    if (rows == 0) return B2_OK;
    if (!row_pos || !cos_table || !sin_table) return invalid("b2_rope: null pointer");
    if ((q_heads && !q) || (kv_heads && !k)) return invalid("b2_rope: null q/k");
    if (head_dim == 0 || (head_dim & 1u)) return invalid("b2_rope: head_dim must be even");
    if (q_heads + kv_heads == 0) return B2_OK;
    RopeArgs a{q, k, row_pos, cos_table, sin_table, rows, q_heads, kv_heads, head_dim, table_rows};
    cudaStream_t s = as_stream(stream);
    const bool vec = (head_dim % 8) == 0 && (!q || aligned16(q)) && (!k || aligned16(k)) &&
                     aligned16(cos_table) && aligned16(sin_table);
    if (vec) {
        const std::size_t per_row = (q_heads + kv_heads) * (head_dim / 8);
        int threads = static_cast<int>(((per_row + 31) / 32) * 32);
        if (threads > 1024) threads = 1024;
        const std::size_t steps = (rows + kRopeRowsPerStep - 1) / kRopeRowsPerStep;
        const unsigned grid = wave_grid(reinterpret_cast<const void*>(rope_vec), threads, 0, steps);
        launch_pdl(rope_vec, grid, threads, 0, s, a);
    } else {
        const unsigned grid = wave_grid(reinterpret_cast<const void*>(rope_scalar), 256, 0, rows);
        launch_pdl(rope_scalar, grid, 256, 0, s, a);
    }
    return launch_result("b2_rope");
}

}  // extern "C"
