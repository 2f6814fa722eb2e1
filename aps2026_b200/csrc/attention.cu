// Prefix-tree GQA attention core: for every trie row and KV head, the
// softmax-weighted sum of the values of the row's ancestor chain.
//
// Reference: k_attention_tree_gqa4 (src/tensor.cu:2425-2633), launched by
// attention_tree_gpu (:3361-3377) with one 128-thread CTA per (row, KV head)
// that stages 16 keys at a time with half of its threads computing, runs the
// softmax on 4 threads, and reads V straight from global memory one scalar
// per key per thread.
//
// Here, also one CTA per (row, KV head) with the same arithmetic in the
// same order (so B2_FLAG_EXACT_ORDER output is bit-identical), but:
//   - keys: tiles of 64 chain rows staged in shared memory with 128-bit
//     loads (all of a thread's loads of a tile issued before any is
//     stored), every thread computing one key for two of the four query
//     heads from 128-bit shared reads -- the four accumulators over d mod 4
//     and their (a0 + a1) + (a2 + a3) combination are the reference's;
//   - softmax: a warp per query head (max by shuffles, the exponential of
//     fastexp.cuh, the denominator serially by one lane in EXACT_ORDER or
//     by a shuffle tree otherwise, Markstein division);
//   - values: tiles of 64 rows staged like the keys, each thread owning one
//     output dimension and accumulating the four heads in ascending key
//     order with fused multiply-adds, reading p[w][0..3] as one 128-bit
//     shared load.
// FP32 CUDA-core work (the reference's arithmetic has no tensor-core
// equivalent): 2 * 4 * window * head_dim multiply-adds per CTA.
#include "common.cuh"
#include "fastexp.cuh"

namespace b2 {
namespace {

constexpr int kAttnThreads = 128;
constexpr int kGroup = 4;       // query heads per KV head (GQA-4, as the reference requires)
constexpr int kKeyTile = 64;    // chain rows per staged tile

struct AttnArgs {
    const float* q;
    const float* k;
    const float* v;
    float* out;
    const std::uint32_t* row_pos;
    const std::uint32_t* anc;
    std::size_t anc_stride, rows, q_heads, kv_heads, window, max_window;
    float scale;
};

// Division by a row denominator d >= 1 with one reciprocal per row, as in
// softmax.cu (Markstein's correction gives the correctly rounded quotient).
__device__ __forceinline__ float attn_div(float e, float d, float y) {
    if (e < 0x1p-96f) return __fdiv_rn(e, d);
    const float q = __fmul_rn(e, y);
    return __fmaf_rn(__fmaf_rn(-d, q, e), y, q);
}

// Shared layout (floats): scores [max_window][4] | chain [max_window] (u32)
// | q [HD][4] | tile [64][HD + 4] (keys, then values).
template <int HD, bool EXACT>
__global__ void __launch_bounds__(kAttnThreads)
attention_tree_kernel(AttnArgs a) {
    pdl_begin();
    constexpr int PITCH = HD + 4;   // 16-byte row pitch offset: conflict-free 128-bit reads
    constexpr int HD4 = HD / 4;
    extern __shared__ __align__(16) float smem[];
    __shared__ double tab[64];
    __shared__ int bad_s;
    float* scores = smem;                                                   // [w][g]
    std::uint32_t* chain = reinterpret_cast<std::uint32_t*>(scores + kGroup * a.max_window);
    float* qs = reinterpret_cast<float*>(chain + ((a.max_window + 3) & ~std::size_t(3)));  // [d][g]
    float* tile = qs + HD * kGroup;
    load_exp2_table(tab);

    const std::size_t task = blockIdx.x;
    const std::size_t row = task / a.kv_heads, kh = task % a.kv_heads;
    const unsigned tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const std::size_t pos = a.row_pos[row];
    if (tid == 0) bad_s = pos >= a.anc_stride;
    __syncthreads();
    float* out_row = a.out + (row * a.q_heads + kh * kGroup) * HD;
    if (bad_s) {  // position outside the ancestor table: report, output zeros
        if (tid == 0) flag_check(B2_CHECK_ATTENTION);
        for (int i = tid; i < kGroup * HD; i += kAttnThreads) out_row[i] = 0.0f;
        return;
    }
    const std::size_t begin = pos + 1 > a.window ? pos + 1 - a.window : 0;
    const int W = static_cast<int>(pos - begin + 1);
    const std::uint32_t* anc_row = a.anc + row * a.anc_stride + begin;
    for (int i = tid; i < W; i += kAttnThreads) {
        std::uint32_t c = anc_row[i];
        if (c >= a.rows) {
            flag_check(B2_CHECK_ATTENTION);
            c = static_cast<std::uint32_t>(row);  // keep the access in bounds
        }
        chain[i] = c;
    }
    for (int i = tid; i < kGroup * HD; i += kAttnThreads) {
        const int g = i / HD, d = i % HD;
        qs[d * kGroup + g] = a.q[(row * a.q_heads + kh * kGroup + g) * HD + d];
    }
    __syncthreads();

    const std::size_t kv_row = a.kv_heads * HD;
    const float4* k4 = reinterpret_cast<const float4*>(a.k + kh * HD);
    const float4* v4 = reinterpret_cast<const float4*>(a.v + kh * HD);
    constexpr int PER_THREAD = kKeyTile * HD4 / kAttnThreads;  // float4 per thread per tile

    // ---- scores: s[w][g] = ((a0 + a1) + (a2 + a3)) * scale ----
    const int key = tid % kKeyTile, g0 = (tid / kKeyTile) * 2;  // this thread: key slot, heads g0, g0+1
    const bool hi = g0 != 0;
    for (int base = 0; base < W; base += kKeyTile) {
        const int count = min(kKeyTile, W - base);
        float4 stage[PER_THREAD];
#pragma unroll
        for (int u = 0; u < PER_THREAD; ++u) {
            const int i = tid + u * kAttnThreads, ks = i / HD4, c = i % HD4;
            stage[u] = ks < count ? __ldg(k4 + static_cast<std::size_t>(chain[base + ks]) * (kv_row / 4) + c)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < PER_THREAD; ++u) {
            const int i = tid + u * kAttnThreads, ks = i / HD4, c = i % HD4;
            reinterpret_cast<float4*>(tile + ks * PITCH)[c] = stage[u];
        }
        __syncthreads();
        if (key < count) {
            float acc[2][4] = {};
            const float4* kr = reinterpret_cast<const float4*>(tile + key * PITCH);
#pragma unroll 8
            for (int c = 0; c < HD4; ++c) {
                const float4 kv = kr[c];
                const float4 qa = reinterpret_cast<const float4*>(qs)[4 * c + 0];  // d = 4c, heads 0..3
                const float4 qb = reinterpret_cast<const float4*>(qs)[4 * c + 1];
                const float4 qc = reinterpret_cast<const float4*>(qs)[4 * c + 2];
                const float4 qd = reinterpret_cast<const float4*>(qs)[4 * c + 3];
                // this thread's two heads (g0 = 0: heads 0, 1; g0 = 2: heads 2, 3)
                const float qa0 = hi ? qa.z : qa.x, qa1 = hi ? qa.w : qa.y;
                const float qb0 = hi ? qb.z : qb.x, qb1 = hi ? qb.w : qb.y;
                const float qc0 = hi ? qc.z : qc.x, qc1 = hi ? qc.w : qc.y;
                const float qd0 = hi ? qd.z : qd.x, qd1 = hi ? qd.w : qd.y;
                acc[0][0] = __fmaf_rn(qa0, kv.x, acc[0][0]);
                acc[0][1] = __fmaf_rn(qb0, kv.y, acc[0][1]);
                acc[0][2] = __fmaf_rn(qc0, kv.z, acc[0][2]);
                acc[0][3] = __fmaf_rn(qd0, kv.w, acc[0][3]);
                acc[1][0] = __fmaf_rn(qa1, kv.x, acc[1][0]);
                acc[1][1] = __fmaf_rn(qb1, kv.y, acc[1][1]);
                acc[1][2] = __fmaf_rn(qc1, kv.z, acc[1][2]);
                acc[1][3] = __fmaf_rn(qd1, kv.w, acc[1][3]);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float sc = __fadd_rn(__fadd_rn(acc[h][0], acc[h][1]), __fadd_rn(acc[h][2], acc[h][3]));
                scores[(base + key) * kGroup + g0 + h] = __fmul_rn(sc, a.scale);
            }
        }
        __syncthreads();  // the tile is overwritten next
    }

    // ---- softmax per head: warp g ----
    {
        const int g = warp;
        float m = -3.402823466e+38F;
        for (int w = lane; w < W; w += 32) m = fmaxf(m, scores[w * kGroup + g]);
        m = warp_max(m);
        float part = 0.0f;
        for (int w = lane; w < W; w += 32) {
            const float e = exp_ref(__fsub_rn(scores[w * kGroup + g], m), tab);
            scores[w * kGroup + g] = e;
            part = __fadd_rn(part, e);
        }
        float denom;
        if (EXACT) {
            __syncwarp();
            float d = 0.0f;
            if (lane == 0)
                for (int w = 0; w < W; ++w) d = __fadd_rn(d, scores[w * kGroup + g]);
            denom = __shfl_sync(0xffffffffu, d, 0);
        } else {
            denom = warp_sum(part);
        }
        const float y = __frcp_rn(denom);
        for (int w = lane; w < W; w += 32) scores[w * kGroup + g] = attn_div(scores[w * kGroup + g], denom, y);
    }
    __syncthreads();

    // ---- out[g][d] = sum_w p[w][g] * v[chain[w]][d], ascending w ----
    float value[kGroup] = {};
    for (int base = 0; base < W; base += kKeyTile) {
        const int count = min(kKeyTile, W - base);
        float4 stage[PER_THREAD];
#pragma unroll
        for (int u = 0; u < PER_THREAD; ++u) {
            const int i = tid + u * kAttnThreads, ks = i / HD4, c = i % HD4;
            stage[u] = ks < count ? __ldg(v4 + static_cast<std::size_t>(chain[base + ks]) * (kv_row / 4) + c)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int u = 0; u < PER_THREAD; ++u) {
            const int i = tid + u * kAttnThreads, ks = i / HD4, c = i % HD4;
            reinterpret_cast<float4*>(tile + ks * PITCH)[c] = stage[u];
        }
        __syncthreads();
        for (int d = tid; d < HD; d += kAttnThreads) {
            float acc[kGroup] = {value[0], value[1], value[2], value[3]};
            for (int w = 0; w < count; ++w) {
                const float vv = tile[w * PITCH + d];
                const float4 p = reinterpret_cast<const float4*>(scores)[base + w];
                acc[0] = __fmaf_rn(p.x, vv, acc[0]);
                acc[1] = __fmaf_rn(p.y, vv, acc[1]);
                acc[2] = __fmaf_rn(p.z, vv, acc[2]);
                acc[3] = __fmaf_rn(p.w, vv, acc[3]);
            }
#pragma unroll
            for (int g = 0; g < kGroup; ++g) value[g] = acc[g];
        }
        __syncthreads();
    }
    for (int d = tid; d < HD; d += kAttnThreads)
#pragma unroll
        for (int g = 0; g < kGroup; ++g) out_row[g * HD + d] = value[g];
}

template <int HD, bool EXACT>
int launch_attention(const AttnArgs& a, cudaStream_t s) {
    const std::size_t chain_words = (a.max_window + 3) & ~std::size_t(3);
    const std::size_t smem = (kGroup * a.max_window + chain_words + HD * kGroup + kKeyTile * (HD + 4)) * 4;
    auto kernel = attention_tree_kernel<HD, EXACT>;
    if (smem > 200 * 1024) return set_error(B2_ERR_UNSUPPORTED, "b2_attention_tree: window too large");
    if (allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem) != cudaSuccess)
        return launch_result("b2_attention_tree: shared memory attribute");
    launch_pdl(kernel, static_cast<unsigned>(a.rows * a.kv_heads), kAttnThreads, smem, s, a);
    return B2_OK;
}

}  // namespace
}  // namespace b2

B2_DEFINE_CHECK_TAKER(attention)

extern "C" int b2_attention_tree(const float* q, const float* k, const float* v, float* out,
                                 const uint32_t* row_pos, const uint32_t* anc, size_t anc_stride, size_t rows,
                                 size_t q_heads, size_t kv_heads, size_t head_dim, size_t window, uint32_t flags,
                                 b2_stream_t stream) {
    using namespace b2;
    if (rows == 0) return B2_OK;
    if (!q || !k || !v || !out || !row_pos || !anc) return invalid("b2_attention_tree: null pointer");
    if (kv_heads == 0 || q_heads != kGroup * kv_heads)
        return invalid("attention_tree_gpu expects GQA-4");
    if (head_dim != 128 && head_dim != 64)
        return set_error(B2_ERR_UNSUPPORTED, "b2_attention_tree: head_dim must be 64 or 128");
    if (window == 0 || anc_stride == 0) return invalid("b2_attention_tree: window / anc_stride is 0");
    if (rows * kv_heads > 0x7FFFFFFFu) return invalid("b2_attention_tree: too many rows");
    if (!aligned16(k) || !aligned16(v)) return invalid("b2_attention_tree: k / v not 16-byte aligned");
    AttnArgs a{q, k, v, out, row_pos, anc, anc_stride, rows, q_heads, kv_heads, window,
               window < anc_stride ? window : anc_stride, 1.0f / sqrtf(static_cast<float>(head_dim))};
    const bool exact = (flags & B2_FLAG_EXACT_ORDER) != 0;
    cudaStream_t s = as_stream(stream);
    int rc;
    if (head_dim == 128) rc = exact ? launch_attention<128, true>(a, s) : launch_attention<128, false>(a, s);
    else rc = exact ? launch_attention<64, true>(a, s) : launch_attention<64, false>(a, s);
    if (rc) return rc;
    return launch_result("b2_attention_tree");
}
