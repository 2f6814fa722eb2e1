// Prefix-tree GQA attention core: for every trie row and KV head, the
// softmax-weighted sum of the values of the row's ancestor chain.
//
// Reference: k_attention_tree_gqa4 (src/tensor.cu:2425-2633), launched by
// attention_tree_gpu (:3361-3377) with one 128-thread CTA per (row, KV head)
// that stages 16 keys at a time with half of its threads computing, runs the
// softmax on 4 threads, and reads V straight from global memory one scalar
// per key per thread.
//
// Two kernels with the reference's arithmetic in its order (so
// B2_FLAG_EXACT_ORDER output is bit-identical). head_dim 128 runs the
// query-blocked attention_tree_block below; other head dims (64) and
// windows too large for its shared memory run attention_tree_kernel, one
// CTA per (row, KV head) like the reference, but:
//   - keys: tiles of 64 chain rows staged in shared memory with 128-bit
//     loads (all of a thread's loads of a tile issued before any is
//     stored), every thread computing one key for two of the four query
//     heads from 128-bit shared reads -- the four accumulators over d mod 4
//     and their (a0 + a1) + (a2 + a3) combination are the reference's;
//   - softmax: a warp per query head (max by shuffles; in EXACT_ORDER the
//     reference's exponential (fastexp.cuh), the denominator serially by one
//     lane and Markstein division; otherwise CUDA's expf, a shuffle-tree
//     denominator and a multiplication by its reciprocal);
//   - values: tiles of 64 rows staged like the keys, each thread owning one
//     output dimension and accumulating the four heads in ascending key
//     order with fused multiply-adds, reading p[w][0..3] as one 128-bit
//     shared load.
// FP32 CUDA-core work (the reference's arithmetic has no tensor-core
// equivalent): 2 * 4 * window * head_dim multiply-adds per CTA.
#include "common.cuh"
#include "fastexp.cuh"
#include "rowload.cuh"
#include "tcgen05.cuh"

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
    const std::uint32_t* anc;          // dense chains [rows][anc_stride], or null: compact chains
    std::size_t anc_stride, rows, q_heads, kv_heads, window, max_window;
    float scale;
    // compact chains: node n's keys 0..pos are token_node[prompt_off[p] ..], p = node_prompt[n]
    const std::uint32_t* node_prompt;
    const std::uint32_t* prompt_off;   // [prompts + 1]
    const std::uint32_t* token_node;   // [total]
    std::size_t prompts, total;
    int tc_paths;                      // attention_tree_tc ran: path blocks of 32 rows are done
    // with tc_paths: the count and list of the (32-row block, KV head) pairs
    // attention_tree_tc left to attention_tree_block
    const std::uint32_t* tc_rest_count;
    const std::uint32_t* tc_rest;
};

// First key of the ancestor chain of row n at position pos (its keys are
// [0, pos]), or null when the chain is not available: pos outside the dense
// table's stride (or the longest prompt), or a compact witness prompt that
// does not reach depth pos.
__device__ __forceinline__ const std::uint32_t* chain_of(const AttnArgs& a, std::size_t n, std::size_t pos) {
    if (pos >= a.anc_stride) return nullptr;
    if (a.anc) return a.anc + n * a.anc_stride;
    const std::uint32_t p = a.node_prompt[n];
    if (p >= a.prompts) return nullptr;
    const std::uint32_t o0 = a.prompt_off[p], o1 = a.prompt_off[p + 1];
    if (o0 > o1 || o1 > a.total || pos >= o1 - o0) return nullptr;
    return a.token_node + o0;
}

// Division by a row denominator d >= 1 with one reciprocal per row, as in
// softmax.cu (in EXACT_ORDER Markstein's correction gives the correctly
// rounded quotient).
template <bool EXACT>
__device__ __forceinline__ float attn_div(float e, float d, float y) {
    if (!EXACT) return __fmul_rn(e, y);  // tree-order mode: within 1.5 ulp
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
    const std::uint32_t* row_chain = chain_of(a, row, pos);
    if (tid == 0) bad_s = row_chain == nullptr;
    __syncthreads();
    float* out_row = a.out + (row * a.q_heads + kh * kGroup) * HD;
    if (bad_s) {  // no ancestor chain for this position: report, output zeros
        if (tid == 0) flag_check(B2_CHECK_ATTENTION);
        for (int i = tid; i < kGroup * HD; i += kAttnThreads) out_row[i] = 0.0f;
        return;
    }
    const std::size_t begin = pos + 1 > a.window ? pos + 1 - a.window : 0;
    const int W = static_cast<int>(pos - begin + 1);
    const std::uint32_t* anc_row = row_chain + begin;
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
            const float e = exp_mode<EXACT>(__fsub_rn(scores[w * kGroup + g], m), tab);
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
        for (int w = lane; w < W; w += 32) scores[w * kGroup + g] = attn_div<EXACT>(scores[w * kGroup + g], denom, y);
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

// ---- tensor-core attention core (tree-order mode, head_dim 128) -------------
//
// The default (tree-order) mode only has to land within 1e-5 relative OR
// 1e-6 absolute of the reference, so its contractions run on the tcgen05
// tensor cores with FP32-level products: every operand x is split into
// hi = x rounded to TF32 and lo = (x - hi) rounded to TF32, and each product
// is hi.hi + hi.lo + lo.hi -- kind::tf32 MMAs with FP32 accumulators in
// tensor memory (relative error ~2^-22 per product).
//
// tc_split_kv writes the hi / lo planes of K and V once per call. One CTA of
// attention_tree_tc per (block of 32 consecutive trie rows that form a path,
// KV head): M = 32 rows x 4 query heads = 128 rows of the MMA, and the keys
// of every row are a prefix of the deepest row's chain, so each 32-key tile
// of that chain is staged once for all 128 rows.
//   tensor memory  Q hi / lo [128 x 128] (the A operands of the scores), S
//                  [128 x 64]: columns 0-31 Qh.Kh, 32-63 Qh.Kl + Ql.Kh (one
//                  N = 64 MMA per k-step against the stacked [Kh; Kl] tile
//                  costs what an N = 32 one does), P hi / lo [128 x 32] (the
//                  A operand of P V), the tile's P V [128 x 128];
//   shared memory  a ring of 2 key tiles, per 32-dim block the hi then the
//                  lo rows of the 32 keys (K-major, 128-byte swizzle), and a
//                  ring of 2 value tiles hi / lo [32 keys x 128 dims] (the B
//                  operand of P V with N = dims contiguous: MN-major,
//                  128-byte rows with 32-byte swizzle granules);
//   registers      O, 64 floats per softmax thread (its half of a row's 128
//                  dims; 128 registers a thread is the cap for 13 warps, as
//                  the SM's four register-file quarters hold 4, 3, 3 and 3
//                  of them).
// Warp roles: 8-9 stage key tiles, 10-11 value tiles (16-byte cp.async
// copies of the planes into the swizzled layouts); 12 issues the MMAs --
// S(t + 1) as soon as S(t) has been read, P V(t) once P(t) is written; 0-7
// run the softmax, two threads per MMA row m (tensor-memory lane m: row m / 4
// of the block, query head m % 4 of the group), thread half h taking keys
// 16h .. 16h + 15 of each tile and dims 64h .. 64h + 63 of O. The softmax is
// online in base 2: with s2 = s * scale * log2(e) per key, the row's
// running maximum m (the pair exchanges its halves' maxima once per tile)
// and sum l are updated per tile (l = l * 2^(m_old - m) + sum p,
// p = 2^(s2 - m), 0 outside the row's window), and the previous tile's P V
// is folded into O as O = O * 2^(m_old - m) + PV in FP32 round-to-nearest
// (the tensor core's accumulator truncates; chaining every tile there biased
// long windows by ~1e-6), after P(t) is stored and before P V(t) may
// overwrite the P V columns. The epilogue writes O * (1 / l): the softmax of
// the tree-order SIMT kernel, formed in another order. Blocks that are not a
// path (prompt boundaries, shared-prefix branch points) are listed for
// attention_tree_block.
constexpr int kTcRows = 32;  // trie rows per CTA (x 4 heads = M 128)
constexpr int kTcKeys = 32;  // chain keys per tile
constexpr int kTcSoftmaxThreads = 256;  // warps 0-7
constexpr int kTcStageWarps = 2;        // per operand
constexpr int kTcStageThreads = 32 * kTcStageWarps;
constexpr int kTcThreads = kTcSoftmaxThreads + 2 * kTcStageThreads + 32;  // + key, value and MMA warps
constexpr int kTcKStages = 2, kTcVStages = 2;
constexpr std::uint32_t kColQh = 0, kColQl = 128, kColO = 256, kColS = 384, kColPh = 448, kColPl = 480;
constexpr std::uint32_t kTcCols = 512;
constexpr int kTcTileBytes = 16 * 1024;  // one operand plane of a tile: 32 x 128 fp32
constexpr int kTcStageBytes = 2 * kTcTileBytes;  // hi, lo
// rings + 1024-byte alignment (129 KB; one CTA per SM, by its registers, and
// each allocates all 512 tensor-memory columns)
constexpr std::size_t kTcSmem = (kTcKStages + kTcVStages) * kTcStageBytes + 1024;

// Byte offset of dims 4c .. 4c + 3 of key j's hi row in a key stage: per
// 32-dim block (8192 bytes) the 32 hi rows then the 32 lo rows (the lo row
// is 4096 bytes further), K-major rows of 128 bytes in 8-row atoms of 1024
// bytes, 16-byte chunks swizzled by j % 8.
__device__ __forceinline__ int tc_key_offset(int j, int c) { return (c >> 3) * 8192 + tc::sw128_offset(j, c & 7); }
// ... in a value tile: rows of 128 bytes (32 dims) per key, 4-key groups of
// 512 bytes, the four 32-dim blocks 4096 bytes apart, 32-byte granules
// swizzled by j % 4 (the MN-major SWIZZLE_128B_BASE32B layout).
__device__ __forceinline__ int tc_value_offset(int j, int c) {
    return (c >> 3) * 4096 + (j >> 2) * 512 + (j & 3) * 128 + ((((c >> 1) & 3) ^ (j & 3)) << 5) + (c & 1) * 16;
}
// P V's B descriptor at key group ks (8 keys = two 4-key groups): MN-major,
// 32-dim blocks 4096 bytes apart (leading byte offset), 4-key groups 512
// bytes apart (stride byte offset).
__device__ __forceinline__ std::uint64_t tc_value_desc(const void* p) {
    std::uint64_t d = static_cast<std::uint64_t>((smem_addr(p) >> 4) & 0x3FFFu);
    d |= static_cast<std::uint64_t>(4096 >> 4) << 16;
    d |= static_cast<std::uint64_t>(512 >> 4) << 32;
    d |= static_cast<std::uint64_t>(1) << 46;  // descriptor version (sm_100)
    d |= static_cast<std::uint64_t>(1) << 61;  // layout: 128-byte swizzle, 32-byte base
    return d;
}

// Whether rows n0 .. n0 + nr - 1 form a path whose chains are prefixes of the
// last row's chain: consecutive positions, each row found in the last row's
// chain at its own position. Evaluated by one full warp; on success *chain
// and *pos0 describe the block.
__device__ __forceinline__ bool tc_block_is_path(const AttnArgs& a, std::size_t n0, int nr,
                                                 const std::uint32_t** chain, std::size_t* pos0) {
    const unsigned lane = threadIdx.x & 31u;
    const std::size_t n1 = n0 + nr - 1;
    const std::size_t p1 = a.row_pos[n1];
    const std::uint32_t* c = chain_of(a, n1, p1);
    const std::size_t p0 = a.row_pos[n0];
    bool ok = c != nullptr && p1 == p0 + static_cast<std::size_t>(nr - 1);
    if (ok && static_cast<int>(lane) < nr) {
        const std::size_t pi = a.row_pos[n0 + lane];
        ok = pi == p0 + lane && c[pi] == n0 + lane;
    }
    ok = __all_sync(0xffffffffu, ok);
    *chain = c;
    *pos0 = p0;
    return ok;
}

// Waits for a barrier phase; gives up (false) when another warp of the CTA
// has given up, or after kMbarWaitNs, in which case it raises the CTA's flag.
__device__ __forceinline__ bool tc_wait(std::uint64_t* bar, unsigned parity, volatile int* abort) {
    const unsigned long long t0 = global_ns();
    for (unsigned i = 0; i < kMbarMaxPolls; ++i) {
        unsigned done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(done)
            : "r"(smem_addr(bar)), "r"(parity)
            : "memory");
        if (done) return true;
        if ((i & 63u) == 63u) {
            if (*abort) return false;
            if (global_ns() - t0 > kMbarWaitNs) break;
        }
    }
    *abort = 1;
    flag_check(B2_CHECK_WAIT);
    return false;
}

// Barrier 1 over the 128 softmax threads, returning whether any of them
// passed `pred`.
__device__ __forceinline__ bool softmax_group_any(bool pred) {
    unsigned r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, 1, %2, p;\n selp.u32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"(static_cast<unsigned>(pred)), "n"(kTcSoftmaxThreads)
        : "memory");
    return r != 0;
}

// The trie row of key kp of the chain (none past `last`); out-of-range
// entries are reported and replaced by an in-range row.
__device__ __forceinline__ std::uint32_t tc_key_row(const AttnArgs& a, const std::uint32_t* chain, std::size_t kp,
                                                    std::size_t last, std::size_t n0) {
    if (kp > last) return 0xFFFFFFFFu;
    std::uint32_t r = chain[kp];
    if (r >= a.rows) {
        flag_check(B2_CHECK_ATTENTION);
        r = static_cast<std::uint32_t>(n0);
    }
    return r;
}

// x -> (TF32 hi, TF32 lo) of the 3 x TF32 split.
__device__ __forceinline__ void tc_split(float x, float& hi, float& lo) {
    hi = tc::tf32_round(x);
    lo = tc::tf32_round(__fsub_rn(x, hi));
}

// 2^x (ex2.approx: relative error ~2^-22; 2^-inf = 0).
__device__ __forceinline__ float tc_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 16-byte copy global -> shared (L2 only), zero-filled when !valid.
__device__ __forceinline__ void tc_copy16(void* dst, const void* src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
                 "r"(valid ? 16u : 0u)
                 : "memory");
}

// K and V -> hi / lo planes: split[0..3] = K hi, K lo, V hi, V lo, each
// [rows][kv_heads * 128]; zeroes the count of blocks attention_tree_tc leaves.
__global__ void __launch_bounds__(256) tc_split_kv(const float4* k, const float4* v, float4* split,
                                                   std::size_t n4, std::uint32_t* rest_count) {
    pdl_begin();
    if (blockIdx.x == 0 && threadIdx.x == 0) *rest_count = 0;
    for (std::size_t i = blockIdx.x * std::size_t(256) + threadIdx.x; i < n4; i += std::size_t(gridDim.x) * 256) {
        const float4 kx = ld_plain(k + i), vx = ld_plain(v + i);
        float4 h, l;
        tc_split(kx.x, h.x, l.x);
        tc_split(kx.y, h.y, l.y);
        tc_split(kx.z, h.z, l.z);
        tc_split(kx.w, h.w, l.w);
        split[i] = h;
        split[n4 + i] = l;
        tc_split(vx.x, h.x, l.x);
        tc_split(vx.y, h.y, l.y);
        tc_split(vx.z, h.z, l.z);
        tc_split(vx.w, h.w, l.w);
        split[2 * n4 + i] = h;
        split[3 * n4 + i] = l;
    }
}

__global__ void __launch_bounds__(kTcThreads, 1)
attention_tree_tc(AttnArgs a, const float* split, std::uint32_t* rest_count, std::uint32_t* rest) {
    pdl_begin();
    extern __shared__ __align__(16) unsigned char tc_raw[];
    __shared__ std::uint32_t tmem_base;
    __shared__ __align__(8) std::uint64_t kfull[kTcKStages], kempty[kTcKStages], vfull[kTcVStages],
        vempty[kTcVStages], sfull, sempty, qfull, pfull, ofull;
    __shared__ float max_x[2][2][128];  // [tile % 2][half][MMA row]: the halves' tile maxima
    __shared__ float sum_x[2][128];     // [half][MMA row]: the halves' sums
    __shared__ int path_s;
    __shared__ volatile int abort_s;
    __shared__ std::size_t pos0_s;
    __shared__ const std::uint32_t* chain_s;
    // 1024-byte aligned stages (swizzle atoms): keys, then values
    unsigned char* kring = tc_raw + ((1024 - (smem_addr(tc_raw) & 1023u)) & 1023u);
    unsigned char* vring = kring + kTcKStages * kTcStageBytes;

    const unsigned tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const std::size_t kh = blockIdx.x % a.kv_heads;
    const std::size_t n0 = (blockIdx.x / a.kv_heads) * kTcRows;
    const int nr = static_cast<int>(a.rows - n0 < kTcRows ? a.rows - n0 : kTcRows);
    if (warp == 0) {
        const std::uint32_t* c;
        std::size_t p0;
        const bool path = tc_block_is_path(a, n0, nr, &c, &p0);
        if (lane == 0) {
            path_s = path;
            chain_s = c;
            pos0_s = p0;
            abort_s = 0;
            for (int s = 0; s < kTcKStages; ++s) {
                mbar_init(&kfull[s], kTcStageThreads);
                mbar_init(&kempty[s], 1);
            }
            for (int s = 0; s < kTcVStages; ++s) {
                mbar_init(&vfull[s], kTcStageThreads);
                mbar_init(&vempty[s], 1);
            }
            mbar_init(&sfull, 1);
            mbar_init(&sempty, kTcSoftmaxThreads);
            mbar_init(&qfull, kTcSoftmaxThreads);
            mbar_init(&pfull, kTcSoftmaxThreads);
            mbar_init(&ofull, 1);
        }
    }
    __syncthreads();
    if (!path_s) {  // attention_tree_block takes this block
        if (tid == 0) rest[atomicAdd(rest_count, 1u)] = blockIdx.x;
        return;
    }
    if (warp == 0) tc::tmem_alloc(&tmem_base, kTcCols);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const std::uint32_t tmem = tmem_base;
    const std::uint32_t* chain = chain_s;
    const std::size_t pos0 = pos0_s;
    const std::size_t last = pos0 + nr - 1;
    const std::size_t kb0 = pos0 + 1 > a.window ? pos0 + 1 - a.window : 0;
    const int tiles_n = static_cast<int>((last - kb0 + kTcKeys) / kTcKeys);
    const std::size_t kv_row = a.kv_heads * 128;
    constexpr unsigned kSoftmaxWarps = kTcSoftmaxThreads / 32;
    constexpr unsigned kMmaWarp = kSoftmaxWarps + 2 * kTcStageWarps;

    if (warp >= kSoftmaxWarps && warp < kMmaWarp) {
        // ---- staging: warps 8-9 the key tiles into a ring of 2, 10-11 the
        // value tiles into a ring of 2; warp w takes keys 16 (w % 2) .. + 15,
        // lane = 16-byte chunk c of a key's 128 dims. Each lane's copies of a
        // tile arrive on the stage's barrier when they have landed
        // (cp.async.mbarrier.arrive.noinc: one of its 64 arrivals). ----
        const bool keys = warp < kSoftmaxWarps + kTcStageWarps;
        const int j0 = static_cast<int>((warp - kSoftmaxWarps) % kTcStageWarps) * (kTcKeys / kTcStageWarps);
        const int stages = keys ? kTcKStages : kTcVStages;
        unsigned char* ring = keys ? kring : vring;
        std::uint64_t* full = keys ? kfull : vfull;
        std::uint64_t* empty = keys ? kempty : vempty;
        const std::size_t plane = a.rows * kv_row;
        const float* hi_p = split + (keys ? 0 : 2 * plane) + kh * 128 + 4 * lane;
        const float* lo_p = hi_p + plane;
        const int lo_off = keys ? 4096 : kTcTileBytes;  // the lo row of a chunk, from its hi row
        for (int t = 0; t < tiles_n; ++t) {
            const int s = t % stages;
            if (t >= stages && !__all_sync(0xffffffffu, tc_wait(&empty[s], ((t / stages) - 1) & 1, &abort_s)))
                break;
            unsigned char* st = ring + s * kTcStageBytes;
            const std::uint32_t r = tc_key_row(a, chain, kb0 + static_cast<std::size_t>(t) * kTcKeys + lane, last, n0);
#pragma unroll 8
            for (int i = 0; i < kTcKeys / kTcStageWarps; ++i) {
                const int j = j0 + i;
                const std::uint32_t rk = __shfl_sync(0xffffffffu, r, j);
                const bool valid = rk != 0xFFFFFFFFu;
                const std::size_t src = valid ? rk * kv_row : 0;
                const int off = keys ? tc_key_offset(j, static_cast<int>(lane)) : tc_value_offset(j, static_cast<int>(lane));
                tc_copy16(st + off, hi_p + src, valid);
                tc_copy16(st + off + lo_off, lo_p + src, valid);
            }
            asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(&full[s])) : "memory");
        }
        asm volatile("cp.async.wait_all;" ::: "memory");  // none in flight when the CTA ends
    } else if (warp == kMmaWarp) {
        // ---- MMA issue (one thread) ----
        if (lane == 0) {
            // S(t): Qh . [Kh; Kl] (N = 64) into columns 0-63, then Ql . Kh
            // (N = 32) added to columns 32-63
            auto scores = [&](int t) -> bool {
                const int s = t % kTcKStages;
                if (!tc_wait(&kfull[s], (t / kTcKStages) & 1, &abort_s)) return false;
                tc::fence_after_sync();
                const unsigned char* kst = kring + s * kTcStageBytes;
                for (int ks = 0; ks < 16; ++ks)
                    tc::mma_tf32_ts(tmem + kColS, tmem + kColQh + ks * 8,
                                    tc::sw128_desc(kst + (ks >> 2) * 8192 + (ks & 3) * 32), tc::tf32_idesc(128, 64),
                                    ks > 0);
                for (int ks = 0; ks < 16; ++ks)
                    tc::mma_tf32_ts(tmem + kColS + 32, tmem + kColQl + ks * 8,
                                    tc::sw128_desc(kst + (ks >> 2) * 8192 + (ks & 3) * 32), tc::tf32_idesc(128, 32),
                                    true);
                tc::commit(&sfull);
                if (t + kTcKStages < tiles_n) tc::commit(&kempty[s]);
                return true;
            };
            bool ok = tc_wait(&qfull, 0, &abort_s) && scores(0);
            for (int t = 0; t < tiles_n && ok; ++t) {
                // S(t + 1) once every softmax thread has read S(t)
                if (t + 1 < tiles_n && !(tc_wait(&sempty, t & 1, &abort_s) && scores(t + 1))) break;
                // P V(t) = Pl Vh + Ph Vl + Ph Vh (B = V MN-major), once P(t) is in tensor memory
                const int s = t % kTcVStages;
                if (!tc_wait(&pfull, t & 1, &abort_s) || !tc_wait(&vfull[s], (t / kTcVStages) & 1, &abort_s)) break;
                tc::fence_after_sync();
                constexpr std::uint32_t idesc = tc::tf32_idesc(128, 128) | (1u << 16);
                const unsigned char* v_hi = vring + s * kTcStageBytes;
                const unsigned char* vb[3] = {v_hi, v_hi + kTcTileBytes, v_hi};
                const std::uint32_t pa[3] = {kColPl, kColPh, kColPh};
                for (int part = 0; part < 3; ++part)
                    for (int ks = 0; ks < kTcKeys / 8; ++ks)
                        tc::mma_tf32_ts(tmem + kColO, tmem + pa[part] + ks * 8, tc_value_desc(vb[part] + ks * 1024),
                                        idesc, part > 0 || ks > 0);
                tc::commit(&ofull);
                if (t + kTcVStages < tiles_n) tc::commit(&vempty[s]);
            }
        }
        __syncwarp();
    } else {
        // ---- softmax warps: thread (m, h), m = MMA row / tensor-memory lane ----
        const unsigned m = tid & 127u, h = tid >> 7;
        const std::uint32_t lane_base = static_cast<std::uint32_t>((warp & 3u) * 32) << 16;
        const int ri = static_cast<int>(m >> 2), hg = static_cast<int>(m & 3);  // this row and head
        const bool row_ok = ri < nr;
        const std::size_t pos_i = pos0 + ri;
        // Q hi / lo, dims 64h .. 64h + 63, into tensor memory; this half of O = 0
        {
            const float* qr = a.q + ((n0 + (row_ok ? ri : 0)) * a.q_heads + kh * kGroup + hg) * 128 + 64 * h;
            for (int c0 = 0; c0 < 64; c0 += 32) {
                float hi[32], lo[32];
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    const float4 v = row_ok ? ld_plain(reinterpret_cast<const float4*>(qr + c0 + j)) : zero4();
                    tc_split(v.x, hi[j], lo[j]);
                    tc_split(v.y, hi[j + 1], lo[j + 1]);
                    tc_split(v.z, hi[j + 2], lo[j + 2]);
                    tc_split(v.w, hi[j + 3], lo[j + 3]);
                }
                tc::st32(tmem + lane_base + kColQh + 64 * h + c0, hi);
                tc::st32(tmem + lane_base + kColQl + 64 * h + c0, lo);
            }
            tc::st_wait();
            tc::fence_before_sync();
            mbar_arrive(&qfull);
        }
        float oreg[64];  // this half of the row's O: dims 64h .. 64h + 63
#pragma unroll
        for (int c = 0; c < 64; ++c) oreg[c] = 0.0f;
        // folds this half of the P V of the tile issued last into O: O = O * alpha + PV
        auto fold = [&](float alpha) {
#pragma unroll
            for (int c0 = 0; c0 < 64; c0 += 16) {
                float o[16];
                tc::ld16(tmem + lane_base + kColO + 64 * h + c0, o);
#pragma unroll
                for (int j = 0; j < 16; ++j) oreg[c0 + j] = __fmaf_rn(oreg[c0 + j], alpha, o[j]);
            }
        };
        const float scale2 = __fmul_rn(a.scale, 1.4426950408889634f);  // scale * log2(e)
        // keys kb0 + lo_k .. kb0 + hi_k are in this row's window
        const long long lo_k = row_ok ? static_cast<long long>(pos_i + 1 > a.window ? pos_i + 1 - a.window : 0) -
                                            static_cast<long long>(kb0)
                                      : 1;
        const long long hi_k = row_ok ? static_cast<long long>(pos_i - kb0) : 0;
        float mx = -INFINITY, l = 0.0f, alpha_prev = 1.0f;
        bool ok = true;
        for (int t = 0; t < tiles_n; ++t) {
            float p[16], pl[16];
            float mt = -INFINITY;
            if (ok) ok = __all_sync(0xffffffffu, tc_wait(&sfull, t & 1, &abort_s));
            if (ok) {
                tc::fence_after_sync();
                float x[16];
                tc::ld16(tmem + lane_base + kColS + 16 * h, p);        // Qh.Kh
                tc::ld16(tmem + lane_base + kColS + 32 + 16 * h, x);   // Qh.Kl + Ql.Kh
                tc::fence_before_sync();
                mbar_arrive(&sempty);  // S(t + 1) may be computed into these columns
                // this row's window within the tile: keys jlo .. jhi of it
                const long long t0 = static_cast<long long>(t) * kTcKeys + 16 * h;
                const int jlo = static_cast<int>(lo_k - t0 < 0 ? 0 : (lo_k - t0 > 16 ? 16 : lo_k - t0));
                const int jhi = static_cast<int>(hi_k - t0 > 15 ? 15 : (hi_k - t0 < -1 ? -1 : hi_k - t0));
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    p[j] = (j >= jlo && j <= jhi) ? __fmul_rn(__fadd_rn(p[j], x[j]), scale2) : -INFINITY;
                    mt = fmaxf(mt, p[j]);
                }
                max_x[t & 1][h][m] = mt;
            }
            // the pair's maxima meet here; also the group-wide decision to stop
            if (softmax_group_any(!ok)) {
                ok = false;
                break;
            }
            mt = fmaxf(mt, max_x[t & 1][h ^ 1u][m]);
            const float mn = fmaxf(mx, mt);
            const float mref = mn == -INFINITY ? 0.0f : mn;
            const float alpha = tc_exp2(__fsub_rn(mx, mref));  // 0 while mx is -inf, 1 while it holds
            float l0 = 0.0f, l1 = 0.0f;
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
                const float p0 = tc_exp2(__fsub_rn(p[j], mref));
                const float p1 = tc_exp2(__fsub_rn(p[j + 1], mref));
                l0 = __fadd_rn(l0, p0);
                l1 = __fadd_rn(l1, p1);
                tc_split(p0, p[j], pl[j]);
                tc_split(p1, p[j + 1], pl[j + 1]);
            }
            l = __fmaf_rn(l, alpha, __fadd_rn(l0, l1));
            mx = mn;
            if (t > 0) {  // P V(t - 1) done: P's columns are free, and it can be folded
                ok = __all_sync(0xffffffffu, tc_wait(&ofull, (t - 1) & 1, &abort_s));
                if (ok) tc::fence_after_sync();
            }
            if (ok) {
                tc::st16(tmem + lane_base + kColPh + 16 * h, p);
                tc::st16(tmem + lane_base + kColPl + 16 * h, pl);
                if (t > 0) fold(alpha_prev);  // (P V's columns are read before pfull lets P V(t) overwrite them)
                tc::st_wait();
            }
            alpha_prev = alpha;
            tc::fence_before_sync();
            mbar_arrive(&pfull);  // also: this thread's reads of the P V columns are done
        }
        if (ok) {
            ok = __all_sync(0xffffffffu, tc_wait(&ofull, (tiles_n - 1) & 1, &abort_s));
            if (ok) {
                tc::fence_after_sync();
                fold(alpha_prev);
            }
        }
        // ---- epilogue: out = O / l, l the sum of the halves' sums ----
        sum_x[h][m] = l;
        if (!softmax_group_any(!ok) && row_ok) {
            const float inv = __fdiv_rn(1.0f, __fadd_rn(sum_x[0][m], sum_x[1][m]));
            float4* orow =
                reinterpret_cast<float4*>(a.out + ((n0 + ri) * a.q_heads + kh * kGroup + hg) * 128 + 64 * h);
#pragma unroll
            for (int c = 0; c < 16; ++c)
                st_plain(orow + c, make_float4(__fmul_rn(oreg[4 * c], inv), __fmul_rn(oreg[4 * c + 1], inv),
                                               __fmul_rn(oreg[4 * c + 2], inv), __fmul_rn(oreg[4 * c + 3], inv)));
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_free(tmem, kTcCols);
}

// ---- query-blocked kernel (head_dim 128) --------------------------------------
//
// The rows of a trie path -- node n + 1 the child of node n, as prefix-trie
// numbering makes every run of new nodes along one prompt -- have nested
// ancestor chains: the chain of the deepest row holds every other row's
// keys. attention_tree_block gives one CTA a block of kBlkRows such rows and
// one KV head, stages each K and V tile of that chain once for all of them
// (cp.async into two alternating buffers, so no registers wait on the
// copies and two CTAs fit an SM at a 1024-key window), and keeps each lane's
// query slices in registers, so every value read from shared memory feeds 8
// (QK) or 16 (PV) fused multiply-adds. The arithmetic
// per (row, head) is the reference's, in its order: four accumulators over
// d mod 4 (chain j sums q[d] k[d] for d = j, j + 4, ... in ascending d, one
// lane per chain), combined ((a0 + a1) + (a2 + a3)) by shuffles, times the
// scale; the softmax over the row's own window; the output a fused
// multiply-add chain over the window in ascending key order.
// Blocks that are not a path (prompt starts, bad positions, or an ancestor
// table whose rows disagree) fall back to one row at a time in the same code.
constexpr int kBlkRows = 4;                    // query rows per CTA
constexpr int kBlkThreads = 256;
constexpr int kBlkKeys = 32;                   // chain keys per staged tile (two tiles in flight)
constexpr int kCombos = kBlkRows * kGroup;     // (row, head) pairs: 16
constexpr int kJStride = 36;                   // floats between the 4 d-mod-4 slices of a staged key
constexpr int kKeyPitch = 4 * kJStride;        // floats per staged key (also holds a value row)
constexpr int kTileFloats = kBlkKeys * kKeyPitch;

// Shared layout (floats): scores [wcap][16] | chain [wcap] (u32) | 2 tiles [32][144].
// At a 1024-key window that is 107 KB and two CTAs share an SM.
inline std::size_t block_smem_bytes(std::size_t wcap) {
    return (wcap * kCombos + wcap + 2 * static_cast<std::size_t>(kTileFloats)) * 4;
}


template <bool EXACT>
struct BlockAttention {
    const AttnArgs& a;
    float* scores;
    std::uint32_t* chain;
    float* tile;
    const double* tab;
    float* red;  // [8 warps][16 combos] reduction scratch
    std::size_t kh;
    unsigned tid, lane, warp;

    // Issues the copies of the 32 chain rows of tile t into buffer t & 1:
    // keys transposed to [key][j][i] (d = 4i + j), one 4-byte copy per
    // element; values as [key][d], one 16-byte copy per 4 elements. Rows past
    // wg are skipped. For the keys, 8 threads share a key row: thread x
    // copies d = x, x + 8, ..., so a warp's copy covers four whole 32-byte
    // sectors, each thread looks up its chain entry once, and its elements
    // all fall in one d-mod-4 slice (j = x mod 4), two positions apart.
    __device__ __forceinline__ void issue_keys(int t, int wg) const {
        static_assert(kBlkKeys * 8 == kBlkThreads, "8 threads per staged key row");
        const int ks = static_cast<int>(tid >> 3), x = static_cast<int>(tid & 7);
        const int w = t * kBlkKeys + ks;
        if (w < wg) {
            const float* src = a.k + static_cast<std::size_t>(chain[w]) * (a.kv_heads * 128) + kh * 128 + x;
            float* dst = tile + (t & 1) * kTileFloats + ks * kKeyPitch + (x & 3) * kJStride + (x >> 2);
#pragma unroll
            for (int u = 0; u < 16; ++u) cp_async4(dst + 2 * u, src + 8 * u);
        }
        cp_async_commit();
    }
    __device__ __forceinline__ void issue_values(int t, int wg) const {
        const std::size_t row = a.kv_heads * 128;
        float* buf = tile + (t & 1) * kTileFloats;
#pragma unroll
        for (int u = 0; u < kBlkKeys * 32 / kBlkThreads; ++u) {
            const int i = static_cast<int>(tid) + u * kBlkThreads, ks = i >> 5, c = i & 31;
            const int w = t * kBlkKeys + ks;
            if (w < wg)
                cp_async16(buf + ks * kKeyPitch + 4 * c, a.v + static_cast<std::size_t>(chain[w]) * row + kh * 128 + 4 * c);
        }
        cp_async_commit();
    }
    // Tile t has landed for every thread (the next one may still be in flight).
    __device__ __forceinline__ void tile_ready(int t, int tiles) const {
        if (t + 1 < tiles) cp_async_wait<1>();
        else cp_async_wait<0>();
        __syncthreads();
    }

    // Rows first .. first + g - 1 (a path, g <= kBlkRows). With `verify`,
    // returns false (computing nothing) when some row's ancestors in its
    // window differ from the deepest row's.
    __device__ bool run(std::size_t first, int g, bool verify) const {
        const std::size_t last = first + g - 1;
        const std::size_t p0 = a.row_pos[first], P = a.row_pos[last];
        const std::size_t begin = p0 + 1 > a.window ? p0 + 1 - a.window : 0;
        const int wg = static_cast<int>(P - begin + 1);
        const std::uint32_t* anc_last = chain_of(a, last, P) + begin;  // checked by the caller
        for (int i = tid; i < wg; i += kBlkThreads) {
            std::uint32_t c = anc_last[i];
            if (c >= a.rows) {
                flag_check(B2_CHECK_ATTENTION);
                c = static_cast<std::uint32_t>(last);
            }
            chain[i] = c;
        }
        __syncthreads();  // chain complete (fetch reads other threads' entries)
        if (verify && g > 1 && a.anc) {  // compact chains of one prompt agree by construction
            int differs = 0;
            for (int r = 0; r + 1 < g; ++r) {
                const std::size_t pr = p0 + r;
                const std::size_t br = pr + 1 > a.window ? pr + 1 - a.window : 0;
                const std::uint32_t* own = a.anc + (first + r) * a.anc_stride;
                for (std::size_t k = br + tid; k <= pr; k += kBlkThreads)
                    differs |= own[k] != anc_last[k - begin];
            }
            if (__syncthreads_or(differs)) return false;
        }

        // ---- scores[w][r * 4 + h] ----
        const unsigned j = lane & 3, cp = lane >> 2;        // chain j; combos 2cp, 2cp + 1
        const int rq = static_cast<int>(cp >> 1), hq = static_cast<int>(cp & 1) * 2;
        float qa[32], qb[32];
        {
            const std::size_t qrow = first + (rq < g ? rq : g - 1);
            const float* q0 = a.q + (qrow * a.q_heads + kh * kGroup + hq) * 128 + j;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                qa[i] = __ldg(q0 + 4 * i);
                qb[i] = __ldg(q0 + 128 + 4 * i);
            }
        }
        const int tiles = (wg + kBlkKeys - 1) / kBlkKeys;
        issue_keys(0, wg);
        for (int t = 0; t < tiles; ++t) {
            if (t + 1 < tiles) issue_keys(t + 1, wg);  // into the other buffer, read two iterations ago
            tile_ready(t, tiles);
            const float* buf = tile + (t & 1) * kTileFloats;
#pragma unroll 1
            for (int m = 0; m < kBlkKeys / 16; ++m) {
                const int ka = static_cast<int>(warp) + 16 * m, kb = ka + 8;  // this warp's two keys
                const int wa = t * kBlkKeys + ka;
                if (wa >= wg) break;
                const float4* xa = reinterpret_cast<const float4*>(buf + ka * kKeyPitch + j * kJStride);
                const float4* xb = reinterpret_cast<const float4*>(buf + kb * kKeyPitch + j * kJStride);
                float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;   // (a, combo 0), (a, 1), (b, 0), (b, 1)
#pragma unroll
                for (int t4 = 0; t4 < 8; ++t4) {
                    const float4 x = xa[t4], y = xb[t4];
                    s0 = __fmaf_rn(qa[4 * t4], x.x, s0); s0 = __fmaf_rn(qa[4 * t4 + 1], x.y, s0);
                    s0 = __fmaf_rn(qa[4 * t4 + 2], x.z, s0); s0 = __fmaf_rn(qa[4 * t4 + 3], x.w, s0);
                    s1 = __fmaf_rn(qb[4 * t4], x.x, s1); s1 = __fmaf_rn(qb[4 * t4 + 1], x.y, s1);
                    s1 = __fmaf_rn(qb[4 * t4 + 2], x.z, s1); s1 = __fmaf_rn(qb[4 * t4 + 3], x.w, s1);
                    s2 = __fmaf_rn(qa[4 * t4], y.x, s2); s2 = __fmaf_rn(qa[4 * t4 + 1], y.y, s2);
                    s2 = __fmaf_rn(qa[4 * t4 + 2], y.z, s2); s2 = __fmaf_rn(qa[4 * t4 + 3], y.w, s2);
                    s3 = __fmaf_rn(qb[4 * t4], y.x, s3); s3 = __fmaf_rn(qb[4 * t4 + 1], y.y, s3);
                    s3 = __fmaf_rn(qb[4 * t4 + 2], y.z, s3); s3 = __fmaf_rn(qb[4 * t4 + 3], y.w, s3);
                }
                // ((a0 + a1) + (a2 + a3)) across the four chain lanes
                s0 = __fadd_rn(s0, __shfl_xor_sync(0xffffffffu, s0, 1));
                s1 = __fadd_rn(s1, __shfl_xor_sync(0xffffffffu, s1, 1));
                s2 = __fadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, 1));
                s3 = __fadd_rn(s3, __shfl_xor_sync(0xffffffffu, s3, 1));
                s0 = __fadd_rn(s0, __shfl_xor_sync(0xffffffffu, s0, 2));
                s1 = __fadd_rn(s1, __shfl_xor_sync(0xffffffffu, s1, 2));
                s2 = __fadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, 2));
                s3 = __fadd_rn(s3, __shfl_xor_sync(0xffffffffu, s3, 2));
                if (j == 0) {
                    float* sa = scores + static_cast<std::size_t>(wa) * kCombos + 2 * cp;
                    sa[0] = __fmul_rn(s0, a.scale);
                    sa[1] = __fmul_rn(s1, a.scale);
                    if (wa + 8 < wg) {
                        sa[8 * kCombos] = __fmul_rn(s2, a.scale);
                        sa[8 * kCombos + 1] = __fmul_rn(s3, a.scale);
                    }
                }
            }
            __syncthreads();  // buffer t & 1 is refilled by the next iteration's issue
        }

        // ---- softmax of every (row, head) over the row's window: warp `warp`
        // takes keys [wg * warp / 8, wg * (warp + 1) / 8), lane (combo c,
        // parity) every other key of them, so each access is two whole
        // 64-byte score rows (no bank conflicts) ----
        {
            const int c = static_cast<int>(lane & 15), par = static_cast<int>(lane >> 4), rc = c >> 2;
            int lo = 1, hi = 0;  // empty for rows past the group
            if (rc < g) {
                const std::size_t pr = p0 + rc;
                lo = static_cast<int>((pr + 1 > a.window ? pr + 1 - a.window : 0) - begin);
                hi = static_cast<int>(pr - begin);
            }
            const int wb = max(wg * static_cast<int>(warp) / 8, lo);
            const int we = min(wg * (static_cast<int>(warp) + 1) / 8 - 1, hi);
            float m = -3.402823466e+38F;
            for (int w = wb + par; w <= we; w += 2) m = fmaxf(m, scores[w * kCombos + c]);
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 16));
            if (lane < 16) red[warp * 16 + c] = m;
            __syncthreads();
            m = red[c];
#pragma unroll
            for (int k = 1; k < 8; ++k) m = fmaxf(m, red[k * 16 + c]);
            __syncthreads();  // red is reused
            float part = 0.0f;
            for (int w = wb + par; w <= we; w += 2) {
                const float e = exp_mode<EXACT>(__fsub_rn(scores[w * kCombos + c], m), tab);
                scores[w * kCombos + c] = e;
                part = __fadd_rn(part, e);
            }
            float d;
            if (EXACT) {  // serial ascending sums, one lane per (row, head)
                __syncthreads();
                if (warp == 0 && lane < 16) {
                    float acc = 0.0f;
#pragma unroll 8
                    for (int w = lo; w <= hi; ++w) acc = __fadd_rn(acc, scores[w * kCombos + c]);
                    red[c] = acc;
                }
                __syncthreads();
                d = red[c];
            } else {
                part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, 16));
                if (lane < 16) red[warp * 16 + c] = part;
                __syncthreads();
                d = red[c];
#pragma unroll
                for (int k = 1; k < 8; ++k) d = __fadd_rn(d, red[k * 16 + c]);
            }
            const float y = __frcp_rn(d);
            for (int w = wb + par; w <= we; w += 2)
                scores[w * kCombos + c] = attn_div<EXACT>(scores[w * kCombos + c], d, y);
        }

        // ---- out[r][h][d] = sum_w p[w][r * 4 + h] v[w][d], ascending w ----
        // Threads 0..127: rows ra = 2 * (tid / 64) and ra + 1, dimensions
        // 2 * (tid % 64) and + 1, all four heads: 16 chains per thread, each
        // value pair read once for both rows, run as 8 packed pairs (heads
        // 2j and 2j + 1 in the two lanes of one fma.rn.f32x2, each lane its
        // own chain). The deeper row's window is the shallower one's shifted
        // by at most one key at each end, so each tile splits into
        // (shallower only) (both) (deeper only) key runs.
        const bool pv = tid < 128;
        const int ra = 2 * static_cast<int>(tid >> 6), dp = static_cast<int>(tid & 63);
        constexpr int kNone = 1 << 30;
        int loa = kNone, hia = -1, lob = kNone, hib = -1;
        if (pv && ra < g) {
            const std::size_t pr = p0 + ra;
            loa = static_cast<int>((pr + 1 > a.window ? pr + 1 - a.window : 0) - begin);
            hia = static_cast<int>(pr - begin);
        }
        if (pv && ra + 1 < g) {
            const std::size_t pr = p0 + ra + 1;
            lob = static_cast<int>((pr + 1 > a.window ? pr + 1 - a.window : 0) - begin);
            hib = static_cast<int>(pr - begin);
        }
        unsigned long long acc[2][2][2];  // [row][head pair][d]: heads (2j, 2j + 1)
#pragma unroll
        for (int i = 0; i < 8; ++i) (&acc[0][0][0])[i] = 0ull;
        issue_values(0, wg);  // the key buffers were released by the last QK barrier
        for (int t = 0; t < tiles; ++t) {
            if (t + 1 < tiles) issue_values(t + 1, wg);
            tile_ready(t, tiles);  // (the first also orders the softmax before PV)
            const float* buf = tile + (t & 1) * kTileFloats + 2 * dp;
            if (hia >= 0) {
                const int tb = t * kBlkKeys;
                const int w0a = max(loa - tb, 0), w1a = min(hia - tb, kBlkKeys - 1);
                const int w0b = lob == kNone ? kNone : max(lob - tb, 0), w1b = min(hib - tb, kBlkKeys - 1);
                const float* prow = scores + static_cast<std::size_t>(tb) * kCombos + 4 * ra;
                // one key for row r: p = (heads 0,1 | heads 2,3), v = (d0, d1)
                auto step = [&](int r, const ulonglong2 p, const unsigned long long vx, const unsigned long long vy) {
                    acc[r][0][0] = f2_fma(p.x, vx, acc[r][0][0]);
                    acc[r][0][1] = f2_fma(p.x, vy, acc[r][0][1]);
                    acc[r][1][0] = f2_fma(p.y, vx, acc[r][1][0]);
                    acc[r][1][1] = f2_fma(p.y, vy, acc[r][1][1]);
                };
                const int e1 = min(w1a, w0b - 1);
                for (int w = w0a; w <= e1; ++w) {  // shallower row only
                    const ulonglong2 pa = *reinterpret_cast<const ulonglong2*>(prow + w * kCombos);
                    const float2 vv = *reinterpret_cast<const float2*>(buf + w * kKeyPitch);
                    step(0, pa, f2_pack(vv.x, vv.x), f2_pack(vv.y, vv.y));
                }
                const int e2 = min(w1a, w1b);
#pragma unroll 8
                for (int w = max(w0a, w0b); w <= e2; ++w) {  // both rows
                    const ulonglong2 pa = *reinterpret_cast<const ulonglong2*>(prow + w * kCombos);
                    const ulonglong2 pb = *reinterpret_cast<const ulonglong2*>(prow + w * kCombos + 4);
                    const float2 vv = *reinterpret_cast<const float2*>(buf + w * kKeyPitch);
                    const unsigned long long vx = f2_pack(vv.x, vv.x), vy = f2_pack(vv.y, vv.y);
                    step(0, pa, vx, vy);
                    step(1, pb, vx, vy);
                }
                for (int w = max(w1a + 1, w0b); w <= w1b; ++w) {  // deeper row only
                    const ulonglong2 pb = *reinterpret_cast<const ulonglong2*>(prow + w * kCombos + 4);
                    const float2 vv = *reinterpret_cast<const float2*>(buf + w * kKeyPitch);
                    step(1, pb, f2_pack(vv.x, vv.x), f2_pack(vv.y, vv.y));
                }
            }
            __syncthreads();  // buffer t & 1 is refilled next
        }
#pragma unroll
        for (int rr = 0; rr < 2; ++rr)
            if (pv && ra + rr < g) {
                float* o = a.out + ((first + ra + rr) * a.q_heads + kh * kGroup) * 128 + 2 * dp;
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const float2 d0 = f2_unpack(acc[rr][j][0]), d1 = f2_unpack(acc[rr][j][1]);  // (head 2j, 2j + 1)
                    *reinterpret_cast<float2*>(o + (2 * j) * 128) = make_float2(d0.x, d1.x);
                    *reinterpret_cast<float2*>(o + (2 * j + 1) * 128) = make_float2(d0.y, d1.y);
                }
            }
        __syncthreads();  // scores / chain / tile are reused by the next group
        return true;
    }
};

template <bool EXACT>
__global__ void __launch_bounds__(kBlkThreads, 2)
attention_tree_block(AttnArgs a, std::size_t wcap) {
    pdl_begin();
    extern __shared__ __align__(16) float smem[];
    __shared__ double tab[64];
    __shared__ int seg_s[kBlkRows + 1], bad_s[kBlkRows], nseg_s;
    __shared__ float red_s[(kBlkThreads / 32) * kCombos];
    load_exp2_table(tab);
    // Alone, CTA i takes the kBlkRows rows of block i / kv_heads and KV head
    // i % kv_heads. After attention_tree_tc (tc_paths), the CTAs stride over
    // the blocks of kBlkRows rows inside the (32-row block, KV head) pairs it
    // left, listed in tc_rest.
    constexpr std::size_t kSub = kTcRows / kBlkRows;
    const std::size_t units = (!EXACT && a.tc_paths) ? std::size_t(*a.tc_rest_count) * kSub : gridDim.x;
    const std::size_t stride = (!EXACT && a.tc_paths) ? gridDim.x : units;
    for (std::size_t u = blockIdx.x; u < units; u += stride) {
        std::size_t kh, n0;
        if (!EXACT && a.tc_paths) {
            const std::uint32_t e = a.tc_rest[u / kSub];
            kh = e % a.kv_heads;
            n0 = (e / a.kv_heads) * kTcRows + (u % kSub) * kBlkRows;
            if (n0 >= a.rows) continue;
        } else {
            kh = blockIdx.x % a.kv_heads;
            n0 = (blockIdx.x / a.kv_heads) * kBlkRows;
        }
        const int nrows = static_cast<int>(a.rows - n0 < kBlkRows ? a.rows - n0 : kBlkRows);
        if (threadIdx.x == 0) {
            // segments: maximal runs in which row n is the child of row n - 1
            int nseg = 0;
            seg_s[0] = 0;
            std::size_t prev = 0;
            for (int r = 0; r < nrows; ++r) {
                const std::size_t n = n0 + r, pos = a.row_pos[n];
                bad_s[r] = chain_of(a, n, pos) == nullptr;
                if (r > 0) {
                    // dense: the parent entry of row n is n - 1; compact: the same
                    // witness prompt one position further
                    const bool link = !bad_s[r] && !bad_s[r - 1] && pos == prev + 1 &&
                                      (a.anc ? a.anc[n * a.anc_stride + pos - 1] == n - 1
                                             : a.node_prompt[n] == a.node_prompt[n - 1]);
                    if (!link) seg_s[++nseg] = r;
                }
                prev = pos;
            }
            seg_s[++nseg] = nrows;
            nseg_s = nseg;
        }
        __syncthreads();
        BlockAttention<EXACT> b{a, smem, reinterpret_cast<std::uint32_t*>(smem + wcap * kCombos),
                                smem + wcap * kCombos + wcap, tab, red_s, kh,
                                threadIdx.x, threadIdx.x & 31u, threadIdx.x >> 5};
        for (int sgi = 0; sgi < nseg_s; ++sgi) {
            const int r0 = seg_s[sgi], r1 = seg_s[sgi + 1];
            if (r1 - r0 == 1 && bad_s[r0]) {  // position outside the ancestor table: report, output zeros
                if (threadIdx.x == 0) flag_check(B2_CHECK_ATTENTION);
                float* o = a.out + ((n0 + r0) * a.q_heads + kh * kGroup) * 128;
                for (int i = threadIdx.x; i < kGroup * 128; i += kBlkThreads) o[i] = 0.0f;
                continue;
            }
            if (!b.run(n0 + r0, r1 - r0, true))
                for (int r = r0; r < r1; ++r) b.run(n0 + r, 1, false);
        }
        __syncthreads();  // the shared state is rewritten by the next block
    }
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

namespace b2 {
namespace {

// Shared by both entry points once the chain source is set in `a`.
int attention_launch(AttnArgs& a, std::size_t head_dim, std::uint32_t flags, b2_stream_t stream) {
    const std::size_t rows = a.rows, kv_heads = a.kv_heads, q_heads = a.q_heads, window = a.window;
    const std::size_t anc_stride = a.anc_stride;
    const float *q = a.q, *k = a.k, *v = a.v;
    float* out = a.out;
    if (kv_heads == 0 || q_heads != kGroup * kv_heads)
        return invalid("attention_tree_gpu expects GQA-4");
    if (head_dim != 128 && head_dim != 64)
        return set_error(B2_ERR_UNSUPPORTED, "b2_attention_tree: head_dim must be 64 or 128");
    if (window == 0 || anc_stride == 0) return invalid("b2_attention_tree: window / anc_stride is 0");
    if (rows * kv_heads > 0x7FFFFFFFu) return invalid("b2_attention_tree: too many rows");
    if (!aligned16(k) || !aligned16(v)) return invalid("b2_attention_tree: k / v not 16-byte aligned");
    a.max_window = window < anc_stride ? window : anc_stride;
    a.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    const bool exact = (flags & B2_FLAG_EXACT_ORDER) != 0;
    cudaStream_t s = as_stream(stream);
    const std::size_t wcap = (a.max_window + kBlkRows - 1 + 3) & ~std::size_t(3);
    if (head_dim == 128 && block_smem_bytes(wcap) <= 200 * 1024 && aligned16(q) && aligned16(out) &&
        (rows + kBlkRows - 1) / kBlkRows * kv_heads <= 0x7FFFFFFFu) {
        const std::size_t smem = block_smem_bytes(wcap);
        auto kernel = exact ? attention_tree_block<true> : attention_tree_block<false>;
        if (allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem) != cudaSuccess)
            return launch_result("b2_attention_tree: shared memory attribute");
        // tree order: the path blocks on the tensor cores first, from the hi /
        // lo planes of K and V in stream-ordered scratch (then the count and
        // list of the blocks left over); the block kernel below then strides
        // over the rows of the blocks left over
        void* scratch = nullptr;
        const std::size_t n4 = rows * kv_heads * 32;  // float4s per plane
        const std::size_t tc_blocks = (rows + kTcRows - 1) / kTcRows * kv_heads;
        const std::size_t scratch_bytes = 4 * n4 * sizeof(float4) + (1 + tc_blocks) * sizeof(std::uint32_t);
        unsigned grid = static_cast<unsigned>((rows + kBlkRows - 1) / kBlkRows * kv_heads);
        if (!exact && tc_blocks <= 0x7FFFFFFFu) {
            if (scratch_alloc(&scratch, scratch_bytes, s) != cudaSuccess) {
                cudaGetLastError();  // no scratch: every block on the block kernel
                scratch = nullptr;
            }
        }
        if (scratch) {
            if (allow_dynamic_smem(reinterpret_cast<const void*>(attention_tree_tc), kTcSmem) != cudaSuccess) {
                cudaFreeAsync(scratch, s);
                return launch_result("b2_attention_tree: shared memory attribute");
            }
            float4* split = static_cast<float4*>(scratch);
            std::uint32_t* rest_count = reinterpret_cast<std::uint32_t*>(split + 4 * n4);
            std::uint32_t* rest = rest_count + 1;
            const std::size_t want = (n4 + 255) / 256;
            launch_pdl(tc_split_kv, static_cast<unsigned>(want < 148 * 8 ? want : 148 * 8), 256, 0, s,
                       reinterpret_cast<const float4*>(k), reinterpret_cast<const float4*>(v), split, n4, rest_count);
            launch_pdl(attention_tree_tc, static_cast<unsigned>(tc_blocks), kTcThreads, kTcSmem, s, a,
                       static_cast<const float*>(scratch), rest_count, rest);
            a.tc_paths = 1;
            a.tc_rest_count = rest_count;
            a.tc_rest = rest;
            const std::size_t wave = static_cast<std::size_t>(sm_count()) *
                                     static_cast<std::size_t>(resident_ctas(reinterpret_cast<const void*>(kernel),
                                                                            kBlkThreads, smem));
            grid = static_cast<unsigned>(wave < grid ? wave : grid);
        }
        launch_pdl(kernel, grid, kBlkThreads, smem, s, a, wcap);
        if (scratch) cudaFreeAsync(scratch, s);
        return launch_result("b2_attention_tree");
    }
    int rc;
    if (head_dim == 128) rc = exact ? launch_attention<128, true>(a, s) : launch_attention<128, false>(a, s);
    else rc = exact ? launch_attention<64, true>(a, s) : launch_attention<64, false>(a, s);
    if (rc) return rc;
    return launch_result("b2_attention_tree");
}

}  // namespace
}  // namespace b2

extern "C" int b2_attention_tree(const float* q, const float* k, const float* v, float* out,
                                 const uint32_t* row_pos, const uint32_t* anc, size_t anc_stride, size_t rows,
                                 size_t q_heads, size_t kv_heads, size_t head_dim, size_t window, uint32_t flags,
                                 b2_stream_t stream) {
    using namespace b2;
    if (rows == 0) return B2_OK;
    if (!q || !k || !v || !out || !row_pos || !anc) return invalid("b2_attention_tree: null pointer");
    AttnArgs a{};
    a.q = q; a.k = k; a.v = v; a.out = out; a.row_pos = row_pos; a.anc = anc; a.anc_stride = anc_stride;
    a.rows = rows; a.q_heads = q_heads; a.kv_heads = kv_heads; a.window = window;
    return attention_launch(a, head_dim, flags, stream);
}

extern "C" int b2_attention_tree_compact(const float* q, const float* k, const float* v, float* out,
                                         const uint32_t* row_pos, const uint32_t* node_prompt,
                                         const uint32_t* prompt_offsets, size_t prompts, const uint32_t* token_node,
                                         size_t total_tokens, size_t max_len, size_t rows, size_t q_heads,
                                         size_t kv_heads, size_t head_dim, size_t window, uint32_t flags,
                                         b2_stream_t stream) {
    using namespace b2;
    if (rows == 0) return B2_OK;
    if (!q || !k || !v || !out || !row_pos || !node_prompt || !prompt_offsets || !token_node)
        return invalid("b2_attention_tree_compact: null pointer");
    if (prompts == 0 || total_tokens == 0) return invalid("b2_attention_tree_compact: empty batch");
    AttnArgs a{};
    a.q = q; a.k = k; a.v = v; a.out = out; a.row_pos = row_pos; a.anc = nullptr; a.anc_stride = max_len;
    a.rows = rows; a.q_heads = q_heads; a.kv_heads = kv_heads; a.window = window;
    a.node_prompt = node_prompt; a.prompt_off = prompt_offsets; a.token_node = token_node;
    a.prompts = prompts; a.total = total_tokens;
    return attention_launch(a, head_dim, flags, stream);
}
