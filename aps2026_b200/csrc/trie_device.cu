// Prefix-trie dedup of a packed prompt batch ON THE DEVICE.
//
// Reference: the host walk of PhiTinyMoEModel::generate (src/model.cu:64-117),
// which visits prompts in order and creates a node whenever (parent, token)
// has no child yet, numbering nodes in creation order. The same numbering
// follows from longest common prefixes, without a walk:
//   L(b)   = max over earlier prompts b' < b of LCP(b', b)   (0 for b = 0)
//   b*(b)  = the first earlier prompt reaching that maximum
// Position d of prompt b is a NEW node iff d >= L(b) (no earlier prompt shares
// its prefix 0..d), numbered base(b) + d - L(b), base = exclusive scan of
// len(b) - L(b) over prompts. For d < L(b) the prefix 0..d is b*'s, so the
// node is b*'s node at depth d -- new in b* or found by following b* again
// (b* < b, so the chain ends).
//
// Three launches: trie_lcp (one CTA per prompt, a warp per earlier prompt,
// 32 positions per ballot, so unrelated prompts cost one step), trie_scan
// (one CTA), trie_nodes (one thread per token). Work: O(batch^2) LCP steps
// plus O(total tokens) -- the host walk's hash lookups are gone. The witness
// array node_prompt gives each node a prompt that contains it, so its
// ancestor chain is token_node[offsets[p] .. offsets[p] + depth]: the compact
// form of the [nodes, max_len] ancestor table.
#include "common.cuh"

namespace b2 {
namespace {

constexpr int kLcpThreads = 256;
constexpr int kScanThreads = 1024;
constexpr unsigned kNoPrompt = 0xFFFFFFFFu;

struct TrieArgs {
    const std::int32_t* ids;
    const std::uint32_t* offsets;  // [batch + 1]
    std::size_t batch, total, vocab, max_len;
    std::uint32_t* token_node;
    std::uint32_t* node_token;
    std::uint32_t* node_depth;
    std::uint32_t* node_prompt;  // may be null
    std::uint32_t* node_count;   // device scalar
    std::uint32_t* lcp;          // workspace [batch]: L(b)
    std::uint32_t* from;         // workspace [batch]: b*(b)
    std::uint32_t* base;         // workspace [batch]: first new node of b
};

// Tokens of prompt b; 0 (and a reported check) when the offsets are not a
// non-decreasing split of [0, total), so no read leaves the id array.
__device__ __forceinline__ std::uint32_t prompt_len(const TrieArgs& a, std::size_t b) {
    const std::uint32_t o0 = a.offsets[b], o1 = a.offsets[b + 1];
    if (o0 > o1 || o1 > a.total) return 0;
    return o1 - o0;
}

__global__ void __launch_bounds__(kLcpThreads)
trie_lcp(TrieArgs a) {
    pdl_begin();
    constexpr int WARPS = kLcpThreads / 32;
    __shared__ unsigned best_s[WARPS], from_s[WARPS];
    const std::size_t b = blockIdx.x;
    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const std::uint32_t ob = a.offsets[b], len_b = prompt_len(a, b);
    if (threadIdx.x == 0 && (len_b == 0 || len_b > a.max_len)) flag_check(B2_CHECK_TRIE);
    unsigned best = 0, best_from = kNoPrompt;
    for (std::size_t p = warp; p < b; p += WARPS) {
        const std::uint32_t op = a.offsets[p], len_p = prompt_len(a, p);
        const std::uint32_t n = len_p < len_b ? len_p : len_b;
        unsigned l = n;
        for (std::uint32_t s = 0; s < n; s += 32) {
            const std::uint32_t j = s + lane;
            const unsigned stop = __ballot_sync(0xffffffffu, !(j < n && a.ids[op + j] == a.ids[ob + j]));
            if (stop) {
                const unsigned at = s + __ffs(stop) - 1;
                l = at < n ? at : n;
                break;
            }
        }
        if (l > best) {  // p ascending within the warp: the first maximum is kept
            best = l;
            best_from = static_cast<unsigned>(p);
        }
    }
    if (lane == 0) {
        best_s[warp] = best;
        from_s[warp] = best_from;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned l = 0, f = kNoPrompt;
        for (int w = 0; w < WARPS; ++w)  // ties: the smallest prompt index
            if (best_s[w] > l || (best_s[w] == l && l > 0 && from_s[w] < f)) {
                l = best_s[w];
                f = from_s[w];
            }
        a.lcp[b] = l;
        a.from[b] = f;
    }
}

// base(b) = sum over b' < b of len(b') - L(b'); node_count = the total.
__global__ void __launch_bounds__(kScanThreads)
trie_scan(TrieArgs a) {
    pdl_begin();
    constexpr int WARPS = kScanThreads / 32;
    __shared__ unsigned warp_tot[WARPS];
    __shared__ unsigned carry_s;
    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) carry_s = 0;
    __syncthreads();
    for (std::size_t c0 = 0; c0 < a.batch; c0 += kScanThreads) {
        const std::size_t b = c0 + threadIdx.x;
        const unsigned v = b < a.batch ? prompt_len(a, b) - a.lcp[b] : 0;
        unsigned incl = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned n = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= static_cast<unsigned>(o)) incl += n;
        }
        if (lane == 31) warp_tot[warp] = incl;
        __syncthreads();
        if (warp == 0) {
            unsigned t = warp_tot[lane], ti = t;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned n = __shfl_up_sync(0xffffffffu, ti, o);
                if (lane >= static_cast<unsigned>(o)) ti += n;
            }
            warp_tot[lane] = ti - t;  // exclusive over warps
        }
        __syncthreads();
        const unsigned carry = carry_s;
        if (b < a.batch) a.base[b] = carry + warp_tot[warp] + incl - v;
        __syncthreads();
        if (threadIdx.x == kScanThreads - 1) carry_s = carry + warp_tot[warp] + incl;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        *a.node_count = carry_s;
        if (a.offsets[0] != 0 || a.offsets[a.batch] != a.total) flag_check(B2_CHECK_TRIE);
    }
}

__global__ void __launch_bounds__(256)
trie_nodes(TrieArgs a) {
    pdl_begin();
    for (std::size_t t = static_cast<std::size_t>(blockIdx.x) * 256 + threadIdx.x; t < a.total;
         t += static_cast<std::size_t>(gridDim.x) * 256) {
        // prompt of token t: the last b with offsets[b] <= t
        std::size_t lo = 0, hi = a.batch;  // offsets[lo] <= t < offsets[hi]
        while (hi - lo > 1) {
            const std::size_t mid = (lo + hi) / 2;
            if (a.offsets[mid] <= t) lo = mid;
            else hi = mid;
        }
        const std::int32_t token = a.ids[t];
        if (token < 0 || static_cast<std::size_t>(token) >= a.vocab) flag_check(B2_CHECK_TRIE);
        const std::uint32_t d = static_cast<std::uint32_t>(t - a.offsets[lo]);
        std::size_t b = lo;
        // follow b* while the prefix 0..d is an earlier prompt's (at most batch steps)
        for (std::size_t hop = 0; d < a.lcp[b] && hop < a.batch; ++hop) b = a.from[b];
        const std::uint32_t node = a.base[b] + d - a.lcp[b];
        if (node >= a.total) {  // only from offsets that do not split [0, total)
            flag_check(B2_CHECK_TRIE);
            continue;
        }
        a.token_node[t] = node;
        if (b == lo) {  // created by this token
            a.node_token[node] = static_cast<std::uint32_t>(token);
            a.node_depth[node] = d;
            if (a.node_prompt) a.node_prompt[node] = static_cast<std::uint32_t>(lo);
        }
    }
}

}  // namespace
}  // namespace b2

B2_DEFINE_CHECK_TAKER(trie)

extern "C" {

int b2_prefix_trie_device_workspace_size(size_t batch, size_t* bytes) {
    if (!bytes) return b2::invalid("b2_prefix_trie_device_workspace_size: null bytes");
    *bytes = 3 * batch * sizeof(uint32_t);
    return B2_OK;
}

int b2_prefix_trie_device(const int32_t* ids, const uint32_t* offsets, size_t batch, size_t total, size_t vocab,
                          size_t max_len, uint32_t* token_node, uint32_t* node_token, uint32_t* node_depth,
                          uint32_t* node_prompt, uint32_t* node_count, void* workspace, size_t workspace_bytes,
                          b2_stream_t stream) {
    using namespace b2;
    if (batch == 0) return invalid("generate received an empty input batch");
    if (!offsets || !token_node || !node_token || !node_depth || !node_count || !workspace || (total && !ids))
        return invalid("b2_prefix_trie_device: null pointer");
    if (batch > 0x7FFFFFFFu || total >= 0xFFFFFFFFu) return invalid("b2_prefix_trie_device: batch or total too large");
    size_t need = 0;
    b2_prefix_trie_device_workspace_size(batch, &need);
    if (workspace_bytes < need) return invalid("b2_prefix_trie_device: workspace too small");
    if (reinterpret_cast<std::uintptr_t>(workspace) & 3u) return invalid("b2_prefix_trie_device: misaligned workspace");
    TrieArgs a{ids, offsets, batch, total, vocab, max_len, token_node, node_token, node_depth, node_prompt, node_count,
               nullptr, nullptr, nullptr};
    a.lcp = static_cast<uint32_t*>(workspace);
    a.from = a.lcp + batch;
    a.base = a.from + batch;
    cudaStream_t s = as_stream(stream);
    launch_pdl(trie_lcp, static_cast<unsigned>(batch), kLcpThreads, 0, s, a);
    launch_pdl(trie_scan, 1, kScanThreads, 0, s, a);
    if (total) {
        const unsigned grid = wave_grid(reinterpret_cast<const void*>(trie_nodes), 256, 0, (total + 255) / 256);
        launch_pdl(trie_nodes, grid, 256, 0, s, a);
    }
    return launch_result("b2_prefix_trie_device");
}

}  // extern "C"
