// Prefix-trie dedup of a packed prefill batch (host side).
//
// Reference: PhiTinyMoEModel::generate (src/model.cu:64-117) walks the
// prompts in order with a std::unordered_map keyed by (parent + 1) << 32 |
// token and numbers nodes in order of creation; per node it records the
// token, the depth (= RoPE position) and the ancestor chain root -> node.
//
// Same walk and the same numbering here, with an open-addressing table sized
// once for the whole batch (power of two, linear probing) instead of a
// node-allocating map, and the ancestor table filled only when the caller
// asks for it (only the attention core reads it; at 64 x 2048 tokens it is
// 1 GB).
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/aps2026_b200.h"

namespace b2 {
int set_error(int code, const std::string& message);
}

namespace {

struct ChildTable {
    std::vector<std::uint64_t> keys;
    std::vector<std::uint32_t> vals;
    std::uint64_t mask = 0;

    explicit ChildTable(std::size_t entries) {
        std::size_t cap = 16;
        while (cap < entries * 2) cap <<= 1;
        keys.assign(cap, ~std::uint64_t{0});
        vals.resize(cap);
        mask = cap - 1;
    }

    static std::uint64_t mix(std::uint64_t k) {
        k ^= k >> 33;
        k *= 0xff51afd7ed558ccdULL;
        k ^= k >> 33;
        k *= 0xc4ceb9fe1a85ec53ULL;
        k ^= k >> 33;
        return k;
    }

    // Returns the slot of `key`; *found tells whether it was present.
    std::size_t find(std::uint64_t key, bool* found) const {
        std::size_t i = mix(key) & mask;
        while (true) {
            if (keys[i] == key) { *found = true; return i; }
            if (keys[i] == ~std::uint64_t{0}) { *found = false; return i; }
            i = (i + 1) & mask;
        }
    }
};

}  // namespace

extern "C" int b2_prefix_trie_build(const int32_t* ids, const uint32_t* seq_lens, size_t batch,
                                    size_t vocab, size_t max_len, uint32_t* token_node,
                                    uint32_t* node_token, uint32_t* node_depth,
                                    uint32_t* node_anc, size_t anc_stride, size_t* nodes_out) {
    if (batch == 0) return b2::set_error(B2_ERR_INVALID_ARGUMENT, "generate received an empty input batch");
    if (!ids || !seq_lens || !token_node || !node_token || !node_depth || !nodes_out)
        return b2::set_error(B2_ERR_INVALID_ARGUMENT, "b2_prefix_trie_build: null pointer");
    std::size_t total = 0, longest = 0;
    for (std::size_t b = 0; b < batch; ++b) {
        if (seq_lens[b] == 0) return b2::set_error(B2_ERR_INVALID_ARGUMENT, "empty input");
        if (seq_lens[b] > max_len) return b2::set_error(B2_ERR_INVALID_ARGUMENT, "sequence is too long");
        total += seq_lens[b];
        if (seq_lens[b] > longest) longest = seq_lens[b];
    }
    if (total >= 0xFFFFFFFFu) return b2::set_error(B2_ERR_INVALID_ARGUMENT, "b2_prefix_trie_build: too many tokens");
    if (node_anc && anc_stride < longest)
        return b2::set_error(B2_ERR_INVALID_ARGUMENT, "b2_prefix_trie_build: anc_stride < longest prompt");

    ChildTable table(total);
    std::vector<std::uint32_t> chain(longest);
    std::size_t row = 0;
    std::uint32_t nodes = 0;
    for (std::size_t b = 0; b < batch; ++b) {
        std::uint32_t parent = 0xFFFFFFFFu;  // virtual root
        for (std::size_t si = 0; si < seq_lens[b]; ++si, ++row) {
            const int32_t token = ids[row];
            if (token < 0 || static_cast<std::size_t>(token) >= vocab)
                return b2::set_error(B2_ERR_INVALID_ARGUMENT, "token out of vocabulary");
            const std::uint64_t key = (static_cast<std::uint64_t>(parent + 1u) << 32) |
                                      static_cast<std::uint32_t>(token);
            bool found = false;
            const std::size_t slot = table.find(key, &found);
            std::uint32_t node;
            if (found) {
                node = table.vals[slot];
            } else {
                node = nodes++;
                table.keys[slot] = key;
                table.vals[slot] = node;
                node_token[node] = static_cast<std::uint32_t>(token);
                node_depth[node] = static_cast<std::uint32_t>(si);
                if (node_anc) {
                    std::uint32_t* a = node_anc + static_cast<std::size_t>(node) * anc_stride;
                    chain[si] = node;
                    std::memcpy(a, chain.data(), (si + 1) * sizeof(std::uint32_t));
                    std::memset(a + si + 1, 0, (anc_stride - si - 1) * sizeof(std::uint32_t));
                }
            }
            chain[si] = node;
            token_node[row] = node;
            parent = node;
        }
    }
    *nodes_out = nodes;
    return B2_OK;
}
