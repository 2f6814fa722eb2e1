// Drop-in implementation of the reference's non-GEMM tensor_ops GPU ops
// (ezzy0654/aps2026 include/tensor.h:63-161) over the aps2026_b200 C ABI.
//
// A maintainer adds this file to the reference build, links
// libaps2026_b200.so, and deletes the functions defined here from
// src/tensor.cu (add_inplace_gpu, silu_mul_gpu, layer_norm_gpu,
// add_layer_norm_gpu, apply_rope_gpu, apply_rope_tree_gpu, attention_gpu,
// attention_tree_gpu, both gather_rows_gpu overloads). src/layer.cu,
// src/model.cu and src/main.cpp
// compile unchanged: same signatures, same Tensor handling (inputs through
// cuda_data(), outputs through cuda_data_write(), the legacy default
// stream), and the same exception types with the reference's messages
// (std::invalid_argument on a shape mismatch, std::runtime_error on a CUDA
// failure). The routing and un-permute inside moe_forward_grouped_gpu are
// replaced in place (see the b2 calls its body makes in the integration
// notes), because that function also launches the reference's GEMMs.
//
// Reductions keep the reference's serial order (B2_FLAG_EXACT_ORDER) so the
// drop-in reproduces the reference's outputs bit for bit, which its
// end-to-end validation against answers.bin relies on (routing downstream of
// a LayerNorm flips on a last-ulp change).
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "aps2026_b200.h"
#include "config.h"
#include "tensor.h"

namespace tensor_ops {
namespace {

constexpr std::uint32_t kFlags = B2_FLAG_EXACT_ORDER;

void check(int rc, const char* what) {
    if (rc == B2_OK) return;
    const std::string msg = std::string(what) + ": " + b2_last_error();
    if (rc == B2_ERR_INVALID_ARGUMENT || rc == B2_ERR_UNSUPPORTED) throw std::invalid_argument(msg);
    throw std::runtime_error(msg);
}

void cuda_check(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// Device RoPE table, built on the host by b2_rope_table and cached like the
// reference's rope_table() static (src/tensor.cu:2695-2737).
struct RopeTable {
    float* cosine = nullptr;
    float* sine = nullptr;
    std::size_t max_seq = 0, half = 0;
    float theta = 0.0f;
};

RopeTable& rope_table(std::size_t max_seq, std::size_t head_dim, float theta) {
    static RopeTable t;
    const std::size_t half = head_dim / 2;
    if (t.cosine && t.max_seq >= max_seq && t.half == half && t.theta == theta) return t;
    if (t.cosine) cudaFree(t.cosine);
    if (t.sine) cudaFree(t.sine);
    t = RopeTable{};
    std::vector<float> c(max_seq * half), s(max_seq * half);
    check(b2_rope_table(max_seq, head_dim, theta, c.data(), s.data()), "rope table");
    cuda_check(cudaMalloc(&t.cosine, c.size() * sizeof(float)), "cudaMalloc rope cosine");
    cuda_check(cudaMalloc(&t.sine, s.size() * sizeof(float)), "cudaMalloc rope sine");
    cuda_check(cudaMemcpy(t.cosine, c.data(), c.size() * sizeof(float), cudaMemcpyHostToDevice),
               "copy rope cosine");
    cuda_check(cudaMemcpy(t.sine, s.data(), s.size() * sizeof(float), cudaMemcpyHostToDevice), "copy rope sine");
    t.max_seq = max_seq;
    t.half = half;
    t.theta = theta;
    return t;
}

// Per-segment positions of a packed batch, cached per seq_lens like the
// reference's packed_meta() (src/tensor.cu:2662-2693).
const std::uint32_t* packed_positions(const std::vector<std::size_t>& lens, std::size_t* rows,
                                      std::size_t* max_seq) {
    static std::vector<std::size_t> key;
    static std::uint32_t* pos = nullptr;
    static std::size_t n = 0, longest = 0;
    if (pos && key == lens) {
        *rows = n;
        *max_seq = longest;
        return pos;
    }
    std::vector<std::uint32_t> host;
    longest = 0;
    for (std::size_t len : lens) {
        for (std::size_t p = 0; p < len; ++p) host.push_back(static_cast<std::uint32_t>(p));
        if (len > longest) longest = len;
    }
    if (pos) cudaFree(pos);
    pos = nullptr;
    n = host.size();
    if (n) {
        cuda_check(cudaMalloc(&pos, n * sizeof(std::uint32_t)), "cudaMalloc packed positions");
        cuda_check(cudaMemcpy(pos, host.data(), n * sizeof(std::uint32_t), cudaMemcpyHostToDevice),
                   "copy packed positions");
    }
    key = lens;
    *rows = n;
    *max_seq = longest;
    return pos;
}

// The packed-segment layout of attention_gpu in the compact chain form of
// b2_attention_tree_compact: segment b's rows offsets[b] .. offsets[b + 1]
// are their own chain, so row r's keys are rows offsets[seg[r]] .. + pos
// (token_node = identity). Cached per seq_lens like packed_positions.
struct SegmentChains {
    std::uint32_t* seg = nullptr;       // [rows] segment of each row
    std::uint32_t* offsets = nullptr;   // [segments + 1]
    std::uint32_t* identity = nullptr;  // [rows]
};

const SegmentChains& segment_chains(const std::vector<std::size_t>& lens) {
    static std::vector<std::size_t> key;
    static SegmentChains c;
    if (c.seg && key == lens) return c;
    for (std::uint32_t* p : {c.seg, c.offsets, c.identity})
        if (p) cudaFree(p);
    c = SegmentChains{};
    std::vector<std::uint32_t> seg, offsets{0}, identity;
    for (std::size_t b = 0; b < lens.size(); ++b) {
        for (std::size_t p = 0; p < lens[b]; ++p) {
            seg.push_back(static_cast<std::uint32_t>(b));
            identity.push_back(static_cast<std::uint32_t>(identity.size()));
        }
        offsets.push_back(static_cast<std::uint32_t>(identity.size()));
    }
    auto upload = [](const std::vector<std::uint32_t>& h, std::uint32_t** d, const char* what) {
        if (h.empty()) return;
        cuda_check(cudaMalloc(d, h.size() * sizeof(std::uint32_t)), what);
        cuda_check(cudaMemcpy(*d, h.data(), h.size() * sizeof(std::uint32_t), cudaMemcpyHostToDevice), what);
    };
    upload(seg, &c.seg, "segment chains: rows");
    upload(offsets, &c.offsets, "segment chains: offsets");
    upload(identity, &c.identity, "segment chains: identity");
    key = lens;
    return c;
}

// Staging for the std::vector gather overload (the reference's
// device_rows(), src/tensor.cu:2739-2753).
const std::uint32_t* device_rows(const std::vector<std::size_t>& rows) {
    static std::uint32_t* ptr = nullptr;
    static std::size_t capacity = 0;
    if (capacity < rows.size()) {
        if (ptr) cudaFree(ptr);
        cuda_check(cudaMalloc(&ptr, rows.size() * sizeof(std::uint32_t)), "cudaMalloc row indices");
        capacity = rows.size();
    }
    std::vector<std::uint32_t> compact(rows.begin(), rows.end());
    cuda_check(cudaMemcpy(ptr, compact.data(), compact.size() * sizeof(std::uint32_t), cudaMemcpyHostToDevice),
               "copy row indices");
    return ptr;
}

}  // namespace

void add_inplace_gpu(Tensor& a, const Tensor& b) {
    if (a.size() != b.size()) throw std::invalid_argument("add shape");
    a.cuda_data();
    check(b2_add(a.cuda_data_write(), b.cuda_data(), a.size(), nullptr), "k_add launch");
}

void silu_mul_gpu(const Tensor& gate, const Tensor& up, Tensor& out) {
    if (gate.size() != up.size() || out.size() != gate.size()) throw std::invalid_argument("silu_mul shape");
    const std::size_t n = gate.size();
    check(b2_silu_mul(gate.cuda_data(), n, up.cuda_data(), n, out.cuda_data_write(), n, 1, n, nullptr),
          "k_silu_mul launch");
}

void layer_norm_gpu(const Tensor& x, const Tensor& weight, const Tensor& bias, float eps, Tensor& y) {
    const std::size_t h = x.size(x.ndim() - 1);
    const std::size_t rows = x.size() / h;
    if (weight.size() != h || bias.size() != h || y.size() != x.size())
        throw std::invalid_argument("layer norm shape");
    check(b2_layer_norm(x.cuda_data(), weight.cuda_data(), bias.cuda_data(), y.cuda_data_write(), rows, h, eps,
                        kFlags, nullptr),
          "k_layer_norm launch");
}

void add_layer_norm_gpu(Tensor& x, const Tensor& residual, const Tensor& weight, const Tensor& bias, float eps,
                        Tensor& y) {
    const std::size_t h = x.size(x.ndim() - 1);
    const std::size_t rows = x.size() / h;
    if (residual.size() != x.size() || weight.size() != h || bias.size() != h || y.size() != x.size())
        throw std::invalid_argument("add layer norm shape");
    x.cuda_data();
    check(b2_add_layer_norm(x.cuda_data_write(), residual.cuda_data(), weight.cuda_data(), bias.cuda_data(),
                            y.cuda_data_write(), rows, h, eps, kFlags, nullptr),
          "k_add_layer_norm launch");
}

void apply_rope_gpu(Tensor& q, Tensor& k, const std::vector<std::size_t>& seq_lens, std::size_t q_heads,
                    std::size_t kv_heads, std::size_t head_dim, float theta) {
    std::size_t rows = 0, max_seq = 0;
    const std::uint32_t* pos = packed_positions(seq_lens, &rows, &max_seq);
    RopeTable& t = rope_table(max_seq, head_dim, theta);
    q.cuda_data();
    k.cuda_data();
    check(b2_rope(q.cuda_data_write(), k.cuda_data_write(), pos, rows, q_heads, kv_heads, head_dim, t.cosine,
                  t.sine, t.max_seq, nullptr),
          "k_rope launch");
}

void apply_rope_tree_gpu(Tensor& q, Tensor& k, const std::uint32_t* row_pos, std::size_t rows,
                         std::size_t max_seq, std::size_t q_heads, std::size_t kv_heads, std::size_t head_dim,
                         float theta) {
    RopeTable& t = rope_table(max_seq, head_dim, theta);
    q.cuda_data();
    k.cuda_data();
    check(b2_rope(q.cuda_data_write(), k.cuda_data_write(), row_pos, rows, q_heads, kv_heads, head_dim, t.cosine,
                  t.sine, t.max_seq, nullptr),
          "k_rope(tree) launch");
}

// GQA-4 (the model's layout) runs the prefix-tree kernel over segment chains,
// whose arithmetic is k_attention_grouped_gqa4's; other head groupings
// (the reference's k_attention) are not implemented here.
void attention_gpu(const Tensor& q, const Tensor& k, const Tensor& v, Tensor& out,
                   const std::vector<std::size_t>& seq_lens, std::size_t q_heads, std::size_t kv_heads,
                   std::size_t head_dim) {
    if (q_heads != 4 * kv_heads)
        throw std::invalid_argument("attention_gpu: only GQA-4 is implemented by the B200 library");
    std::size_t rows = 0, max_seq = 0;
    const std::uint32_t* pos = packed_positions(seq_lens, &rows, &max_seq);
    if (rows == 0) return;
    const SegmentChains& c = segment_chains(seq_lens);
    check(b2_attention_tree_compact(q.cuda_data(), k.cuda_data(), v.cuda_data(), out.cuda_data_write(), pos, c.seg,
                                    c.offsets, seq_lens.size(), c.identity, rows, max_seq, rows, q_heads, kv_heads,
                                    head_dim, apss26::SLIDING_WINDOW, kFlags, nullptr),
          "k_attention_grouped_gqa4 launch");
}

void attention_tree_gpu(const Tensor& q, const Tensor& k, const Tensor& v, Tensor& out,
                        const std::uint32_t* row_pos, const std::uint32_t* anc, std::size_t anc_stride,
                        std::size_t rows, std::size_t max_seq, std::size_t q_heads, std::size_t kv_heads,
                        std::size_t head_dim) {
    (void)max_seq;  // positions are bounded by anc_stride
    check(b2_attention_tree(q.cuda_data(), k.cuda_data(), v.cuda_data(), out.cuda_data_write(), row_pos, anc,
                            anc_stride, rows, q_heads, kv_heads, head_dim, apss26::SLIDING_WINDOW, kFlags, nullptr),
          "k_attention_tree_gqa4 launch");
}

void gather_rows_gpu(const Tensor& x, const std::vector<std::size_t>& rows, Tensor& out) {
    const std::size_t h = x.size(x.ndim() - 1);
    check(b2_gather_rows(x.cuda_data(), x.size() / h, h, device_rows(rows), rows.size(), out.cuda_data_write(),
                         nullptr),
          "k_gather_rows launch");
}

void gather_rows_gpu(const Tensor& x, const RowIndexBuffer& rows, Tensor& out) {
    if (rows.empty()) return;
    const std::size_t h = x.size(x.ndim() - 1);
    check(b2_gather_rows(x.cuda_data(), x.size() / h, h, rows.data(), rows.size(), out.cuda_data_write(), nullptr),
          "k_gather_rows(dev) launch");
}

}  // namespace tensor_ops
