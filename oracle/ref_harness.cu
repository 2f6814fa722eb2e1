// TEST INFRASTRUCTURE ONLY -- builds the reference itself as a checker.
//
// This translation unit compiles ezzy0654/aps2026's own src/tensor.cu from
// where it lies (oracle/Makefile passes its directory with -I; no reference
// source is copied into this repository) and exposes, through extern "C":
//   - ref_k_*   : launchers of the reference's non-GEMM CUDA kernels
//                 (anonymous namespace inside tensor_ops, reachable because
//                 they are in this same translation unit), with the launch
//                 shapes of the reference wrappers (src/tensor.cu:3236-3438,
//                 :2804-2821, :2922-2926);
//   - ref_cpu_* : the reference's host ops (tensor_ops::layer_norm,
//                 apply_rope, silu, mul, add_inplace; src/tensor.cu:302-367)
//                 through its own Tensor class on host memory.
// Output goes to oracle/_ref/libref.so. Tests use it to pin the CPU oracle
// and the product kernels to the reference on identical inputs; the product
// never loads it.

#include "tensor.cu"

#include <chrono>
#include <cstdint>
#include <vector>

namespace {
cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }
int launch_status() { return static_cast<int>(cudaGetLastError()); }
unsigned blocks_for(std::size_t n) { return static_cast<unsigned>((n + 255) / 256); }

Tensor host_tensor(const float* src, std::vector<std::size_t> shape) {
    Tensor t(std::move(shape));
    float* d = t.data();
    std::copy(src, src + t.size(), d);
    return t;
}
// The reference's host ops write outputs through operator[] from inside
// OpenMP loops, and operator[] lazily allocates host storage on first touch
// (Tensor::ensure_host, src/tensor.cu:88-90): on a fresh output tensor the
// threads would race on that allocation. Touch data() once first.
Tensor host_output(std::vector<std::size_t> shape) {
    Tensor t(std::move(shape));
    (void)t.data();
    return t;
}
void copy_out(const Tensor& t, float* dst) {
    const float* s = t.data();
    std::copy(s, s + t.size(), dst);
}

// Times `op` alone (not the copies into and out of the reference Tensors);
// stores seconds into *seconds when it is not null.
template <typename F>
void timed(double* seconds, F&& op) {
    const auto t0 = std::chrono::steady_clock::now();
    op();
    const auto t1 = std::chrono::steady_clock::now();
    if (seconds) *seconds = std::chrono::duration<double>(t1 - t0).count();
}
}  // namespace

extern "C" {

// ---- GPU kernels of the reference (device pointers) -----------------------

int ref_k_gather_rows(const float* x, const std::uint32_t* rows, float* out,
                      std::size_t count, std::size_t h, void* stream) {
    tensor_ops::k_gather_rows<<<blocks_for(count * h), 256, 0, as_stream(stream)>>>(
        x, rows, out, count, h);
    return launch_status();
}

int ref_k_layer_norm(const float* x, const float* w, const float* b, float* y,
                     std::size_t rows, std::size_t h, float eps, void* stream) {
    tensor_ops::k_layer_norm<<<static_cast<unsigned>(rows), 256, h * sizeof(float),
                               as_stream(stream)>>>(x, w, b, y, h, eps);
    return launch_status();
}

int ref_k_add_layer_norm(float* x, const float* r, const float* w,
                         const float* b, float* y, std::size_t rows,
                         std::size_t h, float eps, void* stream) {
    tensor_ops::k_add_layer_norm<<<static_cast<unsigned>(rows), 256, h * sizeof(float),
                                   as_stream(stream)>>>(x, r, w, b, y, h, eps);
    return launch_status();
}

// Two launches, Q then K, as apply_rope_tree_gpu does (src/tensor.cu:3352-3357).
int ref_k_rope(float* q, float* k, const std::uint32_t* row_pos,
               const float* cosine, const float* sine, std::size_t rows,
               std::size_t q_heads, std::size_t kv_heads, std::size_t head_dim,
               void* stream) {
    const std::size_t half = head_dim / 2;
    tensor_ops::k_rope<<<blocks_for(rows * q_heads * half), 256, 0, as_stream(stream)>>>(
        q, row_pos, cosine, sine, rows, q_heads, head_dim);
    tensor_ops::k_rope<<<blocks_for(rows * kv_heads * half), 256, 0, as_stream(stream)>>>(
        k, row_pos, cosine, sine, rows, kv_heads, head_dim);
    return launch_status();
}

// The routing sequence of moe_forward_grouped_gpu (src/tensor.cu:2804-2821)
// with caller buffers. Queue lengths follow moe_scratch (:1244-1247).
int ref_k_moe_route(const float* router, std::size_t rows, std::uint8_t* routes,
                    std::uint32_t* counts, std::uint32_t* offsets,
                    std::uint32_t* assignment_rows,
                    std::uint32_t* route_positions, std::uint32_t* we64,
                    std::uint32_t* ws64, std::uint32_t* we128,
                    std::uint32_t* ws128, void* stream) {
    cudaStream_t s = as_stream(stream);
    const std::size_t max_work = (2 * rows + tensor_ops::BIG_BM - 1) / tensor_ops::BIG_BM + apss26::NUM_EXPERTS;
    const std::size_t max_tall = (2 * rows + tensor_ops::T8_BM - 1) / tensor_ops::T8_BM + apss26::NUM_EXPERTS;
    cudaMemsetAsync(we64, 0xff, max_work * sizeof(std::uint32_t), s);
    cudaMemsetAsync(we128, 0xff, max_tall * sizeof(std::uint32_t), s);
    cudaMemsetAsync(counts, 0, apss26::NUM_EXPERTS * sizeof(std::uint32_t), s);
    tensor_ops::k_moe_top2<<<blocks_for(rows), 256, 0, s>>>(router, routes, counts, rows);
    tensor_ops::k_moe_offsets_work<<<1, 32, 0, s>>>(counts, offsets, we64, ws64, we128, ws128);
    tensor_ops::k_moe_fill_stable<<<apss26::NUM_EXPERTS, 256, 0, s>>>(
        routes, offsets, assignment_rows, route_positions, rows);
    return launch_status();
}

int ref_k_silu_mul(const float* gate, const float* up, float* out,
                   std::size_t n, void* stream) {
    tensor_ops::k_silu_mul<<<blocks_for(n), 256, 0, as_stream(stream)>>>(gate, up, out, n);
    return launch_status();
}

int ref_k_moe_combine(const float* expert_out, const std::uint8_t* routes,
                      const std::uint32_t* route_positions, float* out,
                      std::size_t rows, std::size_t h, void* stream) {
    tensor_ops::k_moe_combine<<<blocks_for(rows * h), 256, 0, as_stream(stream)>>>(
        expert_out, routes, route_positions, out, rows, h);
    return launch_status();
}

// k_moe_gather_compact with the launch of moe_forward_grouped_gpu
// (src/tensor.cu:1420-1428, :2828-2833): compact[i,:] = x[assignment_rows[i],:].
int ref_k_moe_gather_compact(const float* x, const std::uint32_t* assignment_rows, float* out,
                             std::size_t assignments, std::size_t h, void* stream) {
    tensor_ops::k_moe_gather_compact<<<blocks_for(assignments * h), 256, 0, as_stream(stream)>>>(
        x, assignment_rows, out, assignments, h);
    return launch_status();
}

int ref_k_add(float* a, const float* b, std::size_t n, void* stream) {
    tensor_ops::k_add<<<blocks_for(n), 256, 0, as_stream(stream)>>>(a, b, n);
    return launch_status();
}

// k_attention_tree_gqa4 with the launch of attention_tree_gpu
// (src/tensor.cu:3361-3377). Its shared-memory need grows with max_seq, so
// the harness raises the kernel's dynamic shared-memory limit when needed.
int ref_k_attention_tree(const float* q, const float* k, const float* v,
                         float* out, const std::uint32_t* row_pos,
                         const std::uint32_t* anc, std::size_t anc_stride,
                         std::size_t rows, std::size_t max_seq,
                         std::size_t q_heads, std::size_t kv_heads,
                         std::size_t head_dim, void* stream) {
    const std::size_t shared =
        (4 * max_seq + 4 * head_dim + tensor_ops::ATTN_KEY_TILE * (head_dim + 1) + max_seq) *
        sizeof(float);
    if (shared > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(
            tensor_ops::k_attention_tree_gqa4,
            cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(shared));
        if (e != cudaSuccess) return static_cast<int>(e);
    }
    tensor_ops::k_attention_tree_gqa4<<<static_cast<unsigned>(rows * kv_heads), 128, shared,
                                        as_stream(stream)>>>(
        q, k, v, out, row_pos, anc, anc_stride, rows, q_heads, kv_heads, head_dim, max_seq);
    return launch_status();
}

// k_attention_grouped_gqa4 with the launch of attention_gpu
// (src/tensor.cu:3316-3330): seg_offset[r] is the first row of row r's
// segment, seg_pos[r] its position in it.
int ref_k_attention_grouped(const float* q, const float* k, const float* v, float* out,
                            const std::uint32_t* seg_offset, const std::uint32_t* seg_pos, std::size_t rows,
                            std::size_t max_seq, std::size_t q_heads, std::size_t kv_heads, std::size_t head_dim,
                            void* stream) {
    const std::size_t shared =
        (4 * max_seq + 4 * head_dim + tensor_ops::ATTN_KEY_TILE * (head_dim + 1)) * sizeof(float);
    if (shared > 48 * 1024) {
        const cudaError_t e = cudaFuncSetAttribute(
            tensor_ops::k_attention_grouped_gqa4,
            cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(shared));
        if (e != cudaSuccess) return static_cast<int>(e);
    }
    tensor_ops::k_attention_grouped_gqa4<<<static_cast<unsigned>(rows * kv_heads), 128, shared,
                                           as_stream(stream)>>>(
        q, k, v, out, seg_offset, seg_pos, rows, q_heads, kv_heads, head_dim, max_seq);
    return launch_status();
}

int ref_sliding_window(void) { return static_cast<int>(apss26::SLIDING_WINDOW); }

// ---- host ops of the reference (host pointers) -----------------------------
// Each takes an optional `seconds` out-parameter: the time of the reference
// op itself, without the copies through its Tensor class.

int ref_cpu_layer_norm(const float* x, const float* w, const float* b, float* y,
                       std::size_t rows, std::size_t h, float eps, double* seconds) {
    Tensor tx = host_tensor(x, {rows, h}), tw = host_tensor(w, {h}),
           tb = host_tensor(b, {h}), ty = host_output({rows, h});
    timed(seconds, [&] { tensor_ops::layer_norm(tx, tw, tb, eps, ty); });
    copy_out(ty, y);
    return 0;
}

// apply_rope over packed segments (src/tensor.cu:343-367); q/k in place.
int ref_cpu_apply_rope(float* q, float* k, const std::size_t* seq_lens,
                       std::size_t segments, std::size_t q_heads,
                       std::size_t kv_heads, std::size_t head_dim, float theta,
                       double* seconds) {
    std::vector<std::size_t> lens(seq_lens, seq_lens + segments);
    std::size_t rows = 0;
    for (std::size_t l : lens) rows += l;
    Tensor tq = host_tensor(q, {rows, q_heads * head_dim});
    Tensor tk = host_tensor(k, {rows, kv_heads * head_dim});
    timed(seconds, [&] { tensor_ops::apply_rope(tq, tk, lens, q_heads, kv_heads, head_dim, theta); });
    copy_out(tq, q);
    copy_out(tk, k);
    return 0;
}

// silu then mul, as PhiMLP::forward does on the CPU (src/layer.cu:60-61).
int ref_cpu_silu_mul(const float* gate, const float* up, float* out, std::size_t n,
                     double* seconds) {
    Tensor tg = host_tensor(gate, {n}), tu = host_tensor(up, {n}), act = host_output({n});
    timed(seconds, [&] {
        tensor_ops::silu(tg, act);
        tensor_ops::mul(act, tu, act);
    });
    copy_out(act, out);
    return 0;
}

int ref_cpu_add_inplace(float* a, const float* b, std::size_t n, double* seconds) {
    Tensor ta = host_tensor(a, {n}), tb = host_tensor(b, {n});
    timed(seconds, [&] { tensor_ops::add_inplace(ta, tb); });
    copy_out(ta, a);
    return 0;
}

}  // extern "C"
