/*
 * aps2026_b200.h -- C ABI of the B200 (sm_100a) non-GEMM prefill layer ops of
 * Phi-tiny-MoE: embedding gather, LayerNorm (+ fused residual add), RoPE on
 * Q/K, causal scaled softmax, deterministic top-2 routing with the
 * token->expert permutation, gated SiLU, weighted un-permute, residual add,
 * and the prefix-trie dedup that feeds them.
 *
 * The reference exposes these as C++ free functions in `namespace tensor_ops`
 * that take `Tensor&` (ezzy0654/aps2026 include/tensor.h:63-161). This ABI
 * replaces each of them with a plain-C entry point:
 *   - every tensor is a raw DEVICE pointer (row-major, fp32 unless noted) plus
 *     explicit sizes -- shapes that the reference read from Tensor::size();
 *   - every device entry point takes the stream to run on (NULL = legacy
 *     default stream, which is what the reference always used);
 *   - no hot-path entry point allocates device memory; scratch is
 *     caller-provided and sized by a *_workspace_size() query (the
 *     diagnostic b2_selfcheck_exp allocates a 24-byte counter block);
 *   - there is no hidden per-process state except one status word per device
 *     that in-kernel bounds checks write (b2_device_status) and the fixed
 *     scratch of b2_moe_route_noalloc, so one host thread per GPU may call
 *     concurrently on different devices/streams;
 *   - errors are status codes instead of the reference's exceptions:
 *     B2_ERR_INVALID_ARGUMENT where the reference throws
 *     std::invalid_argument, B2_ERR_CUDA where its check_cuda throws
 *     std::runtime_error (src/tensor.cu:370-374), B2_ERR_IO where the
 *     harness's file reader / writer throws (src/main.cpp:144-192).
 *     b2_last_error() returns the message of the calling thread's last
 *     failure.
 *
 * Floating point: by default reductions (LayerNorm moments, softmax
 * denominators) are tree-shaped, the softmax and SiLU exponentials
 * (b2_silu_mul_flags, and inside b2_prefill_layers) are CUDA's expf and their
 * quotients a multiplication by a rounded reciprocal, and results agree with
 * the reference kernels within 1e-5 relative OR 1e-6 absolute. With
 * B2_FLAG_EXACT_ORDER reductions run in the reference's serial ascending
 * order, exponentials are the reference's (float)exp((double)x) and
 * divisions correctly rounded, and results agree bit for bit. Functions
 * without a flags argument (b2_silu_mul, b2_rope, b2_moe_combine, b2_add)
 * are always bit-exact; b2_silu_mul_flags is the SiLU with a mode. Index/integer outputs (gather, routing,
 * permutation) are always bit-exact.
 */
#ifndef APS2026_B200_H
#define APS2026_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* A cudaStream_t passed as an opaque pointer; NULL selects stream 0. */
typedef void* b2_stream_t;

enum b2_status {
    B2_OK = 0,
    B2_ERR_INVALID_ARGUMENT = 1, /* bad shape / size / null / alignment      */
    B2_ERR_CUDA = 2,             /* kernel launch or CUDA runtime failure     */
    B2_ERR_DEVICE_CHECK = 3,     /* an in-kernel bounds check saw a bad index */
    B2_ERR_TIMEOUT = 4,          /* a bounded device wait gave up             */
    B2_ERR_UNSUPPORTED = 5,      /* valid request outside what is built       */
    B2_ERR_IO = 6                /* a file could not be opened, read, written */
};

/* Flags for the floating-point reductions. */
#define B2_FLAG_EXACT_ORDER 1u /* serial ascending sums, bit-exact to reference */

/* ---- library / status ---------------------------------------------------- */

/* Version string of the library ("aps2026_b200 <semver> sm_100a"). */
const char* b2_version(void);

/* Message of this thread's last non-OK status ("" if none). */
const char* b2_last_error(void);

/*
 * Reads, then clears, the current device's in-kernel check word. Waits for
 * `stream` first. *status_out is 0 when no kernel since the last call saw an
 * out-of-range index; otherwise a bitmask of B2_CHECK_* (which kernel
 * family). Kernels that see a bad index skip that access (their output for
 * that row is zero) instead of reading out of bounds.
 */
#define B2_CHECK_GATHER 1u
#define B2_CHECK_ROPE 2u
#define B2_CHECK_COMBINE 4u
#define B2_CHECK_ATTENTION 8u
#define B2_CHECK_TRIE 16u
#define B2_CHECK_WAIT 32u    /* a bounded wait for a bulk copy gave up; the CTA stopped */
int b2_device_status(uint32_t* status_out, b2_stream_t stream);

/* ---- embedding / row gather ---------------------------------------------- */

/*
 * out[i, :] = x[rows[i], :] for i < count; x is [x_rows, h], out [count, h],
 * rows a device uint32 array. Bit-exact copy.
 * Replaces tensor_ops::gather_rows_gpu (include/tensor.h:115-116 and :138;
 * src/tensor.cu:3379-3387, :3419-3426; kernel k_gather_rows :2635-2642).
 * count == 0 is a no-op (as the RowIndexBuffer overload, :3420).
 */
int b2_gather_rows(const float* x, size_t x_rows, size_t h,
                   const uint32_t* rows, size_t count, float* out,
                   b2_stream_t stream);

/*
 * The MoE permutation gather: compact[i, :] = x[assignment_rows[i], :] for
 * i < assignments (2T), the expert-ordered GEMM input. Replaces
 * k_moe_gather_compact (src/tensor.cu:1420-1428) as moe_forward_grouped_gpu
 * launches it when the gather is not fused into its GEMM (:2824-2833).
 * The same kernel as b2_gather_rows (one CTA per row, 128-bit copies).
 */
int b2_moe_gather_compact(const float* x, size_t x_rows, size_t h,
                          const uint32_t* assignment_rows, size_t assignments,
                          float* compact, b2_stream_t stream);

/* ---- LayerNorm ------------------------------------------------------------ */

/*
 * y[r, :] = (x[r, :] - mean) * (1 / sqrtf(var + eps)) * gamma + beta, with
 * mean and var the two-pass row moments over h. x, y: [rows, h].
 * Replaces tensor_ops::layer_norm_gpu (include/tensor.h:86-87;
 * src/tensor.cu:3262-3280; kernel k_layer_norm :2130-2142).
 */
int b2_layer_norm(const float* x, const float* gamma, const float* beta,
                  float* y, size_t rows, size_t h, float eps, uint32_t flags,
                  b2_stream_t stream);

/*
 * The per-row statistics of b2_layer_norm without its output: mean[r] and
 * inv[r] = 1 / sqrtf(var / h + eps) of x[r, :] (x: [rows, h]; mean, inv:
 * [rows] floats). No reference counterpart as an entry point: they are the
 * moments k_layer_norm forms internally (ln_moments, src/tensor.cu:2063-2128),
 * exposed so that a GEMM can normalise its operand in its prologue
 * (b2_fusion::layer_norm_value, include/aps2026_b200_fusion.cuh) instead of
 * reading b2_layer_norm's output. With B2_FLAG_EXACT_ORDER they are the
 * reference's serial sums, bit-identical to what b2_layer_norm uses;
 * otherwise a tree reduction, within tolerance.
 */
int b2_layer_norm_stats(const float* x, size_t rows, size_t h, float eps,
                        uint32_t flags, float* mean, float* inv,
                        b2_stream_t stream);

/*
 * x[r, :] += residual[r, :] (written back), then y = LayerNorm(x).
 * Replaces tensor_ops::add_layer_norm_gpu (include/tensor.h:88-90;
 * src/tensor.cu:3282-3295; kernel k_add_layer_norm :2144-2178).
 */
int b2_add_layer_norm(float* x, const float* residual, const float* gamma,
                      const float* beta, float* y, size_t rows, size_t h,
                      float eps, uint32_t flags, b2_stream_t stream);

/*
 * Fused MoE un-permute + carried residual add + LayerNorm:
 *   x_out[t, :] = combine(expert_out)[t, :] + carry[t, :]
 *   y[t, :]     = LayerNorm(x_out[t, :])
 * where combine is exactly b2_moe_combine. This is the reference's
 * k_moe_combine (src/tensor.cu:1968-1988) followed by the next layer's
 * k_add_layer_norm of the carry protocol (src/layer.cu:273-300,
 * src/model.cu:145-150) in one pass: the MoE output row never goes to HBM.
 * Same arithmetic in the same order, so it equals the two-call sequence.
 */
int b2_moe_combine_add_layer_norm(const float* expert_out, size_t expert_rows,
                                  const uint8_t* routes,
                                  const uint32_t* route_positions,
                                  const float* carry, const float* gamma,
                                  const float* beta, float* x_out, float* y,
                                  size_t rows, size_t h, float eps,
                                  uint32_t flags, b2_stream_t stream);

/* ---- rotary embedding ----------------------------------------------------- */

/*
 * HOST function. Fills cos_host / sin_host ([max_seq, head_dim/2] floats)
 * with cos/sin(p * theta^(-2j/head_dim)) evaluated exactly as the
 * reference's host-built table (src/tensor.cu:2716-2724: powf, cosf, sinf in
 * float), so the device lookups are bit-identical.
 */
int b2_rope_table(size_t max_seq, size_t head_dim, float theta,
                  float* cos_host, float* sin_host);

/*
 * Rotate-half RoPE in place on q [rows, q_heads*head_dim] and
 * k [rows, kv_heads*head_dim] in ONE launch; row r uses table row
 * row_pos[r] (< table_rows) of the device tables from b2_rope_table.
 * Replaces tensor_ops::apply_rope_tree_gpu / apply_rope_gpu
 * (include/tensor.h:91-94, :104-108; src/tensor.cu:3297-3314, :3342-3359;
 * kernel k_rope :2180-2197, launched twice there).
 */
int b2_rope(float* q, float* k, const uint32_t* row_pos, size_t rows,
            size_t q_heads, size_t kv_heads, size_t head_dim,
            const float* cos_table, const float* sin_table, size_t table_rows,
            b2_stream_t stream);

/* ---- causal scaled softmax ------------------------------------------------ */

/*
 * probs[h, i, j] = softmax_j(scores[h, i, j] * scale) over the causal
 * sliding window j in [max(0, i + 1 - window), i]; entries outside it are 0.
 * scores, probs: [heads, T, ld] (ld >= T; columns >= T are not touched).
 * Max, exp(double) rounded to float, ascending denominator and division are
 * the softmax section of k_attention_tree_gqa4 (src/tensor.cu:2448, :2526,
 * :2549-2585; window rule :2435-2439). The reference declares
 * softmax_last_dim (include/tensor.h:152) but defines no standalone kernel.
 */
int b2_causal_softmax(const float* scores, float* probs, size_t heads,
                      size_t T, size_t ld, float scale, size_t window,
                      uint32_t flags, b2_stream_t stream);

/*
 * Prefix-tree GQA attention core: for trie row r and KV head h, the keys
 * and values are the rows of r's ancestor chain anc[r * anc_stride + begin
 * .. + pos] (pos = row_pos[r], begin = max(0, pos + 1 - window)); each of
 * the 4 query heads of h gets softmax(q . k * 1/sqrt(head_dim)) . v.
 * q, out: [rows, q_heads*head_dim]; k, v: [rows, kv_heads*head_dim];
 * q_heads = 4 * kv_heads; head_dim 64 or 128. Same arithmetic and order as
 * k_attention_tree_gqa4 (src/tensor.cu:2425-2633; wrapper
 * tensor_ops::attention_tree_gpu, include/tensor.h:109-114, :3361-3377;
 * the reference's window is SLIDING_WINDOW = 2047): bit-identical with
 * B2_FLAG_EXACT_ORDER, within tolerance with tree-order softmax sums.
 * A row whose position is >= anc_stride, or a chain entry >= rows, is
 * reported through b2_device_status (B2_CHECK_ATTENTION).
 * Without B2_FLAG_EXACT_ORDER and at head_dim 128, blocks of 32 trie rows
 * that form a path run on the tensor cores (three TF32 products per FP32
 * product) from TF32 hi / lo copies of k and v in stream-ordered scratch of
 * 16 * rows * kv_heads * 128 + 4 * (rows / 32 + 2) * kv_heads bytes, taken
 * from a memory pool the library keeps per device (its memory stays
 * reserved between calls) or, during stream capture, a graph allocation;
 * the scratch is freed on `stream` after the launches. If it cannot be had,
 * every block runs on the CUDA cores instead.
 */
int b2_attention_tree(const float* q, const float* k, const float* v,
                      float* out, const uint32_t* row_pos,
                      const uint32_t* anc, size_t anc_stride, size_t rows,
                      size_t q_heads, size_t kv_heads, size_t head_dim,
                      size_t window, uint32_t flags, b2_stream_t stream);

/*
 * b2_attention_tree with the compact ancestor form of b2_prefix_trie_device
 * instead of the dense [rows, anc_stride] table (1 GB at 64 x 2048 tokens;
 * no reference counterpart): row r's chain is
 * token_node[prompt_offsets[p] .. + pos], p = node_prompt[r], so only the
 * packed token_node array [total_tokens] is read. max_len bounds the
 * positions (the longest prompt). Same kernels, arithmetic and results as
 * b2_attention_tree on the equivalent dense table; a row whose witness
 * prompt does not reach its position is reported like a bad position.
 */
int b2_attention_tree_compact(const float* q, const float* k, const float* v,
                              float* out, const uint32_t* row_pos,
                              const uint32_t* node_prompt,
                              const uint32_t* prompt_offsets, size_t prompts,
                              const uint32_t* token_node, size_t total_tokens,
                              size_t max_len, size_t rows, size_t q_heads,
                              size_t kv_heads, size_t head_dim, size_t window,
                              uint32_t flags, b2_stream_t stream);

/* ---- MoE routing (bit-exact) ---------------------------------------------- */

/* Bytes of caller workspace b2_moe_route needs for T tokens, E experts. */
int b2_moe_route_workspace_size(size_t T, size_t E, size_t* bytes);

/*
 * Top-2 routing + token->expert permutation, replacing the routing part of
 * tensor_ops::moe_forward_grouped_gpu (include/tensor.h:146-147;
 * src/tensor.cu:2790-2821: memsets, k_moe_top2 :1293-1331,
 * k_moe_offsets_work :1337-1374, k_moe_fill_stable :1376-1418).
 *   logits            [T, E] fp32 (E <= 32)
 *   routes            [T, 2] uint8: first, second expert of each token
 *   counts            [E]    tokens per expert
 *   offsets           [E+1]  exclusive prefix of counts
 *   assignment_rows   [2T]   token of each expert-ordered assignment
 *   route_positions   [2T]   position of (token t, slot s) at [2t+s]
 *   work_expert64 / work_start64    [ceil(2T/64)+E]  64-row chunks
 *   work_expert128 / work_start128  [ceil(2T/128)+E] 128-row chunks
 *     (unused queue entries are 0xFFFFFFFF, as the reference memsets them;
 *      any queue pointer may be NULL to skip it)
 * Scores are quantized to `quantum` (reference 1e-3) and picked by an
 * ascending scan that only replaces on > best + tie_eps (reference 2e-2).
 * The workspace (b2_moe_route_workspace_size bytes, 16-byte aligned) holds
 * per-tile expert histograms between the two launches; it needs no
 * initialisation. Calls that overlap on the GPU must not share it.
 */
int b2_moe_route(const float* logits, size_t T, size_t E, float quantum,
                 float tie_eps, uint8_t* routes, uint32_t* counts,
                 uint32_t* offsets, uint32_t* assignment_rows,
                 uint32_t* route_positions, uint32_t* work_expert64,
                 uint32_t* work_start64, uint32_t* work_expert128,
                 uint32_t* work_start128, void* workspace,
                 size_t workspace_bytes, b2_stream_t stream);

/*
 * b2_moe_route without a caller workspace -- no counterpart in the
 * reference. For callers that cannot allocate device memory (a plugin whose
 * host framework owns all device allocations and forbids allocating on its
 * execution path, or code that must not call cudaMalloc because it can
 * synchronize the device). Same arguments and outputs as b2_moe_route minus
 * the workspace; allocates nothing: the per-tile histograms live in a fixed
 * 128 KB array compiled into the library (held by every GPU that loads it
 * until the process exits), which limits ceil(T/256) * E' to 32768 words
 * with E' = E rounded up to a power of two >= 4 (524,288 tokens at E = 16);
 * larger requests return B2_ERR_UNSUPPORTED. Each call looks up the array's
 * device address on the current device (cudaGetSymbolAddress, a host-side
 * lookup), so a context reset between calls is safe; the first call on a
 * device also loads the library's device code there, so make that first call
 * before any stream capture. All calls on a device share the array: calls
 * that overlap on the GPU (other streams, other host threads) race on it.
 * Every word a call reads it has written first, so nothing needs clearing.
 */
int b2_moe_route_noalloc(const float* logits, size_t T, size_t E,
                         float quantum, float tie_eps, uint8_t* routes,
                         uint32_t* counts, uint32_t* offsets,
                         uint32_t* assignment_rows,
                         uint32_t* route_positions, uint32_t* work_expert64,
                         uint32_t* work_start64, uint32_t* work_expert128,
                         uint32_t* work_start128, b2_stream_t stream);

/* ---- expert activation, un-permute, residual ------------------------------ */

/*
 * out[r, c] = g / (1 + (float)exp((double)-g)) * up[r, c], g = gate[r, c];
 * gate/up/out rows strided by ld_gate/ld_up/ld_out elements, so both the
 * split [2T,448] and the concatenated [2T,896] gate|up layouts work.
 * Replaces tensor_ops::silu_mul_gpu (include/tensor.h:85;
 * src/tensor.cu:3254-3260; kernel k_silu_mul :2001-2010; the same math is
 * the epilogue of k_moe_pair_silu_8x8 :1953-1965).
 */
int b2_silu_mul(const float* gate, size_t ld_gate, const float* up,
                size_t ld_up, float* out, size_t ld_out, size_t rows,
                size_t cols, b2_stream_t stream);

/*
 * b2_silu_mul with the numerics mode of `flags`, like the other
 * floating-point ops: B2_FLAG_EXACT_ORDER is b2_silu_mul (bit-exact); 0
 * evaluates exp(-g) with CUDA's expf and the quotient with __fdividef
 * (within 1e-5 relative OR 1e-6 absolute of the reference; no reference
 * counterpart of its own).
 */
int b2_silu_mul_flags(const float* gate, size_t ld_gate, const float* up,
                      size_t ld_up, float* out, size_t ld_out, size_t rows,
                      size_t cols, uint32_t flags, b2_stream_t stream);

/*
 * out[t, :] = 0.5 * expert_out[p_lo, :] + 0.5 * expert_out[p_hi, :], where
 * p_lo/p_hi are the route_positions of token t's two assignments in
 * ascending EXPERT id order; expert_out is [expert_rows, h].
 * Replaces k_moe_combine (src/tensor.cu:1968-1988, launched at :2922-2926).
 */
int b2_moe_combine(const float* expert_out, size_t expert_rows,
                   const uint8_t* routes, const uint32_t* route_positions,
                   float* out, size_t T, size_t h, b2_stream_t stream);

/*
 * a[i] += b[i] for i < n.
 * Replaces tensor_ops::add_inplace_gpu (include/tensor.h:83;
 * src/tensor.cu:3236-3242; kernel k_add :1990-1993).
 */
int b2_add(float* a, const float* b, size_t n, b2_stream_t stream);

/* ---- prefix-trie dedup ------------------------------------------------------ */

/*
 * HOST function. Builds the prefix trie of `batch` prompts packed in `ids`
 * (prompt b has seq_lens[b] tokens, all in [0, vocab)), numbering nodes in
 * order of creation exactly as PhiTinyMoEModel::generate does
 * (src/model.cu:64-117):
 *   token_node [sum(seq_lens)] node of each packed token row
 *   node_token [nodes]  token id of each node        (capacity: total tokens)
 *   node_depth [nodes]  depth = RoPE position        (capacity: total tokens)
 *   node_anc   [nodes * anc_stride] ancestor chain root->node, zero padded;
 *              may be NULL (it only feeds the attention core)
 * *nodes_out receives the node count. anc_stride must be >= max seq_len.
 * Returns B2_ERR_INVALID_ARGUMENT for an empty batch or prompt, a token out
 * of the vocabulary, or a prompt longer than max_len (the reference's
 * MAX_POSITION_EMBEDDINGS check, src/model.cu:55-58).
 */
int b2_prefix_trie_build(const int32_t* ids, const uint32_t* seq_lens,
                         size_t batch, size_t vocab, size_t max_len,
                         uint32_t* token_node, uint32_t* node_token,
                         uint32_t* node_depth, uint32_t* node_anc,
                         size_t anc_stride, size_t* nodes_out);

/*
 * DEVICE twin of b2_prefix_trie_build, no reference counterpart as a kernel
 * (the reference walks the trie on the host, src/model.cu:64-117): the same
 * token_node / node_token / node_depth, numbered identically, computed from
 * longest common prefixes with earlier prompts on the GPU, so an end-to-end
 * step uploads token ids only. All pointers are device memory:
 *   ids        [total]      int32 token ids, prompts packed back to back
 *   offsets    [batch + 1]  prompt b is ids[offsets[b] .. offsets[b + 1]),
 *                           offsets[0] = 0, offsets[batch] = total
 *   token_node [total]; node_token, node_depth [total] (the first
 *   *node_count entries are written); node_prompt [total] or NULL: a prompt
 *   containing each node, so its ancestor chain root..node is
 *   token_node[offsets[p] .. offsets[p] + node_depth[node]] (the compact form
 *   of node_anc); node_count: device uint32 scalar.
 * Workspace: b2_prefix_trie_device_workspace_size bytes, 4-byte aligned.
 * Inputs the host version rejects (an empty or over-long prompt, a token
 * outside [0, vocab), offsets that do not split [0, total)) are reported
 * through b2_device_status (B2_CHECK_TRIE); no access leaves the arrays.
 * Cost: O(batch^2) prefix comparisons (one 32-token step for unrelated
 * prompts) plus O(total).
 */
int b2_prefix_trie_device_workspace_size(size_t batch, size_t* bytes);
int b2_prefix_trie_device(const int32_t* ids, const uint32_t* offsets,
                          size_t batch, size_t total, size_t vocab,
                          size_t max_len, uint32_t* token_node,
                          uint32_t* node_token, uint32_t* node_depth,
                          uint32_t* node_prompt, uint32_t* node_count,
                          void* workspace, size_t workspace_bytes,
                          b2_stream_t stream);

/* ---- input and output files of the prefill harness ----------------------------- */

/*
 * HOST function, replaces read_inputs (src/main.cpp:144-181). Reads the
 * variable-length prompt file:
 *   uint32 batch, uint32 max_seq_len, then `batch` times
 *   uint32 len, int32 ids[len]                      (little-endian)
 * and returns the prompts packed back to back in file order -- the `ids` /
 * `seq_lens` pair that b2_prefix_trie_build takes (b2_prefix_trie_device
 * takes ids and the running sum of seq_lens as offsets).
 * Call it with seq_lens = ids = NULL to learn the sizes (*batch_out,
 * *max_seq_out, *total_out = sum of the lengths; any of the three may be
 * NULL), then with buffers of at least batch and total entries. Token ids
 * are returned as stored (b2_prefix_trie_build checks the vocabulary, as
 * src/model.cu:55-58 does). max_len is the largest accepted max_seq_len
 * (MAX_POSITION_EMBEDDINGS = 4096 in include/config.h:16). The whole file is
 * validated on every call. Errors, in the reference's order and with its
 * messages (b2_last_error): B2_ERR_IO "cannot open input: <path>", "invalid
 * input header" (shorter than 8 bytes, batch or max_seq_len 0, max_seq_len
 * above max_len), "invalid sequence length in input" (a length field cut
 * short, 0, or above max_seq_len), "truncated input" (fewer ids than the
 * length says); bytes after the last prompt are ignored, as there.
 * B2_ERR_INVALID_ARGUMENT: null path, only one of seq_lens / ids given, or
 * a buffer below the sizes.
 */
int b2_read_inputs(const char* path, size_t max_len, uint32_t* batch_out,
                   uint32_t* max_seq_out, size_t* total_out, uint32_t* seq_lens,
                   size_t seq_lens_cap, int32_t* ids, size_t ids_cap);

/*
 * HOST function, replaces write_outputs (src/main.cpp:183-192). Writes the
 * prefill output file byte for byte as the reference does:
 *   uint32 batch, uint32 vocab, float logits[batch][vocab]  (little-endian)
 * logits is row-major [batch, vocab] fp32, in device memory when
 * logits_on_device != 0 (streamed through two 4 MiB pinned staging buffers
 * by copies on `stream`, one chunk written while the next copies; the call
 * orders itself after the work already on `stream`), else host memory
 * (written directly; no CUDA call is made). Synchronous: returns once the
 * file is closed. The pinned buffers are allocated and freed per call (a
 * file write, not a hot-path step). Errors: B2_ERR_IO "cannot open output:
 * <path>" / "failed while writing output: <path>" (the reference's
 * messages); B2_ERR_INVALID_ARGUMENT for a null path, null logits with
 * batch * vocab > 0, or batch / vocab above UINT32_MAX (the reference would
 * truncate them to 32 bits); B2_ERR_CUDA for a failed copy.
 */
int b2_write_outputs(const char* path, const float* logits, size_t batch,
                     size_t vocab, int logits_on_device, b2_stream_t stream);

/* ---- diagnostics --------------------------------------------------------------- */

/*
 * Checks the kernels' fast (float)exp((double)x) -- a table-driven double
 * evaluation that defers to exp(double) near float rounding midpoints --
 * against exp(double) itself for every float whose bit pattern lies in
 * [lo_bits, hi_bits). Synchronous; allocates a 24-byte counter block (a
 * diagnostic, not a hot-path call). *mismatches must come back 0;
 * *slow_path counts arguments that took the exp(double) path.
 */
int b2_selfcheck_exp(uint32_t lo_bits, uint32_t hi_bits, uint64_t* checked,
                     uint64_t* mismatches, uint64_t* slow_path);

/*
 * Diagnostic, no reference counterpart: launches one warp that waits on a
 * shared-memory barrier nothing completes, with the bounded wait the bulk-copy
 * kernels use (limit_ns of the global timer, at most 10 s). The wait gives
 * up, the kernel returns, and b2_device_status then reports B2_CHECK_WAIT;
 * the context stays usable. Tests the failure path without any fault.
 */
int b2_selfcheck_wait(uint64_t limit_ns);

/* ---- non-GEMM layer pipeline ------------------------------------------------ */

/* Model shape and numerics of one prefill batch (config.h defaults in
 * brackets: include/config.h:6-26). */
typedef struct b2_prefill_shape {
    size_t rows;          /* trie-node rows of the batch                  */
    size_t hidden;        /* [4096]                                       */
    size_t q_heads;       /* [16]                                         */
    size_t kv_heads;      /* [4]                                          */
    size_t head_dim;      /* [128]                                        */
    size_t experts;       /* [16]                                         */
    size_t intermediate;  /* [448]                                        */
    float eps;            /* [1e-5]                                       */
    float router_quantum; /* [1e-3]                                       */
    float router_tie_eps; /* [2e-2]                                       */
    uint32_t flags;       /* B2_FLAG_EXACT_ORDER or 0                     */
} b2_prefill_shape;

/* One decoder layer's GEMM outputs (device pointers; in the real model the
 * projections and experts write them) and LayerNorm parameters. */
typedef struct b2_prefill_layer {
    float* q;                   /* [rows, q_heads*head_dim], RoPE in place   */
    float* k;                   /* [rows, kv_heads*head_dim], RoPE in place  */
    float* attn;                /* [rows, hidden] o_proj output; += x in     */
                                /* place, then carried to the next layer     */
    const float* router_logits; /* [rows, experts]                           */
    const float* gate;          /* [2*rows, .] rows strided by ld_gate_up    */
    const float* up;            /* [2*rows, .]                               */
    size_t ld_gate_up;
    const float* expert_out;    /* [2*rows, hidden] W2 output, expert order  */
    const float* ln1_gamma;     /* input_layernorm [hidden]                  */
    const float* ln1_beta;
    const float* ln2_gamma;     /* post_attention_layernorm [hidden]         */
    const float* ln2_beta;
} b2_prefill_layer;

/* Caller-owned working buffers (nothing is allocated by the library). */
typedef struct b2_prefill_work {
    float* x;                   /* [rows, hidden] residual stream            */
    float* normed;              /* [rows, hidden] input LN out (-> q/k/v)     */
    float* post;                /* [rows, hidden] post-attn LN out (-> MoE)   */
    float* act;                 /* [2*rows, intermediate] SiLU(gate)*up       */
    uint8_t* routes;            /* b2_moe_route outputs, sized for rows       */
    uint32_t* counts;
    uint32_t* offsets;
    uint32_t* assignment_rows;
    uint32_t* route_positions;
    uint32_t* work_expert64;    /* may be NULL                                */
    uint32_t* work_start64;
    uint32_t* work_expert128;
    uint32_t* work_start128;
    void* route_ws;             /* b2_moe_route_workspace_size(rows, experts) */
    size_t route_ws_bytes;
} b2_prefill_work;

/*
 * Runs the non-GEMM path of all `num_layers` decoder layers plus the final
 * add + LayerNorm on trie-node rows, in the order of
 * PhiDecoderLayer::forward_carry (src/layer.cu:273-300) and
 * PhiTinyMoEModel::generate (src/model.cu:119-150):
 * embedding gather of node_token; per layer: LN1 (layer 0) or the previous
 * layer's un-permute + carried add + LN1 (fused), RoPE at node_depth,
 * attn += x + LN2, top-2 routing, SiLU(gate)*up; finally the last
 * un-permute + carried add + final LN. final_x receives the final residual
 * stream and final_out its LayerNorm ([rows, hidden] each).
 *
 * `events` (NULL for none) is an array of 2 * (5 * num_layers + 1)
 * cudaEvent_t handles recorded on `stream` around each launch, pair i at
 * [2i, 2i+1]: i = l < num_layers is layer l's LN1 step (plain LN for l = 0,
 * the fused un-permute + add + LN otherwise), i = num_layers the final fused
 * step, i = num_layers + 1 + 4l + s layer l's RoPE (s = 0), add + LN2 (1),
 * routing (2) and SiLU (3); a NULL handle in the array skips that record.
 * Kernel launches issued: B2_PREFILL_LAUNCHES(L).
 */
#define B2_PREFILL_LAUNCHES(num_layers) (2 + 6 * (num_layers))
int b2_prefill_layers(const b2_prefill_shape* shape, const float* emb, size_t vocab,
                      const uint32_t* node_token, const uint32_t* node_depth,
                      const float* rope_cos, const float* rope_sin, size_t rope_rows,
                      const b2_prefill_layer* layers, size_t num_layers,
                      const float* final_gamma, const float* final_beta,
                      const b2_prefill_work* work, float* final_x, float* final_out,
                      void* const* events, b2_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* APS2026_B200_H */
