// Layer pipeline of the non-GEMM prefill path: the per-layer op sequence of
// PhiDecoderLayer::forward_carry (src/layer.cu:273-300) over all layers and
// the final add + LayerNorm of PhiTinyMoEModel::generate
// (src/model.cu:119-156), on prefix-trie node rows, with every GEMM output
// supplied by the caller (b2_prefill_layer).
//
// Per layer l, on the stream, in the reference's order:
//   l == 0 : x = emb[node_token]                       (b2_gather_rows)
//            normed = LN1(x)                           (b2_layer_norm)
//   l  > 0 : x = combine(expert_out[l-1]) + carry      (fused: the previous
//            normed = LN1(x)                            layer's un-permute,
//                                                       the carried residual
//                                                       add and this LN)
//            [q, k, v = GEMM(normed)]
//   RoPE(q, k) at node depths                          (b2_rope)
//            [attn = attention core + o_proj]
//   attn += x; post = LN2(attn)                        (b2_add_layer_norm)
//            [router logits = GEMM(post)]
//   route(logits)                                      (b2_moe_route)
//            [gate, up = grouped GEMM(post[assignment_rows])]
//   act = silu(gate) * up      (b2_silu_mul; expf in the tree-order mode)
//            [expert_out = grouped GEMM(act)]
//   carry = attn
// and finally x = combine(expert_out[L-1]) + carry, out = LN_final(x)
// (fused again). The fusion of the un-permute into the next LayerNorm keeps
// the MoE output row from ever being written to HBM; every other op is
// separated from its neighbours by a GEMM in the real model and so stays a
// kernel of its own.
#include <cstring>
#include <vector>

#include "common.cuh"

namespace {

int check_layer(const b2_prefill_layer& L, size_t i) {
    if (!L.q || !L.k || !L.attn || !L.router_logits || !L.gate || !L.up || !L.expert_out ||
        !L.ln1_gamma || !L.ln1_beta || !L.ln2_gamma || !L.ln2_beta)
        return b2::invalid("b2_prefill_layers: null pointer in layer " + std::to_string(i));
    return B2_OK;
}

}  // namespace

extern "C" {

int b2_prefill_layers(const b2_prefill_shape* shape, const float* emb, size_t vocab,
                      const uint32_t* node_token, const uint32_t* node_depth,
                      const float* rope_cos, const float* rope_sin, size_t rope_rows,
                      const b2_prefill_layer* layers, size_t num_layers,
                      const float* final_gamma, const float* final_beta,
                      const b2_prefill_work* work, float* final_x, float* final_out,
                      void* const* events, b2_stream_t stream) {
    using namespace b2;
    if (!shape || !layers || !work) return invalid("b2_prefill_layers: null argument");
    const b2_prefill_shape& s = *shape;
    if (s.rows == 0) return B2_OK;
    if (num_layers == 0) return invalid("b2_prefill_layers: no layers");
    if (!emb || !node_token || !node_depth || !rope_cos || !rope_sin || !final_gamma || !final_beta ||
        !final_x || !final_out)
        return invalid("b2_prefill_layers: null pointer");
    if (!work->x || !work->normed || !work->post || !work->act || !work->routes || !work->counts ||
        !work->offsets || !work->assignment_rows || !work->route_positions || !work->route_ws)
        return invalid("b2_prefill_layers: null work buffer");
    for (size_t i = 0; i < num_layers; ++i)
        if (int rc = check_layer(layers[i], i)) return rc;

    const size_t rows = s.rows, h = s.hidden, nl = num_layers;
    const float eps = s.eps;
    const uint32_t flags = s.flags;
    cudaStream_t cs = as_stream(stream);
    // Optional timing: event pair i brackets launch i (layout in the header).
    auto mark = [&](size_t pair, int end) -> int {
        if (!events || !events[2 * pair + end]) return B2_OK;
        const cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(events[2 * pair + end]), cs);
        return e == cudaSuccess ? B2_OK : set_error(B2_ERR_CUDA, std::string("event record: ") + cudaGetErrorString(e));
    };
    int rc;
    // layer 0 input: embedding gather onto trie nodes (src/model.cu:128)
    if ((rc = b2_gather_rows(emb, vocab, h, node_token, rows, work->x, stream))) return rc;
    for (size_t l = 0; l < nl; ++l) {
        const b2_prefill_layer& L = layers[l];
        const size_t stage = nl + 1 + 4 * l;
        if ((rc = mark(l, 0))) return rc;
        if (l == 0) {
            rc = b2_layer_norm(work->x, L.ln1_gamma, L.ln1_beta, work->normed, rows, h, eps, flags, stream);
        } else {
            const b2_prefill_layer& P = layers[l - 1];
            rc = b2_moe_combine_add_layer_norm(P.expert_out, 2 * rows, work->routes, work->route_positions,
                                               P.attn, L.ln1_gamma, L.ln1_beta, work->x, work->normed,
                                               rows, h, eps, flags, stream);
        }
        if (rc || (rc = mark(l, 1)) || (rc = mark(stage, 0))) return rc;
        if ((rc = b2_rope(L.q, L.k, node_depth, rows, s.q_heads, s.kv_heads, s.head_dim, rope_cos, rope_sin,
                          rope_rows, stream)))
            return rc;
        if ((rc = mark(stage, 1)) || (rc = mark(stage + 1, 0))) return rc;
        if ((rc = b2_add_layer_norm(L.attn, work->x, L.ln2_gamma, L.ln2_beta, work->post, rows, h, eps, flags,
                                    stream)))
            return rc;
        if ((rc = mark(stage + 1, 1)) || (rc = mark(stage + 2, 0))) return rc;
        if ((rc = b2_moe_route(L.router_logits, rows, s.experts, s.router_quantum, s.router_tie_eps,
                               work->routes, work->counts, work->offsets, work->assignment_rows,
                               work->route_positions, work->work_expert64, work->work_start64,
                               work->work_expert128, work->work_start128, work->route_ws,
                               work->route_ws_bytes, stream)))
            return rc;
        if ((rc = mark(stage + 2, 1)) || (rc = mark(stage + 3, 0))) return rc;
        if ((rc = b2::silu_mul_launch(L.gate, L.ld_gate_up, L.up, L.ld_gate_up, work->act, s.intermediate,
                                      2 * rows, s.intermediate, (flags & B2_FLAG_EXACT_ORDER) != 0, stream)))
            return rc;
        if ((rc = mark(stage + 3, 1))) return rc;
    }
    // the last layer's pending add folds into the final LayerNorm (src/model.cu:145-150)
    const b2_prefill_layer& Z = layers[nl - 1];
    if ((rc = mark(nl, 0))) return rc;
    if ((rc = b2_moe_combine_add_layer_norm(Z.expert_out, 2 * rows, work->routes, work->route_positions, Z.attn,
                                            final_gamma, final_beta, final_x, final_out, rows, h, eps, flags,
                                            stream)))
        return rc;
    return mark(nl, 1);
}

}  // extern "C"
