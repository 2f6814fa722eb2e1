// TEST INFRASTRUCTURE ONLY: the reference's own model code behind a C entry
// point, for checking the drop-in claim end to end.
//
// oracle/Makefile compiles this file with the reference's src/model.cu,
// src/layer.cu, src/model_loader.cu and src/tensor.cu (from where they lie,
// unmodified) twice:
//   _ref/libdropin_ref.so  the reference as it is;
//   _ref/libdropin_b2.so   the same sources, except that the tensor_ops
//                          functions aps2026_b200/shim/tensor_ops_b2.cu
//                          defines are renamed out of tensor.cu (a -D
//                          name=ref_name per function, on that translation
//                          unit only -- the build-system form of deleting
//                          them) and the shim, over libaps2026_b200.so, is
//                          linked in their place.
// layer.cu and model.cu are compiled unchanged in both. The two libraries
// export the same functions; each is loaded in its own process.
//
// Entry points run PhiTinyMoEModel::generate (src/model.cu:45-159: trie
// dedup, embedding gather, 32 x forward_carry over the node rows with the
// tree RoPE and tree attention, final add + LayerNorm, last-row gather,
// lm_head) and PhiTinyMoEModel::forward with use_gpu = true
// (src/model.cu:20-39: per-layer LayerNorm, packed RoPE and attention,
// add + LayerNorm, MoE, residual add). Status: 0 ok, 1 std::invalid_argument,
// 2 any other exception; the message is returned by dropin_error().
#include <chrono>
#include <cstring>
#include <exception>
#include <stdexcept>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "config.h"
#include "model.h"

namespace {

thread_local std::string g_error;

int fail(const std::exception& e, int code) {
    g_error = e.what();
    return code;
}

double now_ms() {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

}  // namespace

extern "C" {

const char* dropin_error() { return g_error.c_str(); }

void* dropin_load(const char* model_path) {
    try {
        return new PhiTinyMoEModel(model_path);
    } catch (const std::exception& e) {
        g_error = e.what();
        return nullptr;
    }
}

void dropin_free(void* model) { delete static_cast<PhiTinyMoEModel*>(model); }

// Prompts packed in ids, prompt b = ids[offsets[b] .. offsets[b + 1]);
// logits: [batch, VOCAB_SIZE] on the host. *ms: the generate call's wall time,
// device synchronised on both sides, the logits' copy to the host included.
int dropin_generate(void* model, const int* ids, const int* offsets, int batch, float* logits, double* ms) {
    try {
        std::vector<std::vector<int>> prompts(static_cast<std::size_t>(batch));
        for (int b = 0; b < batch; ++b) prompts[b].assign(ids + offsets[b], ids + offsets[b + 1]);
        Tensor out;
        cudaDeviceSynchronize();
        const double t0 = now_ms();
        static_cast<const PhiTinyMoEModel*>(model)->generate(prompts, out);
        const float* host = static_cast<const Tensor&>(out).data();
        cudaDeviceSynchronize();
        if (ms) *ms = now_ms() - t0;
        if (out.size() != static_cast<std::size_t>(batch) * apss26::VOCAB_SIZE)
            throw std::runtime_error("generate returned an unexpected logits shape");
        std::memcpy(logits, host, out.size() * sizeof(float));
        return 0;
    } catch (const std::invalid_argument& e) {
        return fail(e, 1);
    } catch (const std::exception& e) {
        return fail(e, 2);
    }
}

// One prompt through forward(ids, logits, use_gpu = true); logits [VOCAB_SIZE].
int dropin_forward(void* model, const int* ids, int n, float* logits, double* ms) {
    try {
        const std::vector<int> prompt(ids, ids + n);
        Tensor out;
        cudaDeviceSynchronize();
        const double t0 = now_ms();
        static_cast<const PhiTinyMoEModel*>(model)->forward(prompt, out, /*use_gpu=*/true);
        const float* host = static_cast<const Tensor&>(out).data();
        cudaDeviceSynchronize();
        if (ms) *ms = now_ms() - t0;
        if (out.size() != apss26::VOCAB_SIZE) throw std::runtime_error("forward returned an unexpected logits shape");
        std::memcpy(logits, host, out.size() * sizeof(float));
        return 0;
    } catch (const std::invalid_argument& e) {
        return fail(e, 1);
    } catch (const std::exception& e) {
        return fail(e, 2);
    }
}

// The packed-segment ops of PhiAttention::forward's GPU branch
// (src/layer.cu:232-240) on host arrays: q [rows, 16*128], k, v
// [rows, 4*128], segments of lengths lens[0..segments); q and k are rotated
// in place, attention written to out [rows, 16*128].
int dropin_packed_attention(float* q, float* k, const float* v, const size_t* lens, int segments, float* out) {
    try {
        std::vector<std::size_t> seq_lens(lens, lens + segments);
        std::size_t rows = 0;
        for (std::size_t n : seq_lens) rows += n;
        const std::size_t qd = apss26::NUM_ATTENTION_HEADS * apss26::HEAD_DIM;
        const std::size_t kd = apss26::NUM_KV_HEADS * apss26::HEAD_DIM;
        Tensor tq({rows, qd}), tk({rows, kd}), tv({rows, kd}), to({rows, qd});
        std::memcpy(tq.data(), q, rows * qd * sizeof(float));
        std::memcpy(tk.data(), k, rows * kd * sizeof(float));
        std::memcpy(tv.data(), v, rows * kd * sizeof(float));
        tensor_ops::apply_rope_gpu(tq, tk, seq_lens, apss26::NUM_ATTENTION_HEADS, apss26::NUM_KV_HEADS,
                                   apss26::HEAD_DIM, apss26::ROPE_THETA);
        tensor_ops::attention_gpu(tq, tk, tv, to, seq_lens, apss26::NUM_ATTENTION_HEADS, apss26::NUM_KV_HEADS,
                                  apss26::HEAD_DIM);
        std::memcpy(q, static_cast<const Tensor&>(tq).data(), rows * qd * sizeof(float));
        std::memcpy(k, static_cast<const Tensor&>(tk).data(), rows * kd * sizeof(float));
        std::memcpy(out, static_cast<const Tensor&>(to).data(), rows * qd * sizeof(float));
        return 0;
    } catch (const std::invalid_argument& e) {
        return fail(e, 1);
    } catch (const std::exception& e) {
        return fail(e, 2);
    }
}

// add_inplace_gpu (src/layer.cu:322): a += b over n floats, on host arrays.
int dropin_add_inplace(float* a, const float* b, size_t n) {
    try {
        Tensor ta({n}), tb({n});
        std::memcpy(ta.data(), a, n * sizeof(float));
        std::memcpy(tb.data(), b, n * sizeof(float));
        tensor_ops::add_inplace_gpu(ta, tb);
        std::memcpy(a, static_cast<const Tensor&>(ta).data(), n * sizeof(float));
        return 0;
    } catch (const std::invalid_argument& e) {
        return fail(e, 1);
    } catch (const std::exception& e) {
        return fail(e, 2);
    }
}

}  // extern "C"
