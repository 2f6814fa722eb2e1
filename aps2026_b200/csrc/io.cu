// Prefill input and output files of the course harness (host side).
//
// Reference: src/main.cpp:144-181 (read_inputs) and :183-192
// (write_outputs). Both files are little-endian and unpadded:
//   inputs:  uint32 batch, uint32 max_seq_len, then per prompt
//            uint32 len, int32 ids[len]
//   outputs: uint32 batch, uint32 vocab, float logits[batch][vocab]
//
// The reader parses the whole file from one buffer and returns the prompts
// packed back to back with their lengths -- exactly what
// b2_prefix_trie_build / b2_prefix_trie_device take -- instead of a vector
// per prompt; it applies the reference's checks in the reference's order and
// fails with its messages. The writer takes the logits where they are: from
// device memory it streams them through two pinned staging buffers (chunk
// i + 1 copies while chunk i is written), where the reference first copies
// the whole tensor into a pageable host vector (Tensor::data ->
// sync_cuda_to_host) and writes it afterwards.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/aps2026_b200.h"

namespace b2 {
int set_error(int code, const std::string& message);
}

namespace {

constexpr std::size_t kStageBytes = std::size_t(4) << 20;  // per staging buffer

int io_error(const std::string& message) { return b2::set_error(B2_ERR_IO, message); }

// Closes the file on every return path.
struct File {
    std::FILE* f = nullptr;
    File(const char* path, const char* mode) : f(std::fopen(path, mode)) {}
    ~File() {
        if (f) std::fclose(f);
    }
    // fclose flushes: a failure there is a failed write too.
    bool close() {
        const bool ok = std::fclose(f) == 0;
        f = nullptr;
        return ok;
    }
};

bool read_all(const char* path, std::vector<unsigned char>* out) {
    File file(path, "rb");
    if (!file.f) return false;
    unsigned char buf[1 << 16];
    std::size_t n = 0;
    while ((n = std::fread(buf, 1, sizeof buf, file.f)) > 0) out->insert(out->end(), buf, buf + n);
    return !std::ferror(file.f);
}

std::uint32_t load_u32(const unsigned char* p) {
    std::uint32_t v;
    std::memcpy(&v, p, sizeof v);
    return v;
}

// Pinned staging buffers and their events, released on every return path --
// after the copies last recorded on them have landed, so an early return
// never frees a buffer a copy is still writing.
struct Staging {
    void* buf[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    ~Staging() {
        for (int i = 0; i < 2; ++i) {
            if (done[i]) {
                cudaEventSynchronize(done[i]);
                cudaEventDestroy(done[i]);
            }
            if (buf[i]) cudaFreeHost(buf[i]);
        }
    }
};

int cuda_error(const char* what, cudaError_t e) {
    return b2::set_error(B2_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Streams `bytes` of device memory at `src` into `f`: chunk i is copied on
// `stream` into staging buffer i % 2 while chunk i - 1 is written.
int write_from_device(std::FILE* f, const unsigned char* src, std::size_t bytes, cudaStream_t stream,
                      const std::string& fail_message) {
    Staging st;
    const std::size_t stage = std::min(bytes, kStageBytes);
    const int nbuf = bytes > stage ? 2 : 1;
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < nbuf; ++i) {
        if ((e = cudaMallocHost(&st.buf[i], stage)) != cudaSuccess) return cuda_error("pinned staging", e);
        if ((e = cudaEventCreateWithFlags(&st.done[i], cudaEventDisableTiming)) != cudaSuccess)
            return cuda_error("staging event", e);
    }
    const std::size_t chunks = (bytes + stage - 1) / stage;
    auto enqueue = [&](std::size_t c) -> cudaError_t {
        const std::size_t off = c * stage, n = std::min(stage, bytes - off);
        const int b = static_cast<int>(c % 2);
        cudaError_t r = cudaMemcpyAsync(st.buf[b], src + off, n, cudaMemcpyDeviceToHost, stream);
        return r != cudaSuccess ? r : cudaEventRecord(st.done[b], stream);
    };
    if ((e = enqueue(0)) != cudaSuccess) return cuda_error("copy logits to host", e);
    for (std::size_t c = 0; c < chunks; ++c) {
        const int b = static_cast<int>(c % 2);
        if ((e = cudaEventSynchronize(st.done[b])) != cudaSuccess) return cuda_error("copy logits to host", e);
        // the other buffer was written out in the previous iteration: refill it
        if (c + 1 < chunks && (e = enqueue(c + 1)) != cudaSuccess) return cuda_error("copy logits to host", e);
        const std::size_t n = std::min(stage, bytes - c * stage);
        if (std::fwrite(st.buf[b], 1, n, f) != n) return io_error(fail_message);
    }
    return B2_OK;
}

}  // namespace

extern "C" int b2_write_outputs(const char* path, const float* logits, size_t batch, size_t vocab,
                                int logits_on_device, b2_stream_t stream) {
    if (path == nullptr) return b2::set_error(B2_ERR_INVALID_ARGUMENT, "write_outputs: null path");
    if (batch > UINT32_MAX || vocab > UINT32_MAX)
        return b2::set_error(B2_ERR_INVALID_ARGUMENT, "write_outputs: batch and vocab must fit in uint32");
    if (batch != 0 && vocab > SIZE_MAX / sizeof(float) / batch)
        return b2::set_error(B2_ERR_INVALID_ARGUMENT, "write_outputs: batch * vocab overflows");
    const std::size_t bytes = batch * vocab * sizeof(float);
    if (bytes != 0 && logits == nullptr) return b2::set_error(B2_ERR_INVALID_ARGUMENT, "write_outputs: null logits");

    File file(path, "wb");
    if (!file.f) return io_error(std::string("cannot open output: ") + path);
    const std::string fail = std::string("failed while writing output: ") + path;
    const std::uint32_t header[2] = {static_cast<std::uint32_t>(batch), static_cast<std::uint32_t>(vocab)};
    if (std::fwrite(header, sizeof header[0], 2, file.f) != 2) return io_error(fail);
    if (bytes != 0) {
        if (logits_on_device) {
            const int rc = write_from_device(file.f, reinterpret_cast<const unsigned char*>(logits), bytes,
                                             static_cast<cudaStream_t>(stream), fail);
            if (rc != B2_OK) return rc;
        } else if (std::fwrite(logits, 1, bytes, file.f) != bytes) {
            return io_error(fail);
        }
    }
    if (!file.close()) return io_error(fail);
    return B2_OK;
}

extern "C" int b2_read_inputs(const char* path, size_t max_len, uint32_t* batch_out, uint32_t* max_seq_out,
                              size_t* total_out, uint32_t* seq_lens, size_t seq_lens_cap, int32_t* ids,
                              size_t ids_cap) {
    if (path == nullptr) return b2::set_error(B2_ERR_INVALID_ARGUMENT, "read_inputs: null path");
    if ((seq_lens == nullptr) != (ids == nullptr))
        return b2::set_error(B2_ERR_INVALID_ARGUMENT, "read_inputs: give both seq_lens and ids, or neither");
    std::vector<unsigned char> buf;
    if (!read_all(path, &buf)) return io_error(std::string("cannot open input: ") + path);

    const std::size_t size = buf.size();
    const unsigned char* p = buf.data();
    if (size < 8) return io_error("invalid input header");
    const std::uint32_t batch = load_u32(p), max_seq = load_u32(p + 4);
    if (batch == 0 || max_seq == 0 || max_seq > max_len) return io_error("invalid input header");

    // one pass validates the whole file and counts the tokens; the second
    // (when buffers are given) copies them
    std::size_t pos = 8, total = 0;
    for (std::uint32_t b = 0; b < batch; ++b) {
        if (size - pos < 4) return io_error("invalid sequence length in input");
        const std::uint32_t len = load_u32(p + pos);
        pos += 4;
        if (len == 0 || len > max_seq) return io_error("invalid sequence length in input");
        if ((size - pos) / 4 < len) return io_error("truncated input");
        pos += std::size_t(len) * 4;
        total += len;
    }
    if (seq_lens != nullptr) {
        if (seq_lens_cap < batch || ids_cap < total)
            return b2::set_error(B2_ERR_INVALID_ARGUMENT, "read_inputs: seq_lens or ids buffer too small");
        pos = 8;
        std::size_t at = 0;
        for (std::uint32_t b = 0; b < batch; ++b) {
            const std::uint32_t len = load_u32(p + pos);
            std::memcpy(ids + at, p + pos + 4, std::size_t(len) * 4);
            seq_lens[b] = len;
            pos += 4 + std::size_t(len) * 4;
            at += len;
        }
    }
    if (batch_out) *batch_out = batch;
    if (max_seq_out) *max_seq_out = max_seq;
    if (total_out) *total_out = total;
    return B2_OK;
}
