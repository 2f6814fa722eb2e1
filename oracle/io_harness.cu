// TEST INFRASTRUCTURE ONLY: the reference harness's own prompt-file reader
// and output-file writer (src/main.cpp:144-192) behind C entry points, for
// checking b2_read_inputs / b2_write_outputs against them.
//
// oracle/Makefile compiles this file against the reference tree where it
// lies: src/main.cpp is included as it is, with its `main` renamed so the
// library has no entry point of its own, and linked with the reference's
// model objects that main.cpp refers to. read_inputs and write_outputs are
// `static` there, so only code in this translation unit can call them.
// Both work on host memory only (write_outputs reads Tensor::data, which
// never touches a GPU for a host tensor), so this library runs on a machine
// without one.
//
// Status: 0 ok, 2 an exception (message from io_ref_error()).
#define main aps2026_ref_cli_main_unused
#include "main.cpp"
#undef main

#include <cstring>

namespace {
thread_local std::string g_io_error;
}

extern "C" const char* io_ref_error() { return g_io_error.c_str(); }

// write_outputs(path, logits) of a host [batch, vocab] tensor holding `logits`.
extern "C" int io_ref_write_outputs(const char* path, const float* logits, std::size_t batch,
                                    std::size_t vocab) {
    try {
        Tensor t({batch, vocab});
        if (batch * vocab) std::memcpy(t.data(), logits, batch * vocab * sizeof(float));
        write_outputs(path, t);
        return 0;
    } catch (const std::exception& e) {
        g_io_error = e.what();
        return 2;
    }
}

// read_inputs(path, max_seq_len); the prompts packed into ids (capacity
// ids_cap) and their lengths into seq_lens (capacity lens_cap).
extern "C" int io_ref_read_inputs(const char* path, std::uint32_t* batch, std::uint32_t* max_seq,
                                  std::size_t* total, std::uint32_t* seq_lens, std::size_t lens_cap,
                                  std::int32_t* ids, std::size_t ids_cap) {
    try {
        std::size_t max_seq_len = 0;
        const std::vector<std::vector<int>> rows = read_inputs(path, max_seq_len);
        std::size_t at = 0;
        for (std::size_t b = 0; b < rows.size(); ++b) {
            if (b < lens_cap) seq_lens[b] = static_cast<std::uint32_t>(rows[b].size());
            for (int t : rows[b]) {
                if (at < ids_cap) ids[at] = t;
                ++at;
            }
        }
        *batch = static_cast<std::uint32_t>(rows.size());
        *max_seq = static_cast<std::uint32_t>(max_seq_len);
        *total = at;
        return 0;
    } catch (const std::exception& e) {
        g_io_error = e.what();
        return 2;
    }
}
