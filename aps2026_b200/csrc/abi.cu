// Library-level entry points of the C ABI: version, error messages, the
// per-device check word, and cached device properties used for grid sizing.
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace b2 {

namespace {
thread_local std::string t_last_error;

struct DeviceInfo {
    int sms = 0;
};
std::mutex g_info_mutex;
std::vector<DeviceInfo> g_info;
}  // namespace

int set_error(int code, const std::string& message) {
    t_last_error = message;
    return code;
}

int sm_count() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    std::lock_guard<std::mutex> lock(g_info_mutex);
    if (static_cast<std::size_t>(dev) >= g_info.size()) g_info.resize(dev + 1);
    DeviceInfo& info = g_info[dev];
    if (info.sms == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
            n = 148;
        info.sms = n;
    }
    return info.sms;
}

int resident_ctas(const void* kernel, int threads, std::size_t smem) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = 1;
    }
    return n;
}

int take_check_gather(cudaStream_t, unsigned int*);
int take_check_layernorm(cudaStream_t, unsigned int*);
int take_check_rope(cudaStream_t, unsigned int*);
int take_check_moe(cudaStream_t, unsigned int*);
int take_check_attention(cudaStream_t, unsigned int*);
int take_check_trie(cudaStream_t, unsigned int*);
int take_check_selfcheck(cudaStream_t, unsigned int*);

}  // namespace b2

extern "C" {

const char* b2_version(void) { return "aps2026_b200 0.1.0 sm_100a"; }

const char* b2_last_error(void) { return b2::t_last_error.c_str(); }

int b2_device_status(uint32_t* status_out, b2_stream_t stream) {
    if (!status_out) return b2::invalid("b2_device_status: null status_out");
    cudaStream_t s = b2::as_stream(stream);
    unsigned int acc = 0;
    int rc;
    if ((rc = b2::take_check_gather(s, &acc)) != B2_OK) return rc;
    if ((rc = b2::take_check_layernorm(s, &acc)) != B2_OK) return rc;
    if ((rc = b2::take_check_rope(s, &acc)) != B2_OK) return rc;
    if ((rc = b2::take_check_moe(s, &acc)) != B2_OK) return rc;
    if ((rc = b2::take_check_attention(s, &acc)) != B2_OK) return rc;
    if ((rc = b2::take_check_trie(s, &acc)) != B2_OK) return rc;
    if ((rc = b2::take_check_selfcheck(s, &acc)) != B2_OK) return rc;
    *status_out = acc;
    return B2_OK;
}

}  // extern "C"
