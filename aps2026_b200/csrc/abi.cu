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
    cudaMemPool_t scratch = nullptr;  // scratch_alloc's pool on this device
};

cudaError_t make_scratch_pool(int dev, cudaMemPool_t* pool) {
    cudaMemPoolProps props{};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaError_t e = cudaMemPoolCreate(pool, &props);
    if (e != cudaSuccess) return e;
    std::uint64_t keep = ~std::uint64_t(0);  // never trim at synchronisation points
    return cudaMemPoolSetAttribute(*pool, cudaMemPoolAttrReleaseThreshold, &keep);
}
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

cudaError_t scratch_alloc(void** p, std::size_t bytes, cudaStream_t stream) {
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &capture) != cudaSuccess) {
        cudaGetLastError();
        capture = cudaStreamCaptureStatusNone;
    }
    if (capture != cudaStreamCaptureStatusNone) return cudaMallocAsync(p, bytes, stream);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(g_info_mutex);
    if (static_cast<std::size_t>(dev) >= g_info.size()) g_info.resize(dev + 1);
    DeviceInfo& info = g_info[dev];
    for (int attempt = 0; attempt < 2; ++attempt) {
        if (!info.scratch && (e = make_scratch_pool(dev, &info.scratch)) != cudaSuccess) {
            info.scratch = nullptr;
            return e;
        }
        e = cudaMallocFromPoolAsync(p, bytes, info.scratch, stream);
        if (e == cudaSuccess || e == cudaErrorMemoryAllocation) return e;
        cudaGetLastError();  // a pool of an earlier context (device reset): make a new one
        info.scratch = nullptr;
    }
    return e;
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
