// Shared helpers of the aps2026_b200 kernels: status reporting, 128-bit
// global memory access, block reductions and launch geometry for sm_100a.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/aps2026_b200.h"
#include "../../include/aps2026_b200_fusion.cuh"

namespace b2 {

// ---- host-side status -------------------------------------------------------

// Records the calling thread's last failure message; returns `code`.
int set_error(int code, const std::string& message);

inline int invalid(const std::string& message) {
    return set_error(B2_ERR_INVALID_ARGUMENT, message);
}

// Converts the launch status of the kernels just enqueued into a b2 status.
inline int launch_result(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return set_error(B2_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    return B2_OK;
}

inline cudaStream_t as_stream(b2_stream_t s) { return static_cast<cudaStream_t>(s); }

__host__ __device__ inline bool aligned16(const void* p) {
    return (reinterpret_cast<std::uintptr_t>(p) & 15u) == 0;
}

// Number of SMs of the current device (148 on B200), cached per device.
int sm_count();

// Stream-ordered device scratch of `bytes`: from a memory pool of this
// library on the current device that keeps its memory reserved between
// calls (so a repeated call does not go back to the driver), or, while
// `stream` is being captured, a graph allocation (cudaMallocAsync). Free it
// with cudaFreeAsync on the same stream.
cudaError_t scratch_alloc(void** p, std::size_t bytes, cudaStream_t stream);

// Gated SiLU launch (moe.cu) with the exponential mode chosen by the caller:
// b2_silu_mul passes exact = true (bit-exact always); b2_silu_mul_flags and
// b2_prefill_layers the mode of their flags.
int silu_mul_launch(const float* gate, std::size_t ld_gate, const float* up, std::size_t ld_up, float* out,
                    std::size_t ld_out, std::size_t rows, std::size_t cols, bool exact, b2_stream_t stream);

// Resident CTAs per SM for `kernel` at `threads` threads and `smem` bytes of
// dynamic shared memory on the current device.
int resident_ctas(const void* kernel, int threads, std::size_t smem);

// Grid for a grid-stride loop over `units`: at most the number of CTAs that
// are resident at once (one full wave), at least 1.
inline unsigned wave_grid(const void* kernel, int threads, std::size_t smem,
                          std::size_t units) {
    const std::size_t wave =
        static_cast<std::size_t>(sm_count()) * static_cast<std::size_t>(resident_ctas(kernel, threads, smem));
    std::size_t g = units < wave ? units : wave;
    if (g == 0) g = 1;
    return static_cast<unsigned>(g);
}

// Allows `kernel` to launch with `bytes` of dynamic shared memory: above the
// 48 KB default (static shared memory counts against it too) the opt-in
// attribute must be raised first.
inline cudaError_t allow_dynamic_smem(const void* kernel, std::size_t bytes) {
    if (bytes <= 40 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(bytes));
}

// ---- programmatic dependent launch ---------------------------------------------
//
// Every kernel is launched with programmatic stream serialization: its CTAs
// may be scheduled while the previous kernel on the stream drains, which
// hides the launch gap and the previous grid's tail. pdl_begin() is the
// first statement of every kernel: it waits until the previous grid has
// completed and its writes are visible (griddepcontrol.wait -- a hardware
// dependency, not a spin), then lets the next kernel start its own launch.
// When the previous kernel was not launched this way (or there is none),
// the wait returns at once.
__device__ __forceinline__ void pdl_begin() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, std::size_t smem, cudaStream_t s,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---- asynchronous global -> shared copies ------------------------------------
//
// cp.async: the copy holds no registers while in flight; a thread's copies
// are complete (and visible to that thread) after cp_async_wait<N>() leaves at
// most N of its committed groups pending; other threads see them after a
// barrier.
__device__ __forceinline__ void cp_async4(float* dst, const float* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(
                     static_cast<unsigned>(__cvta_generic_to_shared(dst))), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(
                     static_cast<unsigned>(__cvta_generic_to_shared(dst))), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// ---- packed FP32 pairs (sm_100 fma.rn.f32x2) ------------------------------------
//
// Two independent round-to-nearest FMAs in one instruction: lane k of the
// result is fma(a_k, b_k, c_k) exactly as __fmaf_rn computes it, so chains
// kept in the two lanes keep their own order.
__device__ __forceinline__ unsigned long long f2_pack(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 f2_unpack(unsigned long long v) {
    float2 r;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
    return r;
}
__device__ __forceinline__ unsigned long long f2_fma(unsigned long long a, unsigned long long b,
                                                     unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// ---- bulk (TMA) copies completing on an mbarrier ------------------------------
//
// One thread arms the CTA's barrier with the byte count of a phase and issues
// 1-D bulk copies global -> shared (no multicast); every thread then waits
// for the phase with mbar_wait, which gives up after kMbarWaitNs of the
// global timer (or kMbarMaxPolls polls) so no wait can hang the GPU.
constexpr unsigned kMbarMaxPolls = 1u << 26;
constexpr unsigned long long kMbarWaitNs = 1000000000ull;  // 1 s

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned smem_addr(const void* p) {
    return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(std::uint64_t* bar, unsigned arrivals) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(arrivals) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(std::uint64_t* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
// Orders this thread's earlier generic accesses to shared memory before
// later async-proxy (bulk copy) writes to it.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, std::uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}
// Completes the barrier's phase with no bytes expected (a slot whose copy
// was skipped keeps its phase count in step).
__device__ __forceinline__ void mbar_arrive(std::uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// 1-D bulk copy shared -> global, in this thread's current bulk group.
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, unsigned bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_addr(src)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until at most N of this thread's bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Waits until at most N of this thread's bulk groups are incomplete.
template <int N>
__device__ __forceinline__ void bulk_wait() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// Waits for the barrier phase of parity `parity`; false if it did not
// complete within `limit_ns` (or kMbarMaxPolls polls).
__device__ __forceinline__ bool mbar_wait(std::uint64_t* bar, unsigned parity,
                                          unsigned long long limit_ns = kMbarWaitNs) {
    const unsigned long long t0 = global_ns();
    for (unsigned i = 0; i < kMbarMaxPolls; ++i) {
        unsigned done;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
            : "=r"(done)
            : "r"(smem_addr(bar)), "r"(parity)
            : "memory");
        if (done) return true;
        if ((i & 255u) == 255u && global_ns() - t0 > limit_ns) return false;
    }
    return false;
}

// ---- in-kernel bounds checks -------------------------------------------------
//
// Every kernel that dereferences a caller-provided index checks it, skips
// the access when it is out of range, and ORs a B2_CHECK_* bit into this
// per-translation-unit word, which b2_device_status() collects and clears.
// No kernel traps or asserts.
static __device__ unsigned int g_check_word;

__device__ __forceinline__ void flag_check(unsigned int bit) {
    atomicOr(&g_check_word, bit);
}

// Host side of the per-TU word: adds its value to *acc and clears it.
inline int take_check_word(cudaStream_t stream, unsigned int* acc) {
    unsigned int v = 0;
    cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_check_word, sizeof(v), 0,
                                              cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess && v != 0) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbolAsync(g_check_word, &zero, sizeof(zero), 0,
                                    cudaMemcpyHostToDevice, stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    }
    if (e != cudaSuccess)
        return set_error(B2_ERR_CUDA, std::string("b2_device_status: ") + cudaGetErrorString(e));
    *acc |= v;
    return B2_OK;
}

// ---- 128-bit global access ----------------------------------------------------

// Streaming read of data this kernel reads once (read-only path, no L1
// allocation).
__device__ __forceinline__ float4 ld_stream(const float4* p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

// Plain coherent read, for operands the same kernel also writes (in-place
// x of add-LN, q/k of RoPE), which must not take the read-only path.
__device__ __forceinline__ float4 ld_plain(const float4* p) {
    float4 v;
    asm volatile("ld.global.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void st_plain(float4* p, const float4& v) {
    asm volatile("st.global.v4.f32 [%0], {%1,%2,%3,%4};"
                 :
                 : "l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

// ---- reductions ------------------------------------------------------------------

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum of one value per thread, returned to every thread.
// `scratch` holds at least WARPS floats; consecutive calls must alternate
// scratch buffers (or be separated by a barrier) so a fast warp cannot
// overwrite a slot a slow warp is still reading.
template <int WARPS>
__device__ __forceinline__ float block_sum(float v, float* scratch) {
    v = warp_sum(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = lane < WARPS ? scratch[lane] : 0.0f;
    return warp_sum(t);
}

template <int WARPS>
__device__ __forceinline__ float block_max(float v, float* scratch) {
    v = warp_max(v);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = lane < WARPS ? scratch[lane] : -3.402823466e+38F;
    return warp_max(t);
}

}  // namespace b2

// Per-TU status collector registration: each .cu that has kernels with bounds
// checks defines one of these, and b2_device_status calls them all.
#define B2_DEFINE_CHECK_TAKER(name)                                              \
    namespace b2 {                                                               \
    int take_check_##name(cudaStream_t stream, unsigned int* acc) {              \
        return take_check_word(stream, acc);                                     \
    }                                                                            \
    }
