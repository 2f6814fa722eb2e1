// Exhaustive self-check of the table-driven exponential (fastexp.cuh)
// against CUDA's exp(double) over every float in a range.
#include "fastexp.cuh"
#include "common.cuh"

namespace b2 {
namespace {

struct Counters {
    unsigned long long checked, mismatches, slow;
};

// Every float whose bit pattern lies in [lo, hi) (hi exclusive), grid-strided.
__global__ void __launch_bounds__(256)
exp_selfcheck(unsigned lo, unsigned hi, Counters* out) {
    __shared__ double tab[64];
    load_exp2_table(tab);
    __syncthreads();
    unsigned long long checked = 0, bad = 0, slow = 0;
    const unsigned long long n = static_cast<unsigned long long>(hi) - lo;
    for (unsigned long long i = static_cast<unsigned long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<unsigned long long>(gridDim.x) * blockDim.x) {
        const float x = __uint_as_float(lo + static_cast<unsigned>(i));
        bool s = false;
        const float f = exp_ref(x, tab, &s);
        const float r = exp_ref_slow(x);
        checked += 1;
        bad += __float_as_uint(f) != __float_as_uint(r);
        slow += s;
    }
    atomicAdd(&out->checked, checked);
    atomicAdd(&out->mismatches, bad);
    atomicAdd(&out->slow, slow);
}

// A barrier armed for 16 bytes that no copy delivers: every wait on it must
// give up within `limit_ns` and report B2_CHECK_WAIT (the bounded-wait path
// of the bulk-copy kernels, exercised without any copy in flight).
__global__ void __launch_bounds__(32)
wait_selfcheck(unsigned long long limit_ns) {
    __shared__ __align__(8) std::uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_expect_tx(&bar, 16);
    }
    __syncwarp();
    const bool ok = mbar_wait(&bar, 0, limit_ns);
    if (!ok && threadIdx.x == 0) flag_check(B2_CHECK_WAIT);
}

}  // namespace
}  // namespace b2

B2_DEFINE_CHECK_TAKER(selfcheck)

extern "C" int b2_selfcheck_wait(uint64_t limit_ns) {
    using namespace b2;
    if (limit_ns == 0 || limit_ns > 10000000000ull) return invalid("b2_selfcheck_wait: limit_ns out of (0, 10 s]");
    wait_selfcheck<<<1, 32>>>(limit_ns);
    return launch_result("b2_selfcheck_wait");
}

extern "C" int b2_selfcheck_exp(uint32_t lo_bits, uint32_t hi_bits, uint64_t* checked, uint64_t* mismatches,
                                uint64_t* slow_path) {
    using namespace b2;
    if (!checked || !mismatches || !slow_path) return invalid("b2_selfcheck_exp: null pointer");
    if (hi_bits < lo_bits) return invalid("b2_selfcheck_exp: hi_bits < lo_bits");
    Counters* d = nullptr;
    cudaError_t e = cudaMalloc(&d, sizeof(Counters));
    if (e == cudaSuccess) e = cudaMemset(d, 0, sizeof(Counters));
    if (e == cudaSuccess) {
        exp_selfcheck<<<sm_count() * 8, 256>>>(lo_bits, hi_bits, d);
        e = cudaGetLastError();
    }
    Counters h{};
    if (e == cudaSuccess) e = cudaMemcpy(&h, d, sizeof(h), cudaMemcpyDeviceToHost);
    if (d) cudaFree(d);
    if (e != cudaSuccess) return set_error(B2_ERR_CUDA, std::string("b2_selfcheck_exp: ") + cudaGetErrorString(e));
    *checked = h.checked;
    *mismatches = h.mismatches;
    *slow_path = h.slow;
    return B2_OK;
}
