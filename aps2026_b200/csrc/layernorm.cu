// LayerNorm family: plain LN, residual add + LN, and MoE un-permute +
// carried residual add + LN, each one pass over the row.
//
// Reference: k_layer_norm / k_add_layer_norm (src/tensor.cu:2130-2178) with
// ln_stage / ln_moments / ln_write (:2017-2128). There a whole 256-thread
// CTA waits while thread 0 sums the row twice serially from shared memory.
//
// Here (default, tree order) the row lives in registers: THREADS x V float4
// (at h = 4096: 256 x 4 for plain LN, 512 x 2 for the two- and three-input
// forms), loaded with 128-bit streaming loads, mean and variance come from
// two register passes with warp shuffles and one shared slot per warp, and
// the output is written straight from registers -- the row crosses HBM
// exactly once in each direction. CTAs loop over rows (grid = one resident
// wave of the device). Rows too long for registers are staged in shared
// memory by bulk (TMA) copies.
//
// With B2_FLAG_EXACT_ORDER the moments are formed in ascending order exactly
// as ln_serial_sum / ln_serial_var do (var += t * t as a fused
// multiply-add), so the output is bit-identical to the reference: over many
// rows by the chain pipeline (ln_exact_pipe: warps whose lanes run 16 rows'
// chains side by side, fed by a ring of staged chunks), otherwise by one
// thread per row over the row staged in shared memory, with 128-thread CTAs
// keeping more rows resident per SM to overlap those serial chains.
//
// Output: y = fma((x - mean) * inv, gamma, beta), inv = 1 / sqrtf(var / h +
// eps), the reference's ln_write arithmetic (:2043-2047).
#include "rowload.cuh"

namespace b2 {
namespace {

enum LnMode { kLN = 0, kAddLN = 1, kCombineAddLN = 2 };

struct LnArgs {
    const float* x;             // kLN: input; kAddLN: in/out residual stream
    const float* res;           // kAddLN: residual; kCombineAddLN: carry
    const float* gamma;
    const float* beta;
    float* y;                   // normalised output
    float* x_out;               // kAddLN: x (in place); kCombineAddLN: sum
    const float* expert_out;    // kCombineAddLN
    const std::uint8_t* routes;
    const std::uint32_t* route_positions;
    std::size_t expert_rows;
    std::size_t rows;
    std::size_t h;
    float eps;
};

__device__ __forceinline__ float sum4(const float4& v) {
    return __fadd_rn(__fadd_rn(v.x, v.y), __fadd_rn(v.z, v.w));
}

__device__ __forceinline__ float sqdev4(const float4& v, float m) {
    const float a = __fsub_rn(v.x, m), b = __fsub_rn(v.y, m);
    const float c = __fsub_rn(v.z, m), d = __fsub_rn(v.w, m);
    return __fadd_rn(__fmaf_rn(a, a, __fmul_rn(b, b)), __fmaf_rn(c, c, __fmul_rn(d, d)));
}

// the public prologue hook of aps2026_b200_fusion.cuh: a GEMM that forms
// its operand with it matches this kernel's output bit for bit
__device__ __forceinline__ float ln_out(float s, float mean, float inv, float w, float b) {
    return b2_fusion::layer_norm_value(s, mean, inv, w, b);
}

__device__ __forceinline__ float4 ln_out4(const float4& s, float mean, float inv,
                                          const float4& w, const float4& b) {
    return make_float4(ln_out(s.x, mean, inv, w.x, b.x), ln_out(s.y, mean, inv, w.y, b.y),
                       ln_out(s.z, mean, inv, w.z, b.z), ln_out(s.w, mean, inv, w.w, b.w));
}

__device__ __forceinline__ float inv_std(float var_sum, float h, float eps) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(var_sum, h), eps)));
}

// Serial ascending moments over a shared-memory row (ln_serial_sum /
// ln_serial_var / ln_moments, src/tensor.cu:2063-2128), float4 reads for
// latency, the additions in index order.
__device__ __forceinline__ void serial_moments(const float* s, std::size_t h, float eps,
                                               float* mean_out, float* inv_out) {
    float sum = 0.0f;
    std::size_t j = 0;
    if ((h & 15u) == 0) {
        const float4* s4 = reinterpret_cast<const float4*>(s);
        for (std::size_t v = 0; v < h / 4; v += 4) {
            const float4 a = s4[v], b = s4[v + 1], c = s4[v + 2], d = s4[v + 3];
            sum = __fadd_rn(sum, a.x); sum = __fadd_rn(sum, a.y);
            sum = __fadd_rn(sum, a.z); sum = __fadd_rn(sum, a.w);
            sum = __fadd_rn(sum, b.x); sum = __fadd_rn(sum, b.y);
            sum = __fadd_rn(sum, b.z); sum = __fadd_rn(sum, b.w);
            sum = __fadd_rn(sum, c.x); sum = __fadd_rn(sum, c.y);
            sum = __fadd_rn(sum, c.z); sum = __fadd_rn(sum, c.w);
            sum = __fadd_rn(sum, d.x); sum = __fadd_rn(sum, d.y);
            sum = __fadd_rn(sum, d.z); sum = __fadd_rn(sum, d.w);
        }
        j = h;
    }
    for (; j < h; ++j) sum = __fadd_rn(sum, s[j]);
    const float m = __fdiv_rn(sum, static_cast<float>(h));
    float var = 0.0f;
    j = 0;
    if ((h & 15u) == 0) {
        const float4* s4 = reinterpret_cast<const float4*>(s);
        for (std::size_t v = 0; v < h / 4; v += 4) {
            const float4 q[4] = {s4[v], s4[v + 1], s4[v + 2], s4[v + 3]};
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                float t;
                t = __fsub_rn(q[u].x, m); var = __fmaf_rn(t, t, var);
                t = __fsub_rn(q[u].y, m); var = __fmaf_rn(t, t, var);
                t = __fsub_rn(q[u].z, m); var = __fmaf_rn(t, t, var);
                t = __fsub_rn(q[u].w, m); var = __fmaf_rn(t, t, var);
            }
        }
        j = h;
    }
    for (; j < h; ++j) {
        const float t = __fsub_rn(s[j], m);
        var = __fmaf_rn(t, t, var);
    }
    *mean_out = m;
    *inv_out = inv_std(var, static_cast<float>(h), eps);
}

// Produces float4 chunk j of row r of the value to normalise, and writes it
// back to x_out where the mode keeps the sum.
template <int MODE>
__device__ __forceinline__ float4 load_chunk(const LnArgs& a, std::size_t r, std::size_t h4,
                                             std::size_t j, const CombineRows& cr) {
    const std::size_t o = r * h4 + j;
    if (MODE == kLN) return ld_stream(reinterpret_cast<const float4*>(a.x) + o);
    if (MODE == kAddLN)
        return add4(ld_plain(reinterpret_cast<const float4*>(a.x) + o),
                    ld_stream(reinterpret_cast<const float4*>(a.res) + o));
    const float4* e = reinterpret_cast<const float4*>(a.expert_out);
    const float4 lo = cr.lo < a.expert_rows ? ld_stream(e + cr.lo * h4 + j) : zero4();
    const float4 hi = cr.hi < a.expert_rows ? ld_stream(e + cr.hi * h4 + j) : zero4();
    return add4(combine4(lo, hi), ld_stream(reinterpret_cast<const float4*>(a.res) + o));
}

// Register-resident rows: h / 4 <= THREADS * V.
template <int MODE, int THREADS, int V, bool EXACT>
__global__ void __launch_bounds__(THREADS)
ln_rows_reg(LnArgs a) {
    pdl_begin();
    constexpr int WARPS = THREADS / 32;
    __shared__ float red[2][WARPS];
    __shared__ float stats[2];
    extern __shared__ __align__(16) float staged[];  // EXACT only: h floats
    const std::size_t h4 = a.h / 4;
    const float hf = static_cast<float>(a.h);
    const float4* g4 = reinterpret_cast<const float4*>(a.gamma);
    const float4* b4 = reinterpret_cast<const float4*>(a.beta);

    for (std::size_t r = blockIdx.x; r < a.rows; r += gridDim.x) {
        CombineRows cr{0, 0};
        if (MODE == kCombineAddLN) cr = combine_rows(a.routes, a.route_positions, r, a.expert_rows);
        float4 v[V];
#pragma unroll
        for (int k = 0; k < V; ++k) {
            const std::size_t j = threadIdx.x + static_cast<std::size_t>(k) * THREADS;
            v[k] = j < h4 ? load_chunk<MODE>(a, r, h4, j, cr) : zero4();
        }
        if (MODE != kLN) {
#pragma unroll
            for (int k = 0; k < V; ++k) {
                const std::size_t j = threadIdx.x + static_cast<std::size_t>(k) * THREADS;
                if (j < h4) st_plain(reinterpret_cast<float4*>(a.x_out) + r * h4 + j, v[k]);
            }
        }
        float mean, inv;
        if (EXACT) {
            float4* s4 = reinterpret_cast<float4*>(staged);
#pragma unroll
            for (int k = 0; k < V; ++k) {
                const std::size_t j = threadIdx.x + static_cast<std::size_t>(k) * THREADS;
                if (j < h4) s4[j] = v[k];
            }
            __syncthreads();
            if (threadIdx.x == 0) serial_moments(staged, a.h, a.eps, &stats[0], &stats[1]);
            __syncthreads();
            mean = stats[0];
            inv = stats[1];
        } else {
            float part = 0.0f;
#pragma unroll
            for (int k = 0; k < V; ++k) part = __fadd_rn(part, sum4(v[k]));
            mean = __fdiv_rn(block_sum<WARPS>(part, red[0]), hf);
            float part2 = 0.0f;
#pragma unroll
            for (int k = 0; k < V; ++k) {
                const std::size_t j = threadIdx.x + static_cast<std::size_t>(k) * THREADS;
                if (j < h4) part2 = __fadd_rn(part2, sqdev4(v[k], mean));
            }
            inv = inv_std(block_sum<WARPS>(part2, red[1]), hf, a.eps);
        }
#pragma unroll
        for (int k = 0; k < V; ++k) {
            const std::size_t j = threadIdx.x + static_cast<std::size_t>(k) * THREADS;
            if (j < h4)
                st_plain(reinterpret_cast<float4*>(a.y) + r * h4 + j,
                         ln_out4(v[k], mean, inv, __ldg(g4 + j), __ldg(b4 + j)));
        }
    }
}

// Any h / alignment: the row is staged in shared memory (h floats).
template <int MODE, bool EXACT>
__global__ void __launch_bounds__(256)
ln_rows_smem(LnArgs a) {
    pdl_begin();
    constexpr int THREADS = 256, WARPS = 8;
    __shared__ float red[2][WARPS];
    __shared__ float stats[2];
    extern __shared__ __align__(16) float staged[];
    const std::size_t h = a.h;
    const float hf = static_cast<float>(h);
    for (std::size_t r = blockIdx.x; r < a.rows; r += gridDim.x) {
        const std::size_t base = r * h;
        CombineRows cr{0, 0};
        if (MODE == kCombineAddLN) cr = combine_rows(a.routes, a.route_positions, r, a.expert_rows);
        for (std::size_t j = threadIdx.x; j < h; j += THREADS) {
            float s;
            if (MODE == kLN) {
                s = a.x[base + j];
            } else if (MODE == kAddLN) {
                s = __fadd_rn(a.x[base + j], a.res[base + j]);
            } else {
                const float lo = cr.lo < a.expert_rows ? a.expert_out[cr.lo * h + j] : 0.0f;
                const float hi = cr.hi < a.expert_rows ? a.expert_out[cr.hi * h + j] : 0.0f;
                s = __fadd_rn(combine_one(lo, hi), a.res[base + j]);
            }
            if (MODE != kLN) a.x_out[base + j] = s;
            staged[j] = s;
        }
        __syncthreads();
        float mean, inv;
        if (EXACT) {
            if (threadIdx.x == 0) serial_moments(staged, h, a.eps, &stats[0], &stats[1]);
            __syncthreads();
            mean = stats[0];
            inv = stats[1];
        } else {
            float part = 0.0f;
            for (std::size_t j = threadIdx.x; j < h; j += THREADS) part = __fadd_rn(part, staged[j]);
            mean = __fdiv_rn(block_sum<WARPS>(part, red[0]), hf);
            float part2 = 0.0f;
            for (std::size_t j = threadIdx.x; j < h; j += THREADS) {
                const float t = __fsub_rn(staged[j], mean);
                part2 = __fmaf_rn(t, t, part2);
            }
            inv = inv_std(block_sum<WARPS>(part2, red[1]), hf, a.eps);
        }
        for (std::size_t j = threadIdx.x; j < h; j += THREADS)
            a.y[base + j] = ln_out(staged[j], mean, inv, a.gamma[j], a.beta[j]);
        __syncthreads();  // staged[] is rewritten by the next row
    }
}

// Rows too long for registers, h % 4 == 0 and 16-byte aligned: each row's
// inputs (x; x and the residual; or the two expert rows and the carry) are
// staged in shared memory by 1-D bulk (TMA) copies issued by one thread and
// completing on an mbarrier, then reduced and written like ln_rows_smem.
// Copies of an expert row outside expert_out are not issued (the row reads
// as zeros, as in the register path). A wait that does not complete stops the
// CTA and reports B2_CHECK_WAIT.
template <int MODE, bool EXACT>
__global__ void __launch_bounds__(256)
ln_rows_bulk(LnArgs a) {
    pdl_begin();
    constexpr int THREADS = 256, WARPS = 8;
    __shared__ float red[2][WARPS];
    __shared__ float stats[2];
    __shared__ __align__(8) std::uint64_t bar;
    extern __shared__ __align__(128) float in[];  // NIN rows of h floats; in[0..h) becomes the sum
    const std::size_t h = a.h;
    const unsigned bytes = static_cast<unsigned>(h * sizeof(float));
    const float hf = static_cast<float>(h);
    if (threadIdx.x == 0) mbar_init(&bar, 1);
    __syncthreads();
    unsigned parity = 0;
    for (std::size_t r = blockIdx.x; r < a.rows; r += gridDim.x, parity ^= 1u) {
        CombineRows cr{0, 0};
        if (MODE == kCombineAddLN) cr = combine_rows(a.routes, a.route_positions, r, a.expert_rows);
        const bool lo_ok = MODE == kCombineAddLN && cr.lo < a.expert_rows;
        const bool hi_ok = MODE == kCombineAddLN && cr.hi < a.expert_rows;
        if (threadIdx.x == 0) {
            fence_proxy_async_smem();  // the previous row's shared accesses come first
            if (MODE == kLN) {
                mbar_expect_tx(&bar, bytes);
                bulk_g2s(in, a.x + r * h, bytes, &bar);
            } else if (MODE == kAddLN) {
                mbar_expect_tx(&bar, 2 * bytes);
                bulk_g2s(in, a.x + r * h, bytes, &bar);
                bulk_g2s(in + h, a.res + r * h, bytes, &bar);
            } else {
                mbar_expect_tx(&bar, (1u + lo_ok + hi_ok) * bytes);
                bulk_g2s(in, a.res + r * h, bytes, &bar);
                if (lo_ok) bulk_g2s(in + h, a.expert_out + cr.lo * h, bytes, &bar);
                if (hi_ok) bulk_g2s(in + 2 * h, a.expert_out + cr.hi * h, bytes, &bar);
            }
        }
        if (__syncthreads_or(!mbar_wait(&bar, parity))) {  // a copy never landed: stop, report
            if (threadIdx.x == 0) {
                flag_check(B2_CHECK_WAIT);
                // One more bounded wait for the copies in flight. A global ->
                // shared bulk copy that completes on an mbarrier has no other
                // completion signal (cp.async.bulk.wait_group tracks bulk-group
                // copies only), and an unbounded wait would hang the GPU; if this
                // wait also gives up, the copy engine has stopped, the CTA
                // returns, and B2_CHECK_WAIT tells the host that the context is
                // no longer usable (b2_device_status).
                mbar_wait(&bar, parity);
            }
            return;
        }
        float4* s4 = reinterpret_cast<float4*>(in);
        const std::size_t h4 = h / 4;
        if (MODE != kLN) {
            for (std::size_t j = threadIdx.x; j < h4; j += THREADS) {
                float4 v;
                if (MODE == kAddLN) {
                    v = add4(s4[j], s4[h4 + j]);
                } else {
                    const float4 lo = lo_ok ? s4[h4 + j] : zero4(), hi = hi_ok ? s4[2 * h4 + j] : zero4();
                    v = add4(combine4(lo, hi), s4[j]);
                }
                s4[j] = v;
                st_plain(reinterpret_cast<float4*>(a.x_out) + r * h4 + j, v);
            }
            __syncthreads();
        }
        float mean, inv;
        if (EXACT) {
            if (threadIdx.x == 0) serial_moments(in, h, a.eps, &stats[0], &stats[1]);
            __syncthreads();
            mean = stats[0];
            inv = stats[1];
        } else {
            float part = 0.0f;
            for (std::size_t j = threadIdx.x; j < h4; j += THREADS) part = __fadd_rn(part, sum4(s4[j]));
            mean = __fdiv_rn(block_sum<WARPS>(part, red[0]), hf);
            float part2 = 0.0f;
            for (std::size_t j = threadIdx.x; j < h4; j += THREADS) part2 = __fadd_rn(part2, sqdev4(s4[j], mean));
            inv = inv_std(block_sum<WARPS>(part2, red[1]), hf, a.eps);
        }
        const float4* g4 = reinterpret_cast<const float4*>(a.gamma);
        const float4* b4 = reinterpret_cast<const float4*>(a.beta);
        for (std::size_t j = threadIdx.x; j < h4; j += THREADS)
            st_plain(reinterpret_cast<float4*>(a.y) + r * h4 + j,
                     ln_out4(s4[j], mean, inv, __ldg(g4 + j), __ldg(b4 + j)));
        __syncthreads();  // in[] is refilled for the next row
    }
}

// ---- reference-order LayerNorm of many rows: the chain pipeline ----------------
//
// B2_FLAG_EXACT_ORDER forms the mean and the variance as the reference does
// (ln_serial_sum / ln_serial_var, src/tensor.cu:2063-2128): one ascending
// chain of h dependent additions per row for each, about 17 us of FP32
// latency per row at h = 4096. Over many rows that latency has to overlap
// the HBM traffic, so rows go through a pipeline of persistent CTAs (two per
// SM), in batches of 16 rows and "ticks" of one 128-float chunk of each row:
//
//   compute warps   stage, a ring of shared-memory stages ahead (6 stages
//                   for plain LN, 4 with the residual, 2 with the
//                   un-permute, as many as fit), the pass-A inputs of batch
//                   b (x; x and the residual; or the carry and the two
//                   expert rows), the pass-B tile of batch b - 1 and gamma
//                   and beta, by cp.async (16 bytes a thread; completion
//                   tracked by the stage's mbarrier, so no copy holds
//                   registers); in the add modes they form the row values of
//                   batch b (x + res, or combine + carry) and write them to
//                   x_out (with the un-permute also into a tile for chain
//                   A); and they write y of batch b - 2 from its row values,
//                   loaded into registers two ticks ahead, and the stats
//                   chain B published;
//   chain warp A    lane r adds row r of batch b in ascending order -> mean;
//                   with the residual it forms x + res itself from the
//                   staged inputs (the compute warps' operation, so the same
//                   values; independent of the chain, they fill its issue
//                   slots), with the un-permute it reads the compute warps'
//                   tile (forming combine + carry there would make the
//                   chain warp issue-bound);
//   chain warp B    lane r accumulates (x - mean)^2 of row r of batch b - 1
//                   as a fused multiply-add, ascending -> 1/sqrt(var/h+eps).
//
// The chains take 128 x 4 cycles a tick, less than a tick's HBM time. The
// row values are read once from HBM and twice more (pass B, y), with L2
// priorities that keep them resident for those re-reads. A thread stages,
// reads back and re-reads only its own rows' float4 column, so its writes
// of x_out order its later copies of them. Every wait is bounded; a wait
// that gives up sets a shared abort flag that stops every role, and each
// thread waits for its own copies before the CTA exits. Same operations in
// the same order as serial_moments, so y is bit-identical to the reference.
constexpr int kPipeRows = 16;
constexpr int kPipeChunk = 128;                // floats of a row per tick
constexpr int kPipePitch = kPipeChunk + 4;     // 528 B: lanes' rows start on distinct banks
constexpr int kPipeTile = kPipeRows * kPipePitch;
constexpr int kPipeMaxStages = 8;
constexpr int kPipeComputeWarps = 8;
constexpr int kPipeThreads = 32 * (2 + kPipeComputeWarps);

template <int MODE>
constexpr int pipe_inputs() {
    return MODE == kLN ? 1 : (MODE == kAddLN ? 2 : 3);
}

// Stages of the ring (as many as fit in shared memory; each holds a tick's
// pass-A inputs, pass-B tile and gamma / beta chunk).
// CTAs per SM: a tick's time is set by the chain warps, so two CTAs (twice
// the chains, half the ring each). At 131,072 x 4096 that took 17% (LN),
// 10% (add + LN) and 15% (un-permute) off one CTA with a deeper ring (8, 8
// and 5 stages).
template <int MODE>
constexpr int pipe_ctas_per_sm() {
    return 2;
}

template <int MODE>
constexpr int pipe_stages() {
    return MODE == kLN ? 6 : (MODE == kAddLN ? 4 : 2);
}

// floats of one stage: NIN pass-A tiles, the pass-B tile,
// and gamma | beta of the chunk
template <int MODE>
constexpr int pipe_stage_floats() {
    return (pipe_inputs<MODE>() + 1) * kPipeTile + 2 * kPipeChunk;
}

// Whether chain A reads the stage's pass-A inputs itself (LN, add + LN) or
// a tile of row values the compute warps formed (the un-permute).
template <int MODE>
constexpr bool chain_reads_stage() {
    return MODE != kCombineAddLN;
}

// Dynamic shared memory: the stages, then (un-permute) two tiles of row
// values for chain A.
template <int MODE>
constexpr std::size_t pipe_smem() {
    return (static_cast<std::size_t>(pipe_stages<MODE>()) * pipe_stage_floats<MODE>() +
            (chain_reads_stage<MODE>() ? 0 : 2) * kPipeTile) * sizeof(float);
}

struct PipeShared {
    std::uint64_t full[kPipeMaxStages], empty[kPipeMaxStages];
    std::uint64_t sfull[2], sempty[2];  // compute -> chain A: row-value tiles (un-permute)
    std::uint64_t mfull[2], mempty[2];  // chain A -> chain B: means
    std::uint64_t ifull[2], iempty[2];  // chain B -> compute: mean and 1/std
    float mean_a[2][kPipeRows];
    float mean_o[2][kPipeRows], inv_o[2][kPipeRows];
    int abort;
};

__device__ __forceinline__ bool mbar_try(std::uint64_t* bar, unsigned parity) {
    unsigned done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// Gives up (and stops every role) after kMbarWaitNs of the global timer.
__device__ __forceinline__ bool pipe_stop(volatile int* abort_flag, unsigned long long t0) {
    if (*abort_flag) return true;
    if (global_ns() - t0 > kMbarWaitNs) {
        *abort_flag = 1;
        flag_check(B2_CHECK_WAIT);
        return true;
    }
    return false;
}

// Every lane of the warp waits for the phase; the result is warp-uniform.
__device__ __forceinline__ bool warp_wait(std::uint64_t* bar, unsigned parity, volatile int* abort_flag) {
    const unsigned long long t0 = global_ns();
    for (unsigned i = 0; i < kMbarMaxPolls; ++i) {
        const bool done = mbar_try(bar, parity);
        if (__all_sync(0xffffffffu, done)) return true;
        if ((i & 63u) == 63u) {
            int stop = 0;
            if ((threadIdx.x & 31u) == 0) stop = pipe_stop(abort_flag, t0);
            if (__shfl_sync(0xffffffffu, stop, 0)) return false;
        }
    }
    if ((threadIdx.x & 31u) == 0) *abort_flag = 1;
    return false;
}

__device__ __forceinline__ void warp_arrive(std::uint64_t* bar) {
    __syncwarp();
    if ((threadIdx.x & 31u) == 0) mbar_arrive(bar);
}

// Arrives on the barrier once all of this thread's earlier cp.async copies
// have landed (the arrival is one of the barrier's expected count).
__device__ __forceinline__ void cp_async_arrive(std::uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// L2 eviction priorities: the row values a batch re-reads twice (pass B, y)
// are kept ahead of the data read or written once (the pass-A inputs of the
// add modes, y), so the re-reads find them in L2 at steady state.
__device__ __forceinline__ std::uint64_t l2_keep() {
    std::uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ std::uint64_t l2_stream() {
    std::uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void cp_async16_l2(void* dst, const void* src, std::uint64_t policy) {
    asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;\n" ::"r"(smem_addr(dst)), "l"(src),
                 "l"(policy)
                 : "memory");
}
__device__ __forceinline__ float4 ld_l2(const float4* p, std::uint64_t policy) {
    float4 v;
    asm volatile("ld.global.L2::cache_hint.v4.f32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p), "l"(policy));
    return v;
}
__device__ __forceinline__ void st_l2(float4* p, const float4& v, std::uint64_t policy) {
    asm volatile("st.global.L2::cache_hint.v4.f32 [%0], {%1,%2,%3,%4}, %5;" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w), "l"(policy)
                 : "memory");
}

template <int MODE>
__global__ void __launch_bounds__(kPipeThreads, pipe_ctas_per_sm<MODE>())
ln_exact_pipe(LnArgs a) {
    pdl_begin();
    constexpr int NIN = pipe_inputs<MODE>();
    constexpr int S = pipe_stages<MODE>();
    constexpr int AHEAD = S - 1;  // ticks staged ahead of the one being used
    constexpr int CW = kPipeComputeWarps;
    constexpr int Q = kPipeChunk / 4;  // float4 of a row chunk (one per lane)
    // readers of a stage: the compute warps (gamma / beta, their
    // own pass-A copies), chain B (pass-B tile), chain A (pass-A inputs,
    // unless it reads the compute warps' row values)
    constexpr bool kChainStage = chain_reads_stage<MODE>();
    constexpr unsigned kStageReaders = CW + (kChainStage ? 2u : 1u);
    extern __shared__ __align__(128) float smem[];
    __shared__ PipeShared sh;
    const unsigned tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const std::size_t h = a.h, h4 = h / 4;
    const int NT = static_cast<int>(h / kPipeChunk);
    const std::size_t total_batches = (a.rows + kPipeRows - 1) / kPipeRows;
    const int nb = blockIdx.x < total_batches
                       ? static_cast<int>((total_batches - 1 - blockIdx.x) / gridDim.x + 1)
                       : 0;
    const long long G = static_cast<long long>(nb + 2) * NT;  // ticks, two batches of drain
    volatile int* abort_flag = &sh.abort;

    auto stage_base = [&](int st) { return smem + st * pipe_stage_floats<MODE>(); };
    auto tile_in = [&](int st, int input) { return stage_base(st) + input * kPipeTile; };
    auto tile_b = [&](int st) { return stage_base(st) + NIN * kPipeTile; };
    auto tile_gb = [&](int st) { return stage_base(st) + (NIN + 1) * kPipeTile; };  // gamma | beta
    float* svals = smem + S * pipe_stage_floats<MODE>();  // [2] tiles (un-permute)
    auto row0 = [&](int j) {
        return (static_cast<std::size_t>(blockIdx.x) + static_cast<std::size_t>(j) * gridDim.x) * kPipeRows;
    };
    auto nrows = [&](int j) {
        const std::size_t r = a.rows - row0(j);
        return static_cast<int>(r < static_cast<std::size_t>(kPipeRows) ? r : kPipeRows);
    };
    // the row values passes B and y read: x itself, or the sum written to x_out
    const float* sval = MODE == kLN ? a.x : a.x_out;

    if (tid == 0) {
        for (int i = 0; i < S; ++i) {
            mbar_init(&sh.full[i], 32 * CW);
            mbar_init(&sh.empty[i], kStageReaders);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&sh.sfull[i], CW);
            mbar_init(&sh.sempty[i], 1);
            mbar_init(&sh.mfull[i], 1);
            mbar_init(&sh.mempty[i], 1);
            mbar_init(&sh.ifull[i], 1);
            mbar_init(&sh.iempty[i], CW);
        }
        sh.abort = 0;
    }
    __syncthreads();

    if (warp == 0) {
        // ---- chain A: ascending sums of the row values of batch b ----
        float acc = 0.0f;
        unsigned q = 0;  // row-value tiles so far (un-permute)
        for (long long g = 0; g < G; ++g) {
            const int st = static_cast<int>(g % S);
            const unsigned use = static_cast<unsigned>(g / S);
            const int jb = static_cast<int>(g / NT), c = static_cast<int>(g % NT);
            if (kChainStage && !warp_wait(&sh.full[st], use & 1u, abort_flag)) break;
            if (jb < nb) {
                const float* tile = tile_in(st, 0);
                if (!kChainStage) {
                    if (!warp_wait(&sh.sfull[q & 1u], (q >> 1) & 1u, abort_flag)) break;
                    tile = svals + (q & 1u) * kPipeTile;
                }
                if (static_cast<int>(lane) < nrows(jb)) {
                    const float4* r0 = reinterpret_cast<const float4*>(tile + lane * kPipePitch);
                    const float4* r1 = reinterpret_cast<const float4*>(tile_in(st, NIN > 1 ? 1 : 0) + lane * kPipePitch);
#pragma unroll 8
                    for (int i = 0; i < Q; ++i) {
                        float4 v = r0[i];
                        if (MODE == kAddLN) v = add4(v, r1[i]);  // x + res, as the compute warps form it
                        acc = __fadd_rn(acc, v.x);
                        acc = __fadd_rn(acc, v.y);
                        acc = __fadd_rn(acc, v.z);
                        acc = __fadd_rn(acc, v.w);
                    }
                }
                if (!kChainStage) {
                    warp_arrive(&sh.sempty[q & 1u]);
                    ++q;
                }
                if (c == NT - 1) {
                    const float mean = __fdiv_rn(acc, static_cast<float>(h));
                    acc = 0.0f;
                    if (!warp_wait(&sh.mempty[jb & 1], ((jb >> 1) & 1) ^ 1, abort_flag)) break;
                    if (lane < kPipeRows) sh.mean_a[jb & 1][lane] = mean;
                    warp_arrive(&sh.mfull[jb & 1]);
                }
            }
            if (kChainStage) warp_arrive(&sh.empty[st]);
        }
    } else if (warp == 1) {
        // ---- chain B: ascending sums of squared deviations ----
        float acc = 0.0f, mean = 0.0f;
        for (long long g = 0; g < G; ++g) {
            const int st = static_cast<int>(g % S);
            const unsigned use = static_cast<unsigned>(g / S);
            const int jb = static_cast<int>(g / NT), c = static_cast<int>(g % NT);
            const int j = jb - 1;  // batch in pass B
            if (!warp_wait(&sh.full[st], use & 1u, abort_flag)) break;
            if (j >= 0 && j < nb) {
                if (c == 0) {
                    if (!warp_wait(&sh.mfull[j & 1], (j >> 1) & 1, abort_flag)) break;
                    mean = lane < kPipeRows ? sh.mean_a[j & 1][lane] : 0.0f;
                    warp_arrive(&sh.mempty[j & 1]);
                }
                if (static_cast<int>(lane) < nrows(j)) {
                    const float4* row = reinterpret_cast<const float4*>(tile_b(st) + lane * kPipePitch);
#pragma unroll 8
                    for (int i = 0; i < Q; ++i) {
                        const float4 v = row[i];
                        float t;
                        t = __fsub_rn(v.x, mean); acc = __fmaf_rn(t, t, acc);
                        t = __fsub_rn(v.y, mean); acc = __fmaf_rn(t, t, acc);
                        t = __fsub_rn(v.z, mean); acc = __fmaf_rn(t, t, acc);
                        t = __fsub_rn(v.w, mean); acc = __fmaf_rn(t, t, acc);
                    }
                }
                if (c == NT - 1) {
                    const float inv = inv_std(acc, static_cast<float>(h), a.eps);
                    acc = 0.0f;
                    if (!warp_wait(&sh.iempty[j & 1], ((j >> 1) & 1) ^ 1, abort_flag)) break;
                    if (lane < kPipeRows) {
                        sh.mean_o[j & 1][lane] = mean;
                        sh.inv_o[j & 1][lane] = inv;
                    }
                    warp_arrive(&sh.ifull[j & 1]);
                }
            }
            warp_arrive(&sh.empty[st]);
        }
    } else {
        // ---- compute warps: staging, row values of batch b, y of batch b - 2 ----
        const int cw = static_cast<int>(warp) - 2;  // rows cw and cw + 8 of each tile, float4 column `lane`
        const float4* g4 = reinterpret_cast<const float4*>(a.gamma);
        const float4* b4 = reinterpret_cast<const float4*>(a.beta);
        const float4* sv4 = reinterpret_cast<const float4*>(sval);
        const float4* x4 = reinterpret_cast<const float4*>(a.x);
        const float4* r4 = reinterpret_cast<const float4*>(a.res);
        const float4* e4 = reinterpret_cast<const float4*>(a.expert_out);
        float4* xo4 = reinterpret_cast<float4*>(a.x_out);
        float4* y4 = reinterpret_cast<float4*>(a.y);
        const int o_lane = 4 * static_cast<int>(lane);
        const std::uint64_t keep = l2_keep(), stream = l2_stream();
        // expert rows of this thread's two rows (combine mode): of the batch
        // being staged (is_*), and which of them the batch being formed has (ps_*)
        std::size_t is_lo[2] = {0, 0}, is_hi[2] = {0, 0};
        bool is_lok[2] = {false, false}, is_hok[2] = {false, false};
        bool ps_lok[2] = {false, false}, ps_hok[2] = {false, false};
        auto expert_rows = [&](int j, int k, std::size_t& lo, std::size_t& hi, bool& lok, bool& hok) {
            lok = hok = false;
            if (cw + 8 * k >= nrows(j)) return;
            const std::size_t t = row0(j) + cw + 8 * k;
            const std::uint8_t e0 = __ldg(a.routes + 2 * t), e1 = __ldg(a.routes + 2 * t + 1);
            const std::size_t p0 = __ldg(a.route_positions + 2 * t);
            const std::size_t p1 = __ldg(a.route_positions + 2 * t + 1);
            lo = e0 < e1 ? p0 : p1;
            hi = e0 < e1 ? p1 : p0;
            lok = lo < a.expert_rows;
            hok = hi < a.expert_rows;
        };
        // stages this thread's part of tick t: the pass-A inputs of batch
        // t / NT, the pass-B tile of the batch before (and, warps 0 / 1, the
        // gamma / beta chunk for the y pass of the batch before that)
        auto stage = [&](long long t) -> bool {
            if (t >= G) return true;
            const int st = static_cast<int>(t % S);
            const unsigned use = static_cast<unsigned>(t / S);
            const int jb = static_cast<int>(t / NT), c = static_cast<int>(t % NT);
            if (!warp_wait(&sh.empty[st], (use & 1u) ^ 1u, abort_flag)) return false;
            const std::size_t c4 = static_cast<std::size_t>(c) * Q + lane;
            if (jb < nb) {
                if (MODE == kCombineAddLN && c == 0)
                    for (int k = 0; k < 2; ++k) {
                        expert_rows(jb, k, is_lo[k], is_hi[k], is_lok[k], is_hok[k]);
                        if (lane == 0 && cw + 8 * k < nrows(jb) && (!is_lok[k] || !is_hok[k]))
                            flag_check(B2_CHECK_COMBINE);
                    }
                const int nra = nrows(jb);
                for (int k = 0; k < 2; ++k) {
                    const int r = cw + 8 * k;
                    if (r >= nra) continue;
                    const std::size_t row = row0(jb) + r;
                    const int o = r * kPipePitch + o_lane;
                    if (MODE == kLN) {  // x is the row value: kept for the re-reads
                        cp_async16_l2(tile_in(st, 0) + o, x4 + row * h4 + c4, keep);
                    } else if (MODE == kAddLN) {
                        cp_async16_l2(tile_in(st, 0) + o, x4 + row * h4 + c4, stream);
                        cp_async16_l2(tile_in(st, 1) + o, r4 + row * h4 + c4, stream);
                    } else {
                        cp_async16_l2(tile_in(st, 0) + o, r4 + row * h4 + c4, stream);
                        if (is_lok[k]) cp_async16_l2(tile_in(st, 1) + o, e4 + is_lo[k] * h4 + c4, stream);
                        if (is_hok[k]) cp_async16_l2(tile_in(st, 2) + o, e4 + is_hi[k] * h4 + c4, stream);
                    }
                }
            }
            if (jb >= 1 && jb - 1 < nb) {
                const int nrb = nrows(jb - 1);
                for (int k = 0; k < 2; ++k) {
                    const int r = cw + 8 * k;
                    if (r < nrb)
                        cp_async16_l2(tile_b(st) + r * kPipePitch + o_lane, sv4 + (row0(jb - 1) + r) * h4 + c4,
                                      keep);
                }
            }
            if (jb >= 2 && jb - 2 < nb && cw < 2)
                cp_async16(tile_gb(st) + cw * kPipeChunk + o_lane, (cw == 0 ? g4 : b4) + c4);
            cp_async_arrive(&sh.full[st]);
            return true;
        };
        float m_o[2] = {0.f, 0.f}, i_o[2] = {0.f, 0.f};
        // the y pass's row values (the last read of them), loaded into
        // registers two ticks ahead: tick t's for rows cw + 8k of batch t / NT - 2
        auto yload = [&](long long t, int k) -> float4 {
            const int j = static_cast<int>(t / NT) - 2, cc = static_cast<int>(t % NT);
            if (t >= G || j < 0 || j >= nb || cw + 8 * k >= nrows(j)) return zero4();
            return ld_l2(sv4 + (row0(j) + cw + 8 * k) * h4 + static_cast<std::size_t>(cc) * Q + lane, stream);
        };
        float4 ya[2] = {yload(0, 0), yload(0, 1)}, yb[2] = {yload(1, 0), yload(1, 1)};
        bool ok = true;
        for (int d = 0; d < AHEAD && ok; ++d) ok = stage(d);
        unsigned q = 0;  // row-value tiles so far (un-permute)
        for (long long g = 0; g < G && ok; ++g) {
            const float4 yc[2] = {ya[0], ya[1]};
            ya[0] = yb[0];
            ya[1] = yb[1];
            yb[0] = yload(g + 2, 0);
            yb[1] = yload(g + 2, 1);
            if (!stage(g + AHEAD)) break;
            const int st = static_cast<int>(g % S);
            const unsigned use = static_cast<unsigned>(g / S);
            const int jb = static_cast<int>(g / NT), c = static_cast<int>(g % NT);
            const int jo = jb - 2;  // batch whose y this tick writes
            if (!warp_wait(&sh.full[st], use & 1u, abort_flag)) break;
            if (MODE != kLN && jb < nb) {
                if (MODE == kCombineAddLN && c == 0) {
                    std::size_t lo, hi;
                    for (int k = 0; k < 2; ++k) expert_rows(jb, k, lo, hi, ps_lok[k], ps_hok[k]);
                }
                if (!kChainStage && !warp_wait(&sh.sempty[q & 1u], ((q >> 1) & 1u) ^ 1u, abort_flag)) break;
                float* tile = svals + (q & 1u) * kPipeTile;
                const int nra = nrows(jb);
                const std::size_t c4 = static_cast<std::size_t>(c) * Q + lane;
                for (int k = 0; k < 2; ++k) {
                    const int r = cw + 8 * k;
                    if (r >= nra) continue;
                    const int o = r * kPipePitch + o_lane;
                    const float4 v0 = *reinterpret_cast<const float4*>(tile_in(st, 0) + o);
                    float4 v;
                    if (MODE == kAddLN) {
                        v = add4(v0, *reinterpret_cast<const float4*>(tile_in(st, 1) + o));
                    } else {
                        const float4 lo4 = ps_lok[k] ? *reinterpret_cast<const float4*>(tile_in(st, 1) + o) : zero4();
                        const float4 hi4 = ps_hok[k] ? *reinterpret_cast<const float4*>(tile_in(st, 2) + o) : zero4();
                        v = add4(combine4(lo4, hi4), v0);
                    }
                    st_l2(xo4 + (row0(jb) + r) * h4 + c4, v, keep);
                    if (!kChainStage) *reinterpret_cast<float4*>(tile + o) = v;
                }
                if (!kChainStage) {
                    warp_arrive(&sh.sfull[q & 1u]);
                    ++q;
                }
            }
            if (jo >= 0 && jo < nb) {
                if (c == 0) {
                    if (!warp_wait(&sh.ifull[jo & 1], (jo >> 1) & 1, abort_flag)) break;
                    for (int k = 0; k < 2; ++k) {
                        m_o[k] = sh.mean_o[jo & 1][cw + 8 * k];
                        i_o[k] = sh.inv_o[jo & 1][cw + 8 * k];
                    }
                    warp_arrive(&sh.iempty[jo & 1]);
                }
                const float4 gw = *reinterpret_cast<const float4*>(tile_gb(st) + o_lane);
                const float4 bw = *reinterpret_cast<const float4*>(tile_gb(st) + kPipeChunk + o_lane);
                const std::size_t c4 = static_cast<std::size_t>(c) * Q + lane;
                const int nro = nrows(jo);
                for (int k = 0; k < 2; ++k) {
                    const int r = cw + 8 * k;
                    if (r < nro) st_l2(y4 + (row0(jo) + r) * h4 + c4, ln_out4(yc[k], m_o[k], i_o[k], gw, bw), stream);
                }
            }
            warp_arrive(&sh.empty[st]);
        }
        cp_async_wait_all();  // no copy may land after the CTA has gone
    }
    __syncthreads();
}

// Per-row statistics only (b2_layer_norm_stats): the mean and 1/std every
// LayerNorm kernel here forms, for a GEMM that applies the normalisation in
// its prologue. CTA per row (grid-stride), the row staged in shared memory;
// reference order: thread 0's serial ascending sums (serial_moments, as the
// exact kernels), otherwise a block tree reduction.
template <bool EXACT>
__global__ void __launch_bounds__(128)
ln_row_stats(const float* x, std::size_t rows, std::size_t h, float eps, float* mean_out, float* inv_out) {
    pdl_begin();
    constexpr int THREADS = 128, WARPS = 4;
    __shared__ float red[2][WARPS];
    __shared__ float stats[2];
    extern __shared__ __align__(16) float staged[];
    const float hf = static_cast<float>(h);
    for (std::size_t r = blockIdx.x; r < rows; r += gridDim.x) {
        for (std::size_t j = threadIdx.x; j < h; j += THREADS) staged[j] = x[r * h + j];
        __syncthreads();
        float mean, inv;
        if (EXACT) {
            if (threadIdx.x == 0) serial_moments(staged, h, eps, &stats[0], &stats[1]);
            __syncthreads();
            mean = stats[0];
            inv = stats[1];
        } else {
            float part = 0.0f;
            for (std::size_t j = threadIdx.x; j < h; j += THREADS) part = __fadd_rn(part, staged[j]);
            mean = __fdiv_rn(block_sum<WARPS>(part, red[0]), hf);
            float part2 = 0.0f;
            for (std::size_t j = threadIdx.x; j < h; j += THREADS) {
                const float t = __fsub_rn(staged[j], mean);
                part2 = __fmaf_rn(t, t, part2);
            }
            inv = inv_std(block_sum<WARPS>(part2, red[1]), hf, eps);
        }
        if (threadIdx.x == 0) {
            mean_out[r] = mean;
            inv_out[r] = inv;
        }
        __syncthreads();  // staged[] and stats are reused by the next row
    }
}

constexpr std::size_t kMaxSmemRow = 220 * 1024;  // + static reduction slots <= 227 KB

template <int MODE, int THREADS, int V, bool EXACT>
int launch_reg(const LnArgs& a, cudaStream_t s) {
    const std::size_t smem = EXACT ? a.h * sizeof(float) : 0;
    auto kernel = ln_rows_reg<MODE, THREADS, V, EXACT>;
    if (allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem) != cudaSuccess)
        return launch_result("layer norm: shared memory attribute");
    const unsigned grid = wave_grid(reinterpret_cast<const void*>(kernel), THREADS, smem, a.rows);
    launch_pdl(kernel, grid, THREADS, smem, s, a);
    return B2_OK;
}

template <int MODE>
int launch_exact_pipe(const LnArgs& a, cudaStream_t s) {
    constexpr std::size_t smem = pipe_smem<MODE>();
    auto kernel = ln_exact_pipe<MODE>;
    if (allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem) != cudaSuccess)
        return launch_result("layer norm: shared memory attribute");
    const std::size_t batches = (a.rows + kPipeRows - 1) / kPipeRows;
    const std::size_t ctas = static_cast<std::size_t>(pipe_ctas_per_sm<MODE>()) * sm_count();
    launch_pdl(kernel, static_cast<unsigned>(batches < ctas ? batches : ctas), kPipeThreads, smem, s, a);
    return B2_OK;
}

template <int MODE, bool EXACT>
int launch_bulk(const LnArgs& a, cudaStream_t s) {
    constexpr int NIN = MODE == kLN ? 1 : (MODE == kAddLN ? 2 : 3);
    const std::size_t smem = NIN * a.h * sizeof(float);
    auto kernel = ln_rows_bulk<MODE, EXACT>;
    if (allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem) != cudaSuccess)
        return launch_result("layer norm: shared memory attribute");
    const unsigned grid = wave_grid(reinterpret_cast<const void*>(kernel), 256, smem, a.rows);
    launch_pdl(kernel, grid, 256, smem, s, a);
    return B2_OK;
}

template <int MODE, bool EXACT>
int launch_smem(const LnArgs& a, cudaStream_t s) {
    const std::size_t smem = a.h * sizeof(float);
    auto kernel = ln_rows_smem<MODE, EXACT>;
    if (allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem) != cudaSuccess)
        return launch_result("layer norm: shared memory attribute");
    const unsigned grid = wave_grid(reinterpret_cast<const void*>(kernel), 256, smem, a.rows);
    launch_pdl(kernel, grid, 256, smem, s, a);
    return B2_OK;
}

// Picks, in reference order over enough rows (h a multiple of 128, aligned),
// the chain pipeline; otherwise the register-resident variant whose
// THREADS * V covers h / 4, else bulk-copy staging (aligned rows,
// h % 4 == 0), else the scalar shared-memory one. From one 16-row batch per
// SM the pipeline beats the per-row kernels (at 6,144 and 8,192 rows by
// 15% / 24% with the residual, 8% / 19% with the un-permute; they tie at
// 2,048).
constexpr int kPipeMinBatchesPerSm = 1;
template <int MODE>
int dispatch(const LnArgs& a, bool exact, bool vec_ok, cudaStream_t s, const char* what) {
    if (a.h * sizeof(float) > kMaxSmemRow && exact)
        return set_error(B2_ERR_UNSUPPORTED, std::string(what) + ": h too large");
    int rc = B2_OK;
    const std::size_t h4 = a.h / 4;
    // (h >= pipe_stages chunks in the add modes: a thread's copies of the
    // x_out chunks it wrote are then staged after it wrote them)
    if (vec_ok && exact && a.h % kPipeChunk == 0 &&
        a.h >= static_cast<std::size_t>(MODE == kLN ? 1 : pipe_stages<MODE>()) * kPipeChunk &&
        a.rows >= static_cast<std::size_t>(kPipeMinBatchesPerSm) * kPipeRows * sm_count()) {
        rc = launch_exact_pipe<MODE>(a, s);  // a 16-row batch or more per SM
    } else if (vec_ok && !exact && h4 <= 256 * 8) {
        if (h4 <= 256) rc = launch_reg<MODE, 256, 1, false>(a, s);
        else if (h4 <= 512) rc = launch_reg<MODE, 256, 2, false>(a, s);
        // (at h = 4096 the two- and three-input forms run at 99% of the HBM
        // copy rate as 512 x 2 against 94-96% as 256 x 4; plain LN is 10%
        // slower as 512 x 2)
        else if (h4 <= 1024) rc = MODE != kLN ? launch_reg<MODE, 512, 2, false>(a, s)
                                              : launch_reg<MODE, 256, 4, false>(a, s);
        else rc = launch_reg<MODE, 256, 8, false>(a, s);
    } else if (vec_ok && exact && h4 <= 128 * 8) {
        if (h4 <= 128) rc = launch_reg<MODE, 128, 1, true>(a, s);
        else if (h4 <= 256) rc = launch_reg<MODE, 128, 2, true>(a, s);
        else if (h4 <= 512) rc = launch_reg<MODE, 128, 4, true>(a, s);
        else rc = launch_reg<MODE, 128, 8, true>(a, s);
    } else if (vec_ok && (MODE == kLN ? 1 : MODE == kAddLN ? 2 : 3) * a.h * sizeof(float) <= kMaxSmemRow) {
        rc = exact ? launch_bulk<MODE, true>(a, s) : launch_bulk<MODE, false>(a, s);
    } else {
        if (a.h * sizeof(float) > kMaxSmemRow)
            return set_error(B2_ERR_UNSUPPORTED, std::string(what) + ": h too large");
        rc = exact ? launch_smem<MODE, true>(a, s) : launch_smem<MODE, false>(a, s);
    }
    if (rc != B2_OK) return rc;
    return launch_result(what);
}

bool all_aligned(std::initializer_list<const void*> ps) {
    for (const void* p : ps)
        if (p && !aligned16(p)) return false;
    return true;
}

}  // namespace
}  // namespace b2

B2_DEFINE_CHECK_TAKER(layernorm)

extern "C" {

int b2_layer_norm(const float* x, const float* gamma, const float* beta, float* y,
                  size_t rows, size_t h, float eps, uint32_t flags, b2_stream_t stream) {
    using namespace b2;
    if (rows == 0) return B2_OK;
    if (!x || !gamma || !beta || !y) return invalid("layer norm: null pointer");
    if (h == 0) return invalid("layer norm shape");
    LnArgs a{};
    a.x = x; a.gamma = gamma; a.beta = beta; a.y = y;
    a.rows = rows; a.h = h; a.eps = eps;
    const bool vec = (h & 3u) == 0 && all_aligned({x, gamma, beta, y});
    return dispatch<kLN>(a, (flags & B2_FLAG_EXACT_ORDER) != 0, vec, as_stream(stream),
                         "b2_layer_norm");
}

int b2_layer_norm_stats(const float* x, size_t rows, size_t h, float eps, uint32_t flags, float* mean,
                        float* inv, b2_stream_t stream) {
    using namespace b2;
    if (rows == 0) return B2_OK;
    if (!x || !mean || !inv) return invalid("layer norm stats: null pointer");
    if (h == 0) return invalid("layer norm stats shape");
    const std::size_t smem = h * sizeof(float);
    if (smem > kMaxSmemRow) return set_error(B2_ERR_UNSUPPORTED, "b2_layer_norm_stats: h too large");
    const bool exact = (flags & B2_FLAG_EXACT_ORDER) != 0;
    auto kernel = exact ? ln_row_stats<true> : ln_row_stats<false>;
    if (allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem) != cudaSuccess)
        return launch_result("b2_layer_norm_stats: shared memory attribute");
    const unsigned grid = wave_grid(reinterpret_cast<const void*>(kernel), 128, smem, rows);
    launch_pdl(kernel, grid, 128, smem, as_stream(stream), x, rows, h, eps, mean, inv);
    return launch_result("b2_layer_norm_stats");
}

int b2_add_layer_norm(float* x, const float* residual, const float* gamma, const float* beta,
                      float* y, size_t rows, size_t h, float eps, uint32_t flags,
                      b2_stream_t stream) {
    using namespace b2;
    if (rows == 0) return B2_OK;
    if (!x || !residual || !gamma || !beta || !y) return invalid("add layer norm: null pointer");
    if (h == 0) return invalid("add layer norm shape");
    LnArgs a{};
    a.x = x; a.res = residual; a.gamma = gamma; a.beta = beta; a.y = y; a.x_out = x;
    a.rows = rows; a.h = h; a.eps = eps;
    const bool vec = (h & 3u) == 0 && all_aligned({x, residual, gamma, beta, y});
    return dispatch<kAddLN>(a, (flags & B2_FLAG_EXACT_ORDER) != 0, vec, as_stream(stream),
                            "b2_add_layer_norm");
}

int b2_moe_combine_add_layer_norm(const float* expert_out, size_t expert_rows,
                                  const uint8_t* routes, const uint32_t* route_positions,
                                  const float* carry, const float* gamma, const float* beta,
                                  float* x_out, float* y, size_t rows, size_t h, float eps,
                                  uint32_t flags, b2_stream_t stream) {
    using namespace b2;
    if (rows == 0) return B2_OK;
    if (!expert_out || !routes || !route_positions || !carry || !gamma || !beta || !x_out || !y)
        return invalid("combine add layer norm: null pointer");
    if (h == 0) return invalid("combine add layer norm shape");
    LnArgs a{};
    a.res = carry; a.gamma = gamma; a.beta = beta; a.y = y; a.x_out = x_out;
    a.expert_out = expert_out; a.routes = routes; a.route_positions = route_positions;
    a.expert_rows = expert_rows; a.rows = rows; a.h = h; a.eps = eps;
    const bool vec = (h & 3u) == 0 && all_aligned({expert_out, carry, gamma, beta, x_out, y});
    return dispatch<kCombineAddLN>(a, (flags & B2_FLAG_EXACT_ORDER) != 0, vec,
                                   as_stream(stream), "b2_moe_combine_add_layer_norm");
}

}  // extern "C"
