// MoE routing (top-2 selection + stable token->expert permutation), gated
// SiLU, weighted un-permute, and the plain residual add.
//
// Routing reference (src/tensor.cu): k_moe_top2 (:1293-1331) picks experts
// and bumps 16 global atomics per token pair; k_moe_offsets_work
// (:1337-1374) scans the counts on ONE thread and fills the work queues;
// k_moe_fill_stable (:1376-1418) runs 16 CTAs, each scanning ALL T tokens
// for its expert -- 16x the routes traffic on 16 of 148 SMs.
//
// Here the same outputs come from two launches over 256-token tiles, with
// no serial step and no waiting between CTAs:
//   1. route_select: per token the quantized scores and the scan-order
//      top-2 pick (same float operations and comparisons as k_moe_top2);
//      per tile an expert histogram (shared-memory atomics) written to the
//      workspace.
//   2. route_scatter: every CTA reads the whole histogram table from L2
//      (128-bit loads, E padded to a power of two >= 4) and forms, per
//      expert, the total and the count in tiles before its own -- so
//      offsets and its tile base need no global scan pass; warp ballots then
//      give each token's stable rank among the tile's tokens of the same
//      expert, and rank + tile base + expert offset is the position written
//      to assignment_rows and route_positions. CTA 0 writes counts/offsets;
//      all CTAs together write the two work queues.
// Token order within an expert is ascending, exactly what
// k_moe_fill_stable produces; all integer outputs are bit-identical.
#include <string>

#include "fastexp.cuh"
#include "rowload.cuh"

namespace b2 {
namespace {

constexpr int kTile = 256;          // tokens per routing tile = threads per CTA
constexpr int kMaxExperts = 32;

// Histogram row stride: E rounded up to a power of two >= 4, so a tile's
// counts are whole 16-byte vectors.
inline unsigned padded_experts(std::size_t E) {
    unsigned p = 4;
    while (p < E) p <<= 1;
    return p;
}

struct RouteArgs {
    const float* logits;
    std::size_t T, E;
    unsigned EP;                 // padded_experts(E)
    float quantum, tie_eps;
    std::uint8_t* routes;
    std::uint32_t* counts;
    std::uint32_t* offsets;
    std::uint32_t* assignment_rows;
    std::uint32_t* route_positions;
    std::uint32_t* we64;
    std::uint32_t* ws64;
    std::uint32_t* we128;
    std::uint32_t* ws128;
    std::uint32_t* tile_counts;  // [tiles][EP]
    std::size_t tiles;
};

// sign(s) * floorf(|s| / quantum + 0.5f) * quantum, the reference's
// canonicalisation (src/tensor.cu:1301-1305), with every operation rounded
// separately (no contraction is possible in the reference expression).
__device__ __forceinline__ float quantize(float s, float quantum) {
    const float r = __fmul_rn(floorf(__fadd_rn(__fdiv_rn(fabsf(s), quantum), 0.5f)), quantum);
    return s < 0.0f ? -r : r;
}

// The two experts of token t, first | second << 8, as k_moe_top2 picks
// them (src/tensor.cu:1299-1328): the first scan takes an expert when its
// quantized score beats the best so far by more than tie_eps, the second
// scan does the same skipping the first pick; also stored to routes[t].
__device__ __forceinline__ unsigned pick_top2(const RouteArgs& a, std::size_t t) {
    const unsigned E = static_cast<unsigned>(a.E);
    float sc[kMaxExperts];
    const float* row = a.logits + t * a.E;
    if ((E & 3u) == 0 && aligned16(row)) {
#pragma unroll
        for (unsigned e = 0; e < kMaxExperts; e += 4)
            if (e < E) {
                const float4 v = ld_stream(reinterpret_cast<const float4*>(row + e));
                sc[e] = v.x; sc[e + 1] = v.y; sc[e + 2] = v.z; sc[e + 3] = v.w;
            }
    } else {
#pragma unroll
        for (unsigned e = 0; e < kMaxExperts; ++e)
            if (e < E) sc[e] = __ldg(row + e);
    }
    int first = -1;
    float first_value = -3.402823466e+38F;
#pragma unroll
    for (unsigned e = 0; e < kMaxExperts; ++e)
        if (e < E) {
            sc[e] = quantize(sc[e], a.quantum);
            if (first < 0 || sc[e] > __fadd_rn(first_value, a.tie_eps)) {
                first = static_cast<int>(e);
                first_value = sc[e];
            }
        }
    int second = -1;
    float second_value = -3.402823466e+38F;
#pragma unroll
    for (unsigned e = 0; e < kMaxExperts; ++e)
        if (e < E && static_cast<int>(e) != first) {
            if (second < 0 || sc[e] > __fadd_rn(second_value, a.tie_eps)) {
                second = static_cast<int>(e);
                second_value = sc[e];
            }
        }
    const unsigned short pair =
        static_cast<unsigned short>(first) | (static_cast<unsigned short>(second) << 8);
    reinterpret_cast<unsigned short*>(a.routes)[t] = pair;
    return pair;
}

__global__ void __launch_bounds__(kTile)
route_select(RouteArgs a) {
    pdl_begin();
    __shared__ unsigned int hist[kMaxExperts];
    if (threadIdx.x < kMaxExperts) hist[threadIdx.x] = 0;
    __syncthreads();

    const std::size_t t = static_cast<std::size_t>(blockIdx.x) * kTile + threadIdx.x;
    if (t < a.T) {
        const unsigned pair = pick_top2(a, t);
        atomicAdd(&hist[pair & 0xFFu], 1u);
        atomicAdd(&hist[pair >> 8], 1u);
    }
    __syncthreads();
    if (threadIdx.x < a.EP)
        a.tile_counts[static_cast<std::size_t>(blockIdx.x) * a.EP + threadIdx.x] = hist[threadIdx.x];
}

__device__ __forceinline__ uint4 add_u4(uint4 a, const uint4& b) {
    a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w;
    return a;
}

__device__ __forceinline__ uint4 shfl_xor_u4(const uint4& v, int o) {
    return make_uint4(__shfl_xor_sync(0xffffffffu, v.x, o), __shfl_xor_sync(0xffffffffu, v.y, o),
                      __shfl_xor_sync(0xffffffffu, v.z, o), __shfl_xor_sync(0xffffffffu, v.w, o));
}

// Shared-memory results of the per-expert scan.
struct ExpertScan {
    unsigned offs[kMaxExperts + 1];  // offsets; [E] = 2T
    unsigned q64[kMaxExperts + 1];   // first 64-row queue entry per expert; [E] = entries used
    unsigned q128[kMaxExperts + 1];
    unsigned base[kMaxExperts];      // offsets[e] + rows of expert e in earlier tokens
};

// Warp-wide (lane = expert): from each expert's total and its count in
// tokens before this CTA's, the exclusive scans over experts -- offsets and
// the bases of the two work queues -- into `sc`; `write_counts` also stores
// counts/offsets (one CTA does).
__device__ __forceinline__ void scan_experts(const RouteArgs& a, unsigned lane, unsigned tot, unsigned bef,
                                             bool write_counts, ExpertScan& sc) {
    const unsigned E = static_cast<unsigned>(a.E);
    const unsigned e = lane;
    unsigned incl = tot, c64 = (tot + 63) / 64, c128 = (tot + 127) / 128;
    unsigned i64 = c64, i128 = c128;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned n = __shfl_up_sync(0xffffffffu, incl, o);
        const unsigned n64 = __shfl_up_sync(0xffffffffu, i64, o);
        const unsigned n128 = __shfl_up_sync(0xffffffffu, i128, o);
        if (lane >= static_cast<unsigned>(o)) { incl += n; i64 += n64; i128 += n128; }
    }
    if (e < E) {
        sc.offs[e] = incl - tot;
        sc.q64[e] = i64 - c64;
        sc.q128[e] = i128 - c128;
        sc.base[e] = incl - tot + bef;
    }
    // lane 31's inclusive sums are the grand totals (lanes >= E add 0)
    const unsigned all_rows = __shfl_sync(0xffffffffu, incl, 31);
    const unsigned all64 = __shfl_sync(0xffffffffu, i64, 31);
    const unsigned all128 = __shfl_sync(0xffffffffu, i128, 31);
    if (lane == 0) {
        sc.offs[E] = all_rows;
        sc.q64[E] = all64;
        sc.q128[E] = all128;
    }
    if (write_counts) {
        if (e < E) {
            a.counts[e] = tot;
            a.offsets[e] = incl - tot;
        }
        if (lane == 0) a.offsets[E] = all_rows;
    }
}

// Work queues, entries first, first + stride, ...: entry i belongs to the
// expert whose chunk range holds it; entries past the last chunk are
// 0xFFFFFFFF (the reference memsets the expert queues to 0xff; the start
// queues get the same marker).
__device__ __forceinline__ void fill_queues(const RouteArgs& a, const ExpertScan& sc, std::size_t first,
                                            std::size_t stride) {
    const unsigned E = static_cast<unsigned>(a.E);
    const std::size_t n64 = (2 * a.T + 63) / 64 + a.E, n128 = (2 * a.T + 127) / 128 + a.E;
    const std::size_t nq = n64 > n128 ? n64 : n128;
    for (std::size_t i = first; i < nq; i += stride) {
        if (i < n64) {
            std::uint32_t ex = 0xFFFFFFFFu, st = 0xFFFFFFFFu;
            if (i < sc.q64[E]) {
                unsigned e = 0;
                while (i >= sc.q64[e + 1]) ++e;
                ex = e;
                st = sc.offs[e] + static_cast<std::uint32_t>(i - sc.q64[e]) * 64u;
            }
            if (a.we64) a.we64[i] = ex;
            if (a.ws64) a.ws64[i] = st;
        }
        if (i < n128) {
            std::uint32_t ex = 0xFFFFFFFFu, st = 0xFFFFFFFFu;
            if (i < sc.q128[E]) {
                unsigned e = 0;
                while (i >= sc.q128[e + 1]) ++e;
                ex = e;
                st = sc.offs[e] + static_cast<std::uint32_t>(i - sc.q128[e]) * 128u;
            }
            if (a.we128) a.we128[i] = ex;
            if (a.ws128) a.ws128[i] = st;
        }
    }
}

__global__ void __launch_bounds__(kTile)
route_scatter(RouteArgs a) {
    pdl_begin();
    constexpr int WARPS = kTile / 32;
    __shared__ uint4 red_all[WARPS][kMaxExperts / 4], red_before[WARPS][kMaxExperts / 4];
    __shared__ ExpertScan sc;
    __shared__ unsigned int warp_cnt[WARPS][kMaxExperts];
    __shared__ unsigned int warp_base[WARPS][kMaxExperts];
    const unsigned E = static_cast<unsigned>(a.E);
    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    // ---- expert totals and this tile's base, from the histogram table ----
    const unsigned ep4 = a.EP / 4;              // 16-byte vectors per tile
    const unsigned sub = threadIdx.x % ep4, trow = threadIdx.x / ep4;
    const unsigned per_pass = kTile / ep4;      // tiles covered per pass
    const uint4* tc4 = reinterpret_cast<const uint4*>(a.tile_counts);
    uint4 all = make_uint4(0, 0, 0, 0), before = make_uint4(0, 0, 0, 0);
#pragma unroll 4
    for (std::size_t tile = trow; tile < a.tiles; tile += per_pass) {
        const uint4 v = __ldcg(tc4 + tile * ep4 + sub);
        all = add_u4(all, v);
        if (tile < blockIdx.x) before = add_u4(before, v);
    }
    for (int o = 16; o >= static_cast<int>(ep4); o >>= 1) {  // lanes of equal `sub`
        all = add_u4(all, shfl_xor_u4(all, o));
        before = add_u4(before, shfl_xor_u4(before, o));
    }
    if (lane < ep4) {
        red_all[warp][lane] = all;
        red_before[warp][lane] = before;
    }
    __syncthreads();
    if (warp == 0) {
        const unsigned e = lane;
        unsigned tot = 0, bef = 0;
        if (e < E) {
            const unsigned* ra = reinterpret_cast<const unsigned*>(&red_all[0][0]);
            const unsigned* rb = reinterpret_cast<const unsigned*>(&red_before[0][0]);
            for (int w = 0; w < WARPS; ++w) {
                tot += ra[w * (kMaxExperts) + e];
                bef += rb[w * (kMaxExperts) + e];
            }
        }
        scan_experts(a, lane, tot, bef, blockIdx.x == 0, sc);
    }

    // ---- stable ranks inside the tile ----
    const std::size_t t = static_cast<std::size_t>(blockIdx.x) * kTile + threadIdx.x;
    const bool valid = t < a.T;
    unsigned e0 = 0xFFu, e1 = 0xFFu;
    if (valid) {
        const unsigned short pair = reinterpret_cast<const unsigned short*>(a.routes)[t];
        e0 = pair & 0xFFu;
        e1 = pair >> 8;
    }
    unsigned my_mask = 0;
    for (unsigned e = 0; e < E; ++e) {
        const unsigned m = __ballot_sync(0xffffffffu, valid && (e0 == e || e1 == e));
        if (lane == e) my_mask = m;
        if (lane == 0) warp_cnt[warp][e] = __popc(m);
    }
    __syncthreads();
    if (threadIdx.x < E) {
        const unsigned e = threadIdx.x;
        unsigned base = sc.base[e];
        for (int w = 0; w < WARPS; ++w) {
            warp_base[w][e] = base;
            base += warp_cnt[w][e];
        }
    }
    __syncthreads();
    const unsigned m0 = __shfl_sync(0xffffffffu, my_mask, e0 & 31u);
    const unsigned m1 = __shfl_sync(0xffffffffu, my_mask, e1 & 31u);
    if (valid) {
        const unsigned lt = (1u << lane) - 1u;
        const unsigned p0 = warp_base[warp][e0] + __popc(m0 & lt);
        const unsigned p1 = warp_base[warp][e1] + __popc(m1 & lt);
        a.assignment_rows[p0] = static_cast<std::uint32_t>(t);
        a.assignment_rows[p1] = static_cast<std::uint32_t>(t);
        reinterpret_cast<uint2*>(a.route_positions)[t] = make_uint2(p0, p1);
    }

    fill_queues(a, sc, static_cast<std::size_t>(blockIdx.x) * kTile + threadIdx.x,
                static_cast<std::size_t>(gridDim.x) * kTile);
}

// ---- gated SiLU -------------------------------------------------------------

// g / (1 + (float)exp((double)-g)) * u, k_silu_mul (src/tensor.cu:2005-2008):
// EXACT bit for bit (exp_ref of fastexp.cuh and an IEEE division); the
// tree-order mode of b2_prefill_layers uses CUDA's expf and __fdividef
// (within 2 ulp each: a few 1e-7 relative; a quotient whose denominator
// exceeds 2^126 becomes 0 instead of |g| / (1 + e) < 1e-36).
template <bool EXACT>
__device__ __forceinline__ float silu_mul1(float g, float u, const double* tab) {
    if (EXACT) return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, exp_ref(-g, tab))), u);
    return __fmul_rn(__fdividef(g, __fadd_rn(1.0f, expf(-g))), u);
}

constexpr int kSiluThreads = 256;

// One 128-bit chunk per thread per step over the flattened (row, chunk)
// space, grid-stride: every thread keeps two independent 16-byte loads in
// flight and the register budget (<= 64, four CTAs per SM) leaves room for
// enough warps to cover the exponentials' latency. (A warp-per-row layout
// with four chunks per lane in flight measured 40% slower: the 448-column
// rows leave a quarter of the lanes idle on the last chunk and the extra
// registers halved the resident warps.)
template <bool EXACT>
__global__ void __launch_bounds__(kSiluThreads, 4)
silu_mul_vec(const float* __restrict__ gate, std::size_t ldg, const float* __restrict__ up,
             std::size_t ldu, float* __restrict__ out, std::size_t ldo, std::size_t rows,
             std::size_t c4) {
    pdl_begin();
    __shared__ double tab[64];
    if (EXACT) {
        load_exp2_table(tab);
        __syncthreads();
    }
    // (row, chunk) of flat index i, advanced by the grid stride without a
    // division per step
    const std::size_t stride = static_cast<std::size_t>(gridDim.x) * kSiluThreads;
    const std::size_t step_r = stride / c4, step_c = stride % c4;
    const std::size_t i0 = static_cast<std::size_t>(blockIdx.x) * kSiluThreads + threadIdx.x;
    std::size_t r = i0 / c4, c = i0 % c4;
    for (; r < rows; r += step_r, c += step_c) {
        if (c >= c4) {
            c -= c4;
            ++r;
            if (r >= rows) break;
        }
        const float4 g = ld_stream(reinterpret_cast<const float4*>(gate + r * ldg) + c);
        const float4 u = ld_stream(reinterpret_cast<const float4*>(up + r * ldu) + c);
        st_plain(reinterpret_cast<float4*>(out + r * ldo) + c,
                 make_float4(silu_mul1<EXACT>(g.x, u.x, tab), silu_mul1<EXACT>(g.y, u.y, tab),
                             silu_mul1<EXACT>(g.z, u.z, tab), silu_mul1<EXACT>(g.w, u.w, tab)));
    }
}

template <bool EXACT>
__global__ void __launch_bounds__(kSiluThreads)
silu_mul_scalar(const float* __restrict__ gate, std::size_t ldg, const float* __restrict__ up,
                std::size_t ldu, float* __restrict__ out, std::size_t ldo, std::size_t rows,
                std::size_t cols) {
    pdl_begin();
    __shared__ double tab[64];
    if (EXACT) {
        load_exp2_table(tab);
        __syncthreads();
    }
    const unsigned lane = threadIdx.x & 31;
    const std::size_t warps = static_cast<std::size_t>(gridDim.x) * (kSiluThreads / 32);
    for (std::size_t r = static_cast<std::size_t>(blockIdx.x) * (kSiluThreads / 32) + (threadIdx.x >> 5);
         r < rows; r += warps)
        for (std::size_t j = lane; j < cols; j += 32)
            out[r * ldo + j] = silu_mul1<EXACT>(__ldg(gate + r * ldg + j), __ldg(up + r * ldu + j), tab);
}

// ---- weighted un-permute ----------------------------------------------------

// One float4 of each expert row per thread, 1024 threads per row: measured
// at 32,768 x 4096 as 6664 GB/s against 6342 for 256 threads x 4 float4 and
// 6554 for 512 x 2.
constexpr int kRowThreads = 1024;
constexpr int kRowUnroll = 1;

template <bool VEC>
__global__ void __launch_bounds__(kRowThreads)
moe_combine_rows(const float* __restrict__ expert_out, std::size_t expert_rows,
                 const std::uint8_t* __restrict__ routes,
                 const std::uint32_t* __restrict__ route_positions, float* __restrict__ out,
                 std::size_t T, std::size_t h) {
    pdl_begin();
    for (std::size_t t = blockIdx.x; t < T; t += gridDim.x) {
        const CombineRows cr = combine_rows(routes, route_positions, t, expert_rows);
        if (VEC) {
            const std::size_t h4 = h / 4;
            const float4* e4 = reinterpret_cast<const float4*>(expert_out);
            float4* o4 = reinterpret_cast<float4*>(out) + t * h4;
            for (std::size_t j0 = threadIdx.x; j0 < h4; j0 += kRowThreads * kRowUnroll) {
                float4 lo[kRowUnroll], hi[kRowUnroll];
#pragma unroll
                for (int k = 0; k < kRowUnroll; ++k) {
                    const std::size_t j = j0 + static_cast<std::size_t>(k) * kRowThreads;
                    if (j < h4) {
                        lo[k] = cr.lo < expert_rows ? ld_stream(e4 + cr.lo * h4 + j) : zero4();
                        hi[k] = cr.hi < expert_rows ? ld_stream(e4 + cr.hi * h4 + j) : zero4();
                    }
                }
#pragma unroll
                for (int k = 0; k < kRowUnroll; ++k) {
                    const std::size_t j = j0 + static_cast<std::size_t>(k) * kRowThreads;
                    if (j < h4) st_plain(o4 + j, combine4(lo[k], hi[k]));
                }
            }
        } else {
            for (std::size_t j = threadIdx.x; j < h; j += kRowThreads) {
                const float lo = cr.lo < expert_rows ? __ldg(expert_out + cr.lo * h + j) : 0.0f;
                const float hi = cr.hi < expert_rows ? __ldg(expert_out + cr.hi * h + j) : 0.0f;
                out[t * h + j] = combine_one(lo, hi);
            }
        }
    }
}

// ---- residual add -------------------------------------------------------------

__global__ void __launch_bounds__(256)
add_vec(float4* __restrict__ a, const float4* __restrict__ b, std::size_t n4) {
    pdl_begin();
    const std::size_t stride = static_cast<std::size_t>(gridDim.x) * 256;
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * 256 + threadIdx.x; i < n4; i += stride * 2) {
        const std::size_t i2 = i + stride;
        const float4 x0 = ld_plain(a + i), y0 = ld_stream(b + i);
        float4 x1, y1;
        if (i2 < n4) {
            x1 = ld_plain(a + i2);
            y1 = ld_stream(b + i2);
        }
        st_plain(a + i, add4(x0, y0));
        if (i2 < n4) st_plain(a + i2, add4(x1, y1));
    }
}

__global__ void __launch_bounds__(256)
add_scalar(float* __restrict__ a, const float* __restrict__ b, std::size_t n) {
    pdl_begin();
    const std::size_t stride = static_cast<std::size_t>(gridDim.x) * 256;
    for (std::size_t i = static_cast<std::size_t>(blockIdx.x) * 256 + threadIdx.x; i < n; i += stride)
        a[i] = __fadd_rn(a[i], b[i]);
}

std::size_t route_tiles(std::size_t T) { return (T + kTile - 1) / kTile; }

}  // namespace

int silu_mul_launch(const float* gate, std::size_t ld_gate, const float* up, std::size_t ld_up, float* out,
                    std::size_t ld_out, std::size_t rows, std::size_t cols, bool exact, b2_stream_t stream) {
    if (rows == 0 || cols == 0) return B2_OK;
    if (!gate || !up || !out) return invalid("silu_mul: null pointer");
    if (ld_gate < cols || ld_up < cols || ld_out < cols) return invalid("silu_mul shape");
    cudaStream_t s = as_stream(stream);
    const bool vec = (cols % 4) == 0 && (ld_gate % 4) == 0 && (ld_up % 4) == 0 && (ld_out % 4) == 0 &&
                     aligned16(gate) && aligned16(up) && aligned16(out);
    if (vec) {
        auto kernel = exact ? silu_mul_vec<true> : silu_mul_vec<false>;
        const std::size_t chunks = rows * (cols / 4);
        const unsigned grid = wave_grid(reinterpret_cast<const void*>(kernel), kSiluThreads, 0,
                                        (chunks + kSiluThreads - 1) / kSiluThreads);
        launch_pdl(kernel, grid, kSiluThreads, 0, s, gate, ld_gate, up, ld_up, out, ld_out, rows, cols / 4);
    } else {
        auto kernel = exact ? silu_mul_scalar<true> : silu_mul_scalar<false>;
        const std::size_t blocks_needed = (rows + (kSiluThreads / 32) - 1) / (kSiluThreads / 32);
        const unsigned grid = wave_grid(reinterpret_cast<const void*>(kernel), kSiluThreads, 0, blocks_needed);
        launch_pdl(kernel, grid, kSiluThreads, 0, s, gate, ld_gate, up, ld_up, out, ld_out, rows, cols);
    }
    return launch_result("b2_silu_mul");
}

}  // namespace b2

B2_DEFINE_CHECK_TAKER(moe)

extern "C" {

int b2_moe_route_workspace_size(size_t T, size_t E, size_t* bytes) {
    if (!bytes) return b2::invalid("b2_moe_route_workspace_size: null bytes");
    *bytes = b2::route_tiles(T) * b2::padded_experts(E) * sizeof(uint32_t);
    return B2_OK;
}

int b2_moe_route(const float* logits, size_t T, size_t E, float quantum, float tie_eps,
                 uint8_t* routes, uint32_t* counts, uint32_t* offsets, uint32_t* assignment_rows,
                 uint32_t* route_positions, uint32_t* work_expert64, uint32_t* work_start64,
                 uint32_t* work_expert128, uint32_t* work_start128, void* workspace,
                 size_t workspace_bytes, b2_stream_t stream) {
    using namespace b2;
    if (E < 2 || E > static_cast<size_t>(kMaxExperts))
        return invalid("b2_moe_route: E must be in [2, 32]");
    if (T == 0) return B2_OK;
    if (T > 0x7FFFFFFFu) return invalid("b2_moe_route: T too large for uint32 positions");
    if (!logits || !routes || !counts || !offsets || !assignment_rows || !route_positions || !workspace)
        return invalid("b2_moe_route: null pointer");
    size_t need = 0;
    b2_moe_route_workspace_size(T, E, &need);
    if (workspace_bytes < need) return invalid("b2_moe_route: workspace too small");
    if ((reinterpret_cast<std::uintptr_t>(routes) & 1u) || (reinterpret_cast<std::uintptr_t>(route_positions) & 7u) ||
        (reinterpret_cast<std::uintptr_t>(workspace) & 15u))
        return invalid("b2_moe_route: misaligned routes / route_positions / workspace");
    RouteArgs a{};
    a.logits = logits; a.T = T; a.E = E; a.quantum = quantum; a.tie_eps = tie_eps;
    a.routes = routes; a.counts = counts; a.offsets = offsets;
    a.assignment_rows = assignment_rows; a.route_positions = route_positions;
    a.we64 = work_expert64; a.ws64 = work_start64; a.we128 = work_expert128; a.ws128 = work_start128;
    a.EP = padded_experts(E);
    a.tile_counts = static_cast<uint32_t*>(workspace);
    a.tiles = route_tiles(T);
    if (a.tiles > 0x7FFFFFFFu) return invalid("b2_moe_route: too many tiles");
    cudaStream_t s = as_stream(stream);
    launch_pdl(route_select, static_cast<unsigned>(a.tiles), kTile, 0, s, a);
    launch_pdl(route_scatter, static_cast<unsigned>(a.tiles), kTile, 0, s, a);
    return launch_result("b2_moe_route");
}

int b2_silu_mul(const float* gate, size_t ld_gate, const float* up, size_t ld_up, float* out,
                size_t ld_out, size_t rows, size_t cols, b2_stream_t stream) {
    return b2::silu_mul_launch(gate, ld_gate, up, ld_up, out, ld_out, rows, cols, true, stream);
}

int b2_silu_mul_flags(const float* gate, size_t ld_gate, const float* up, size_t ld_up, float* out,
                      size_t ld_out, size_t rows, size_t cols, uint32_t flags, b2_stream_t stream) {
    return b2::silu_mul_launch(gate, ld_gate, up, ld_up, out, ld_out, rows, cols,
                               (flags & B2_FLAG_EXACT_ORDER) != 0, stream);
}

int b2_moe_combine(const float* expert_out, size_t expert_rows, const uint8_t* routes,
                   const uint32_t* route_positions, float* out, size_t T, size_t h,
                   b2_stream_t stream) {
    using namespace b2;
    if (T == 0) return B2_OK;
    if (!expert_out || !routes || !route_positions || !out) return invalid("moe combine: null pointer");
    if (h == 0) return invalid("moe combine shape");
    cudaStream_t s = as_stream(stream);
    if ((h % 4) == 0 && aligned16(expert_out) && aligned16(out)) {
        const unsigned grid = wave_grid(reinterpret_cast<const void*>(moe_combine_rows<true>), kRowThreads, 0, T);
        launch_pdl(moe_combine_rows<true>, grid, kRowThreads, 0, s, expert_out, expert_rows, routes, route_positions, out, T, h);
    } else {
        const unsigned grid = wave_grid(reinterpret_cast<const void*>(moe_combine_rows<false>), kRowThreads, 0, T);
        launch_pdl(moe_combine_rows<false>, grid, kRowThreads, 0, s, expert_out, expert_rows, routes, route_positions, out, T, h);
    }
    return launch_result("b2_moe_combine");
}

int b2_add(float* a, const float* b, size_t n, b2_stream_t stream) {
    using namespace b2;
    if (n == 0) return B2_OK;
    if (!a || !b) return invalid("add: null pointer");
    cudaStream_t s = as_stream(stream);
    if ((n % 4) == 0 && aligned16(a) && aligned16(b)) {
        const std::size_t n4 = n / 4;
        const unsigned grid = wave_grid(reinterpret_cast<const void*>(add_vec), 256, 0, (n4 + 511) / 512);
        launch_pdl(add_vec, grid, 256, 0, s, reinterpret_cast<float4*>(a), reinterpret_cast<const float4*>(b), n4);
    } else {
        const unsigned grid = wave_grid(reinterpret_cast<const void*>(add_scalar), 256, 0, (n + 255) / 256);
        launch_pdl(add_scalar, grid, 256, 0, s, a, b, n);
    }
    return launch_result("b2_add");
}

}  // extern "C"

// ---- routing for callers that cannot allocate device memory -----------------
//
// b2_moe_route takes its scratch (the per-tile expert histograms that pass
// from the selection kernel to the scatter kernel) from the caller. Some
// callers have no way to provide it: a plugin run by a host framework that
// owns every device allocation and forbids allocating on its execution path,
// or code that must not call cudaMalloc because it can synchronize the
// device. b2_moe_route_noalloc runs the same two kernels with that scratch in
// a fixed array compiled into this library instead.

namespace b2 {
namespace {

// Fixed scratch of b2_moe_route_noalloc: 32768 words (128 KB), one histogram
// row of padded_experts(E) words per 256-token tile. Every GPU that loads the
// library holds it until the process exits.
constexpr std::size_t kNoAllocScratchWords = 32768;
static __device__ __align__(256) std::uint32_t g_route_scratch[kNoAllocScratchWords];

// Device address of g_route_scratch in the current device's context (in
// host code the array's name is not a device address). Looked up on every
// call rather than cached: a context torn down and created again
// (cudaDeviceReset) may hold the array at another address.
int route_scratch_address(std::uint32_t** out) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_route_scratch);
    if (e != cudaSuccess)
        return set_error(B2_ERR_CUDA,
                         std::string("b2_moe_route_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    *out = static_cast<std::uint32_t*>(p);
    return B2_OK;
}

}  // namespace
}  // namespace b2

extern "C" int b2_moe_route_noalloc(const float* logits, size_t T, size_t E, float quantum, float tie_eps,
                                    uint8_t* routes, uint32_t* counts, uint32_t* offsets,
                                    uint32_t* assignment_rows, uint32_t* route_positions,
                                    uint32_t* work_expert64, uint32_t* work_start64, uint32_t* work_expert128,
                                    uint32_t* work_start128, b2_stream_t stream) {
    using namespace b2;
    if (E < 2 || E > static_cast<size_t>(kMaxExperts))
        return invalid("b2_moe_route_noalloc: E must be in [2, 32]");
    if (T == 0) return B2_OK;
    if (!logits || !routes || !counts || !offsets || !assignment_rows || !route_positions)
        return invalid("b2_moe_route_noalloc: null pointer");
    if ((reinterpret_cast<std::uintptr_t>(routes) & 1u) || (reinterpret_cast<std::uintptr_t>(route_positions) & 7u))
        return invalid("b2_moe_route_noalloc: misaligned routes / route_positions");
    const std::size_t tiles = route_tiles(T), ep = padded_experts(E);
    if (tiles * ep > kNoAllocScratchWords)
        return set_error(B2_ERR_UNSUPPORTED,
                         "b2_moe_route_noalloc: T = " + std::to_string(T) + " with E = " + std::to_string(E) +
                             " needs " + std::to_string(tiles * ep) + " scratch words, the fixed scratch holds " +
                             std::to_string(kNoAllocScratchWords) + " (at most " +
                             std::to_string(kNoAllocScratchWords / ep * kTile) +
                             " tokens for this E); use b2_moe_route with a caller workspace");
    std::uint32_t* scratch = nullptr;
    if (int rc = route_scratch_address(&scratch)) return rc;
    RouteArgs a{};
    a.logits = logits; a.T = T; a.E = E; a.quantum = quantum; a.tie_eps = tie_eps;
    a.routes = routes; a.counts = counts; a.offsets = offsets;
    a.assignment_rows = assignment_rows; a.route_positions = route_positions;
    a.we64 = work_expert64; a.ws64 = work_start64; a.we128 = work_expert128; a.ws128 = work_start128;
    a.EP = static_cast<unsigned>(ep);
    a.tile_counts = scratch;
    a.tiles = tiles;
    cudaStream_t s = as_stream(stream);
    launch_pdl(route_select, static_cast<unsigned>(a.tiles), kTile, 0, s, a);
    launch_pdl(route_scatter, static_cast<unsigned>(a.tiles), kTile, 0, s, a);
    return launch_result("b2_moe_route_noalloc");
}
