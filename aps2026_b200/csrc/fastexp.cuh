// (float)exp((double)x) for float x, bit for bit, in about a third of the
// double-precision work of calling exp(double).
//
// The reference evaluates its exponentials as (float)exp((double)x) (SiLU,
// src/tensor.cu:2005-2007; softmax, :2563-2564). On B200 that double exp
// is the bottleneck of both kernels (it issues ~25 FP64 operations), so it
// is computed here by Tang's table-driven method (P. T. P. Tang, "Table-driven
// implementation of the exponential function in IEEE floating-point
// arithmetic", ACM TOMS 15(2), 1989):
//   x = (64 m + j) * ln2/64 + r,  |r| <= ln2/128 (+ a float rounding margin)
//   exp(x) = 2^m * 2^(j/64) * e^r,  e^r = 1 + r + r^2/2 + r^3/6 + r^4/24 + O(r^5)
// with r from a two-part ln2/64 (the high part exact in a product with n),
// the polynomial in double, and 2^(j/64) from a 64-entry table of correctly
// rounded doubles (exp2_table.cuh). The double y = 2^(j/64) e^r is within
// 2^-43 (relative) of the exact value -- the O(r^5) term, |r|^5/120 <
// 4e-14, dominates. Rounding y to float then gives the correctly rounded
// float of exp(x) unless y lies within that error of a float rounding
// midpoint, i.e. unless bits 0..28 of its significand are within 2048 units
// of 2^28; CUDA's exp(double) (at most 1 ulp of double from exact) rounds
// to the same float in every other case. In the rare near-midpoint case
// (about 8 in 10^6 arguments), and for |x| > 80 where the float result may
// overflow or be subnormal, exp(double) itself is called. The whole float
// range of |x| <= 80 is checked against exp(double) by b2_selfcheck_exp.
#pragma once

#include "exp2_table.cuh"

namespace b2 {

// Per-CTA shared copy of the 2^(j/64) table (divergent j would serialise a
// __constant__ read). Call once per CTA, then __syncthreads().
__device__ __forceinline__ void load_exp2_table(double* smem64) {
    for (int i = threadIdx.x; i < 64; i += blockDim.x) smem64[i] = kExp2Table[i];
}

// Out of line: each kernel inlines exp_ref many times, and the rare slow
// path inlined at every site would multiply the code size.
static __device__ __noinline__ float exp_ref_slow(float x) {
    return static_cast<float>(exp(static_cast<double>(x)));
}

// Fast path of (float)exp((double)x), without branches so that a thread's
// independent exponentials interleave. Sets *slow when the result must come
// from exp_ref_slow instead: |x| > 80 (the float result may overflow or be
// subnormal) or NaN, or y within the error bound of a float rounding
// midpoint. The returned value is meaningless when *slow is set.
//
// n comes from the low word of x * 64/ln2 + 1.5 * 2^52 (round to nearest
// integer by the addition itself); 2^m is applied by adding m to the
// exponent field of y (y * 2^m stays a normal double), and one
// round-to-nearest conversion gives the float (a normal float for |x| <= 80;
// ties are among the near-midpoint cases sent to the slow path).
__device__ __forceinline__ float exp_ref_fast(float x, const double* tab, bool* slow) {
    const bool out_of_range = !(fabsf(x) <= 80.0f);     // also NaN
    // (out of range, the steps below compute garbage -- j stays a valid table
    // index -- and the result is discarded)
    const double xd = static_cast<double>(x);
    const double shifter = 6755399441055744.0;          // 1.5 * 2^52
    const double tn = fma(xd, 92.332482616893656877, shifter);  // x * 64 / ln2, rounded to an integer
    const int n = __double2loint(tn);                   // that integer (|n| < 2^13)
    const double nd = tn - shifter;                     // exact
    const int j = n & 63, m = n >> 6;                   // n = 64 m + j, m = floor(n / 64)
    double r = fma(-nd, kLn2By64Hi, xd);                // exact: nd * hi has <= 53 bits
    r = fma(-nd, kLn2By64Lo, r);
    double p = fma(r, 1.0 / 24.0, 1.0 / 6.0);
    p = fma(p, r, 0.5);
    p = fma(p, r, 1.0);
    p *= r;                                             // e^r - 1
    const double t = tab[j];
    const double y = fma(t, p, t);                      // 2^(j/64) e^r, in [0.99, 2)
    const int lo = __double2loint(y);
    const int low29 = lo & 0x1FFFFFFF;
    *slow = out_of_range | (static_cast<unsigned>(low29 - (0x10000000 - 2047)) < 4095u);  // |low29 - 2^28| < 2048
    const int hi = __double2hiint(y) + static_cast<int>(static_cast<unsigned>(m) << 20);  // y * 2^m
    return __double2float_rn(__hiloint2double(hi, lo));
}

// Returns (float)exp((double)x); `tab` is the shared table. `slow`, when
// given, is set when the call took the exp(double) path. Below -104 the
// result is +0 without calling it: e^-104 = 6.8e-46 is under half the
// smallest float subnormal (2^-150 = 7.0e-46), so it rounds to zero (this
// also makes -inf, a masked score, cheap).
__device__ __forceinline__ float exp_ref(float x, const double* tab, bool* slow = nullptr) {
    bool s;
    const float f = exp_ref_fast(x, tab, &s);
    if (slow) *slow = s;
    return s ? (x < -104.0f ? 0.0f : exp_ref_slow(x)) : f;
}

// The exponential of a reduction mode: in reference order (EXACT) the
// reference's (float)exp((double)x) bit for bit; in the default tree order,
// whose outputs are held to 1e-5 relative / 1e-6 absolute, CUDA's expf
// (within 2 ulp of exp(x), 2.4e-7 relative; +0 below the float range,
// NaN for NaN) at a quarter of the table method's instructions.
template <bool EXACT>
__device__ __forceinline__ float exp_mode(float x, const double* tab) {
    if (EXACT) return exp_ref(x, tab);
    return expf(x);
}

}  // namespace b2
