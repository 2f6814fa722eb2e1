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

__device__ __forceinline__ float exp_ref_slow(float x) {
    return static_cast<float>(exp(static_cast<double>(x)));
}

// Fast path of (float)exp((double)x), without branches so that a thread's
// independent exponentials interleave. Sets *slow when the result must come
// from exp_ref_slow instead: |x| > 80 (the float result may overflow or be
// subnormal) or NaN, or y within the error bound of a float rounding
// midpoint. The returned value is meaningless when *slow is set.
//
// Conversions are kept off the quarter-rate conversion pipe: n comes from
// the low word of x * 64/ln2 + 1.5 * 2^52 (round to nearest integer by the
// addition itself), and the final rounding of y to float is done on its bit
// pattern (the near-midpoint case being excluded, rounding is "round half
// up" on the 29 dropped bits, and the carry runs into the exponent field
// exactly as the next float up).
__device__ __forceinline__ float exp_ref_fast(float x, const double* tab, bool* slow) {
    const bool out_of_range = !(fabsf(x) <= 80.0f);     // also NaN
    const double xd = static_cast<double>(out_of_range ? 0.0f : x);
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
    const unsigned lo = static_cast<unsigned>(__double2loint(y));
    const unsigned hi = static_cast<unsigned>(__double2hiint(y));
    const int low29 = static_cast<int>(lo & 0x1FFFFFFFu);
    *slow = out_of_range | (abs(low29 - 0x10000000) < 2048);
    // float bits of y * 2^m: exponent (biased 1023 -> 127, plus m), the top
    // 23 of the 52 significand bits, plus one when the dropped bits exceed half
    const unsigned bits = ((((hi >> 20) - 896u) + static_cast<unsigned>(m)) << 23) |
                          ((hi & 0xFFFFFu) << 3) | (lo >> 29);
    return __uint_as_float(bits + (low29 > 0x10000000 ? 1u : 0u));
}

// Returns (float)exp((double)x); `tab` is the shared table. `slow`, when
// given, is set when the call took the exp(double) path.
__device__ __forceinline__ float exp_ref(float x, const double* tab, bool* slow = nullptr) {
    bool s;
    const float f = exp_ref_fast(x, tab, &s);
    if (slow) *slow = s;
    return s ? exp_ref_slow(x) : f;
}

}  // namespace b2
