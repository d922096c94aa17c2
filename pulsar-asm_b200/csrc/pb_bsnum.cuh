// pb_bsnum.cuh -- the Bonsai step's RMS norm and SwiGLU arithmetic (fwd8.c,
// pq1_host.c), shared by the decoder's kernels and the Q1 GEMV's fused
// prologues.
//
// rms (fwd8.c:312-317): s = serial double sum of x*x, sc = 1/sqrtf(float(s/n)
// + 1e-6), y = (x*sc)*w. The serial double sum is not recomputed serially: a
// parallel double sum P of the same (exact) products differs from it by at
// most 2(n-1)u*P (u = 2^-53, every term >= 0), so when P(1 -+ n 2^-51)/n
// round to the same float, that float is float(serial/n); otherwise the
// caller runs the serial chain.
// silu (pq1_host.c:196-227): (g * (1/(1+e^-g))) * u, e^x = pb_expf.
#pragma once
#include "pb_common.cuh"

// s / n in double: a multiply by the exact reciprocal when n is a power of two
// (the same value, sums of squares are far above the subnormal range)
PB_DEV double bs_div_n(double s, int n) {
  return (n & (n - 1)) == 0 ? __dmul_rn(s, 1.0 / (double)n) : __ddiv_rn(s, (double)n);
}
// float(s/n) of the serial double sum of squares from a parallel sum P;
// ok = false: not certified
PB_DEV float bs_mean_sq(double P, int n, bool& ok) {
  const double e = (double)n * 0x1p-51;
  const float lo = __double2float_rn(bs_div_n(__dsub_rn(P, __dmul_rn(P, e)), n));
  const float hi = __double2float_rn(bs_div_n(__dadd_rn(P, __dmul_rn(P, e)), n));
  ok = lo == hi;
  return lo;
}
// The other certified case: every square x^2 = k^2 2^(2e) (k odd) is a
// multiple of 2^m, m = min 2e, and P < 2^(m+53). Every partial sum of these
// non-negative terms, in any order, is then a multiple of 2^m below 2^(m+53),
// hence exact: the serial sum equals P (inputs from fp16 data often sum this
// way and land exactly on a float rounding midpoint, which the interval test
// cannot separate). P >= 2^(m+53) exactly when the exact sum is, rounding
// being monotone and 2^(m+53) a double.
// 2e for x != 0, INT_MAX for 0; branch-free (selects only), so that a load
// loop calling it keeps all its loads in flight
PB_DEV int bs_sq_lowbit(float x) {
  const unsigned u = __float_as_uint(x) & 0x7fffffffu;
  const unsigned E = u >> 23, M = u & 0x7fffffu;
  const unsigned mm = E ? (M | 0x800000u) : M;
  const int e = (E ? (int)E - 150 : -149) + (__ffs((int)mm) - 1);
  return u == 0 ? 0x7fffffff : 2 * e;
}
PB_DEV bool bs_sum_exact(double P, int m) {
  if (m == 0x7fffffff) return true;   // every term zero
  return P < __longlong_as_double((long long)(m + 53 + 1023) << 52);   // 2^(m+53), m in [-298, 208]
}
PB_DEV float bs_mean_sq_serial(const float* v, int n) {
  double s = 0.0;
  for (int i = 0; i < n; i++) { const double d = (double)v[i]; s = __fma_rn(d, d, s); }
  return __double2float_rn(bs_div_n(s, n));
}
PB_DEV double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
PB_DEV float bs_rms_scale(float mean) { return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, 1e-6f))); }
PB_DEV float bs_silu_mul(float g, float u) {
  return __fmul_rn(__fmul_rn(g, __fdiv_rn(1.0f, __fadd_rn(1.0f, pb_expf(-g)))), u);
}
