// pb_q8k.cuh -- the Q8_K activation quantiser for one 256-value block, as a
// device function over a 256-thread CTA (thread t holds value t).
//
// fwd8.c:67-139 as stated in scalar form by pq1_parity.c:131-147: amax = max
// |x| and mx = the value at the FIRST index reaching it; iscale = -127/mx;
// q = min(127, nearest_int(fma(x, iscale, 1.5*2^23))) with nearest_int taking
// the low mantissa bits minus 2^22; d = 1/iscale; int16 bsums per 16 values;
// 292 bytes per block (d f32, qs[256], bsums[16]); an all-zero block is 292
// zero bytes. A NaN out of the fma (0 * inf when iscale overflows) reads as
// the default NaN 0x7fc00000 of the reference's CPU, so q = 0 (the device's
// own NaN would give 127).
#pragma once
#include "pb_common.cuh"

struct Q8kScratch {
  float a[8];
  int i[8];
  float mx;
  int zero;
};

// every thread of the 256-thread CTA calls this (it synchronises the CTA)
PB_DEV void pb_q8k_block256(float v, uint8_t* __restrict__ qb, Q8kScratch& sc) {
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  float a = v != v ? -1.0f : fabsf(v);   // a NaN never reaches amax (serial `>`)
  int idx = t;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float oa = __shfl_down_sync(0xffffffffu, a, o);
    const int oi = __shfl_down_sync(0xffffffffu, idx, o);
    if (oa > a || (oa == a && oi < idx)) { a = oa; idx = oi; }
  }
  if (lane == 0) { sc.a[wid] = a; sc.i[wid] = idx; }
  __syncthreads();
  if (t == 0) {
    float ba = sc.a[0]; int bi = sc.i[0];
    for (int w = 1; w < 8; w++) if (sc.a[w] > ba) { ba = sc.a[w]; bi = sc.i[w]; }
    sc.zero = !(ba > 0.0f);
    sc.i[0] = bi;
  }
  __syncthreads();
  if (t == sc.i[0]) sc.mx = v;
  __syncthreads();
  if (sc.zero) {
    for (int i = t; i < 292; i += 256) qb[i] = 0;
    __syncthreads();
    return;
  }
  const float iscale = __fdiv_rn(-127.0f, sc.mx);
  unsigned f = __float_as_uint(__fmaf_rn(v, iscale, 12582912.0f));
  if ((f & 0x7fffffffu) > 0x7f800000u) f = 0x7fc00000u;
  int q = (int)(f & 0x007fffffu) - 0x00400000;
  q = q < 127 ? q : 127;
  qb[4 + t] = (uint8_t)(int8_t)q;
  int s = q;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) s += __shfl_down_sync(0xffffffffu, s, o, 16);
  if ((lane & 15) == 0) {
    const uint16_t s16 = (uint16_t)(int16_t)s;
    const int g = t >> 4;
    qb[260 + 2 * g] = (uint8_t)(s16 & 0xff);
    qb[261 + 2 * g] = (uint8_t)(s16 >> 8);
  }
  if (t == 0) {
    const unsigned u = __float_as_uint(__fdiv_rn(1.0f, iscale));
    qb[0] = u & 0xff; qb[1] = (u >> 8) & 0xff; qb[2] = (u >> 16) & 0xff; qb[3] = u >> 24;
  }
  __syncthreads();
}

// the same block quantiser run by one warp over 256 values y (thread l reads
// y[l + 32k], k < 8); no CTA barrier
PB_DEV void pb_q8k_block256_warp(const float* __restrict__ y, uint8_t* __restrict__ qb) {
  const int l = threadIdx.x & 31;
  float v[8];
#pragma unroll
  for (int k = 0; k < 8; k++) v[k] = y[l + 32 * k];
  float a = -1.0f;
  int idx = 0;
#pragma unroll
  for (int k = 0; k < 8; k++) {   // ascending index within the lane: strict > keeps the first
    const float ak = v[k] != v[k] ? -1.0f : fabsf(v[k]);
    if (ak > a) { a = ak; idx = l + 32 * k; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float oa = __shfl_xor_sync(0xffffffffu, a, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (oa > a || (oa == a && oi < idx)) { a = oa; idx = oi; }
  }
  if (!(a > 0.0f)) {
    for (int i = l; i < 292; i += 32) qb[i] = 0;
    return;
  }
  const float mx = y[idx];
  const float iscale = __fdiv_rn(-127.0f, mx);
#pragma unroll
  for (int k = 0; k < 8; k++) {
    unsigned f = __float_as_uint(__fmaf_rn(v[k], iscale, 12582912.0f));
    if ((f & 0x7fffffffu) > 0x7f800000u) f = 0x7fc00000u;
    int q = (int)(f & 0x007fffffu) - 0x00400000;
    q = q < 127 ? q : 127;
    qb[4 + l + 32 * k] = (uint8_t)(int8_t)q;
    // value l + 32k lies in 16-group 2k + (l >= 16): sum over each half-warp
    int s = q;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((l & 15) == 0) {
      const uint16_t s16 = (uint16_t)(int16_t)s;
      const int g = 2 * k + (l >> 4);
      qb[260 + 2 * g] = (uint8_t)(s16 & 0xff);
      qb[261 + 2 * g] = (uint8_t)(s16 >> 8);
    }
  }
  if (l == 0) {
    const unsigned u = __float_as_uint(__fdiv_rn(1.0f, iscale));
    qb[0] = u & 0xff; qb[1] = (u >> 8) & 0xff; qb[2] = (u >> 16) & 0xff; qb[3] = u >> 24;
  }
}
