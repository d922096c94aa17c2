// pb_common.cuh -- shared device helpers for the sm_100a kernels.
//
// Numerics contract (the CPU oracle under oracle/ states the same operations):
//  * bf16 is storage only: widen exactly, compute in fp32, round to nearest
//    even at the points the reference rounds (lfm3_nanode.cu:13-22, :116-121).
//  * Every multiply/add that the reference writes as a separate __fmul_rn /
//    __fadd_rn stays separate here (explicit _rn intrinsics, so nvcc cannot
//    contract them); every fma the reference writes is __fmaf_rn.
//  * rsqrtf -> correctly rounded 1/sqrt; expf -> pb_expf (below); cos/sin come
//    from a host-built table. These replace device approximations that have no
//    bit-identical CPU twin, so the oracle and the device agree bit for bit.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#define PB_DEV __device__ __forceinline__
#define PB_HD_INL __host__ __device__ __forceinline__

typedef unsigned short bf16_t;

PB_DEV float pb_bf2f(bf16_t v) { return __uint_as_float(((unsigned)v) << 16); }
PB_DEV bf16_t pb_f2bf(float v) {
  const unsigned u = __float_as_uint(v);
  if (((u >> 23) & 0xffu) == 0xffu) return (bf16_t)(u >> 16);
  return (bf16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}
// packed pair of bf16 (low half = element 0) -> two floats, exact
PB_DEV float pb_lo2f(unsigned w) { return __uint_as_float(w << 16); }
PB_DEV float pb_hi2f(unsigned w) { return __uint_as_float(w & 0xffff0000u); }

PB_DEV float pb_h2f(unsigned short h) { return __half2float(__ushort_as_half(h)); }
PB_DEV unsigned short pb_f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// e^x by Cody-Waite reduction (x = n*ln2 + r with ln2 split into a 16-bit
// high part and a low correction) and the degree-7 Taylor polynomial of e^r in
// Horner form with fused multiply-adds, then an exact scale by 2^n (two
// multiplies below the normal range so that only the last one rounds). Max
// error about 1 ulp; the oracle's pbo_expf performs the same operations.
PB_DEV float pb_expf(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
  if (x < -103.97207708399179f) return 0.0f;
  const float n = rintf(__fmul_rn(x, 1.44269502162933349609375f));
  float r = __fmaf_rn(n, -0.693145751953125f, x);
  r = __fmaf_rn(n, -1.428606765330187e-06f, r);
  float p = 1.98412701138295233249664306640625e-4f;
  p = __fmaf_rn(p, r, 1.38888892251998186111450195312500e-3f);
  p = __fmaf_rn(p, r, 8.33333376795053482055664062500000e-3f);
  p = __fmaf_rn(p, r, 4.16666679084300994873046875000000e-2f);
  p = __fmaf_rn(p, r, 1.66666671633720397949218750000000e-1f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int k = (int)n;
  if (k > 127) { p = __fmul_rn(p, 2.0f); k -= 1; }
  if (k < -126) {
    p = __fmul_rn(p, __uint_as_float((unsigned)(k + 64 + 127) << 23));
    return __fmul_rn(p, 5.42101086242752217003726400434970855712890625e-20f);
  }
  return __fmul_rn(p, __uint_as_float((unsigned)(k + 127) << 23));
}

// sigmoid exactly as the reference writes it: 1 / (1 + e^-x)
PB_DEV float pb_sigmoid(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, pb_expf(-x))); }

// shuffle-down tree over a full warp; lane 0 holds (((v0+v16)+(v8+v24))+...)
PB_DEV float pb_warp_tree(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, o));
  return v;
}

// int8 code k (0..3) of a word already biased by ^0x80808080 -> exact float:
// the byte lands in the low mantissa of 2^23 and the bias 2^23 + 128 is removed.
PB_DEV float pb_code(unsigned ub, int k) {
  return __fadd_rn(__uint_as_float(__byte_perm(ub, 0x4B000000u, 0x7440u + k)), -8388736.0f);
}

// PDL: let the next kernel in the stream start its independent prologue
// (weight prefetch) while this one drains; and wait for the previous one's
// results before reading them. Both are no-ops without the launch attribute.
PB_DEV void pb_grid_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
PB_DEV void pb_grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// streaming 128-bit load that does not allocate in L1 (weights are read once)
PB_DEV uint4 pb_ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
PB_DEV unsigned pb_ldg_stream32(const void* p) {
  unsigned r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}
PB_DEV uint2 pb_ldg_stream64(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
