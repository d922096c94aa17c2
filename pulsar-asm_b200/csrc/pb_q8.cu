// pb_q8.cu -- Q8 weight streaming on sm_100a: packing, the REF_FLOAT GEMV /
// GEMM (bf16 activations, fp32 FMA chains in the reference's reduction order)
// and the Q8_0 x Q8_0 integer GEMV.
//
// Reduction order (lfm3_nanode.cu:222-343, the order the reference's shipped
// q8_partial<bf16,FMA=true> and q8_partial_TLb produce): per row and 2048-code
// chunk, leaf l (l = 0..31) is the chain over blocks b = l, l+32, ... of
// acc = fma(s_b, dot_b, acc), dot_b = fma(code_j, x_j, dot) over j = 0..31;
// the 32 leaves combine by the shuffle-down tree (16, 8, 4, 2, 1); chunk
// partials are summed ascending from 0; the Linear output is bf16(that sum).
//
// Streaming layout (PB_Q8_STREAM): the codes of (row, chunk)
// form one 2048-byte segment of 128 16-byte granules; granule h*32 + l holds
// codes [16(h&1), 16(h&1)+16) of block l + 32(h>>1). Lane l of a warp reads
// granules l, 32+l, 64+l, 96+l -- each warp load instruction is one contiguous
// 512-byte run -- and owns exactly leaf l. Scales of a segment are 32 pairs
// (s_l, s_{l+32}), one 4-byte (fp16) or 8-byte (fp32) load per lane. A K that
// 2048 does not divide is reduced as one chunk (pick(), lfm3_nanode.cu:
// 1763-1768): its rows are padded with zero blocks (codes and scales) to whole
// segments, and lane l's chain runs on from segment to segment before the one
// tree (a zero block adds fma(0, 0, acc) = acc exactly).
#include "pb_common.cuh"
#include "pb_internal.h"
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <algorithm>

// ------------------------------------------------------------------ packing
// Source rows r = 0..R-1 (row-major) land at destination row r*rmul + radd,
// which lets the loader merge tensors (q|k|v|gate) and interleave w1/w3 rows.
__global__ void k_q8_pack_codes(const uint4* __restrict__ src, uint4* __restrict__ dst,
                                int R, int K, int rmul, int radd) {
  // one thread per source granule of the destination order
  const int nch = (K + 2047) / 2048;
  const size_t total = (size_t)R * nch * 128;
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const size_t seg = i >> 7;
  const int gi = (int)(i & 127), h = gi >> 5, l = gi & 31;
  const size_t row = seg / nch;
  const int c = (int)(seg - row * nch);
  const int blk = c * 64 + l + 32 * (h >> 1);
  const size_t drow = row * rmul + radd;
  dst[(drow * nch + c) * 128 + gi] =
      blk < K / 32 ? src[(row * (size_t)K + (size_t)blk * 32 + 16 * (h & 1)) >> 4] : make_uint4(0, 0, 0, 0);
}
template <typename ST>
__global__ void k_q8_pack_scales(const ST* __restrict__ src, ST* __restrict__ dst, int R, int K,
                                 int rmul, int radd) {
  const int nch = (K + 2047) / 2048, nb = K / 32;
  const size_t total = (size_t)R * nch * 32;
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= total) return;
  const size_t seg = i >> 5;
  const int l = (int)(i & 31);
  const size_t row = seg / nch;
  const int c = (int)(seg - row * nch);
  const size_t d = ((row * rmul + radd) * nch + c) * 32 + l;
  dst[2 * d] = c * 64 + l < nb ? src[row * nb + c * 64 + l] : (ST)0;
  dst[2 * d + 1] = c * 64 + l + 32 < nb ? src[row * nb + c * 64 + l + 32] : (ST)0;
}

// ------------------------------------------------------ fast streaming GEMV
// CTA = 8 warps = G = 8/NCH row groups x NCH chunk warps. Warp (g, c) keeps the
// 64 x values of its leaf for chunk c in registers for the whole kernel and
// walks U rows per iteration; with NCH > 1 the chunk partials meet in shared
// memory and one thread per row adds them in chunk order.
template <bool F32S>
struct ScalePair;
template <>
struct ScalePair<false> {
  typedef unsigned T;
  static PB_DEV void load(const void* base, size_t idx, float& lo, float& hi) {
    const unsigned w = pb_ldg_stream32(reinterpret_cast<const unsigned*>(base) + idx);
    lo = pb_h2f((unsigned short)(w & 0xffffu));
    hi = pb_h2f((unsigned short)(w >> 16));
  }
};
template <>
struct ScalePair<true> {
  static PB_DEV void load(const void* base, size_t idx, float& lo, float& hi) {
    const uint2 w = pb_ldg_stream64(reinterpret_cast<const uint2*>(base) + idx);
    lo = __uint_as_float(w.x);
    hi = __uint_as_float(w.y);
  }
};

PB_DEV void pb_load_x64(const bf16_t* __restrict__ xc, int lane, float (&xr)[64], int nvalid = 2048) {
  // xr[0..31] = x[32*lane .. +31], xr[32..63] = x[1024 + 32*lane .. +31];
  // blocks at or past nvalid (a one-chunk tensor's padding) read as zero
#pragma unroll
  for (int half = 0; half < 2; half++) {
    if (half * 1024 + lane * 32 >= nvalid) {
#pragma unroll
      for (int j = 0; j < 32; j++) xr[half * 32 + j] = 0.0f;
      continue;
    }
    const uint4* p = reinterpret_cast<const uint4*>(xc + half * 1024 + lane * 32);
#pragma unroll
    for (int v = 0; v < 4; v++) {
      const uint4 w = p[v];
      const unsigned ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int k = 0; k < 4; k++) {
        xr[half * 32 + v * 8 + 2 * k] = pb_lo2f(ws[k]);
        xr[half * 32 + v * 8 + 2 * k + 1] = pb_hi2f(ws[k]);
      }
    }
  }
}

// 16 codes of one granule against 16 x values, continuing the chain `dot`
PB_DEV float pb_dot16(const uint4 g, const float* xr, float dot) {
  const unsigned ws[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const unsigned ub = ws[k] ^ 0x80808080u;
#pragma unroll
    for (int j = 0; j < 4; j++) dot = __fmaf_rn(pb_code(ub, j), xr[4 * k + j], dot);
  }
  return dot;
}

// the dots of this lane's two blocks (l and l+32 of the segment)
PB_DEV void pb_dots(const uint4 (&q)[4], const float (&xr)[64], float& d0, float& d1) {
  d0 = pb_dot16(q[0], xr, 0.0f);
  d0 = pb_dot16(q[1], xr + 16, d0);
  d1 = pb_dot16(q[2], xr + 32, 0.0f);
  d1 = pb_dot16(q[3], xr + 48, d1);
}

// one-chunk rows: segment c's (dot_lo, dot_hi, s_lo, s_hi) of every lane,
// chained in segment order (acc = fma(s, dot, acc), blocks l, l+32, l+64, ...)
// then one tree; lane 0 holds the row's chunk value
template <int NCH>
PB_DEV float pb_one_chain(const float4* p, int lane) {
  float acc = 0.0f;
#pragma unroll
  for (int c = 0; c < NCH; c++) {
    const float4 v = p[c * 32 + lane];
    acc = __fmaf_rn(v.z, v.x, acc);
    acc = __fmaf_rn(v.w, v.y, acc);
  }
  return pb_warp_tree(acc);
}

// one row's leaf value for this lane: blocks l and l+32 of the chunk
PB_DEV float pb_leaf(const uint4 (&q)[4], float slo, float shi, const float (&xr)[64]) {
  float d0 = pb_dot16(q[0], xr, 0.0f);
  d0 = pb_dot16(q[1], xr + 16, d0);
  float acc = __fmaf_rn(slo, d0, 0.0f);
  float d1 = pb_dot16(q[2], xr + 32, 0.0f);
  d1 = pb_dot16(q[3], xr + 48, d1);
  return __fmaf_rn(shi, d1, acc);
}

template <int NCH, int U, bool F32S, bool OUTF32, bool ONE>
__global__ void __launch_bounds__(256, 2)
k_q8f_stream(const uint4* __restrict__ codes, const void* __restrict__ scales,
             const bf16_t* __restrict__ x, void* __restrict__ y, int N, int K) {
  constexpr int G = 8 / NCH, RB = G * U;
  static_assert(!ONE || (NCH > 1 && RB <= 8), "one-chunk rows: a warp per row");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = warp % NCH, g = warp / NCH;
  __shared__ float part[2][RB][NCH];
  __shared__ float4 partq[ONE ? 2 : 1][ONE ? RB : 1][ONE ? NCH * 32 : 1];
  float xr[64];
  pb_load_x64(x + c * 2048, lane, xr, K - c * 2048);
  int it = 0;
  for (int rb = blockIdx.x; rb * RB < N; rb += gridDim.x, it ^= 1) {
    const int row0 = rb * RB + g * U;
    uint4 q[U][4];
    float slo[U], shi[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int row = row0 + u;
      if (row < N) {
        const size_t seg = (size_t)row * NCH + c;
        const uint4* base = codes + seg * 128 + lane;
#pragma unroll
        for (int h = 0; h < 4; h++) q[u][h] = pb_ldg_stream(base + 32 * h);
        ScalePair<F32S>::load(scales, seg * 32 + lane, slo[u], shi[u]);
      } else {
#pragma unroll
        for (int h = 0; h < 4; h++) q[u][h] = make_uint4(0, 0, 0, 0);
        slo[u] = shi[u] = 0.0f;
      }
    }
    if constexpr (ONE) {
#pragma unroll
      for (int u = 0; u < U; u++) {
        float d0, d1;
        pb_dots(q[u], xr, d0, d1);
        partq[it][g * U + u][c * 32 + lane] = make_float4(d0, d1, slo[u], shi[u]);
      }
      __syncthreads();
      if (warp < RB) {
        const int row = rb * RB + warp;
        const float v = pb_one_chain<NCH>(&partq[it][warp][0], lane);
        if (lane == 0 && row < N) {
          if (OUTF32) reinterpret_cast<float*>(y)[row] = __fadd_rn(0.0f, v);
          else reinterpret_cast<bf16_t*>(y)[row] = pb_f2bf(__fadd_rn(0.0f, v));
        }
      }
    } else {
#pragma unroll
      for (int u = 0; u < U; u++) {
        const float v = pb_warp_tree(pb_leaf(q[u], slo[u], shi[u], xr));
        const int row = row0 + u;
        if (NCH == 1) {
          if (lane == 0 && row < N) {
            if (OUTF32) reinterpret_cast<float*>(y)[row] = __fadd_rn(0.0f, v);
            else reinterpret_cast<bf16_t*>(y)[row] = pb_f2bf(__fadd_rn(0.0f, v));
          }
        } else if (lane == 0) {
          part[it][g * U + u][c] = v;
        }
      }
      if (NCH > 1) {
        __syncthreads();
        if (threadIdx.x < RB) {
          const int row = rb * RB + threadIdx.x;
          if (row < N) {
            float acc = 0.0f;
#pragma unroll
            for (int cc = 0; cc < NCH; cc++) acc = __fadd_rn(acc, part[it][threadIdx.x][cc]);
            if (OUTF32) reinterpret_cast<float*>(y)[row] = acc;
            else reinterpret_cast<bf16_t*>(y)[row] = pb_f2bf(acc);
          }
        }
      }
    }
  }
}

// ------------------------------------------------ T positions (float path)
// pf_gemv_T's values (lfm3_nanode.cu:4840-4968: per position, the GEMV leaf
// and chunk order of q8_partial + k_combine) for a tensor in the streaming
// layout: each row's codes and scales are read once per tile of TT positions.
// A warp takes a whole row: per segment (in chunk order) its lane converts
// the 64 codes of blocks l and l+32 once, then for every position of the tile
// runs the two dot chains as one packed fma.rn.f32x2 chain against the
// positions' x in shared memory (x of blocks l and l+32 side by side). Chunked
// rows: the chunk's leaf (s_lo, s_hi FMAs from 0), the tree, and the chunk
// values summed ascending from 0; one-chunk rows: the lane chain runs on over
// the segments, one tree, 0 + v.
constexpr int Q8T_X2 = 32 * 33;   // float2 per (segment, position): lane-major, padded
typedef unsigned long long q8t_f2;
PB_DEV q8t_f2 q8t_pk(float a, float b) {
  q8t_f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
PB_DEV void q8t_upk(q8t_f2 v, float& a, float& b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
PB_DEV q8t_f2 q8t_fma2(q8t_f2 a, q8t_f2 b, q8t_f2 c) {
  q8t_f2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

template <int NCH, bool ONE, bool F32S, bool OUTF32>
__global__ void __launch_bounds__(256, 1)
k_q8f_tiled(const uint4* __restrict__ codes, const void* __restrict__ scales, const bf16_t* __restrict__ x,
            void* __restrict__ y, int N, int K, int T) {
  constexpr int TT = 16 / NCH;
  extern __shared__ __align__(16) float2 xs[];     // [NCH][TT][Q8T_X2]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t0 = 0; t0 < T; t0 += TT) {
    const int nt = T - t0 < TT ? T - t0 : TT;
    __syncthreads();
    // stage the tile's x: (segment c, position t, lane l, j) = (x[c 2048 + 32 l + j],
    // x[c 2048 + 32 (l + 32) + j]); blocks past K (one-chunk padding) and
    // positions past T are zero
    for (int i = threadIdx.x; i < NCH * TT * 1024; i += blockDim.x) {
      const int j = i & 31, l = (i >> 5) & 31, t = (i >> 10) % TT, c = i / (TT * 1024);
      const int k0 = c * 2048 + 32 * l + j, k1 = k0 + 1024;
      float a = 0.0f, b = 0.0f;
      if (t < nt) {
        const bf16_t* xr = x + (size_t)(t0 + t) * K;
        if (k0 < K) a = pb_bf2f(xr[k0]);
        if (k1 < K) b = pb_bf2f(xr[k1]);
      }
      xs[(c * TT + t) * Q8T_X2 + l * 33 + j] = make_float2(a, b);
    }
    __syncthreads();
    for (int row = blockIdx.x * 8 + warp; row < N; row += gridDim.x * 8) {
      float acc[TT], tot[TT];
#pragma unroll
      for (int t = 0; t < TT; t++) { acc[t] = 0.0f; tot[t] = 0.0f; }
#pragma unroll 1
      for (int c = 0; c < NCH; c++) {
        const size_t seg = (size_t)row * NCH + c;
        const uint4* base = codes + seg * 128 + lane;
        uint4 q[4];
#pragma unroll
        for (int h = 0; h < 4; h++) q[h] = pb_ldg_stream(base + 32 * h);
        float slo, shi;
        ScalePair<F32S>::load(scales, seg * 32 + lane, slo, shi);
        // codes of block l (granules 0, 1) and block l+32 (granules 2, 3), paired
        q8t_f2 cw[32];
#pragma unroll
        for (int g = 0; g < 2; g++) {
          const unsigned wa[4] = {q[g].x, q[g].y, q[g].z, q[g].w}, wb[4] = {q[g + 2].x, q[g + 2].y, q[g + 2].z, q[g + 2].w};
#pragma unroll
          for (int k = 0; k < 4; k++) {
            const unsigned ua = wa[k] ^ 0x80808080u, ub = wb[k] ^ 0x80808080u;
#pragma unroll
            for (int jj = 0; jj < 4; jj++) cw[g * 16 + 4 * k + jj] = q8t_pk(pb_code(ua, jj), pb_code(ub, jj));
          }
        }
        const float2* xc = xs + (size_t)c * TT * Q8T_X2 + lane * 33;
#pragma unroll
        for (int t = 0; t < TT; t++) {
          const float2* xt = xc + t * Q8T_X2;
          q8t_f2 d = q8t_pk(0.0f, 0.0f);
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const float2 xv = xt[j];
            d = q8t_fma2(cw[j], q8t_pk(xv.x, xv.y), d);
          }
          float d0, d1;
          q8t_upk(d, d0, d1);
          if (ONE) {
            acc[t] = __fmaf_rn(slo, d0, acc[t]);
            acc[t] = __fmaf_rn(shi, d1, acc[t]);
          } else {
            const float v = pb_warp_tree(__fmaf_rn(shi, d1, __fmaf_rn(slo, d0, 0.0f)));
            tot[t] = __fadd_rn(tot[t], v);
          }
        }
      }
#pragma unroll
      for (int t = 0; t < TT; t++) {
        const float o = ONE ? __fadd_rn(0.0f, pb_warp_tree(acc[t])) : tot[t];
        if (lane == 0 && t < nt) {
          if (OUTF32) reinterpret_cast<float*>(y)[(size_t)(t0 + t) * N + row] = o;
          else reinterpret_cast<bf16_t*>(y)[(size_t)(t0 + t) * N + row] = pb_f2bf(o);
        }
      }
    }
  }
}

// ---------------------------------------------------- general (row-major) path
// Any K % 32 == 0 and T positions: one warp per row, positions in groups of 4,
// the same leaf chains and trees, chunks per pick(). x is read through L2.
__global__ void __launch_bounds__(256)
k_q8f_general(const int8_t* __restrict__ codes, const void* __restrict__ scales, int f32s,
              const bf16_t* __restrict__ x, void* __restrict__ y, int outf32, int N, int K,
              int T, int KC) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= N) return;
  const int nb = K / 32, nch = K / KC, nbc = KC / 32;
  const int8_t* qr = codes + (size_t)row * K;
  for (int t0 = 0; t0 < T; t0 += 4) {
    float tot[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int c = 0; c < nch; c++) {
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int b = lane; b < nbc; b += 32) {
        const int blk = c * nbc + b;
        const float s = f32s ? reinterpret_cast<const float*>(scales)[(size_t)row * nb + blk]
                             : pb_h2f(reinterpret_cast<const unsigned short*>(scales)[(size_t)row * nb + blk]);
        const int8_t* cb = qr + (size_t)blk * 32;
#pragma unroll
        for (int p = 0; p < 4; p++) {
          if (t0 + p < T) {
            const bf16_t* xb = x + (size_t)(t0 + p) * K + (size_t)blk * 32;
            float dot = 0.0f;
            for (int j = 0; j < 32; j++) dot = __fmaf_rn((float)cb[j], pb_bf2f(xb[j]), dot);
            acc[p] = __fmaf_rn(s, dot, acc[p]);
          }
        }
      }
#pragma unroll
      for (int p = 0; p < 4; p++) tot[p] = __fadd_rn(tot[p], pb_warp_tree(acc[p]));
    }
    if (lane == 0)
#pragma unroll
      for (int p = 0; p < 4; p++) {
        const int t = t0 + p;
        if (t < T) {
          if (outf32) reinterpret_cast<float*>(y)[(size_t)t * N + row] = tot[p];
          else reinterpret_cast<bf16_t*>(y)[(size_t)t * N + row] = pb_f2bf(tot[p]);
        }
      }
  }
}

// --------------------------------------------------------- Q8_0 integer path
// fwd35_ref.c:332-343: one warp per 32-block.
__global__ void k_q80_quantize(const float* __restrict__ x, int K, int8_t* __restrict__ qx,
                               unsigned short* __restrict__ dx) {
  const int b = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (b >= K / 32) return;
  const float v = x[b * 32 + lane];
  float amax = fabsf(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float d = __fdiv_rn(amax, 127.0f);
  const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
  qx[b * 32 + lane] = (int8_t)rintf(__fmul_rn(v, id));
  if (lane == 0) dx[b] = pb_f2h(d);
}

// Streaming layout. A warp takes Q80_R consecutive rows at a time: lane l
// owns blocks l and l+32 of each 2048-code chunk of every row, forms their
// exact int32 dots by dp4a and the products (dw*dx)*(float)isum into a
// shared row buffer (all rows' loads in flight together); then lane r folds
// row r in block order (no contraction), the reference's serial accumulation.
constexpr int Q80_R = 4;
template <bool F32S>
__global__ void __launch_bounds__(256)
k_q80_stream(const uint4* __restrict__ codes, const void* __restrict__ scales,
             const int8_t* __restrict__ qx, const unsigned short* __restrict__ dx,
             float* __restrict__ y, int32_t* __restrict__ isum, int N, int K) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int nch = K / 2048, nb = K / 32, ps = nb + 1;
  int8_t* sq = reinterpret_cast<int8_t*>(smem);                       // K bytes
  float* sdx = reinterpret_cast<float*>(smem + K);                    // nb floats
  float* prod = sdx + nb;                                             // 8 warps x Q80_R x (nb + 1)
  for (int i = threadIdx.x; i < K / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(sq)[i] = reinterpret_cast<const uint4*>(qx)[i];
  for (int i = threadIdx.x; i < nb; i += blockDim.x) sdx[i] = pb_h2f(dx[i]);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* pw = prod + (size_t)warp * Q80_R * ps;
  for (int row0 = (blockIdx.x * 8 + warp) * Q80_R; row0 < N; row0 += gridDim.x * 8 * Q80_R) {
    for (int c = 0; c < nch; c++) {
      uint4 q[Q80_R][4];
      float slo[Q80_R], shi[Q80_R];
#pragma unroll
      for (int r = 0; r < Q80_R; r++) {
        const int row = min(row0 + r, N - 1);
        const size_t seg = (size_t)row * nch + c;
        const uint4* base = codes + seg * 128 + lane;
#pragma unroll
        for (int h = 0; h < 4; h++) q[r][h] = pb_ldg_stream(base + 32 * h);
        ScalePair<F32S>::load(scales, seg * 32 + lane, slo[r], shi[r]);
      }
#pragma unroll
      for (int half = 0; half < 2; half++) {
        const int blk = c * 64 + lane + 32 * half;
        const uint4* xq = reinterpret_cast<const uint4*>(sq + blk * 32);
        const uint4 x0 = xq[0], x1 = xq[1];
        const float sx = sdx[blk];
#pragma unroll
        for (int r = 0; r < Q80_R; r++) {
          const uint4 w0 = q[r][2 * half], w1 = q[r][2 * half + 1];
          int s = 0;
          s = __dp4a((int)w0.x, (int)x0.x, s); s = __dp4a((int)w0.y, (int)x0.y, s);
          s = __dp4a((int)w0.z, (int)x0.z, s); s = __dp4a((int)w0.w, (int)x0.w, s);
          s = __dp4a((int)w1.x, (int)x1.x, s); s = __dp4a((int)w1.y, (int)x1.y, s);
          s = __dp4a((int)w1.z, (int)x1.z, s); s = __dp4a((int)w1.w, (int)x1.w, s);
          if (isum && row0 + r < N) isum[(size_t)(row0 + r) * nb + blk] = s;
          pw[r * ps + blk] = __fmul_rn(__fmul_rn(half ? shi[r] : slo[r], sx), __int2float_rn(s));
        }
      }
    }
    __syncwarp();
    if (lane < Q80_R && row0 + lane < N) {
      const float* pr = pw + lane * ps;
      float acc = 0.0f;
      for (int b = 0; b < nb; b++) acc = __fadd_rn(acc, pr[b]);
      y[row0 + lane] = acc;
    }
    __syncwarp();
  }
}

// ----------------------------------------------------- bf16 table (dtype 3)
// The certified arm's tied table (lfm3_nanode.cu:3505-3534): row-major bf16
// -> the head layout (b16_index: granule h*32 + l of a row holds elements
// l + 32 (8h + m), m = 0..7); one thread per destination granule
__global__ void k_b16_pack(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst, int N, int K) {
  const size_t ng = (size_t)N * (K / 8);
  for (size_t g = (size_t)blockIdx.x * blockDim.x + threadIdx.x; g < ng; g += (size_t)gridDim.x * blockDim.x) {
    const size_t row = g / (K / 8);
    const int gi = (int)(g - row * (K / 8)), h = gi >> 5, l = gi & 31;
    const uint16_t* r = src + row * K;
    unsigned w[4];
#pragma unroll
    for (int m = 0; m < 8; m += 2)
      w[m / 2] = (unsigned)r[l + 32 * (8 * h + m)] | ((unsigned)r[l + 32 * (8 * h + m + 1)] << 16);
    reinterpret_cast<uint4*>(dst + row * K)[gi] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// k_gemv_bf16: a warp per row, lane l chains s = s + bf16(W[k]) * x[k] over
// k = l, l+32, ... (product and sum rounded apart), then the shuffle-down
// tree; y fp32 as is. KG = K / 256: 8 granules per 256 elements and lane.
template <int KG>
__global__ void __launch_bounds__(256) k_b16_gemv(const uint16_t* __restrict__ w, const bf16_t* __restrict__ x,
                                                  float* __restrict__ y, int N) {
  constexpr int K = KG * 256;
  const int lane = threadIdx.x & 31;
  float xr[K / 32];
#pragma unroll
  for (int m = 0; m < K / 32; m++) xr[m] = pb_bf2f(x[lane + 32 * m]);
  for (int row = blockIdx.x * 8 + (threadIdx.x >> 5); row < N; row += gridDim.x * 8) {
    const uint4* g = reinterpret_cast<const uint4*>(w + (size_t)row * K) + lane;
    float s = 0.0f;
#pragma unroll
    for (int h = 0; h < KG; h++) {
      const uint4 q = pb_ldg_stream(g + 32 * h);
      const unsigned ws[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int i = 0; i < 4; i++) {
        s = __fadd_rn(s, __fmul_rn(pb_lo2f(ws[i]), xr[8 * h + 2 * i]));
        s = __fadd_rn(s, __fmul_rn(pb_hi2f(ws[i]), xr[8 * h + 2 * i + 1]));
      }
    }
    const float v = pb_warp_tree(s);
    if (lane == 0) y[row] = v;
  }
}

// =============================================================== host side
static int g_nsm = 0;
int pb_num_sms() {
  if (!g_nsm) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_nsm, cudaDevAttrMultiProcessorCount, dev);
    if (g_nsm <= 0) g_nsm = 148;
  }
  return g_nsm;
}

int pb_q8_pack_into(pb_q8* w, const int8_t* d_codes, const void* d_scales, cudaStream_t st,
                    int src_rows, int rmul, int radd) {
  const int K = w->K, R = src_rows;
  if (R <= 0 || (size_t)(R - 1) * rmul + radd >= (size_t)w->N)
    return pb_set_error(PB_EINVAL, "pack: rows %d x%d +%d exceed %d", R, rmul, radd, w->N);
  const size_t sbr = (size_t)(K / 32) * (w->sdt == PB_DT_F32 ? 4 : 2);   // scale bytes per row
  if (w->layout == PB_Q8_ROWMAJOR) {
    if (rmul == 1) {
      PB_TRY_CUDA(cudaMemcpyAsync(w->codes + (size_t)radd * K, d_codes, (size_t)R * K, cudaMemcpyDeviceToDevice, st));
      PB_TRY_CUDA(cudaMemcpyAsync((char*)w->scales + (size_t)radd * sbr, d_scales, (size_t)R * sbr,
                                  cudaMemcpyDeviceToDevice, st));
    } else {
      PB_TRY_CUDA(cudaMemcpy2DAsync(w->codes + (size_t)radd * K, (size_t)rmul * K, d_codes, K, K, R,
                                    cudaMemcpyDeviceToDevice, st));
      PB_TRY_CUDA(cudaMemcpy2DAsync((char*)w->scales + (size_t)radd * sbr, (size_t)rmul * sbr, d_scales,
                                    sbr, sbr, R, cudaMemcpyDeviceToDevice, st));
    }
    return PB_OK;
  }
  const size_t ng = (size_t)R * w->nch * 128;
  k_q8_pack_codes<<<(unsigned)((ng + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<const uint4*>(d_codes), reinterpret_cast<uint4*>(w->codes), R, K, rmul, radd);
  PB_LAUNCHED("k_q8_pack_codes");
  const size_t ns = (size_t)R * w->nch * 32;
  if (w->sdt == PB_DT_F32)
    k_q8_pack_scales<float><<<(unsigned)((ns + 255) / 256), 256, 0, st>>>(
        reinterpret_cast<const float*>(d_scales), reinterpret_cast<float*>(w->scales), R, K, rmul, radd);
  else
    k_q8_pack_scales<unsigned short><<<(unsigned)((ns + 255) / 256), 256, 0, st>>>(
        reinterpret_cast<const unsigned short*>(d_scales),
        reinterpret_cast<unsigned short*>(w->scales), R, K, rmul, radd);
  PB_LAUNCHED("k_q8_pack_scales");
  return PB_OK;
}

template <int NCH, int U, bool ONE>
static int launch_stream(const pb_q8* w, const uint16_t* x, void* y, int outf32, cudaStream_t st) {
  constexpr int RB = (8 / NCH) * U;
  const int nrb = (w->N + RB - 1) / RB;
  int grid = 2 * pb_num_sms();
  if (grid > nrb) grid = nrb;
  const uint4* q = reinterpret_cast<const uint4*>(w->codes);
  const bool f32s = w->sdt == PB_DT_F32;
  if (f32s && outf32) k_q8f_stream<NCH, U, true, true, ONE><<<grid, 256, 0, st>>>(q, w->scales, x, y, w->N, w->K);
  else if (f32s) k_q8f_stream<NCH, U, true, false, ONE><<<grid, 256, 0, st>>>(q, w->scales, x, y, w->N, w->K);
  else if (outf32) k_q8f_stream<NCH, U, false, true, ONE><<<grid, 256, 0, st>>>(q, w->scales, x, y, w->N, w->K);
  else k_q8f_stream<NCH, U, false, false, ONE><<<grid, 256, 0, st>>>(q, w->scales, x, y, w->N, w->K);
  PB_LAUNCHED("k_q8f_stream");
  return PB_OK;
}

template <int NCH, bool ONE, bool F32S, bool OUTF32>
static int launch_tiled_t(const pb_q8* w, int T, const uint16_t* x, void* y, cudaStream_t st) {
  constexpr int TT = 16 / NCH;
  const size_t smem = (size_t)NCH * TT * Q8T_X2 * sizeof(float2);
  static bool set[64] = {};
  int dev = 0;
  PB_TRY_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !set[dev]) {
    PB_TRY_CUDA(cudaFuncSetAttribute(k_q8f_tiled<NCH, ONE, F32S, OUTF32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem));
    set[dev] = true;
  }
  int grid = pb_num_sms();
  if (grid > (w->N + 7) / 8) grid = (w->N + 7) / 8;
  k_q8f_tiled<NCH, ONE, F32S, OUTF32><<<grid, 256, smem, st>>>(reinterpret_cast<const uint4*>(w->codes), w->scales,
                                                              x, y, w->N, w->K, T);
  PB_LAUNCHED("k_q8f_tiled");
  return PB_OK;
}
template <int NCH, bool ONE>
static int launch_tiled_n(const pb_q8* w, int T, const uint16_t* x, void* y, bool outf32, cudaStream_t st) {
  const bool f = w->sdt == PB_DT_F32;
  if (f) return outf32 ? launch_tiled_t<NCH, ONE, true, true>(w, T, x, y, st) : launch_tiled_t<NCH, ONE, true, false>(w, T, x, y, st);
  return outf32 ? launch_tiled_t<NCH, ONE, false, true>(w, T, x, y, st) : launch_tiled_t<NCH, ONE, false, false>(w, T, x, y, st);
}
// T positions of a streaming-layout tensor (pb_q8_gemm, the prefill's float path)
static int launch_tiled(const pb_q8* w, int T, const uint16_t* x, void* y, bool outf32, cudaStream_t st) {
  switch (w->nch) {
    case 1: return launch_tiled_n<1, false>(w, T, x, y, outf32, st);   // one chunk either way
    case 2: return w->one ? launch_tiled_n<2, true>(w, T, x, y, outf32, st) : launch_tiled_n<2, false>(w, T, x, y, outf32, st);
    case 4: return w->one ? launch_tiled_n<4, true>(w, T, x, y, outf32, st) : launch_tiled_n<4, false>(w, T, x, y, outf32, st);
    case 8: return w->one ? launch_tiled_n<8, true>(w, T, x, y, outf32, st) : launch_tiled_n<8, false>(w, T, x, y, outf32, st);
  }
  return pb_set_error(PB_EINVAL, "stream layout with %d chunks", w->nch);
}

int pb_q8_gemv_launch(const pb_q8* w, const uint16_t* d_x, void* d_y, int y_dtype, cudaStream_t st) {
  const int outf32 = y_dtype == PB_DT_F32;
  if (w->layout == PB_Q8_STREAM) {
    switch (w->nch) {
      case 1: return launch_stream<1, 2, false>(w, d_x, d_y, outf32, st);   // one chunk either way
      case 2: return w->one ? launch_stream<2, 2, true>(w, d_x, d_y, outf32, st) : launch_stream<2, 2, false>(w, d_x, d_y, outf32, st);
      case 4: return w->one ? launch_stream<4, 2, true>(w, d_x, d_y, outf32, st) : launch_stream<4, 2, false>(w, d_x, d_y, outf32, st);
      case 8: return w->one ? launch_stream<8, 2, true>(w, d_x, d_y, outf32, st) : launch_stream<8, 2, false>(w, d_x, d_y, outf32, st);
      default: return pb_set_error(PB_EINVAL, "stream layout with %d chunks", w->nch);
    }
  }
  k_q8f_general<<<(w->N + 7) / 8, 256, 0, st>>>(w->codes, w->scales, w->sdt == PB_DT_F32, d_x,
                                                d_y, outf32, w->N, w->K, 1, w->K >= 2048 && w->K % 2048 == 0 ? 2048 : (w->K == 512 ? 512 : w->K));
  PB_LAUNCHED("k_q8f_general");
  return PB_OK;
}

int pb_b16_pack(const uint16_t* d_src, uint16_t* d_dst, int N, int K, cudaStream_t st) {
  if (N <= 0 || K <= 0 || K % 256) return pb_set_error(PB_EINVAL, "bf16 table: shape %dx%d (K %% 256)", N, K);
  const size_t ng = (size_t)N * (K / 8);
  const int grid = (int)std::min<size_t>((ng + 255) / 256, (size_t)pb_num_sms() * 16);
  k_b16_pack<<<grid, 256, 0, st>>>(d_src, d_dst, N, K);
  PB_LAUNCHED("k_b16_pack");
  return PB_OK;
}

// ---------------------------------------------------------------- C ABI
extern "C" int pb_bf16_relayout(const uint16_t* d_src, uint16_t* d_dst, int N, int K, void* stream) {
  if (!d_src || !d_dst) return pb_set_error(PB_EINVAL, "pb_bf16_relayout: null argument");
  if (((uintptr_t)d_dst & 15) != 0) return pb_set_error(PB_EINVAL, "pb_bf16_relayout: dst must be 16-byte aligned");
  return pb_b16_pack(d_src, d_dst, N, K, (cudaStream_t)stream);
}

extern "C" int pb_bf16_gemv(const uint16_t* d_w, int N, int K, const uint16_t* d_x, float* d_y, void* stream) {
  if (!d_w || !d_x || !d_y || N <= 0) return pb_set_error(PB_EINVAL, "pb_bf16_gemv: bad argument");
  if (((uintptr_t)d_w & 15) != 0) return pb_set_error(PB_EINVAL, "pb_bf16_gemv: w must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  const int grid = (int)std::min<long>((N + 7) / 8, (long)pb_num_sms() * 8);
  switch (K) {
    case 256: k_b16_gemv<1><<<grid, 256, 0, st>>>(d_w, d_x, d_y, N); break;
    case 512: k_b16_gemv<2><<<grid, 256, 0, st>>>(d_w, d_x, d_y, N); break;
    case 1024: k_b16_gemv<4><<<grid, 256, 0, st>>>(d_w, d_x, d_y, N); break;
    case 2048: k_b16_gemv<8><<<grid, 256, 0, st>>>(d_w, d_x, d_y, N); break;
    case 4096: k_b16_gemv<16><<<grid, 256, 0, st>>>(d_w, d_x, d_y, N); break;
    default: return pb_set_error(PB_ENOTSUP, "pb_bf16_gemv: K=%d (256, 512, 1024, 2048 or 4096)", K);
  }
  PB_LAUNCHED("k_b16_gemv");
  return PB_OK;
}
extern "C" int pb_q8_pack(const int8_t* codes, const void* scales, int scale_dtype, int N, int K,
                          int src_on_device, void* stream, pb_q8** out) {
  if (!out || !codes || !scales) return pb_set_error(PB_EINVAL, "pb_q8_pack: null argument");
  *out = nullptr;
  if (N <= 0 || K <= 0 || K % 32) return pb_set_error(PB_EINVAL, "pb_q8_pack: bad shape %dx%d", N, K);
  if (scale_dtype != PB_DT_F16 && scale_dtype != PB_DT_F32)
    return pb_set_error(PB_EINVAL, "pb_q8_pack: scale dtype %d", scale_dtype);
  cudaStream_t st = (cudaStream_t)stream;
  pb_q8* w = new pb_q8();
  w->N = N; w->K = K; w->sdt = scale_dtype;
  const int nch = pb_q8_stream_chunks(K, &w->one);
  w->layout = nch ? PB_Q8_STREAM : PB_Q8_ROWMAJOR;
  w->nch = nch ? nch : 1;
  // source sizes (row-major) and device sizes (the tensor's layout)
  const size_t cb = (size_t)N * K, sb = pb_q8_scale_bytes(N, K, scale_dtype);
  const size_t dcb = pb_q8_code_bytes(N, K), dsb = pb_q8_layout_scale_bytes(N, K, scale_dtype);
  if (cudaMalloc(&w->codes, dcb) != cudaSuccess || cudaMalloc(&w->scales, dsb) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(w->codes); cudaFree(w->scales); delete w;
    return pb_set_error(PB_ENOMEM, "pb_q8_pack: cannot allocate %zu bytes", dcb + dsb);
  }
  int rc = PB_OK;
  int8_t* tc = nullptr; void* ts = nullptr;
  if (src_on_device) {
    rc = pb_q8_pack_into(w, codes, scales, st, N, 1, 0);
  } else {
    if (cudaMalloc(&tc, cb) != cudaSuccess || cudaMalloc(&ts, sb) != cudaSuccess) {
      cudaGetLastError();
      rc = pb_set_error(PB_ENOMEM, "pb_q8_pack: staging");
    } else if (cudaMemcpyAsync(tc, codes, cb, cudaMemcpyHostToDevice, st) != cudaSuccess ||
               cudaMemcpyAsync(ts, scales, sb, cudaMemcpyHostToDevice, st) != cudaSuccess) {
      rc = pb_set_error(PB_ECUDA, "pb_q8_pack: upload failed");
    } else {
      rc = pb_q8_pack_into(w, tc, ts, st, N, 1, 0);
    }
  }
  if (rc == PB_OK && cudaStreamSynchronize(st) != cudaSuccess)
    rc = pb_set_error(PB_ECUDA, "pb_q8_pack: %s", cudaGetErrorString(cudaGetLastError()));
  cudaFree(tc); cudaFree(ts);
  if (rc != PB_OK) { cudaFree(w->codes); cudaFree(w->scales); delete w; return rc; }
  *out = w;
  return PB_OK;
}

extern "C" int pb_q8_free(pb_q8* w) {
  if (!w) return PB_OK;
  if (w->owner) { cudaFree(w->codes); cudaFree(w->scales); }
  delete w;
  return PB_OK;
}

extern "C" int pb_q8_shape(const pb_q8* w, int* N, int* K) {
  if (!w) return pb_set_error(PB_EINVAL, "pb_q8_shape: null tensor");
  if (N) *N = w->N;
  if (K) *K = w->K;
  return PB_OK;
}

extern "C" int pb_q8_gemv(const pb_q8* w, const uint16_t* d_x, void* d_y, int y_dtype, void* stream) {
  if (!w || !d_x || !d_y) return pb_set_error(PB_EINVAL, "pb_q8_gemv: null argument");
  if (w->layout == PB_Q8_UMMA) return pb_set_error(PB_EINVAL, "pb_q8_gemv: tensor packed for pb_q80_gemm");
  if (y_dtype != PB_DT_BF16 && y_dtype != PB_DT_F32) return pb_set_error(PB_EINVAL, "pb_q8_gemv: y dtype");
  if (((uintptr_t)d_x & 15) != 0) return pb_set_error(PB_EINVAL, "pb_q8_gemv: x must be 16-byte aligned");
  return pb_q8_gemv_launch(w, d_x, d_y, y_dtype, (cudaStream_t)stream);
}

extern "C" int pb_q8_gemm(const pb_q8* w, int T, const uint16_t* d_x, void* d_y, int y_dtype,
                          void* stream) {
  if (!w || !d_x || !d_y || T <= 0) return pb_set_error(PB_EINVAL, "pb_q8_gemm: bad argument");
  if (w->layout == PB_Q8_UMMA) return pb_set_error(PB_EINVAL, "pb_q8_gemm: tensor packed for pb_q80_gemm");
  if (y_dtype != PB_DT_BF16 && y_dtype != PB_DT_F32) return pb_set_error(PB_EINVAL, "pb_q8_gemm: y dtype");
  cudaStream_t st = (cudaStream_t)stream;
  if (w->layout == PB_Q8_STREAM) return launch_tiled(w, T, d_x, d_y, y_dtype == PB_DT_F32, st);
  const int KC = w->K >= 2048 && w->K % 2048 == 0 ? 2048 : (w->K == 512 ? 512 : w->K);
  k_q8f_general<<<(w->N + 7) / 8, 256, 0, st>>>(w->codes, w->scales, w->sdt == PB_DT_F32, d_x, d_y,
                                                y_dtype == PB_DT_F32, w->N, w->K, T, KC);
  PB_LAUNCHED("k_q8f_general");
  return PB_OK;
}

extern "C" int pb_q80_quantize(const float* d_x, int K, int8_t* d_qx, uint16_t* d_dx, void* stream) {
  if (!d_x || !d_qx || !d_dx || K <= 0 || K % 32) return pb_set_error(PB_EINVAL, "pb_q80_quantize: bad argument");
  k_q80_quantize<<<(K / 32 + 7) / 8, 256, 0, (cudaStream_t)stream>>>(d_x, K, d_qx, d_dx);
  PB_LAUNCHED("k_q80_quantize");
  return PB_OK;
}

extern "C" int pb_q80_gemv(const pb_q8* w, const int8_t* d_qx, const uint16_t* d_dx, float* d_y,
                           int32_t* d_isum, void* stream) {
  if (!w || !d_qx || !d_dx || !d_y) return pb_set_error(PB_EINVAL, "pb_q80_gemv: null argument");
  if (w->layout == PB_Q8_UMMA) return pb_set_error(PB_EINVAL, "pb_q80_gemv: tensor packed for pb_q80_gemm");
  if (w->layout != PB_Q8_STREAM) return pb_set_error(PB_ENOTSUP, "pb_q80_gemv: needs K %% 2048 == 0 (K=%d)", w->K);
  if (((uintptr_t)d_qx & 15) != 0) return pb_set_error(PB_EINVAL, "pb_q80_gemv: qx must be 16-byte aligned");
  const size_t smem = (size_t)w->K + (size_t)(w->K / 32) * 4 + (size_t)8 * Q80_R * (w->K / 32 + 1) * 4;
  if (smem > 200 * 1024) return pb_set_error(PB_ENOTSUP, "pb_q80_gemv: K=%d too large", w->K);
  int grid = 3 * pb_num_sms();
  if (grid * 8 * Q80_R > w->N) grid = (w->N + 8 * Q80_R - 1) / (8 * Q80_R);
  cudaStream_t st = (cudaStream_t)stream;
  const uint4* q = reinterpret_cast<const uint4*>(w->codes);
  if (w->sdt == PB_DT_F32) {
    cudaFuncSetAttribute(k_q80_stream<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_q80_stream<true><<<grid, 256, smem, st>>>(q, w->scales, d_qx, d_dx, d_y, d_isum, w->N, w->K);
  } else {
    cudaFuncSetAttribute(k_q80_stream<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    k_q80_stream<false><<<grid, 256, smem, st>>>(q, w->scales, d_qx, d_dx, d_y, d_isum, w->N, w->K);
  }
  PB_LAUNCHED("k_q80_stream");
  return PB_OK;
}
