// pb_tq.cu -- TurboQuant K/V cache for the Bonsai decoder's attention
// (pulsar_arm/bonsai2/pq1_swar_sm53.cu:3264-3990, selected by PQ1_KVTQ in the
// reference's glue, pq1_fwd8_glue.c:211-232, where 4 bits is the default).
//
// A 128-value f16 K or V row x is rotated, y = H D x (H the Sylvester Hadamard
// matrix, unnormalised; D a fixed sign pattern), every coordinate of y / |x|
// is replaced by the index of its Lloyd-Max level for the sphere marginal at
// d = 128 (b-1 magnitude bits and a sign bit), and the row keeps one fp32
// scale s = |x| / |c|. Row = 12 words (3 bits: 8 words of 2-bit magnitudes,
// 4 of sign bits) or 16 words (4 bits: one nibble per coordinate).
// Attention never rotates the cache back: q.k = (R q).(R k) with R = H D /
// sqrt(128), and the V sum is formed in the rotated domain and rotated back
// once per head.
//
// Every reduction runs in the reference's order, so that the values are the
// reference's; its kernels' parallel shapes are kept where the order depends
// on them (a row's lane split and butterflies, the softmax's 256-thread
// strided sums and 8-warp fold, the P.V's 256-position chunks split over 4
// warps). Deterministic replacements, as in the rest of this library:
// rsqrtf -> 1 / sqrt (both rounded), expf -> pb_expf.
//
// Layout per layer: K codes [n_kv][ctx][CW(bk)], V codes [n_kv][ctx][CW(bv)],
// K scales [n_kv][ctx], V scales [n_kv][ctx]; ctx is the position stride.
#include "pb_internal.h"
#include "pb_common.cuh"

#include <cuda_fp16.h>

namespace {

// the stored format: codebook and thresholds per bit width (the Lloyd-Max
// levels of the d = 128 sphere marginal) and the rotation's sign pattern, as
// the reference stores them (pq1_swar_sm53.cu:3282-3288)
__constant__ float TQ_C3[4] = {0.24444127f, 0.75336427f, 1.33664119f, 2.13151002f};
__constant__ float TQ_T3[3] = {0.49890277f, 1.04500270f, 1.73407555f};
__constant__ float TQ_C4[8] = {0.12788960f, 0.38643676f, 0.65370631f, 0.93720949f,
                               1.24789774f, 1.60447431f, 2.04605246f, 2.68896675f};
__constant__ float TQ_T4[7] = {0.25716320f, 0.52007151f, 0.79545790f, 1.09255362f,
                               1.42618608f, 1.82526338f, 2.36750960f};
__constant__ uint32_t TQ_D[4] = {0xb5297a4du, 0x68e31da4u, 0x1b56c4e9u, 0xf3c2a581u};

constexpr int TQ_CH = 256;   // positions per P.V chunk (the order of the V sum depends on it)

__host__ __device__ constexpr int tq_cw(int b) { return b == 3 ? 12 : 16; }

PB_DEV float tq_dsign(float v, int j) { return (TQ_D[j >> 5] >> (j & 31)) & 1u ? -v : v; }
PB_DEV float tq_cent(int b, int v) {
  const float m = b == 3 ? TQ_C3[v & 3] : TQ_C4[v & 7];
  return (v >> (b - 1)) & 1 ? -m : m;
}
// lane l holds elements 4l..4l+3; x <- H x (within the lane, then the xor
// butterflies m = 1 .. 16)
PB_DEV void tq_fwht(float x[4], int lane) {
  const float a = __fadd_rn(x[0], x[1]), b = __fsub_rn(x[0], x[1]);
  const float c = __fadd_rn(x[2], x[3]), d = __fsub_rn(x[2], x[3]);
  x[0] = __fadd_rn(a, c); x[1] = __fadd_rn(b, d); x[2] = __fsub_rn(a, c); x[3] = __fsub_rn(b, d);
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float p = __shfl_xor_sync(0xffffffffu, x[i], m);
      x[i] = (lane & m) ? __fsub_rn(p, x[i]) : __fadd_rn(x[i], p);
    }
  }
}
PB_DEV float tq_xor_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// one warp encodes one f16 row into cw[CW(B)] and *sc
template <int B>
PB_DEV void tq_row(const uint16_t* __restrict__ row, uint32_t* __restrict__ cw, float* __restrict__ sc, int l) {
  const uint2 u = reinterpret_cast<const uint2*>(row)[l];
  float x[4] = {__half2float(__ushort_as_half((unsigned short)(u.x & 0xffffu))),
                __half2float(__ushort_as_half((unsigned short)(u.x >> 16))),
                __half2float(__ushort_as_half((unsigned short)(u.y & 0xffffu))),
                __half2float(__ushort_as_half((unsigned short)(u.y >> 16)))};
  float n2 = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    n2 = __fmaf_rn(x[i], x[i], n2);
    x[i] = tq_dsign(x[i], 4 * l + i);
  }
  n2 = tq_xor_sum(n2);
  tq_fwht(x, l);
  const float nrm = __fsqrt_rn(n2), inv = nrm > 0.0f ? __fdiv_rn(1.0f, nrm) : 0.0f;
  int v[4];
  float c2 = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const float z = __fmul_rn(x[i], inv), a = fabsf(z);
    int m = 0;
    if (B == 3) m = (a > TQ_T3[0]) + (a > TQ_T3[1]) + (a > TQ_T3[2]);
    else {
#pragma unroll
      for (int k = 0; k < 7; k++) m += a > TQ_T4[k];
    }
    const float c = B == 3 ? TQ_C3[m] : TQ_C4[m];
    c2 = __fmaf_rn(c, c, c2);
    v[i] = m | ((z < 0.0f) << (B - 1));
  }
  c2 = tq_xor_sum(c2);
  if (B == 3) {
    uint32_t mw = (uint32_t)((v[0] & 3) | (v[1] & 3) << 2 | (v[2] & 3) << 4 | (v[3] & 3) << 6) << (8 * (l & 3));
    uint32_t sw = (uint32_t)((v[0] >> 2) | (v[1] >> 2) << 1 | (v[2] >> 2) << 2 | (v[3] >> 2) << 3) << (4 * (l & 7));
    mw |= __shfl_xor_sync(0xffffffffu, mw, 1);
    mw |= __shfl_xor_sync(0xffffffffu, mw, 2);
    sw |= __shfl_xor_sync(0xffffffffu, sw, 1);
    sw |= __shfl_xor_sync(0xffffffffu, sw, 2);
    sw |= __shfl_xor_sync(0xffffffffu, sw, 4);
    if (!(l & 3)) cw[l >> 2] = mw;
    if (!(l & 7)) cw[8 + (l >> 3)] = sw;
  } else {
    uint32_t nw = (uint32_t)(v[0] | v[1] << 4 | v[2] << 8 | v[3] << 12) << (16 * (l & 1));
    nw |= __shfl_xor_sync(0xffffffffu, nw, 1);
    if (!(l & 1)) cw[l >> 1] = nw;
  }
  if (l == 0) *sc = c2 > 0.0f ? __fmul_rn(nrm, __fdiv_rn(1.0f, __fsqrt_rn(c2))) : 0.0f;
}

// 2 n_kv rows (K rows, then V rows) of position npos, one warp each
template <int BK, int BV>
__global__ void __launch_bounds__(1024) k_tq_store(const uint16_t* __restrict__ rows, const int* __restrict__ d_npos,
                                                   int npos_h, uint32_t* __restrict__ kc, float* __restrict__ ks,
                                                   uint32_t* __restrict__ vc, float* __restrict__ vs, int nkv, int ctx) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  pb_grid_wait();
  pb_grid_launch_dependents();
  if (w >= 2 * nkv) return;
  const int npos = d_npos ? *d_npos : npos_h;
  const uint16_t* row = rows + (size_t)w * 128;
  if (w < nkv) {
    const size_t r = (size_t)w * ctx + npos;
    tq_row<BK>(row, kc + r * tq_cw(BK), ks + r, l);
  } else {
    const size_t r = (size_t)(w - nkv) * ctx + npos;
    tq_row<BV>(row, vc + r * tq_cw(BV), vs + r, l);
  }
}

// scores of the 4 query heads of KV head blockIdx.x: one position per thread;
// per head a = a + fl(q_r[j] c) over j in order, then the row scale
template <int B>
__global__ void __launch_bounds__(256) k_tq_qk(const float* __restrict__ q, const uint32_t* __restrict__ kc,
                                               const float* __restrict__ ks, float* __restrict__ sc, int ctx, int T_h,
                                               const int* __restrict__ d_npos) {
  constexpr int CW = tq_cw(B), NV = 1 << B;
  __shared__ __align__(16) float4 qr[128];   // [j] = the 4 heads' rotated q
  __shared__ float cm[NV];
  const int kh = blockIdx.x, tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  pb_grid_wait();
  pb_grid_launch_dependents();
  const int T = d_npos ? *d_npos + 1 : T_h;
  if ((int)blockIdx.y * 256 >= T) return;   // block-uniform
  if (w < 4) {   // R q with R's 1/sqrt(128) and the score scale 1/sqrt(128): 2^-7
    const float4 q4 = reinterpret_cast<const float4*>(q + (size_t)(kh * 4 + w) * 128)[l];
    float x[4] = {tq_dsign(q4.x, 4 * l), tq_dsign(q4.y, 4 * l + 1), tq_dsign(q4.z, 4 * l + 2), tq_dsign(q4.w, 4 * l + 3)};
    tq_fwht(x, l);
    float* qf = reinterpret_cast<float*>(qr);
#pragma unroll
    for (int i = 0; i < 4; i++) qf[(4 * l + i) * 4 + w] = __fmul_rn(x[i], 0.0078125f);
  }
  if (tid < NV) cm[tid] = tq_cent(B, tid);
  __syncthreads();
  const int t = blockIdx.y * 256 + tid;
  if (t >= T) return;
  const uint4* kb = reinterpret_cast<const uint4*>(kc + ((size_t)kh * ctx + t) * CW);
  uint32_t cw[CW];
#pragma unroll
  for (int k = 0; k < CW / 4; k++) {
    const uint4 u = kb[k];
    cw[4 * k] = u.x; cw[4 * k + 1] = u.y; cw[4 * k + 2] = u.z; cw[4 * k + 3] = u.w;
  }
  float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
#pragma unroll
  for (int j = 0; j < 128; j++) {   // fully unrolled: the code words stay in registers
    int v;
    if (B == 3) v = (int)((cw[j >> 4] >> (2 * (j & 15))) & 3u) | (int)(((cw[8 + (j >> 5)] >> (j & 31)) & 1u) << 2);
    else v = (int)((cw[j >> 3] >> (4 * (j & 7))) & 15u);
    const float c = cm[v];
    const float4 qv = qr[j];
    a0 = __fadd_rn(a0, __fmul_rn(qv.x, c)); a1 = __fadd_rn(a1, __fmul_rn(qv.y, c));
    a2 = __fadd_rn(a2, __fmul_rn(qv.z, c)); a3 = __fadd_rn(a3, __fmul_rn(qv.w, c));
  }
  const float s = ks[(size_t)kh * ctx + t];
  float* so = sc + (size_t)kh * 4 * ctx + t;
  so[0] = __fmul_rn(a0, s); so[ctx] = __fmul_rn(a1, s);
  so[2 * (size_t)ctx] = __fmul_rn(a2, s); so[3 * (size_t)ctx] = __fmul_rn(a3, s);
}

// per query head (256 threads): the max and the sum of exp(s - max) over
// thread-strided positions, the warp xor tree, the 8 warps in order; p in
// place, inv = 1 / sum
__global__ void __launch_bounds__(256) k_tq_softmax(float* __restrict__ sc, float* __restrict__ inv, int ctx, int T_h,
                                                    const int* __restrict__ d_npos) {
  __shared__ float red[8];
  const int h = blockIdx.x, tid = threadIdx.x, l = tid & 31, w = tid >> 5;
  pb_grid_wait();
  pb_grid_launch_dependents();
  const int T = d_npos ? *d_npos + 1 : T_h;
  float* s = sc + (size_t)h * ctx;
  float m = -INFINITY;
  for (int t = tid; t < T; t += 256) m = fmaxf(m, s[t]);
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (!l) red[w] = m;
  __syncthreads();
  m = red[0];
#pragma unroll
  for (int k = 1; k < 8; k++) m = fmaxf(m, red[k]);
  __syncthreads();
  float sum = 0.0f;
  for (int t = tid; t < T; t += 256) {
    const float p = pb_expf(__fsub_rn(s[t], m));
    s[t] = p;
    sum = __fadd_rn(sum, p);
  }
  sum = tq_xor_sum(sum);
  if (!l) red[w] = sum;
  __syncthreads();
  if (!tid) {
    float z = 0.0f;
    for (int k = 0; k < 8; k++) z = __fadd_rn(z, red[k]);
    inv[h] = __fdiv_rn(1.0f, z);
  }
}

// the rotated V sum of one 256-position chunk for the 4 heads of KV head
// blockIdx.x: lane = dims 4l..4l+3, warp w takes positions w, w+4, ...; the
// 4 warps' sums added in warp order
template <int B>
__global__ void __launch_bounds__(128) k_tq_pv(const float* __restrict__ p, const uint32_t* __restrict__ vc,
                                               const float* __restrict__ vs, float* __restrict__ part, int nh, int ctx,
                                               int T_h, const int* __restrict__ d_npos) {
  constexpr int CW = tq_cw(B), NV = 1 << B;
  __shared__ __align__(16) float4 wt[TQ_CH];
  __shared__ __align__(16) uint32_t cs[TQ_CH * CW];   // the chunk's code words
  __shared__ float cent[NV];
  __shared__ __align__(16) float red[3][4][128];
  const int kh = blockIdx.x, c = blockIdx.y, tid = threadIdx.x, w = tid >> 5, l = tid & 31;
  pb_grid_wait();
  pb_grid_launch_dependents();
  const int T = d_npos ? *d_npos + 1 : T_h;
  const int t0 = c * TQ_CH, n = min(TQ_CH, T - t0);
  if (n <= 0) return;   // block-uniform
  if (tid < NV) cent[tid] = tq_cent(B, tid);
  {   // every thread's 16-byte loads of the chunk's codes in flight at once
    const uint4* src = reinterpret_cast<const uint4*>(vc + ((size_t)kh * ctx + t0) * CW);
    for (int i = tid; i < n * CW / 4; i += 128) reinterpret_cast<uint4*>(cs)[i] = src[i];
  }
  for (int t = tid; t < n; t += 128) {
    const float s = vs[(size_t)kh * ctx + t0 + t];
    const float* pp = p + (size_t)kh * 4 * ctx + t0 + t;
    wt[t] = make_float4(__fmul_rn(pp[0], s), __fmul_rn(pp[ctx], s), __fmul_rn(pp[2 * (size_t)ctx], s),
                        __fmul_rn(pp[3 * (size_t)ctx], s));
  }
  __syncthreads();
  float a[4][4];
#pragma unroll
  for (int h = 0; h < 4; h++)
#pragma unroll
    for (int i = 0; i < 4; i++) a[h][i] = 0.0f;
  const int wa = B == 3 ? l >> 2 : l >> 1, wb = 8 + (l >> 3);
#pragma unroll 4
  for (int t = w; t < n; t += 4) {
    const uint32_t* cw = cs + t * CW;
    int v[4];
    if (B == 3) {
      const uint32_t mb = cw[wa] >> (8 * (l & 3)), sb = cw[wb] >> (4 * (l & 7));
#pragma unroll
      for (int i = 0; i < 4; i++) v[i] = (int)((mb >> (2 * i)) & 3u) | (int)(((sb >> i) & 1u) << 2);
    } else {
      const uint32_t nb = cw[wa] >> (16 * (l & 1));
#pragma unroll
      for (int i = 0; i < 4; i++) v[i] = (int)((nb >> (4 * i)) & 15u);
    }
    const float4 g = wt[t];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const float e = cent[v[i]];
      a[0][i] = __fmaf_rn(g.x, e, a[0][i]); a[1][i] = __fmaf_rn(g.y, e, a[1][i]);
      a[2][i] = __fmaf_rn(g.z, e, a[2][i]); a[3][i] = __fmaf_rn(g.w, e, a[3][i]);
    }
  }
  if (w)
#pragma unroll
    for (int h = 0; h < 4; h++)
      reinterpret_cast<float4*>(red[w - 1][h])[l] = make_float4(a[h][0], a[h][1], a[h][2], a[h][3]);
  __syncthreads();
  if (!w)
#pragma unroll
    for (int h = 0; h < 4; h++) {
#pragma unroll
      for (int k = 0; k < 3; k++) {
        const float4 r = reinterpret_cast<const float4*>(red[k][h])[l];
        a[h][0] = __fadd_rn(a[h][0], r.x); a[h][1] = __fadd_rn(a[h][1], r.y);
        a[h][2] = __fadd_rn(a[h][2], r.z); a[h][3] = __fadd_rn(a[h][3], r.w);
      }
      reinterpret_cast<float4*>(part + ((size_t)c * nh + kh * 4 + h) * 128)[l] =
          make_float4(a[h][0], a[h][1], a[h][2], a[h][3]);
    }
}

// per query head (one warp): the chunks summed in order from 0, R^T (H, the
// 1/sqrt(128) and 1/sum, then D)
__global__ void __launch_bounds__(32) k_tq_out(const float* __restrict__ part, const float* __restrict__ inv,
                                               float* __restrict__ atto, int nh, int T_h, const int* __restrict__ d_npos) {
  const int h = blockIdx.x, l = threadIdx.x;
  pb_grid_wait();
  pb_grid_launch_dependents();
  const int T = d_npos ? *d_npos + 1 : T_h;
  const int nc = (T + TQ_CH - 1) / TQ_CH;
  float x[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int c = 0; c < nc; c++) {
    const float4 u = reinterpret_cast<const float4*>(part + ((size_t)c * nh + h) * 128)[l];
    x[0] = __fadd_rn(x[0], u.x); x[1] = __fadd_rn(x[1], u.y); x[2] = __fadd_rn(x[2], u.z); x[3] = __fadd_rn(x[3], u.w);
  }
  tq_fwht(x, l);
  const float k = __fmul_rn(inv[h], 0.0883883476f);
  float4 o;
  o.x = tq_dsign(__fmul_rn(x[0], k), 4 * l); o.y = tq_dsign(__fmul_rn(x[1], k), 4 * l + 1);
  o.z = tq_dsign(__fmul_rn(x[2], k), 4 * l + 2); o.w = tq_dsign(__fmul_rn(x[3], k), 4 * l + 3);
  reinterpret_cast<float4*>(atto + (size_t)h * 128)[l] = o;
}

int tq_bk(int bits) { return bits == 43 ? 4 : bits; }
int tq_bv(int bits) { return bits == 43 ? 3 : bits; }
bool tq_bits_ok(int bits) { return bits == 3 || bits == 4 || bits == 43; }

template <typename... KArgs, typename... Args>
int tq_launch(void (*k)(KArgs...), dim3 grid, int block, cudaStream_t st, bool pdl, const char* name, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(block);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k, args...);
  if (e != cudaSuccess) return pb_set_error(PB_ECUDA, "%s: %s", name, cudaGetErrorString(e));
  pb_count_launch();
  return PB_OK;
}

}  // namespace

size_t pb_tq_scratch_floats(int nkv, int ctx) {
  const int nh = 4 * nkv, nch = (ctx + TQ_CH - 1) / TQ_CH;
  return (size_t)nh * ctx + (size_t)nch * nh * 128 + nh;
}

// device npos (d_npos, when non-null) lets a captured graph store at, and
// attend up to, the position of each replay; pdl: programmatic dependent
// launch (every kernel waits for its predecessor before touching its data)
int pb_tq_store_launch(int bits, const uint16_t* d_rows, const int* d_npos, int npos, uint32_t* kc, float* ks,
                       uint32_t* vc, float* vs, int nkv, int ctx, cudaStream_t st, bool pdl) {
  if (!tq_bits_ok(bits) || nkv <= 0 || nkv > 16 || ctx <= 0 || (!d_npos && (npos < 0 || npos >= ctx)))
    return pb_set_error(PB_EINVAL, "pb_tq_store: bits %d (3, 4 or 43), n_kv %d (1..16), position %d of %d", bits, nkv,
                        npos, ctx);
  const dim3 g(1);
  if (bits == 3) return tq_launch(k_tq_store<3, 3>, g, 64 * nkv, st, pdl, "k_tq_store", d_rows, d_npos, npos, kc, ks, vc, vs, nkv, ctx);
  if (bits == 4) return tq_launch(k_tq_store<4, 4>, g, 64 * nkv, st, pdl, "k_tq_store", d_rows, d_npos, npos, kc, ks, vc, vs, nkv, ctx);
  return tq_launch(k_tq_store<4, 3>, g, 64 * nkv, st, pdl, "k_tq_store", d_rows, d_npos, npos, kc, ks, vc, vs, nkv, ctx);
}

// T positions (host), or d_npos + 1 (device, grids sized for ctx)
int pb_tq_attention_launch(int bits, const float* d_q, const uint32_t* kc, const float* ks, const uint32_t* vc,
                           const float* vs, int nkv, int ctx, int T, const int* d_npos, float* d_atto, float* d_scratch,
                           cudaStream_t st, bool pdl) {
  if (!tq_bits_ok(bits) || nkv <= 0 || ctx <= 0 || (!d_npos && (T <= 0 || T > ctx)) || !d_q || !d_atto || !d_scratch)
    return pb_set_error(PB_EINVAL, "pb_tq_attention: bits %d, n_kv %d, T %d of %d", bits, nkv, T, ctx);
  const int nh = 4 * nkv, bk = tq_bk(bits), bv = tq_bv(bits);
  const int span = d_npos ? ctx : T, nch = (span + TQ_CH - 1) / TQ_CH;
  float* sc = d_scratch;
  float* part = sc + (size_t)nh * ctx;
  float* inv = part + (size_t)((ctx + TQ_CH - 1) / TQ_CH) * nh * 128;
  const dim3 gq((unsigned)nkv, (unsigned)((span + 255) / 256));
  int rc = bk == 3 ? tq_launch(k_tq_qk<3>, gq, 256, st, pdl, "k_tq_qk", d_q, (const uint32_t*)kc, ks, sc, ctx, T, d_npos)
                   : tq_launch(k_tq_qk<4>, gq, 256, st, pdl, "k_tq_qk", d_q, (const uint32_t*)kc, ks, sc, ctx, T, d_npos);
  if (rc) return rc;
  if ((rc = tq_launch(k_tq_softmax, dim3(nh), 256, st, pdl, "k_tq_softmax", sc, inv, ctx, T, d_npos))) return rc;
  const dim3 gp((unsigned)nkv, (unsigned)nch);
  rc = bv == 3 ? tq_launch(k_tq_pv<3>, gp, 128, st, pdl, "k_tq_pv", (const float*)sc, (const uint32_t*)vc, vs, part, nh, ctx, T, d_npos)
               : tq_launch(k_tq_pv<4>, gp, 128, st, pdl, "k_tq_pv", (const float*)sc, (const uint32_t*)vc, vs, part, nh, ctx, T, d_npos);
  if (rc) return rc;
  return tq_launch(k_tq_out, dim3(nh), 32, st, pdl, "k_tq_out", (const float*)part, (const float*)inv, d_atto, nh, T, d_npos);
}

extern "C" int pb_tq_store(int bits, const uint16_t* d_rows, int npos, uint32_t* d_kcode, float* d_kscale,
                           uint32_t* d_vcode, float* d_vscale, int nkv, int ctx, void* stream) {
  if (!d_rows || !d_kcode || !d_kscale || !d_vcode || !d_vscale) return pb_set_error(PB_EINVAL, "pb_tq_store: null argument");
  return pb_tq_store_launch(bits, d_rows, nullptr, npos, d_kcode, d_kscale, d_vcode, d_vscale, nkv, ctx,
                            (cudaStream_t)stream, false);
}

extern "C" long long pb_tq_scratch_bytes(int nkv, int ctx) {
  return nkv <= 0 || ctx <= 0 ? -1 : (long long)pb_tq_scratch_floats(nkv, ctx) * 4;
}

extern "C" int pb_tq_attention(int bits, const float* d_q, const uint32_t* d_kcode, const float* d_kscale,
                               const uint32_t* d_vcode, const float* d_vscale, int nkv, int ctx, int T, float* d_atto,
                               void* d_scratch, void* stream) {
  if (!d_kcode || !d_kscale || !d_vcode || !d_vscale) return pb_set_error(PB_EINVAL, "pb_tq_attention: null argument");
  return pb_tq_attention_launch(bits, d_q, d_kcode, d_kscale, d_vcode, d_vscale, nkv, ctx, T, nullptr, d_atto,
                                static_cast<float*>(d_scratch), (cudaStream_t)stream, false);
}
