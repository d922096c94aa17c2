// pb_bonsai.cu -- the Bonsai Q1_0 decoder's token step (pulsar_arm/bonsai2/
// fwd8.c:812-883 with attn_cpu :529-647 on the f16 cache) on sm_100a, as one
// CUDA graph per state of programmatic-dependent launches, 10 per layer:
//
//   embed | per layer: [residual add +] RMS norm + Q8_K -> q|k|v Q1 GEMV ->
//   head norms + YaRN rope + f16 K/V append -> q.k scores -> online-softmax
//   P.V + Q8_K -> o GEMV -> residual add + RMS norm + Q8_K -> gate|up GEMV ->
//   silu(g)*u + Q8_K -> down GEMV | residual add + output norm + Q8_K -> head
//   GEMV -> greedy argmax
//
// Each kernel waits for its predecessor before it lets the next one launch,
// so at most two kernels of the chain are resident at a time (the next one
// parked in its wait, or prefetching weights that do not depend on this one).
//
// Arithmetic, each step as the reference states it (the CPU oracle performs
// the same operations):
//  * rms and silu: pb_bsnum.cuh (a certified parallel form of the serial
//    double sum, with the serial chain as the fallback, counted in the
//    control block).
//  * rope (fwd8.c:359-369, contracted as gcc builds it, pq1_swar_sm53.cu:2147):
//    x[j] = fma(a, c, -(b*s)), x[j+64] = fma(a, s, b*c), with the (cos, sin)
//    table of every position built on the host (fwd8.c:339-358).
//  * attention (pq1_host.c:404-434): q rounded to f16; q.k as 16 fma chains
//    reduced ((a_l+a_8+l)+(a_4+l+a_12+l)), ((r0+r1)+(r2+r3)), times scale; the
//    online softmax keeps the running max M, ms = e^(Mold-M) at a new maximum
//    (rescaling the f16 accumulator), vs = e^(s-M) otherwise; the accumulator
//    is rounded to f16 after every update, S = fma(S, ms, vs), out = acc/S.
//    The running maxima come from a parallel prefix max (exact); the per-
//    dimension accumulator chain runs in position order.
//  * silu(g)*u (pq1_host.c:196-227): (g * (1/(1+e^-g))) * u.
//  * Q8_K and the Q1 GEMV: pb_q8k.cuh and pb_q1.cu.
// expf is pb_expf (pb_common.cuh) on both sides.
#include "pb_common.cuh"
#include "pb_internal.h"
#include "pb_q8k.cuh"
#include "pb_bsnum.cuh"
#include <cmath>
#include <cstring>
#include <vector>

namespace {

constexpr int BS_HD = 128;          // head_dim (fwd8.c hard-codes 128)
constexpr int BS_AM_CTAS = 296;     // argmax partial slots
constexpr int BS_PV_TT = 64;        // positions per V tile in the P.V chain
constexpr int BS_PV_NST = 4;        // V tiles in flight

struct BsCtl {
  int token;          // input id (the argmax writes the greedy id here)
  int pos;            // position (the argmax advances it)
  int step;           // greedy step counter (index into ids)
  int use_x;          // 1: the step's input row is xin (pq1_token_fused), not the embedding
  unsigned counter;   // argmax last-CTA counter
  int top;            // greedy id of the last step
  float topv;         // its logit
  int fallbacks;      // RMS norms that took the serial double chain
  int* ids;           // optional: greedy id of every step
  unsigned pv_pair[64];   // attention: heads of each pair that have finished (reset by the second)
  int err;            // a bounded wait in a kernel gave up
  float slot_val[BS_AM_CTAS];
  int slot_idx[BS_AM_CTAS];
};

// ------------------------------------------------------------- RMS norm
// the step's RMS norms (pb_bsnum.cuh) with the residual add and Q8_K
struct BsNormArgs {
  const float* xin;   // residual stream in
  const float* r;     // added to it first (null: none)
  float* xout;        // updated residual stream (written when r != null)
  const float* w;     // norm weight [H]
  uint8_t* xq;        // Q8_K of the normalised vector [H/256][292]
  int H;
  BsCtl* ctl;
};
// grid H/256 CTAs of 256 threads; every CTA sums all H squares (from L2) and
// writes its own 256-value slice and Q8_K block
__global__ void __launch_bounds__(256) k_bs_norm(BsNormArgs a) {
  extern __shared__ __align__(16) float sv[];   // [H]
  __shared__ double wsum[8];
  __shared__ int wmin[8];
  __shared__ float s_sc;
  __shared__ Q8kScratch q8s;
  // the norm weight does not depend on the previous kernel: load it before
  // the dependency wait
  const float wv = a.w[blockIdx.x * 256 + threadIdx.x];
  pb_grid_wait();
  pb_grid_launch_dependents();
  const int t = threadIdx.x, H = a.H;
  double ps = 0.0;
  int me = 0x7fffffff;
#pragma unroll 8
  for (int i = t; i < H; i += 256) {
    float v = a.xin[i];
    if (a.r) v = __fadd_rn(v, a.r[i]);
    sv[i] = v;
    const double d = (double)v;
    ps = __fma_rn(d, d, ps);
    me = min(me, bs_sq_lowbit(v));
  }
  ps = warp_sum_d(ps);
  me = __reduce_min_sync(0xffffffffu, me);
  if ((t & 31) == 0) { wsum[t >> 5] = ps; wmin[t >> 5] = me; }
  __syncthreads();
  if (t == 0) {
    double P = 0.0;
    int m = 0x7fffffff;
    for (int w = 0; w < 8; w++) { P = __dadd_rn(P, wsum[w]); m = min(m, wmin[w]); }
    bool ok;
    float mean = bs_mean_sq(P, H, ok);
    if (!ok && bs_sum_exact(P, m)) { ok = true; mean = __double2float_rn(bs_div_n(P, H)); }
    if (!ok) {
      mean = bs_mean_sq_serial(sv, H);
      if (blockIdx.x == 0) atomicAdd(&a.ctl->fallbacks, 1);
    }
    s_sc = bs_rms_scale(mean);
  }
  __syncthreads();
  const int i = blockIdx.x * 256 + t;
  const float v = sv[i];
  if (a.r) a.xout[i] = v;
  const float y = __fmul_rn(__fmul_rn(v, s_sc), wv);
  pb_q8k_block256(y, a.xq + (size_t)blockIdx.x * 292, q8s);
}

// ---------------------------------------------------------------- embed
struct BsEmbedArgs {
  const uint32_t* bits;     // token_embd [vocab][H/32]
  const uint16_t* scales;   // [vocab][H/128]
  const float* xin;         // ctl->use_x: the caller's row
  float* x;
  int H;
  const BsCtl* ctl;
};
// fwd8.c:438-452 (Q1_0 branch): x = bit ? sc : -sc, sc the fp16 scale widened
// with -0 read as +0 (fwd8.c:265-272)
__global__ void __launch_bounds__(256) k_bs_embed(BsEmbedArgs a) {
  pb_grid_wait();
  pb_grid_launch_dependents();
  const int i = blockIdx.x * 256 + threadIdx.x;
  if (i >= a.H) return;
  if (a.ctl->use_x) { a.x[i] = a.xin[i]; return; }
  const size_t tok = (size_t)a.ctl->token;
  const unsigned short h = a.scales[tok * (a.H / 128) + i / 128];
  const float sc = h == 0x8000u ? 0.0f : pb_h2f(h);
  const uint32_t w = a.bits[tok * (a.H / 32) + i / 32];
  a.x[i] = ((w >> (i & 31)) & 1u) ? sc : -sc;
}

// ------------------------------------------------ head norms, rope, K/V
struct BsPreArgs {
  const float* qkv;     // [NH + 2 NKV][128] GEMV output
  const float* qn;      // q_norm [128]
  const float* kn;      // k_norm [128]
  const float* rope;    // [max_ctx][cos 64 | sin 64]
  uint16_t* qh;         // [NH][128] f16 post-rope q
  uint16_t* kc;         // layer's K cache [NKV][max_ctx][128]
  uint16_t* vc;         // layer's V cache
  int NH, NKV, max_ctx;
  BsCtl* ctl;
  float* qf;            // optional: post-rope q as fp32 [NH][128] (TurboQuant attention; the hooks' debug copy)
  uint16_t* stage;      // optional: the K and V rows go here ([2 NKV][128] f16, K heads first), not to the cache
};
// one warp per head: q heads, k heads (rms, rope), then v heads (copied)
__global__ void __launch_bounds__(32) k_bs_attn_pre(BsPreArgs a) {
  __shared__ float sx[BS_HD];
  // the head-norm weights do not depend on the previous kernel: load them
  // before the dependency wait (v heads load and ignore k_norm)
  float wq[4];
  {
    const float* w = (int)blockIdx.x < a.NH ? a.qn : a.kn;
#pragma unroll
    for (int k = 0; k < 4; k++) wq[k] = w[threadIdx.x + 32 * k];
  }
  pb_grid_wait();
  pb_grid_launch_dependents();
  const int hh = blockIdx.x, l = threadIdx.x, pos = a.ctl->pos;
  const float* src = a.qkv + (size_t)hh * BS_HD;
  float x[4];
#pragma unroll
  for (int k = 0; k < 4; k++) x[k] = src[l + 32 * k];
  if (hh >= a.NH + a.NKV) {
    uint16_t* dst = a.stage ? a.stage + (size_t)(hh - a.NH) * BS_HD
                            : a.vc + ((size_t)(hh - a.NH - a.NKV) * a.max_ctx + pos) * BS_HD;
#pragma unroll
    for (int k = 0; k < 4; k++) dst[l + 32 * k] = pb_f2h(x[k]);
    return;
  }
  double ps = 0.0;
  int me = 0x7fffffff;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const double d = (double)x[k];
    ps = __fma_rn(d, d, ps);
    sx[l + 32 * k] = x[k];
    me = min(me, bs_sq_lowbit(x[k]));
  }
  ps = warp_sum_d(ps);
  me = __reduce_min_sync(0xffffffffu, me);
  bool ok;
  float mean = bs_mean_sq(ps, BS_HD, ok);
  if (!ok && bs_sum_exact(ps, me)) { ok = true; mean = __double2float_rn(bs_div_n(ps, BS_HD)); }
  if (!ok) {   // warp-uniform
    __syncwarp();
    if (l == 0) {
      mean = bs_mean_sq_serial(sx, BS_HD);
      atomicAdd(&a.ctl->fallbacks, 1);
    }
    mean = __shfl_sync(0xffffffffu, mean, 0);
  }
  const float sc = bs_rms_scale(mean);
  float y[4];
#pragma unroll
  for (int k = 0; k < 4; k++) y[k] = __fmul_rn(__fmul_rn(x[k], sc), wq[k]);
  const float* rc = a.rope + (size_t)pos * BS_HD;
  float o[4];
#pragma unroll
  for (int k = 0; k < 2; k++) {   // pairs (j, j+64), j = l + 32k
    const float c = rc[l + 32 * k], s = rc[64 + l + 32 * k], av = y[k], bv = y[k + 2];
    o[k] = __fmaf_rn(av, c, -__fmul_rn(bv, s));
    o[k + 2] = __fmaf_rn(av, s, __fmul_rn(bv, c));
  }
  if (a.qf && hh < a.NH) {
#pragma unroll
    for (int k = 0; k < 4; k++) a.qf[(size_t)hh * BS_HD + l + 32 * k] = o[k];
  }
  uint16_t* dst = hh < a.NH ? a.qh + (size_t)hh * BS_HD
                 : a.stage ? a.stage + (size_t)(hh - a.NH) * BS_HD
                           : a.kc + ((size_t)(hh - a.NH) * a.max_ctx + pos) * BS_HD;
#pragma unroll
  for (int k = 0; k < 4; k++) dst[l + 32 * k] = pb_f2h(o[k]);
}

// ----------------------------------------------------------- q.k scores
struct BsQkArgs {
  const uint16_t* qh;   // [NH][128] f16
  const uint16_t* kc;   // layer's K cache [NKV][max_ctx][128]
  float* sc;            // [NH][max_ctx] scaled scores
  int NH, NKV, max_ctx;
  float scale;
  const BsCtl* ctl;
};
constexpr int BS_KROW = 272;   // K row stride in shared memory (bank-conflict-free 16-byte reads)
// grid (max_ctx/32, NKV); warp g = query head kvh*G + g, lane = position
__global__ void __launch_bounds__(256) k_bs_fa_qk(BsQkArgs a) {
  __shared__ __align__(16) unsigned char ks[32 * BS_KROW];
  __shared__ __align__(16) uint16_t qs[8][BS_HD];
  pb_grid_wait();
  pb_grid_launch_dependents();
  const int T = a.ctl->pos + 1, t0 = blockIdx.x * 32;
  if (t0 >= T) return;
  const int kvh = blockIdx.y, G = a.NH / a.NKV;
  for (int i = threadIdx.x; i < 32 * 16; i += blockDim.x) {
    const int r = i >> 4, c = i & 15;
    if (t0 + r < T)
      *reinterpret_cast<uint4*>(ks + r * BS_KROW + c * 16) =
          *reinterpret_cast<const uint4*>(a.kc + ((size_t)kvh * a.max_ctx + t0 + r) * BS_HD + c * 8);
  }
  for (int i = threadIdx.x; i < G * 16; i += blockDim.x) {
    const int g = i >> 4, c = i & 15;
    *reinterpret_cast<uint4*>(&qs[g][c * 8]) =
        *reinterpret_cast<const uint4*>(a.qh + (size_t)(kvh * G + g) * BS_HD + c * 8);
  }
  __syncthreads();
  const int g = threadIdx.x >> 5, r = threadIdx.x & 31, t = t0 + r;
  if (t >= T) return;
  float acc[16];
#pragma unroll
  for (int c = 0; c < 16; c++) acc[c] = 0.0f;
  const unsigned char* kr = ks + r * BS_KROW;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const uint4 k0 = *reinterpret_cast<const uint4*>(kr + 32 * j);
    const uint4 k1 = *reinterpret_cast<const uint4*>(kr + 32 * j + 16);
    const uint4 q0 = *reinterpret_cast<const uint4*>(&qs[g][16 * j]);
    const uint4 q1 = *reinterpret_cast<const uint4*>(&qs[g][16 * j + 8]);
    const unsigned kw[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
    const unsigned qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int c = 0; c < 16; c++) {
      const unsigned short kh = (unsigned short)(c & 1 ? kw[c >> 1] >> 16 : kw[c >> 1] & 0xffffu);
      const unsigned short qv = (unsigned short)(c & 1 ? qw[c >> 1] >> 16 : qw[c >> 1] & 0xffffu);
      acc[c] = __fmaf_rn(pb_h2f(kh), pb_h2f(qv), acc[c]);
    }
  }
  float rr[4];
#pragma unroll
  for (int l = 0; l < 4; l++) rr[l] = __fadd_rn(__fadd_rn(acc[l], acc[8 + l]), __fadd_rn(acc[4 + l], acc[12 + l]));
  const float s = __fmul_rn(__fadd_rn(__fadd_rn(rr[0], rr[1]), __fadd_rn(rr[2], rr[3])), a.scale);
  a.sc[(size_t)(kvh * G + g) * a.max_ctx + t] = s;
}

// ------------------------------------------------- online softmax and P.V
struct BsPvArgs {
  const float* sc;    // [NH][max_ctx]
  const uint16_t* vc; // layer's V cache [NKV][max_ctx][128]
  float* atto;        // [NH][128]
  uint8_t* xq;        // Q8_K of atto (one 256-block per head pair)
  int NH, NKV, max_ctx;
  BsCtl* ctl;
};
PB_DEV float bs_r16(float x) { return __half2float(__float2half_rn(x)); }
// the serial algorithm's "s > M" keeps the earliest of equal maxima and never
// takes a NaN: the prefix max maps NaN to -inf and combines (earlier, later)
PB_DEV float bs_max_comb(float m, float s) { return s > m ? s : m; }
// grid NH CTAs of 256 threads, one head each. Softmax weights (all 256
// threads): thread i owns positions [i*C, i*C + C) of the running-max scan (the scratch copy of the scores is skewed by one
// word per 32 so that these strided walks hit distinct banks). Per position
// the scan leaves the exponent argument (Mold - s at a new maximum, s - M
// otherwise) and a flag; a coalesced pass takes the exponentials into the
// chain's array w (bit 31 = new maximum: w is ms and vs = 1; else w is vs and
// ms = 1) and marks every 16-position group that holds a new maximum.
//
// The chains (four warps, one per SM sub-partition, so that the chain's f16
// rounding conversions spread over all four; thread j owns dimension j) read
// V rows from a ring of BS_PV_NST tiles,
// each tile (contiguous rows of the kv head) one bulk copy completing on its
// slot's mbarrier (bounded waits: a copy that never lands sets the control
// block's error and ends the CTA). A 16-position group with no new maximum
// takes the branch-free form acc = r16(fma(v, vs, acc)), S = S + vs (= fma(S,
// 1, vs)); other groups take the general step.
PB_DEV int bs_skew(int p) { return p + (p >> 5); }
// skewed length, a multiple of 4 floats so that what follows it starts on a
// 16-byte boundary (cp.async destinations)
__host__ __device__ inline int bs_skew_len(int mc) { return (mc + mc / 32 + 3) & ~3; }
// group flags per head, padded to whole words (the chain reads a tile's four at once)
__host__ __device__ inline int bs_nm_len(int mc) { return (mc / 16 + 3) & ~3; }
// one tile of the chain for dim j: vb[r * 128] is row r's value, w the
// tile's encoded weights, nmt its 4 group flags, n <= 64 valid rows. Each
// group's operands are loaded one group ahead; a full group with no new
// maximum takes the branch-free step, any other group the general one.
PB_DEV void bs_chain_tile(const uint16_t* __restrict__ vb, const uint32_t* __restrict__ w,
                          const unsigned char* __restrict__ nmt, int n, float& acc, float& Ssum) {
  uint4 wn[4];
  uint16_t vn[16];
#pragma unroll
  for (int k = 0; k < 4; k++) wn[k] = reinterpret_cast<const uint4*>(w)[k];
#pragma unroll
  for (int k = 0; k < 16; k++) vn[k] = vb[k * BS_HD];
#pragma unroll
  for (int gi = 0; gi < BS_PV_TT / 16; gi++) {
    const int g0 = gi * 16;
    if (g0 >= n) break;
    const uint32_t wc[16] = {wn[0].x, wn[0].y, wn[0].z, wn[0].w, wn[1].x, wn[1].y, wn[1].z, wn[1].w,
                             wn[2].x, wn[2].y, wn[2].z, wn[2].w, wn[3].x, wn[3].y, wn[3].z, wn[3].w};
    uint16_t vc[16];
#pragma unroll
    for (int k = 0; k < 16; k++) vc[k] = vn[k];
    if (gi + 1 < BS_PV_TT / 16) {   // rows past n are stale shared memory, never used
#pragma unroll
      for (int k = 0; k < 4; k++) wn[k] = reinterpret_cast<const uint4*>(w + g0 + 16)[k];
#pragma unroll
      for (int k = 0; k < 16; k++) vn[k] = vb[(g0 + 16 + k) * BS_HD];
    }
    if (g0 + 16 <= n && !nmt[gi]) {
#pragma unroll
      for (int k = 0; k < 16; k++) {
        const float wf = __uint_as_float(wc[k]);
        acc = bs_r16(__fmaf_rn(pb_h2f(vc[k]), wf, acc));
        Ssum = __fadd_rn(Ssum, wf);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 16; k++) {
        if (g0 + k < n) {
          const bool nmax = (wc[k] >> 31) != 0;
          const float wk = __uint_as_float(wc[k] & 0x7fffffffu), ms = nmax ? wk : 1.0f, vs = nmax ? 1.0f : wk;
          if (ms != 1.0f) acc = bs_r16(__fmul_rn(acc, ms));
          acc = bs_r16(__fmaf_rn(pb_h2f(vc[k]), vs, acc));
          Ssum = __fmaf_rn(Ssum, ms, vs);
        }
      }
    }
  }
}
PB_DEV uint32_t bs_smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
PB_DEV bool bs_mbar_try(uint64_t* b, unsigned parity) {
  uint32_t ok;
  asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
               : "=r"(ok) : "r"(bs_smem_u32(b)), "r"(parity) : "memory");
  return ok != 0;
}
PB_DEV bool bs_mbar_wait(uint64_t* b, unsigned parity) {   // bounded
  for (unsigned i = 0; i < (1u << 24); i++)
    if (bs_mbar_try(b, parity)) return true;
  return false;
}
__global__ void __launch_bounds__(256) k_bs_fa_pv(BsPvArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int mc = a.max_ctx, mcs = bs_skew_len(mc);
  uint32_t* sw = reinterpret_cast<uint32_t*>(smem);                  // [mc] encoded weights
  float* sk = reinterpret_cast<float*>(sw + mc);                     // [mcs] skewed scratch
  uint16_t* vt = reinterpret_cast<uint16_t*>(sk + mcs);              // [NST][TT][128] f16 ring
  unsigned char* nm = reinterpret_cast<unsigned char*>(vt + (size_t)BS_PV_NST * BS_PV_TT * BS_HD);   // [nm_len]
  __shared__ __align__(8) uint64_t full[BS_PV_NST];
  __shared__ float wmax[8];
  __shared__ float s_S;
  __shared__ int s_last, s_fail;
  pb_grid_wait();
  pb_grid_launch_dependents();
  const int T = a.ctl->pos + 1, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int h = blockIdx.x, kvh = h / (a.NH / a.NKV);
  const uint16_t* V = a.vc + (size_t)kvh * mc * BS_HD;
  const int ntile = (T + BS_PV_TT - 1) / BS_PV_TT;
  // V tiles (contiguous rows of the kv head) by one bulk copy each into a ring
  // of BS_PV_NST slots, completion on the slot's mbarrier
  if (tid == 0) {
    for (int k = 0; k < BS_PV_NST; k++)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bs_smem_u32(&full[k])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_fail = 0;
  }
  __syncthreads();
  auto issue = [&](int tile) {   // thread 0
    if (tile < ntile) {
      uint64_t* bar = &full[tile % BS_PV_NST];
      const unsigned bytes = (unsigned)min(BS_PV_TT, T - tile * BS_PV_TT) * BS_HD * 2;
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bs_smem_u32(bar)), "r"(bytes) : "memory");
      asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                   ::"r"(bs_smem_u32(vt + (size_t)(tile % BS_PV_NST) * BS_PV_TT * BS_HD)),
                   "l"(V + (size_t)tile * BS_PV_TT * BS_HD), "r"(bytes), "r"(bs_smem_u32(bar)) : "memory");
    }
  };
  if (tid == 0)
    for (int k = 0; k < BS_PV_NST; k++) issue(k);
  {
    // ---- softmax weights, all 256 threads: the head's scores
    const float* S = a.sc + (size_t)h * mc;
    for (int p0 = tid; p0 < T; p0 += 8 * 256) {
      float sv[8];
#pragma unroll
      for (int k = 0; k < 8; k++) { const int p = p0 + 256 * k; sv[k] = p < T ? S[p] : 0.0f; }
#pragma unroll
      for (int k = 0; k < 8; k++) { const int p = p0 + 256 * k; if (p < T) sk[bs_skew(p)] = sv[k]; }
    }
    __syncthreads();
    // ---- running maxima: thread i owns positions [i*C, i*C + C)
    const int C = (T + 255) / 256, p0 = tid * C, p1 = min(T, p0 + C);
    float m = -INFINITY;
    for (int p = p0; p < p1; p++) { const float x = sk[bs_skew(p)]; m = bs_max_comb(m, x != x ? -INFINITY : x); }
    float inc = m;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float u = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc = bs_max_comb(u, inc);
    }
    if (lane == 31) wmax[w] = inc;
    __syncthreads();
    float ex = __shfl_up_sync(0xffffffffu, inc, 1);
    if (lane == 0) ex = -INFINITY;
    float M = -INFINITY;
    for (int ww = 0; ww < w; ww++) M = bs_max_comb(M, wmax[ww]);
    M = bs_max_comb(M, ex);
    for (int p = p0; p < p1; p++) {   // in place: the score becomes |exponent argument| | flag
      const int q = bs_skew(p);
      const float x = sk[q];
      float arg;
      uint32_t flag = 0;
      if (x > M) { arg = __fsub_rn(M, x); M = x; flag = 1; }
      else arg = __fsub_rn(x, M);
      sk[q] = __uint_as_float((__float_as_uint(arg) & 0x7fffffffu) | (flag << 31));
    }
    __syncthreads();
    // ---- exponentials, coalesced; group flags by ballot. Every argument
    // is <= 0 or NaN: its sign is restored.
    for (int pb = w * 32; pb < ((T + 31) & ~31); pb += 8 * 32) {
      const int p = pb + lane;
      bool nmax = false;
      if (p < T) {
        const uint32_t ab = __float_as_uint(sk[bs_skew(p)]);
        nmax = (ab >> 31) != 0;
        const uint32_t mag = ab & 0x7fffffffu;
        const float e = pb_expf(__uint_as_float(mag | (mag ? 0x80000000u : 0u)));
        sw[p] = (__float_as_uint(e) & 0x7fffffffu) | (nmax ? 0x80000000u : 0u);
      }
      const unsigned bal = __ballot_sync(0xffffffffu, nmax);
      if (lane == 0 && pb < T) nm[pb >> 4] = (bal & 0xffffu) != 0;
      if (lane == 16 && pb + 16 < T) nm[(pb >> 4) + 1] = (bal >> 16) != 0;
    }
    __syncthreads();
  }
  if (w >= 4) return;   // the chains are four warps; the others are done
  // ---- the chains (thread j < 128 owns dim j), positions in order; named
  // barrier 1 over the 128 chain threads
  const int j = tid;
  float acc = 0.0f, Ssum = 0.0f;
  int failed = -1;   // the tile whose copy never landed (the CTA gives up)
  for (int tile = 0; tile < ntile; tile++) {
    if (!bs_mbar_wait(&full[tile % BS_PV_NST], (unsigned)(tile / BS_PV_NST) & 1u)) s_fail = 1;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (s_fail) { failed = tile; break; }   // read after the barrier: the same decision in every thread
    const int r0 = tile * BS_PV_TT;
    bs_chain_tile(vt + (size_t)(tile % BS_PV_NST) * BS_PV_TT * BS_HD + j,
                  sw + r0, nm + (r0 >> 4), min(BS_PV_TT, T - r0), acc, Ssum);
    asm volatile("bar.sync 1, 128;" ::: "memory");   // every chain thread has left the slot: refill it
    if (tid == 0) issue(tile + BS_PV_NST);
  }
  if (failed >= 0) {   // wait (bounded) for the copies still in flight, then report
    if (tid == 0) {
      for (int t = failed; t < min(ntile, failed + BS_PV_NST); t++)
        bs_mbar_wait(&full[t % BS_PV_NST], (unsigned)(t / BS_PV_NST) & 1u);
      atomicExch(&a.ctl->err, 1);
    }
    return;
  }
  if (j == 0) s_S = Ssum;
  asm volatile("bar.sync 1, 128;" ::: "memory");
  const float si = s_S == 0.0f ? 0.0f : __fdiv_rn(1.0f, s_S);
  a.atto[(size_t)h * BS_HD + j] = __fmul_rn(acc, si);
  // the second head of each pair to finish quantises the pair's 256 outputs
  // (one Q8_K block); the first one's stores are visible through the fence
  __threadfence();
  asm volatile("bar.sync 1, 128;" ::: "memory");
  if (tid == 0) s_last = atomicAdd(&a.ctl->pv_pair[h >> 1], 1u) == 1u;
  asm volatile("bar.sync 1, 128;" ::: "memory");
  if (!s_last) return;
  __threadfence();
  float* y = reinterpret_cast<float*>(vt);   // [256] staging
  const float* src = a.atto + (size_t)(h & ~1) * BS_HD;
#pragma unroll
  for (int k = 0; k < 2; k++) y[tid + 128 * k] = __ldcg(src + tid + 128 * k);
  asm volatile("bar.sync 1, 128;" ::: "memory");
  if (w == 0) pb_q8k_block256_warp(y, a.xq + (size_t)(h >> 1) * 292);
  if (tid == 0) a.ctl->pv_pair[h >> 1] = 0u;
}

// -------------------------------------------------------- silu(g)*u + Q8_K
struct BsSiluArgs {
  const float* gu;   // [2F]: gate rows then up rows
  uint8_t* xq;       // [F/256][292]
  int F;
};
__global__ void __launch_bounds__(256) k_bs_silu_q8k(BsSiluArgs a) {
  __shared__ Q8kScratch q8s;
  pb_grid_wait();
  pb_grid_launch_dependents();
  const int i = blockIdx.x * 256 + threadIdx.x;
  const float g = a.gu[i], u = a.gu[a.F + i];
  const float v = bs_silu_mul(g, u);
  pb_q8k_block256(v, a.xq + (size_t)blockIdx.x * 292, q8s);
}

// ------------------------------------------------- Q8_K of a vector
// the TurboQuant attention's output (fp32 [QD]) for the o projection
struct BsQ8kArgs {
  const float* x;
  uint8_t* xq;   // [n / 256][292]
};
__global__ void __launch_bounds__(256) k_bs_q8k(BsQ8kArgs a) {
  __shared__ Q8kScratch q8s;
  pb_grid_wait();
  pb_grid_launch_dependents();
  pb_q8k_block256(a.x[blockIdx.x * 256 + threadIdx.x], a.xq + (size_t)blockIdx.x * 292, q8s);
}

// ------------------------------------------------------------- argmax
struct BsArgmaxArgs {
  const float* lg;
  int V;
  BsCtl* ctl;
};
// fwd8.c:465-469: the first index of the maximum. Per-CTA best -> slot; the
// last CTA reduces the slots, publishes the id and advances the step.
__global__ void __launch_bounds__(256) k_bs_argmax(BsArgmaxArgs a) {
  __shared__ float bv[8];
  __shared__ int bi[8];
  __shared__ int am_last;
  pb_grid_wait();
  pb_grid_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float b = -INFINITY;
  int ix = 0x7fffffff;
  for (int i = blockIdx.x * 256 + threadIdx.x; i < a.V; i += gridDim.x * 256) {
    const float v = a.lg[i];
    if (v > b || (v == b && i < ix)) { b = v; ix = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_down_sync(0xffffffffu, b, o);
    const int oi = __shfl_down_sync(0xffffffffu, ix, o);
    if (ov > b || (ov == b && oi < ix)) { b = ov; ix = oi; }
  }
  if (lane == 0) { bv[warp] = b; bi[warp] = ix; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < 8; w++)
      if (bv[w] > bv[0] || (bv[w] == bv[0] && bi[w] < bi[0])) { bv[0] = bv[w]; bi[0] = bi[w]; }
    a.ctl->slot_val[blockIdx.x] = bv[0];
    a.ctl->slot_idx[blockIdx.x] = bi[0];
    __threadfence();
    am_last = atomicAdd(&a.ctl->counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!am_last) return;
  // the last CTA reduces the slots (read through L2) the same way
  __threadfence();
  b = -INFINITY;
  ix = 0x7fffffff;
  for (int k = threadIdx.x; k < (int)gridDim.x; k += 256) {
    const float ov = __ldcg(&a.ctl->slot_val[k]);
    const int oi = __ldcg(&a.ctl->slot_idx[k]);
    if (ov > b || (ov == b && oi < ix)) { b = ov; ix = oi; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_down_sync(0xffffffffu, b, o);
    const int oi = __shfl_down_sync(0xffffffffu, ix, o);
    if (ov > b || (ov == b && oi < ix)) { b = ov; ix = oi; }
  }
  __syncthreads();
  if (lane == 0) { bv[warp] = b; bi[warp] = ix; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float best = bv[0];
    int id = bi[0];
    for (int w = 1; w < 8; w++)
      if (bv[w] > best || (bv[w] == best && bi[w] < id)) { best = bv[w]; id = bi[w]; }
    // no finite maximum (all NaN): index 0, as the serial scan leaves it
    // (and a NaN first logit, which the serial scan never leaves)
    if (id == 0x7fffffff || a.lg[0] != a.lg[0]) { id = 0; best = a.lg[0]; }
    a.ctl->top = id;
    a.ctl->topv = best;
    if (a.ctl->ids) a.ctl->ids[a.ctl->step] = id;
    a.ctl->step += 1;
    a.ctl->token = id;
    a.ctl->pos += 1;
    a.ctl->counter = 0;
  }
}

template <typename Args>
int bs_launch(void (*k)(Args), dim3 grid, int block, size_t smem, cudaStream_t st, const Args& args,
              const char* name) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k, args);
  if (e != cudaSuccess) return pb_set_error(PB_ECUDA, "launch %s: %s", name, cudaGetErrorString(e));
  pb_count_launch();
  return PB_OK;
}

size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

// ===================================================================== host
struct pb_bonsai {
  pb_bonsai_cfg c{};
  int device = 0;
  int QD = 0, KD = 0;
  // per layer: merged q|k|v, o, merged gate|up, down (views into one arena)
  std::vector<pb_q1> qkv, o, gu, down;
  pb_q1 emb, head;
  char* arena = nullptr;
  float* norms = nullptr;   // [layer][attn H | ffn H | q 128 | k 128], then output_norm [H]
  std::vector<unsigned> have;   // per layer bit mask of tensors and norms set
  unsigned have_top = 0;        // embed 1, head 2, output norm 4
  size_t weight_bytes = 0;
};

struct pb_bonsai_state {
  pb_bonsai* m = nullptr;
  int max_ctx = 0;
  char* mem = nullptr;
  char* tq_mem = nullptr;   // the TurboQuant cache's allocation
  uint16_t* kv = nullptr;   // [layer][2][NKV][max_ctx][128]
  float* rope = nullptr;    // [max_ctx][128]
  float* x[2] = {nullptr, nullptr};
  float* xin = nullptr;
  float* qkv = nullptr;
  uint16_t* qh = nullptr;
  float* scores = nullptr;
  float* atto = nullptr;
  float* ao = nullptr;
  float* gu = nullptr;
  float* fo = nullptr;
  uint8_t* xq = nullptr;
  float* logits = nullptr;
  BsCtl* ctl = nullptr;
  BsCtl* h_ctl = nullptr;   // pinned mirror for uploads
  // TurboQuant K/V cache (kv_bits 3, 4 or 43; 0: the f16 cache `kv`)
  int kv_bits = 0;
  uint32_t* tq_kc = nullptr;   // [layer][n_kv][max_ctx][CW(bk)]
  uint32_t* tq_vc = nullptr;   // [layer][n_kv][max_ctx][CW(bv)]
  float* tq_ks = nullptr;      // [layer][n_kv][max_ctx]
  float* tq_vs = nullptr;
  uint16_t* tq_stage = nullptr;   // [2 n_kv][128] f16: the rows of the current position
  float* tq_qf = nullptr;         // [n_heads][128] post-rope q
  float* tq_scratch = nullptr;
  cudaGraphExec_t graph = nullptr;
  uint64_t graph_launches = 0;   // kernels per graph launch
  int final_x = 0;          // which x buffer holds the residual after a step
};

namespace {

size_t pv_smem(int max_ctx) {
  return (size_t)4 * max_ctx + (size_t)4 * bs_skew_len(max_ctx) + (size_t)BS_PV_NST * BS_PV_TT * BS_HD * 2 +
         (size_t)bs_nm_len(max_ctx);
}

// fwd8.c:322-358 (yarn_corr_dim, yarn_init, rope_table) for every position,
// written as gcc's default (contracting) build computes it: msc = fma(0.1,
// ln factor, 1), th = fma(ti, 1 - ramp, te*ramp)
float bs_corr_dim(int n_ctx, float rot, float base) {
  return 128 * logf(n_ctx / (rot * 2 * (float)M_PI)) / (2 * logf(base));
}
void bs_rope_table(const pb_bonsai_cfg& c, int pos, float* cs) {
  const float st = floorf(bs_corr_dim(c.rope_orig_ctx, 32.0f, c.rope_base));
  const float en = ceilf(bs_corr_dim(c.rope_orig_ctx, 1.0f, c.rope_base));
  const float c0 = st > 0 ? st : 0, c1 = en < 127 ? en : 127;
  const float fs = 1.0f / c.rope_factor, msc = fmaf(0.1f, logf(c.rope_factor), 1.0f);
  const float tscale = powf(c.rope_base, -2.0f / 128.0f);
  float theta = (float)pos;
  for (int j = 0; j < 64; j++, theta *= tscale) {
    const float y = (j - c0) / fmaxf(0.001f, c1 - c0);
    const float ramp = 1.0f - fminf(1.0f, fmaxf(0.0f, y));
    const float ti = fs * theta, te = theta;
    const float th = fmaf(ti, 1 - ramp, te * ramp);
    cs[j] = cosf(th) * msc;
    cs[64 + j] = sinf(th) * msc;
  }
}

int bs_check_ready(const pb_bonsai* m) {
  for (int L = 0; L < m->c.n_layers; L++)
    if (m->have[L] != 0x7ffu) return pb_set_error(PB_EINVAL, "bonsai: layer %d incomplete (mask 0x%x)", L, m->have[L]);
  if ((m->have_top & 5u) != 5u) return pb_set_error(PB_EINVAL, "bonsai: token_embd or output_norm missing");
  return PB_OK;
}

// the whole token as launches on st (captured into the state's graph)
int bs_record(pb_bonsai* m, pb_bonsai_state* s, cudaStream_t st) {
  const pb_bonsai_cfg& c = m->c;
  const int H = c.hidden, F = c.inter, NH = c.n_heads, NKV = c.n_kv;
  int rc;
  int cur = 0;
  const pb_q1& hd = (m->have_top & 2u) ? m->head : m->emb;
  {
    BsEmbedArgs a{m->emb.bits, m->emb.scales, s->xin, s->x[cur], H, s->ctl};
    if ((rc = bs_launch(k_bs_embed, dim3((H + 255) / 256), 256, 0, st, a, "k_bs_embed"))) return rc;
  }
  const size_t nsm = (size_t)H * 4;
  for (int L = 0; L < c.n_layers; L++) {
    const float* nw = m->norms + (size_t)L * (2 * H + 2 * BS_HD);
    uint16_t* kc = s->kv + (size_t)L * 2 * NKV * s->max_ctx * BS_HD;
    uint16_t* vc = kc + (size_t)NKV * s->max_ctx * BS_HD;
    {   // [x += down output] ; rms(attn_norm) ; Q8_K
      BsNormArgs a{s->x[cur], L ? s->fo : nullptr, s->x[cur ^ 1], nw, s->xq, H, s->ctl};
      if (L) cur ^= 1;
      if ((rc = bs_launch(k_bs_norm, dim3(H / 256), 256, nsm, st, a, "k_bs_norm"))) return rc;
    }
    if ((rc = pb_q1_gemv_launch(&m->qkv[L], s->xq, s->qkv, nullptr, st, true))) return rc;
    {
      BsPreArgs a{s->qkv, nw + 2 * H, nw + 2 * H + BS_HD, s->rope, s->qh, kc, vc, NH, NKV, s->max_ctx, s->ctl,
                  s->tq_qf, s->tq_stage};
      if ((rc = bs_launch(k_bs_attn_pre, dim3(NH + 2 * NKV), 32, 0, st, a, "k_bs_attn_pre"))) return rc;
    }
    if (s->kv_bits) {   // TurboQuant: code the rows of this position, attend over the codes
      const int bk = pb_tq_bk(s->kv_bits), bv = pb_tq_bv(s->kv_bits);
      const size_t rows = (size_t)NKV * s->max_ctx;
      uint32_t* tkc = s->tq_kc + (size_t)L * rows * pb_tq_cw(bk);
      uint32_t* tvc = s->tq_vc + (size_t)L * rows * pb_tq_cw(bv);
      float* tks = s->tq_ks + (size_t)L * rows;
      float* tvs = s->tq_vs + (size_t)L * rows;
      if ((rc = pb_tq_store_launch(s->kv_bits, s->tq_stage, &s->ctl->pos, 0, tkc, tks, tvc, tvs, NKV, s->max_ctx, st,
                                   true)))
        return rc;
      if ((rc = pb_tq_attention_launch(s->kv_bits, s->tq_qf, tkc, tks, tvc, tvs, NKV, s->max_ctx, 0, &s->ctl->pos,
                                       s->atto, s->tq_scratch, st, true)))
        return rc;
      BsQ8kArgs a{s->atto, s->xq};
      if ((rc = bs_launch(k_bs_q8k, dim3(m->QD / 256), 256, 0, st, a, "k_bs_q8k"))) return rc;
    } else {
      {
        BsQkArgs a{s->qh, kc, s->scores, NH, NKV, s->max_ctx, c.attn_scale, s->ctl};
        if ((rc = bs_launch(k_bs_fa_qk, dim3(s->max_ctx / 32, NKV), 32 * (NH / NKV), 0, st, a, "k_bs_fa_qk"))) return rc;
      }
      {
        BsPvArgs a{s->scores, vc, s->atto, s->xq, NH, NKV, s->max_ctx, s->ctl};
        if ((rc = bs_launch(k_bs_fa_pv, dim3(NH), 256, pv_smem(s->max_ctx), st, a, "k_bs_fa_pv"))) return rc;
      }
    }
    if ((rc = pb_q1_gemv_launch(&m->o[L], s->xq, s->ao, nullptr, st, true))) return rc;
    {   // x += attention output ; rms(ffn_norm) ; Q8_K
      BsNormArgs a{s->x[cur], s->ao, s->x[cur ^ 1], nw + H, s->xq, H, s->ctl};
      cur ^= 1;
      if ((rc = bs_launch(k_bs_norm, dim3(H / 256), 256, nsm, st, a, "k_bs_norm"))) return rc;
    }
    if ((rc = pb_q1_gemv_launch(&m->gu[L], s->xq, s->gu, nullptr, st, true))) return rc;
    {
      BsSiluArgs a{s->gu, s->xq, F};
      if ((rc = bs_launch(k_bs_silu_q8k, dim3(F / 256), 256, 0, st, a, "k_bs_silu_q8k"))) return rc;
    }
    if ((rc = pb_q1_gemv_launch(&m->down[L], s->xq, s->fo, nullptr, st, true))) return rc;
  }
  {   // x += last down output ; rms(output_norm) ; Q8_K
    BsNormArgs a{s->x[cur], s->fo, s->x[cur ^ 1], m->norms + (size_t)c.n_layers * (2 * H + 2 * BS_HD), s->xq, H, s->ctl};
    cur ^= 1;
    if ((rc = bs_launch(k_bs_norm, dim3(H / 256), 256, nsm, st, a, "k_bs_norm"))) return rc;
  }
  if ((rc = pb_q1_gemv_launch(&hd, s->xq, s->logits, nullptr, st, true))) return rc;
  {
    BsArgmaxArgs a{s->logits, c.vocab, s->ctl};
    if ((rc = bs_launch(k_bs_argmax, dim3(BS_AM_CTAS), 256, 0, st, a, "k_bs_argmax"))) return rc;
  }
  s->final_x = cur;
  return PB_OK;
}

int bs_graph(pb_bonsai* m, pb_bonsai_state* s, cudaStream_t st) {
  if (s->graph) return PB_OK;
  if (bs_check_ready(m)) return PB_EINVAL;
  cudaStream_t cap;
  PB_TRY_CUDA(cudaStreamCreateWithFlags(&cap, cudaStreamNonBlocking));
  PB_TRY_CUDA(cudaFuncSetAttribute(k_bs_fa_pv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pv_smem(s->max_ctx)));
  PB_TRY_CUDA(cudaFuncSetAttribute(k_bs_norm, cudaFuncAttributeMaxDynamicSharedMemorySize, m->c.hidden * 4));
  pb_set_capturing(true);
  cudaGraph_t g = nullptr;
  const int L = m->c.n_layers;
  s->graph_launches = (uint64_t)L * (s->kv_bits ? 14 : 10) + 4;
  int rc = PB_OK;
  if (cudaStreamBeginCapture(cap, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
    rc = pb_set_error(PB_ECUDA, "bonsai: begin capture");
  } else {
    rc = bs_record(m, s, cap);
    cudaError_t e = cudaStreamEndCapture(cap, &g);
    if (rc == PB_OK && e != cudaSuccess) rc = pb_set_error(PB_ECUDA, "bonsai: end capture: %s", cudaGetErrorString(e));
  }
  pb_set_capturing(false);
  if (rc == PB_OK && cudaGraphInstantiate(&s->graph, g, 0) != cudaSuccess)
    rc = pb_set_error(PB_ECUDA, "bonsai: instantiate: %s", cudaGetErrorString(cudaGetLastError()));
  if (g) cudaGraphDestroy(g);
  cudaStreamDestroy(cap);
  (void)st;
  return rc;
}

// upload token/pos (and the input-row flag) then run the graph
int bs_step(pb_bonsai* m, pb_bonsai_state* s, int token, int pos, int use_x, cudaStream_t st) {
  if (pos < 0 || pos >= s->max_ctx) return pb_set_error(PB_EINVAL, "bonsai: pos %d outside [0, %d)", pos, s->max_ctx);
  if (!use_x && (token < 0 || token >= m->c.vocab)) return pb_set_error(PB_EINVAL, "bonsai: token %d", token);
  int rc;
  if ((rc = bs_graph(m, s, st))) return rc;
  // from pageable memory: staged at call time, so back-to-back calls cannot
  // overwrite a pending upload
  const int hdr[4] = {token, pos, 0, use_x};
  PB_TRY_CUDA(cudaMemcpyAsync(s->ctl, hdr, sizeof hdr, cudaMemcpyHostToDevice, st));
  PB_TRY_CUDA(cudaGraphLaunch(s->graph, st));
  pb_count_launch(s->graph_launches);
  return PB_OK;
}

}  // namespace

// =================================================================== C ABI
extern "C" int pb_bonsai_create(const pb_bonsai_cfg* cfg, int device, pb_bonsai** out) {
  if (!cfg || !out) return pb_set_error(PB_EINVAL, "pb_bonsai_create: null argument");
  *out = nullptr;
  const pb_bonsai_cfg& c = *cfg;
  if (c.hidden <= 0 || c.hidden % 256 || c.hidden > 8192 || c.inter <= 0 || c.inter % 256 ||
      c.n_layers <= 0 || c.n_heads <= 0 || c.n_kv <= 0 || c.n_heads % c.n_kv || c.n_heads % 2 ||
      c.n_heads > 128 || c.n_heads / c.n_kv > 8 || c.vocab <= 0)
    return pb_set_error(PB_EINVAL, "pb_bonsai_create: unsupported shape (hidden %% 256, <= 8192; "
                                   "inter %% 256; n_heads even and <= 128; n_heads/n_kv <= 8)");
  PB_TRY_CUDA(cudaSetDevice(device));
  pb_bonsai* m = new pb_bonsai();
  m->c = c;
  m->device = device;
  m->QD = c.n_heads * BS_HD;
  m->KD = c.n_kv * BS_HD;
  const int H = c.hidden, F = c.inter, L = c.n_layers;
  auto bytes = [](int rows, int K) { return a256((size_t)rows * (K / 32) * 4) + a256((size_t)rows * (K / 128) * 2); };
  const size_t layer_b = bytes(m->QD + 2 * m->KD, H) + bytes(H, m->QD) + bytes(2 * F, H) + bytes(H, F);
  const size_t norm_b = a256(((size_t)L * (2 * H + 2 * BS_HD) + H) * 4);
  const size_t tot = layer_b * L + 2 * bytes(c.vocab, H) + norm_b;
  if (cudaMalloc(&m->arena, tot) != cudaSuccess) {
    cudaGetLastError();
    delete m;
    return pb_set_error(PB_ENOMEM, "pb_bonsai_create: %zu bytes", tot);
  }
  char* p = m->arena;
  auto carve = [&](pb_q1& t, int rows, int K) {
    t.rows = rows; t.K = K; t.owner = false;
    t.bits = reinterpret_cast<uint32_t*>(p); p += a256((size_t)rows * (K / 32) * 4);
    t.scales = reinterpret_cast<uint16_t*>(p); p += a256((size_t)rows * (K / 128) * 2);
  };
  m->qkv.resize(L); m->o.resize(L); m->gu.resize(L); m->down.resize(L);
  for (int l = 0; l < L; l++) {
    carve(m->qkv[l], m->QD + 2 * m->KD, H);
    carve(m->o[l], H, m->QD);
    carve(m->gu[l], 2 * F, H);
    carve(m->down[l], H, F);
  }
  carve(m->emb, c.vocab, H);
  carve(m->head, c.vocab, H);
  m->norms = reinterpret_cast<float*>(p);
  m->have.assign(L, 0u);
  m->weight_bytes = tot;
  *out = m;
  return PB_OK;
}

extern "C" int pb_bonsai_destroy(pb_bonsai* m) {
  if (!m) return PB_OK;
  cudaSetDevice(m->device);
  cudaFree(m->arena);
  delete m;
  return PB_OK;
}

extern "C" int pb_bonsai_set_q1(pb_bonsai* m, int layer, int slot, const uint8_t* blocks, int src_on_device,
                                void* stream) {
  if (!m || !blocks) return pb_set_error(PB_EINVAL, "pb_bonsai_set_q1: null argument");
  const pb_bonsai_cfg& c = m->c;
  pb_q1* t = nullptr;
  int rows = 0, row0 = 0;
  unsigned bit = 0;
  if (layer < 0) {
    if (slot == PB_BS_EMBED) { t = &m->emb; rows = c.vocab; bit = 1; }
    else if (slot == PB_BS_HEAD) { t = &m->head; rows = c.vocab; bit = 2; }
  } else if (layer < c.n_layers) {
    switch (slot) {
      case PB_BS_Q: t = &m->qkv[layer]; rows = m->QD; row0 = 0; break;
      case PB_BS_K: t = &m->qkv[layer]; rows = m->KD; row0 = m->QD; break;
      case PB_BS_V: t = &m->qkv[layer]; rows = m->KD; row0 = m->QD + m->KD; break;
      case PB_BS_O: t = &m->o[layer]; rows = c.hidden; break;
      case PB_BS_GATE: t = &m->gu[layer]; rows = c.inter; row0 = 0; break;
      case PB_BS_UP: t = &m->gu[layer]; rows = c.inter; row0 = c.inter; break;
      case PB_BS_DOWN: t = &m->down[layer]; rows = c.hidden; break;
      default: break;
    }
    bit = 1u << slot;
  }
  if (!t) return pb_set_error(PB_EINVAL, "pb_bonsai_set_q1: bad layer %d / slot %d", layer, slot);
  PB_TRY_CUDA(cudaSetDevice(m->device));
  cudaStream_t st = (cudaStream_t)stream;
  const size_t nbytes = (size_t)rows * (t->K / 128) * 18;
  const uint8_t* src = blocks;
  uint8_t* tmp = nullptr;
  if (!src_on_device) {
    PB_TRY_CUDA(cudaMalloc(&tmp, nbytes));
    if (cudaMemcpyAsync(tmp, blocks, nbytes, cudaMemcpyHostToDevice, st) != cudaSuccess) {
      cudaFree(tmp);
      return pb_set_error(PB_ECUDA, "pb_bonsai_set_q1: upload");
    }
    src = tmp;
  }
  int rc = pb_q1_pack_into(t, src, rows, row0, st);
  if (rc == PB_OK && cudaStreamSynchronize(st) != cudaSuccess)
    rc = pb_set_error(PB_ECUDA, "pb_bonsai_set_q1: %s", cudaGetErrorString(cudaGetLastError()));
  cudaFree(tmp);
  if (rc == PB_OK) {
    if (layer < 0) m->have_top |= bit; else m->have[layer] |= bit;
  }
  return rc;
}

extern "C" int pb_bonsai_set_norm(pb_bonsai* m, int layer, int slot, const float* w, int src_on_device,
                                  void* stream) {
  if (!m || !w) return pb_set_error(PB_EINVAL, "pb_bonsai_set_norm: null argument");
  const pb_bonsai_cfg& c = m->c;
  const int H = c.hidden;
  size_t off = 0, n = 0;
  if (layer < 0 && slot == PB_BS_OUT_NORM) { off = (size_t)c.n_layers * (2 * H + 2 * BS_HD); n = H; }
  else if (layer >= 0 && layer < c.n_layers && slot >= PB_BS_ATTN_NORM && slot <= PB_BS_K_NORM) {
    const size_t base = (size_t)layer * (2 * H + 2 * BS_HD);
    const size_t offs[4] = {0, (size_t)H, 2 * (size_t)H, 2 * (size_t)H + BS_HD};
    off = base + offs[slot];
    n = slot < PB_BS_Q_NORM ? H : BS_HD;
  } else {
    return pb_set_error(PB_EINVAL, "pb_bonsai_set_norm: bad layer %d / slot %d", layer, slot);
  }
  PB_TRY_CUDA(cudaSetDevice(m->device));
  cudaStream_t st = (cudaStream_t)stream;
  PB_TRY_CUDA(cudaMemcpyAsync(m->norms + off, w, n * 4, src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, st));
  PB_TRY_CUDA(cudaStreamSynchronize(st));
  if (layer < 0) m->have_top |= 4u; else m->have[layer] |= 1u << (7 + slot);
  return PB_OK;
}

namespace {
int bs_state_create(pb_bonsai* m, int max_ctx, uint16_t* kv_ext, int kv_bits, const PbTqCache* tq_ext,
                    pb_bonsai_state** out) {
  if (!m || !out || max_ctx <= 0 || max_ctx % 32) return pb_set_error(PB_EINVAL, "pb_bonsai_state_create: bad argument (max_ctx a positive multiple of 32)");
  *out = nullptr;
  if (pv_smem(max_ctx) > 200 * 1024) return pb_set_error(PB_ENOTSUP, "pb_bonsai_state_create: max_ctx %d too large for the attention kernel (<= 8192)", max_ctx);
  PB_TRY_CUDA(cudaSetDevice(m->device));
  const pb_bonsai_cfg& c = m->c;
  const int H = c.hidden, F = c.inter, NH = c.n_heads, NKV = c.n_kv;
  pb_bonsai_state* s = new pb_bonsai_state();
  s->m = m;
  s->max_ctx = max_ctx;
  if (kv_bits && !(kv_bits == 3 || kv_bits == 4 || kv_bits == 43))
    return pb_set_error(PB_EINVAL, "pb_bonsai_state_create: K/V bits %d (0, 3, 4 or 43)", kv_bits);
  if (kv_bits && (NH != 4 * NKV || NKV > 16))
    return pb_set_error(PB_ENOTSUP, "pb_bonsai_state_create: the TurboQuant cache needs n_heads = 4 n_kv <= 64");
  const size_t kvb = (kv_ext || kv_bits) ? 0 : (size_t)c.n_layers * 2 * NKV * max_ctx * BS_HD * 2;
  const int kmax = std::max(std::max(H, F), m->QD);
  const size_t sizes[] = {kvb, (size_t)max_ctx * BS_HD * 4, (size_t)H * 4, (size_t)H * 4, (size_t)H * 4,
                          (size_t)(m->QD + 2 * m->KD) * 4, (size_t)NH * BS_HD * 2, (size_t)NH * max_ctx * 4,
                          (size_t)m->QD * 4, (size_t)H * 4, (size_t)2 * F * 4, (size_t)H * 4,
                          (size_t)(kmax / 256) * 292, (size_t)c.vocab * 4, sizeof(BsCtl)};
  size_t tot = 0;
  for (size_t x : sizes) tot += a256(x);
  if (cudaMalloc(&s->mem, tot) != cudaSuccess) {
    cudaGetLastError();
    delete s;
    return pb_set_error(PB_ENOMEM, "pb_bonsai_state_create: %zu bytes", tot);
  }
  char* p = s->mem;
  size_t k = 0;
  auto take = [&]() { char* r = p; p += a256(sizes[k++]); return r; };
  s->kv = reinterpret_cast<uint16_t*>(take());
  if (kv_ext) s->kv = kv_ext;
  s->rope = reinterpret_cast<float*>(take());
  s->x[0] = reinterpret_cast<float*>(take());
  s->x[1] = reinterpret_cast<float*>(take());
  s->xin = reinterpret_cast<float*>(take());
  s->qkv = reinterpret_cast<float*>(take());
  s->qh = reinterpret_cast<uint16_t*>(take());
  s->scores = reinterpret_cast<float*>(take());
  s->atto = reinterpret_cast<float*>(take());
  s->ao = reinterpret_cast<float*>(take());
  s->gu = reinterpret_cast<float*>(take());
  s->fo = reinterpret_cast<float*>(take());
  s->xq = reinterpret_cast<uint8_t*>(take());
  s->logits = reinterpret_cast<float*>(take());
  s->ctl = reinterpret_cast<BsCtl*>(take());
  int rc = PB_OK;
  if (cudaMemset(s->mem, 0, tot) != cudaSuccess) rc = pb_set_error(PB_ECUDA, "pb_bonsai_state_create: memset");
  if (rc == PB_OK && kv_bits) {   // the TurboQuant cache (unless the caller's) and its scratch, in a second allocation
    const size_t rows = tq_ext ? 0 : (size_t)c.n_layers * NKV * max_ctx;
    const size_t tsz[] = {rows * pb_tq_cw(pb_tq_bk(kv_bits)) * 4, rows * pb_tq_cw(pb_tq_bv(kv_bits)) * 4, rows * 4,
                          rows * 4, (size_t)2 * NKV * BS_HD * 2, (size_t)m->QD * 4,
                          pb_tq_scratch_floats(NKV, max_ctx) * 4};
    size_t ttot = 0;
    for (size_t x : tsz) ttot += a256(x);
    if (cudaMalloc(&s->tq_mem, ttot) != cudaSuccess || cudaMemset(s->tq_mem, 0, ttot) != cudaSuccess) {
      cudaGetLastError();
      rc = pb_set_error(PB_ENOMEM, "pb_bonsai_state_create: TurboQuant cache of %zu bytes", ttot);
    } else {
      char* q = s->tq_mem;
      int k2 = 0;
      auto tk = [&]() { char* r = q; q += a256(tsz[k2++]); return r; };
      s->tq_kc = reinterpret_cast<uint32_t*>(tk());
      s->tq_vc = reinterpret_cast<uint32_t*>(tk());
      s->tq_ks = reinterpret_cast<float*>(tk());
      s->tq_vs = reinterpret_cast<float*>(tk());
      s->tq_stage = reinterpret_cast<uint16_t*>(tk());
      s->tq_qf = reinterpret_cast<float*>(tk());
      s->tq_scratch = reinterpret_cast<float*>(tk());
      if (tq_ext) { s->tq_kc = tq_ext->kc; s->tq_vc = tq_ext->vc; s->tq_ks = tq_ext->ks; s->tq_vs = tq_ext->vs; }
      s->kv_bits = kv_bits;
    }
  }
  if (rc == PB_OK && cudaMallocHost(&s->h_ctl, sizeof(BsCtl)) != cudaSuccess) rc = pb_set_error(PB_ENOMEM, "pb_bonsai_state_create: pinned");
  if (rc == PB_OK) {
    memset(s->h_ctl, 0, sizeof(BsCtl));
    std::vector<float> tab((size_t)max_ctx * BS_HD);
    for (int pos = 0; pos < max_ctx; pos++) bs_rope_table(c, pos, tab.data() + (size_t)pos * BS_HD);
    if (cudaMemcpy(s->rope, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
      rc = pb_set_error(PB_ECUDA, "pb_bonsai_state_create: rope table");
  }
  if (rc != PB_OK) {
    cudaFree(s->mem); if (s->h_ctl) cudaFreeHost(s->h_ctl); cudaFree(s->tq_mem);
    delete s;
    return rc;
  }
  *out = s;
  return PB_OK;
}
}  // namespace

extern "C" int pb_bonsai_state_create(pb_bonsai* m, int max_ctx, pb_bonsai_state** out) {
  return bs_state_create(m, max_ctx, nullptr, 0, nullptr, out);
}
extern "C" int pb_bonsai_state_create_tq(pb_bonsai* m, int max_ctx, int kv_bits, pb_bonsai_state** out) {
  return bs_state_create(m, max_ctx, nullptr, kv_bits, nullptr, out);
}
int pb_bonsai_state_create_kv(pb_bonsai* m, int max_ctx, uint16_t* d_kv, pb_bonsai_state** out) {
  if (!d_kv) return pb_set_error(PB_EINVAL, "pb_bonsai_state_create_kv: null cache");
  return bs_state_create(m, max_ctx, d_kv, 0, nullptr, out);
}
int pb_bonsai_state_create_tq_ext(pb_bonsai* m, int max_ctx, int kv_bits, const PbTqCache* cache,
                                  pb_bonsai_state** out) {
  if (!cache || !cache->kc || !cache->vc || !cache->ks || !cache->vs || !kv_bits)
    return pb_set_error(PB_EINVAL, "pb_bonsai_state_create_tq_ext: bad cache");
  return bs_state_create(m, max_ctx, nullptr, kv_bits, cache, out);
}

extern "C" int pb_bonsai_state_destroy(pb_bonsai_state* s) {
  if (!s) return PB_OK;
  cudaSetDevice(s->m->device);
  if (s->graph) cudaGraphExecDestroy(s->graph);
  cudaFree(s->mem);
  cudaFree(s->tq_mem);
  cudaFreeHost(s->h_ctl);
  delete s;
  return PB_OK;
}

extern "C" int pb_bonsai_state_kv(pb_bonsai_state* s, int layer, int which, void** d_ptr) {
  if (!s || !d_ptr || layer < 0 || layer >= s->m->c.n_layers || which < 0 || which > 1)
    return pb_set_error(PB_EINVAL, "pb_bonsai_state_kv: bad argument");
  if (s->kv_bits) return pb_set_error(PB_ENOTSUP, "pb_bonsai_state_kv: the state's cache is TurboQuant-coded");
  *d_ptr = s->kv + ((size_t)layer * 2 + which) * s->m->c.n_kv * s->max_ctx * BS_HD;
  return PB_OK;
}

extern "C" int pb_bonsai_state_residual(pb_bonsai_state* s, float* d_x, void* stream) {
  if (!s || !d_x) return pb_set_error(PB_EINVAL, "pb_bonsai_state_residual: null argument");
  PB_TRY_CUDA(cudaMemcpyAsync(d_x, s->x[s->final_x], (size_t)s->m->c.hidden * 4, cudaMemcpyDeviceToDevice,
                              (cudaStream_t)stream));
  return PB_OK;
}

// the caller's rope row for position pos ([cos 64 | sin 64], as fwd8.c's
// host table holds it), for the host hooks; and the device logits
int pb_bonsai_state_set_rope_row(pb_bonsai_state* s, int pos, const float* h_cos, const float* h_sin,
                                 cudaStream_t st) {
  if (!s || pos < 0 || pos >= s->max_ctx) return pb_set_error(PB_EINVAL, "rope row %d", pos);
  PB_TRY_CUDA(cudaMemcpyAsync(s->rope + (size_t)pos * BS_HD, h_cos, 64 * 4, cudaMemcpyHostToDevice, st));
  PB_TRY_CUDA(cudaMemcpyAsync(s->rope + (size_t)pos * BS_HD + 64, h_sin, 64 * 4, cudaMemcpyHostToDevice, st));
  return PB_OK;
}
const float* pb_bonsai_state_logits(const pb_bonsai_state* s) { return s ? s->logits : nullptr; }

extern "C" int pb_bonsai_decode(pb_bonsai* m, pb_bonsai_state* s, int token, int pos, const float* d_x,
                                float* d_logits, int* out_id, void* stream) {
  if (!m || !s || s->m != m) return pb_set_error(PB_EINVAL, "pb_bonsai_decode: bad argument");
  PB_TRY_CUDA(cudaSetDevice(m->device));
  cudaStream_t st = (cudaStream_t)stream;
  if (d_x) PB_TRY_CUDA(cudaMemcpyAsync(s->xin, d_x, (size_t)m->c.hidden * 4, cudaMemcpyDeviceToDevice, st));
  int rc = bs_step(m, s, token, pos, d_x != nullptr, st);
  if (rc) return rc;
  if (d_logits) PB_TRY_CUDA(cudaMemcpyAsync(d_logits, s->logits, (size_t)m->c.vocab * 4, cudaMemcpyDeviceToDevice, st));
  if (out_id) {
    PB_TRY_CUDA(cudaMemcpyAsync(&s->h_ctl->top, &s->ctl->top, sizeof(int), cudaMemcpyDeviceToHost, st));
    PB_TRY_CUDA(cudaStreamSynchronize(st));
    *out_id = s->h_ctl->top;
  }
  return PB_OK;
}

extern "C" int pb_bonsai_decode_greedy(pb_bonsai* m, pb_bonsai_state* s, int token, int pos, int n, int* d_ids,
                                       void* stream) {
  if (!m || !s || s->m != m || n <= 0) return pb_set_error(PB_EINVAL, "pb_bonsai_decode_greedy: bad argument");
  if (pos + n > s->max_ctx) return pb_set_error(PB_EINVAL, "pb_bonsai_decode_greedy: pos %d + %d exceeds max_ctx", pos, n);
  PB_TRY_CUDA(cudaSetDevice(m->device));
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
  if ((rc = bs_graph(m, s, st))) return rc;
  const int hdr[4] = {token, pos, 0, 0};
  PB_TRY_CUDA(cudaMemcpyAsync(s->ctl, hdr, sizeof hdr, cudaMemcpyHostToDevice, st));
  PB_TRY_CUDA(cudaMemcpyAsync(&s->ctl->ids, &d_ids, sizeof(int*), cudaMemcpyHostToDevice, st));
  for (int i = 0; i < n; i++) {
    PB_TRY_CUDA(cudaGraphLaunch(s->graph, st));
    pb_count_launch(s->graph_launches);
  }
  int* null_ids = nullptr;
  PB_TRY_CUDA(cudaMemcpyAsync(&s->ctl->ids, &null_ids, sizeof(int*), cudaMemcpyHostToDevice, st));
  PB_TRY_CUDA(cudaStreamSynchronize(st));
  return PB_OK;
}

extern "C" int pb_bonsai_state_status(pb_bonsai_state* s, void* stream) {
  if (!s) return pb_set_error(PB_EINVAL, "pb_bonsai_state_status: null argument");
  PB_TRY_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  int err = 0;
  PB_TRY_CUDA(cudaMemcpy(&err, &s->ctl->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) return pb_set_error(PB_ECUDA, "bonsai decode: a bounded wait in the attention kernel gave up");
  return PB_OK;
}

extern "C" int pb_bonsai_state_fallbacks(pb_bonsai_state* s, int* out) {
  if (!s || !out) return pb_set_error(PB_EINVAL, "pb_bonsai_state_fallbacks: null argument");
  PB_TRY_CUDA(cudaMemcpy(out, &s->ctl->fallbacks, sizeof(int), cudaMemcpyDeviceToHost));
  return PB_OK;
}

// ====================================================== per-layer blocks
// The attention block and the FFN tail of one layer as fwd8.c's per-layer
// hooks run them (pq1_attn_fused / pq1_ffn_fused, pq1_fwd8_shim.h:24-40; the
// reference's glue: pq1_fwd8_glue.c:1156-1235, :1376-1470): the caller's host
// Q8_K activation of the normed residual in, the block's fp32 output back to
// the host. The kernels are the token step's, so every value equals the one
// the whole-token path computes for that layer.
struct pb_bs_blocks {
  int device = 0;
  // attention: shapes the buffers were sized for
  int H = 0, NH = 0, NKV = 0, max_ctx = 0;
  char* amem = nullptr;
  float *rope = nullptr, *qkv = nullptr, *qf = nullptr, *scores = nullptr, *atto = nullptr, *ao = nullptr;
  uint16_t* qh = nullptr;
  uint8_t* xq = nullptr;   // Q8_K of the block input, then of the attention output
  BsCtl* ctl = nullptr;
  // TurboQuant attention (tq_bits != 0): the current rows, scratch
  int tq_bits = 0, tq_ctx = 0, tq_nkv = 0;
  char* tmem = nullptr;
  uint16_t* stage = nullptr;
  float* tq_scratch = nullptr;
  // FFN tail
  int fH = 0, F = 0;
  char* fmem = nullptr;
  float *gu = nullptr, *fo = nullptr;
  uint8_t *fxq = nullptr, *dxq = nullptr;   // Q8_K of the input; of silu(g)*u (the down activation)
};

namespace {

int bs_carve(const size_t* sizes, int n, char** mem, char** parts) {
  size_t tot = 0;
  for (int i = 0; i < n; i++) tot += a256(sizes[i]);
  if (cudaMalloc(mem, tot) != cudaSuccess) {
    cudaGetLastError();
    *mem = nullptr;
    return pb_set_error(PB_ENOMEM, "bonsai blocks: %zu bytes", tot);
  }
  if (cudaMemset(*mem, 0, tot) != cudaSuccess) {
    cudaFree(*mem);
    *mem = nullptr;
    return pb_set_error(PB_ECUDA, "bonsai blocks: memset");
  }
  char* p = *mem;
  for (int i = 0; i < n; i++) { parts[i] = p; p += a256(sizes[i]); }
  return PB_OK;
}

int bs_blocks_attn_alloc(pb_bs_blocks* b, int H, int NH, int NKV, int max_ctx) {
  if (b->amem && b->H == H && b->NH == NH && b->NKV == NKV && b->max_ctx == max_ctx) return PB_OK;
  cudaFree(b->amem);
  b->amem = nullptr;
  b->H = 0;
  const int QD = NH * BS_HD, KD = NKV * BS_HD;
  const size_t sizes[] = {(size_t)max_ctx * BS_HD * 4, (size_t)(QD + 2 * KD) * 4, (size_t)QD * 4,
                          (size_t)NH * max_ctx * 4, (size_t)QD * 4, (size_t)H * 4, (size_t)QD * 2,
                          (size_t)(std::max(H, QD) / 256) * 292, sizeof(BsCtl)};
  char* parts[9];
  int rc = bs_carve(sizes, 9, &b->amem, parts);
  if (rc) return rc;
  b->rope = reinterpret_cast<float*>(parts[0]);
  b->qkv = reinterpret_cast<float*>(parts[1]);
  b->qf = reinterpret_cast<float*>(parts[2]);
  b->scores = reinterpret_cast<float*>(parts[3]);
  b->atto = reinterpret_cast<float*>(parts[4]);
  b->ao = reinterpret_cast<float*>(parts[5]);
  b->qh = reinterpret_cast<uint16_t*>(parts[6]);
  b->xq = reinterpret_cast<uint8_t*>(parts[7]);
  b->ctl = reinterpret_cast<BsCtl*>(parts[8]);
  b->H = H; b->NH = NH; b->NKV = NKV; b->max_ctx = max_ctx;
  return PB_OK;
}

int bs_blocks_ffn_alloc(pb_bs_blocks* b, int H, int F) {
  if (b->fmem && b->fH == H && b->F == F) return PB_OK;
  cudaFree(b->fmem);
  b->fmem = nullptr;
  b->fH = 0;
  const size_t sizes[] = {(size_t)2 * F * 4, (size_t)H * 4, (size_t)(H / 256) * 292, (size_t)(F / 256) * 292};
  char* parts[4];
  int rc = bs_carve(sizes, 4, &b->fmem, parts);
  if (rc) return rc;
  b->gu = reinterpret_cast<float*>(parts[0]);
  b->fo = reinterpret_cast<float*>(parts[1]);
  b->fxq = reinterpret_cast<uint8_t*>(parts[2]);
  b->dxq = reinterpret_cast<uint8_t*>(parts[3]);
  b->fH = H; b->F = F;
  return PB_OK;
}

}  // namespace

int pb_bs_blocks_create(int device, pb_bs_blocks** out) {
  if (!out) return pb_set_error(PB_EINVAL, "pb_bs_blocks_create: null argument");
  *out = new pb_bs_blocks();
  (*out)->device = device;
  return PB_OK;
}

void pb_bs_blocks_destroy(pb_bs_blocks* b) {
  if (!b) return;
  cudaSetDevice(b->device);
  cudaFree(b->amem);
  cudaFree(b->tmem);
  cudaFree(b->fmem);
  delete b;
}

int pb_bs_attn_block(pb_bs_blocks* b, const pb_q1* wq, const pb_q1* wk, const pb_q1* wv, const pb_q1* wo,
                     const float* d_qn, const float* d_kn, uint16_t* kc, uint16_t* vc, int max_ctx, int npos,
                     float attn_scale, const float* h_cos, const float* h_sin, const uint8_t* h_xq, float* h_ao,
                     cudaStream_t st) {
  if (!b || !wq || !wk || !wv || !wo || !d_qn || !d_kn || !kc || !vc || !h_cos || !h_sin || !h_xq || !h_ao)
    return pb_set_error(PB_EINVAL, "pb_bs_attn_block: null argument");
  const int H = wq->K, QD = wq->rows, KD = wk->rows, NH = QD / BS_HD, NKV = KD / BS_HD;
  if (H % 256 || H > 8192 || QD % 256 || KD % BS_HD || NKV <= 0 || NH % NKV || NH / NKV > 8 || NH > 128 ||
      wk->K != H || wv->K != H || wv->rows != KD || wo->rows != H || wo->K != QD)
    return pb_set_error(PB_EINVAL, "pb_bs_attn_block: shapes q %dx%d k %dx%d v %dx%d o %dx%d", wq->rows, wq->K,
                        wk->rows, wk->K, wv->rows, wv->K, wo->rows, wo->K);
  if (max_ctx <= 0 || max_ctx % 32 || pv_smem(max_ctx) > 200 * 1024 || npos < 0 || npos >= max_ctx)
    return pb_set_error(PB_EINVAL, "pb_bs_attn_block: position %d, cache of %d", npos, max_ctx);
  PB_TRY_CUDA(cudaSetDevice(b->device));
  int rc;
  if ((rc = bs_blocks_attn_alloc(b, H, NH, NKV, max_ctx))) return rc;
  PB_TRY_CUDA(cudaFuncSetAttribute(k_bs_fa_pv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pv_smem(max_ctx)));
  const int hdr[4] = {0, npos, 0, 0};
  PB_TRY_CUDA(cudaMemcpyAsync(b->ctl, hdr, sizeof hdr, cudaMemcpyHostToDevice, st));
  PB_TRY_CUDA(cudaMemcpyAsync(b->rope + (size_t)npos * BS_HD, h_cos, 64 * 4, cudaMemcpyHostToDevice, st));
  PB_TRY_CUDA(cudaMemcpyAsync(b->rope + (size_t)npos * BS_HD + 64, h_sin, 64 * 4, cudaMemcpyHostToDevice, st));
  PB_TRY_CUDA(cudaMemcpyAsync(b->xq, h_xq, (size_t)(H / 256) * 292, cudaMemcpyHostToDevice, st));
  // q, k and v into one [NH + 2 NKV][128] vector, as the merged tensor writes it
  if ((rc = pb_q1_gemv_launch(wq, b->xq, b->qkv, nullptr, st, true))) return rc;
  if ((rc = pb_q1_gemv_launch(wk, b->xq, b->qkv + QD, nullptr, st, true))) return rc;
  if ((rc = pb_q1_gemv_launch(wv, b->xq, b->qkv + QD + KD, nullptr, st, true))) return rc;
  {
    BsPreArgs a{b->qkv, d_qn, d_kn, b->rope, b->qh, kc, vc, NH, NKV, max_ctx, b->ctl, b->qf, nullptr};
    if ((rc = bs_launch(k_bs_attn_pre, dim3(NH + 2 * NKV), 32, 0, st, a, "k_bs_attn_pre"))) return rc;
  }
  {
    BsQkArgs a{b->qh, kc, b->scores, NH, NKV, max_ctx, attn_scale, b->ctl};
    if ((rc = bs_launch(k_bs_fa_qk, dim3(max_ctx / 32, NKV), 32 * (NH / NKV), 0, st, a, "k_bs_fa_qk"))) return rc;
  }
  {
    BsPvArgs a{b->scores, vc, b->atto, b->xq, NH, NKV, max_ctx, b->ctl};
    if ((rc = bs_launch(k_bs_fa_pv, dim3(NH), 256, pv_smem(max_ctx), st, a, "k_bs_fa_pv"))) return rc;
  }
  if ((rc = pb_q1_gemv_launch(wo, b->xq, b->ao, nullptr, st, true))) return rc;
  int err = 0;
  PB_TRY_CUDA(cudaMemcpyAsync(h_ao, b->ao, (size_t)H * 4, cudaMemcpyDeviceToHost, st));
  PB_TRY_CUDA(cudaMemcpyAsync(&err, &b->ctl->err, sizeof(int), cudaMemcpyDeviceToHost, st));
  PB_TRY_CUDA(cudaStreamSynchronize(st));
  if (err) return pb_set_error(PB_ECUDA, "pb_bs_attn_block: a bounded wait in the attention kernel gave up");
  return PB_OK;
}

// the attention block over a TurboQuant cache: the layer's K/V rows of npos are
// coded into it, then the attention runs over the codes (the reference's
// pq1_attn_tq_launch inside pq1_attn_fused)
int pb_bs_attn_block_tq(pb_bs_blocks* b, int bits, const pb_q1* wq, const pb_q1* wk, const pb_q1* wv, const pb_q1* wo,
                        const float* d_qn, const float* d_kn, const PbTqCache* layer, int max_ctx, int npos,
                        const float* h_cos, const float* h_sin, const uint8_t* h_xq, float* h_ao, cudaStream_t st) {
  if (!b || !wq || !wk || !wv || !wo || !d_qn || !d_kn || !layer || !h_cos || !h_sin || !h_xq || !h_ao)
    return pb_set_error(PB_EINVAL, "pb_bs_attn_block_tq: null argument");
  const int H = wq->K, QD = wq->rows, KD = wk->rows, NH = QD / BS_HD, NKV = KD / BS_HD;
  if (H % 256 || H > 8192 || QD % 256 || KD % BS_HD || NKV <= 0 || NKV > 16 || NH != 4 * NKV || wk->K != H ||
      wv->K != H || wv->rows != KD || wo->rows != H || wo->K != QD)
    return pb_set_error(PB_EINVAL, "pb_bs_attn_block_tq: shapes q %dx%d k %dx%d (n_heads = 4 n_kv)", wq->rows, wq->K,
                        wk->rows, wk->K);
  if (max_ctx <= 0 || max_ctx % 32 || npos < 0 || npos >= max_ctx)
    return pb_set_error(PB_EINVAL, "pb_bs_attn_block_tq: position %d, cache of %d", npos, max_ctx);
  PB_TRY_CUDA(cudaSetDevice(b->device));
  int rc;
  if ((rc = bs_blocks_attn_alloc(b, H, NH, NKV, max_ctx))) return rc;
  if (!b->tmem || b->tq_ctx != max_ctx || b->tq_nkv != NKV) {
    cudaFree(b->tmem);
    b->tmem = nullptr;
    const size_t sz[] = {(size_t)2 * NKV * BS_HD * 2, pb_tq_scratch_floats(NKV, max_ctx) * 4};
    char* parts[2];
    if ((rc = bs_carve(sz, 2, &b->tmem, parts))) return rc;
    b->stage = reinterpret_cast<uint16_t*>(parts[0]);
    b->tq_scratch = reinterpret_cast<float*>(parts[1]);
    b->tq_ctx = max_ctx;
    b->tq_nkv = NKV;
  }
  const int hdr[4] = {0, npos, 0, 0};
  PB_TRY_CUDA(cudaMemcpyAsync(b->ctl, hdr, sizeof hdr, cudaMemcpyHostToDevice, st));
  PB_TRY_CUDA(cudaMemcpyAsync(b->rope + (size_t)npos * BS_HD, h_cos, 64 * 4, cudaMemcpyHostToDevice, st));
  PB_TRY_CUDA(cudaMemcpyAsync(b->rope + (size_t)npos * BS_HD + 64, h_sin, 64 * 4, cudaMemcpyHostToDevice, st));
  PB_TRY_CUDA(cudaMemcpyAsync(b->xq, h_xq, (size_t)(H / 256) * 292, cudaMemcpyHostToDevice, st));
  if ((rc = pb_q1_gemv_launch(wq, b->xq, b->qkv, nullptr, st, true))) return rc;
  if ((rc = pb_q1_gemv_launch(wk, b->xq, b->qkv + QD, nullptr, st, true))) return rc;
  if ((rc = pb_q1_gemv_launch(wv, b->xq, b->qkv + QD + KD, nullptr, st, true))) return rc;
  {
    BsPreArgs a{b->qkv, d_qn, d_kn, b->rope, b->qh, nullptr, nullptr, NH, NKV, max_ctx, b->ctl, b->qf, b->stage};
    if ((rc = bs_launch(k_bs_attn_pre, dim3(NH + 2 * NKV), 32, 0, st, a, "k_bs_attn_pre"))) return rc;
  }
  if ((rc = pb_tq_store_launch(bits, b->stage, nullptr, npos, layer->kc, layer->ks, layer->vc, layer->vs, NKV, max_ctx,
                               st, true)))
    return rc;
  if ((rc = pb_tq_attention_launch(bits, b->qf, layer->kc, layer->ks, layer->vc, layer->vs, NKV, max_ctx, npos + 1,
                                   nullptr, b->atto, b->tq_scratch, st, true)))
    return rc;
  {
    BsQ8kArgs a{b->atto, b->xq};
    if ((rc = bs_launch(k_bs_q8k, dim3(QD / 256), 256, 0, st, a, "k_bs_q8k"))) return rc;
  }
  if ((rc = pb_q1_gemv_launch(wo, b->xq, b->ao, nullptr, st, true))) return rc;
  PB_TRY_CUDA(cudaMemcpyAsync(h_ao, b->ao, (size_t)H * 4, cudaMemcpyDeviceToHost, st));
  PB_TRY_CUDA(cudaStreamSynchronize(st));
  return PB_OK;
}

int pb_bs_ffn_block(pb_bs_blocks* b, const pb_q1* wg, const pb_q1* wu, const pb_q1* wd, const uint8_t* h_xq,
                    float* h_fo, cudaStream_t st) {
  if (!b || !wg || !wu || !wd || !h_xq || !h_fo) return pb_set_error(PB_EINVAL, "pb_bs_ffn_block: null argument");
  const int H = wg->K, F = wg->rows;
  if (H % 256 || F % 256 || wu->K != H || wu->rows != F || wd->K != F || wd->rows != H)
    return pb_set_error(PB_EINVAL, "pb_bs_ffn_block: shapes gate %dx%d up %dx%d down %dx%d", wg->rows, wg->K,
                        wu->rows, wu->K, wd->rows, wd->K);
  PB_TRY_CUDA(cudaSetDevice(b->device));
  int rc;
  if ((rc = bs_blocks_ffn_alloc(b, H, F))) return rc;
  PB_TRY_CUDA(cudaMemcpyAsync(b->fxq, h_xq, (size_t)(H / 256) * 292, cudaMemcpyHostToDevice, st));
  if ((rc = pb_q1_gemv_launch(wg, b->fxq, b->gu, nullptr, st, true))) return rc;
  if ((rc = pb_q1_gemv_launch(wu, b->fxq, b->gu + F, nullptr, st, true))) return rc;
  {
    BsSiluArgs a{b->gu, b->dxq, F};
    if ((rc = bs_launch(k_bs_silu_q8k, dim3(F / 256), 256, 0, st, a, "k_bs_silu_q8k"))) return rc;
  }
  if ((rc = pb_q1_gemv_launch(wd, b->dxq, b->fo, nullptr, st, true))) return rc;
  PB_TRY_CUDA(cudaMemcpyAsync(h_fo, b->fo, (size_t)H * 4, cudaMemcpyDeviceToHost, st));
  PB_TRY_CUDA(cudaStreamSynchronize(st));
  return PB_OK;
}

int pb_bs_blocks_attn_debug(pb_bs_blocks* b, float* h_q, float* h_atto, int nh) {
  if (!b || !b->amem || nh != b->NH) return pb_set_error(PB_EINVAL, "pb_bs_blocks_attn_debug: no attention block ran");
  PB_TRY_CUDA(cudaSetDevice(b->device));
  if (h_q) PB_TRY_CUDA(cudaMemcpy(h_q, b->qf, (size_t)nh * BS_HD * 4, cudaMemcpyDeviceToHost));
  if (h_atto) PB_TRY_CUDA(cudaMemcpy(h_atto, b->atto, (size_t)nh * BS_HD * 4, cudaMemcpyDeviceToHost));
  return PB_OK;
}

int pb_bs_blocks_ffn_xq(pb_bs_blocks* b, uint8_t* h_dst, size_t n) {
  if (!b || !b->fmem || !h_dst) return pb_set_error(PB_EINVAL, "pb_bs_blocks_ffn_xq: no FFN block ran");
  PB_TRY_CUDA(cudaSetDevice(b->device));
  const size_t have = (size_t)(b->F / 256) * 292;
  PB_TRY_CUDA(cudaMemcpy(h_dst, b->dxq, n < have ? n : have, cudaMemcpyDeviceToHost));
  return PB_OK;
}
