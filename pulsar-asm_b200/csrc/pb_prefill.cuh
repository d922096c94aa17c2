// pb_prefill.cuh -- the chunked prefill on the integer path: T positions of
// the prompt (T a multiple of 16) through every layer, each projection one
// Q8_0 x Q8_0 GEMM on the tensor cores (pb_q80tc.cu), the per-position steps
// around them (residual, RMSNorm, activation quantiser, short conv, head
// norm, RoPE, GQA attention, SwiGLU, the tied head and the greedy argmax) as
// kernels over the chunk's positions. Each position's values equal the
// decode step's with every projection on the integer path (the oracle's
// integer mode): Linear(x) = bf16(sum_b (dw*dx)*(float)isum_b), x quantised
// per 32-block (fwd35_ref.c:332-343), the layer sequencing of layer_chunk_T
// (lfm3_nanode.cu:4997-5162) with the T=1 step's arithmetic per position.
#pragma once
#include "pb_step.cuh"

namespace {

// Q8_0 activation quantiser on E consecutive values per thread (a 32-block
// spans 32/E threads): d = fp16(amax/127), q = rint(x * 127/amax), 0 when
// amax is 0 -- k_q80_quantize's arithmetic
template <int E>
PB_DEV void pf_quant_store(const float (&x)[E], int8_t* qx, uint16_t* dx, int th) {
  float amax = 0.0f;
#pragma unroll
  for (int j = 0; j < E; j++) amax = fmaxf(amax, fabsf(x[j]));
#pragma unroll
  for (int o = 1; o < 32 / E; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float d = __fdiv_rn(amax, 127.0f);
  const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
  int8_t q[E];
#pragma unroll
  for (int j = 0; j < E; j++) q[j] = (int8_t)rintf(__fmul_rn(x[j], id));
#pragma unroll
  for (int j = 0; j < E; j++) qx[th * E + j] = q[j];
  if (((th * E) & 31) == 0) dx[(th * E) >> 5] = pb_f2h(d);
}

struct PfNormArgs {
  const int* tokens;        // EMBED: the chunk's token ids (null: residual input)
  const uint4* emb_codes;   // tied table, streaming layout
  const void* emb_scales;
  int emb_nch, emb_f32;
  const uint16_t* emb16;    // the bf16 table (head layout) instead
  const bf16_t* rin;        // [T][H] residual (unless EMBED)
  const float* hin;         // [T][H] fp32 projection output to post-normalise and add (null: none)
  const float* wpost;
  const float* wnorm;
  bf16_t* rout;             // [T][H] new residual
  int8_t* qx;               // [T][H]
  uint16_t* dx;             // [T][H/32]
  bf16_t* xout;             // optional [T][H]: x itself (the bf16 head's input)
  int H;
  float eps;
};

// residual (embedding row, or rin + bf16(rms(bf16(hin)))) -> rout; x =
// rms(residual) -> quantised; one CTA per position
template <int E>
__global__ void __launch_bounds__(256) k_pf_norm_quant(PfNormArgs p) {
  __shared__ float red[16];
  const int t = blockIdx.x, th = threadIdx.x, H = p.H;
  float R[E];
  if (p.tokens) {
    // the token's row of the tied table
    const int tok = p.tokens[t];
#pragma unroll
    for (int j = 0; j < E; j++)
      R[j] = emb_value(p.emb_codes, p.emb_scales, p.emb_nch, p.emb_f32, p.emb16, H, tok, th * E + j);
  } else {
    ld_bf<E, 0>(p.rin + (size_t)t * H + (size_t)th * E, R);
    if (p.hin) {
      float Hv[E], wp[E], hn[E];
#pragma unroll
      for (int j = 0; j < E; j++) Hv[j] = pb_bf2f(pb_f2bf(p.hin[(size_t)t * H + th * E + j]));
      ld_f32<E>(p.wpost + (size_t)th * E, wp);
      rms_reg<E, 0>(Hv, wp, hn, H, p.eps, red);
#pragma unroll
      for (int j = 0; j < E; j++) R[j] = pb_bf2f(pb_f2bf(__fadd_rn(R[j], hn[j])));
    }
  }
  st_bf<E>(p.rout + (size_t)t * H + (size_t)th * E, R);
  float wn[E], X[E];
  ld_f32<E>(p.wnorm + (size_t)th * E, wn);
  rms_reg<E, 0>(R, wn, X, H, p.eps, red + 8);
  if (p.xout) st_bf<E>(p.xout + (size_t)t * H + (size_t)th * E, X);
  pf_quant_store<E>(X, p.qx + (size_t)t * H, p.dx + (size_t)t * (H / 32), th);
}

// the head over the bf16 tied table for T positions (k_gemv_bf16,
// lfm3_nanode.cu:3517-3534, per position): a warp per row holds lane l's 64
// weights (k = l + 32 m) and runs each position's chain s = s + bf16(W[k]) *
// x[k] from the positions' x (bf16, up to 32 positions in shared memory at a
// time), then the shuffle-down tree; lg [T][N] fp32 as is. KG = K / 256.
template <int KG>
__global__ void __launch_bounds__(256) k_b16_head_T(const uint16_t* __restrict__ w, const bf16_t* __restrict__ x,
                                                    float* __restrict__ lg, int N, int T) {
  constexpr int K = KG * 256, TG = 32;
  extern __shared__ __align__(16) bf16_t xs[];     // [TG][K]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int t0 = 0; t0 < T; t0 += TG) {
    const int nt = T - t0 < TG ? T - t0 : TG;
    __syncthreads();
    for (int i = threadIdx.x; i < nt * K / 8; i += blockDim.x)
      reinterpret_cast<uint4*>(xs)[i] = reinterpret_cast<const uint4*>(x + (size_t)t0 * K)[i];
    __syncthreads();
    for (int row = blockIdx.x * 8 + warp; row < N; row += gridDim.x * 8) {
      const uint4* g = reinterpret_cast<const uint4*>(w + (size_t)row * K) + lane;
      uint4 q[KG];
#pragma unroll
      for (int h = 0; h < KG; h++) q[h] = pb_ldg_stream(g + 32 * h);
      for (int t = 0; t < nt; t++) {
        const bf16_t* xt = xs + (size_t)t * K + lane;
        float acc = 0.0f;
#pragma unroll
        for (int h = 0; h < KG; h++) {
          const unsigned ws[4] = {q[h].x, q[h].y, q[h].z, q[h].w};
#pragma unroll
          for (int i = 0; i < 4; i++) {
            acc = __fadd_rn(acc, __fmul_rn(pb_lo2f(ws[i]), pb_bf2f(xt[32 * (8 * h + 2 * i)])));
            acc = __fadd_rn(acc, __fmul_rn(pb_hi2f(ws[i]), pb_bf2f(xt[32 * (8 * h + 2 * i + 1)])));
          }
        }
        const float v = pb_warp_tree(acc);
        if (lane == 0) lg[(size_t)(t0 + t) * N + row] = v;
      }
    }
  }
}

struct PfConvArgs {
  const float* y;       // [T][3H] in_proj outputs (B | C | x), fp32
  const bf16_t* ring;   // [W][H] this layer's ring, slot = position mod W (positions before the chunk)
  const float* taps;    // [H][W]
  int8_t* qx;           // [T][H]
  uint16_t* dx;
  int H, pos0;
};

// gated short conv (lfm3_nanode.cu:3790-3818) at one position of the chunk:
// bx_p = bf16(B_p x_p) for the W positions ending at it (from the chunk's
// own in_proj outputs, or the ring before the chunk), y = sum_k taps * bx in
// tap order, out = bf16(C * bf16(y)), then quantised
template <int E, int W>
__global__ void __launch_bounds__(256) k_pf_conv_quant(PfConvArgs p) {
  const int t = blockIdx.x, th = threadIdx.x, H = p.H;
  float out[E];
#pragma unroll
  for (int j = 0; j < E; j++) {
    const int i = th * E + j;
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < W; k++) {
      const int tt = t - (W - 1) + k;
      float bx;
      if (tt >= 0) {
        const float* yr = p.y + (size_t)tt * 3 * H;
        bx = pb_bf2f(pb_f2bf(__fmul_rn(pb_bf2f(pb_f2bf(yr[i])), pb_bf2f(pb_f2bf(yr[2 * H + i])))));
      } else {
        const int pp = p.pos0 + tt;
        bx = pb_bf2f(p.ring[(size_t)(((pp % W) + W) % W) * H + i]);
      }
      acc = __fadd_rn(acc, __fmul_rn(p.taps[(size_t)i * W + k], bx));
    }
    const float C = pb_bf2f(pb_f2bf(p.y[(size_t)t * 3 * H + H + i]));
    out[j] = pb_bf2f(pb_f2bf(__fmul_rn(C, pb_bf2f(pb_f2bf(acc)))));
  }
  pf_quant_store<E>(out, p.qx + (size_t)t * H, p.dx + (size_t)t * (H / 32), th);
}

// the ring after the chunk: slot p mod W holds bx_p of the chunk's last W positions
__global__ void k_pf_ring(const float* __restrict__ y, bf16_t* __restrict__ ring, int H, int W, int T, int pos0) {
  const int k = blockIdx.y;                 // one of the last W positions
  const int tt = T - W + k;
  if (tt < 0) return;
  const int pp = pos0 + tt;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x) {
    const float* yr = y + (size_t)tt * 3 * H;
    ring[(size_t)(pp % W) * H + i] = pb_f2bf(__fmul_rn(pb_bf2f(pb_f2bf(yr[i])), pb_bf2f(pb_f2bf(yr[2 * H + i]))));
  }
}

struct PfQkvArgs {
  const float* y;       // [T][nq] q | k | v | gate projection outputs, fp32
  bf16_t* qkvg;         // [T][nq] the same as bf16
  const float* knorm;
  const float* rope_cos;
  const float* rope_sin;
  unsigned short* kc;   // this layer's caches
  unsigned short* vc;
  int nq, nh, nkv, half, pos0;
  float eps;
};

// one CTA per position: the bf16 projection row, then the new K (head norm,
// RoPE, fp16) and V (fp16) rows of every KV head into the caches -- the rows
// the attention of every later position of the chunk reads
template <int E>
__global__ void __launch_bounds__(256) k_pf_qkv(PfQkvArgs p) {
  constexpr int HD = 32 * E;
  __shared__ float ks[8][HD];
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < p.nq; i += blockDim.x)
    p.qkvg[(size_t)t * p.nq + i] = pb_f2bf(p.y[(size_t)t * p.nq + i]);
  __syncthreads();
  const int pos = p.pos0 + t;
  const size_t koff = (size_t)p.nh * HD, voff = koff + (size_t)p.nkv * HD;
  const bf16_t* row = p.qkvg + (size_t)t * p.nq;
  for (int kvh = warp; kvh < p.nkv; kvh += 8) {
    head_norm_rope<E, 0>(row + koff + (size_t)kvh * HD, p.knorm, p.rope_cos + (size_t)pos * p.half,
                         p.rope_sin + (size_t)pos * p.half, p.half, p.eps, ks[warp]);
#pragma unroll
    for (int j = 0; j < E; j++) {
      const int i = lane * E + j;
      p.kc[((size_t)pos * p.nkv + kvh) * HD + i] = pb_f2h(ks[warp][i]);
      p.vc[((size_t)pos * p.nkv + kvh) * HD + i] = pb_f2h(pb_bf2f(row[voff + (size_t)kvh * HD + i]));
    }
    __syncwarp();
  }
}

// attention of the chunk's positions: CTA (head, position), the decode's
// per-head body (k_attn_head, lfm3_nanode.cu:503-602, gate fused)
template <int E>
__global__ void __launch_bounds__(256) k_pf_attn(AttnArgs a, int pos0, int qstride, int ostride) {
  constexpr int HD = 32 * E;
  extern __shared__ __align__(16) float sl[];     // scores [max_ctx]
  __shared__ float qv[HD], kv[HD], vv[HD];
  __shared__ float red[8];
  __shared__ float segred[8 * HD];
  const int t = blockIdx.y;
  AttnArgs b = a;
  b.qkvg = a.qkvg + (size_t)t * qstride;
  b.out = a.out + (size_t)t * ostride;
  attn_body<E, 0>(b, blockIdx.x, pos0 + t, sl, qv, kv, vv, segred, red);
}

// bf16 rows [T][K] -> quantised (the o_proj input)
template <int E>
__global__ void __launch_bounds__(256) k_pf_quant(const bf16_t* __restrict__ x, int K, int8_t* __restrict__ qx,
                                                  uint16_t* __restrict__ dx) {
  const int t = blockIdx.x, th = threadIdx.x;
  float v[E];
  ld_bf<E, 0>(x + (size_t)t * K + (size_t)th * E, v);
  pf_quant_store<E>(v, qx + (size_t)t * K, dx + (size_t)t * (K / 32), th);
}

// SwiGLU on the interleaved w1|w3 outputs (k_silu_mul_bf, lfm3_nanode.cu:821-829),
// then quantised (the w2 input)
// (F = 256 E, or with E = 32 any multiple of 32 up to 8192: a thread then
// holds one whole 32-block, and threads past F have none)
template <int E>
__global__ void __launch_bounds__(256) k_pf_silu_quant(const float* __restrict__ y, int F, int8_t* __restrict__ qx,
                                                       uint16_t* __restrict__ dx) {
  const int t = blockIdx.x, th = threadIdx.x;
  if (E == 32 && th * E >= F) return;
  float u[E];
#pragma unroll
  for (int j = 0; j < E; j++) {
    const int i = th * E + j;
    const float av = pb_bf2f(pb_f2bf(y[(size_t)t * 2 * F + 2 * i]));
    const float bw = pb_bf2f(pb_f2bf(y[(size_t)t * 2 * F + 2 * i + 1]));
    u[j] = pb_bf2f(pb_f2bf(__fmul_rn(__fmul_rn(av, pb_sigmoid(av)), bw)));
  }
  pf_quant_store<E>(u, qx + (size_t)t * F, dx + (size_t)t * (F / 32), th);
}

// greedy id of each position's logits (ties to the lowest index; a NaN is
// never taken), one CTA per position. Each thread keeps 8 loads in flight:
// the row is read from L2 at its latency once per 8 keys, not once per key.
// The rule does not depend on the order keys are visited in.
constexpr int PF_AM_T = 1024;
__global__ void __launch_bounds__(PF_AM_T) k_pf_argmax(const float* __restrict__ lg, int V, int* __restrict__ ids) {
  __shared__ float bv[PF_AM_T / 32];
  __shared__ int bi[PF_AM_T / 32];
  const int t = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* row = lg + (size_t)t * V;
  float b = -INFINITY;
  int ix = 0x7fffffff;
  for (int base = 0; base < V; base += 8 * PF_AM_T) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int i = base + u * PF_AM_T + threadIdx.x;
      v[u] = i < V ? row[i] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int i = base + u * PF_AM_T + threadIdx.x;
      if (i < V && (v[u] > b || (v[u] == b && i < ix))) { b = v[u]; ix = i; }
    }
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
    for (int w = 1; w < PF_AM_T / 32; w++)
      if (bv[w] > bv[0] || (bv[w] == bv[0] && bi[w] < bi[0])) { bv[0] = bv[w]; bi[0] = bi[w]; }
    ids[t] = bi[0];
  }
}

}  // namespace

// ----------------------------------------------------------- batched decode
// B independent sequences, one position each: the projections are the same
// tensor-core GEMMs (T = B), every per-position step reads and writes its
// own sequence's state.
namespace {

struct SeqPtrs {
  unsigned short* kv;       // [n_attn][2][max_ctx][NKV][HD]
  bf16_t* ring;             // [n_conv][W][H]
  const float* rope_cos;    // [max_ctx][half]: full-attention layers
  const float* rope_sin;
  const float* rope_cos_s;  // [max_ctx][half]: sliding-attention layers
  const float* rope_sin_s;
  int max_ctx;
  int _pad;
};

struct BdArgs {
  const SeqPtrs* seq;       // [B]
  const int* pos;           // [B]
  const float* y;           // [B][nq] projection outputs
  bf16_t* qkvg;             // [B][nq]
  const float* qnorm;
  const float* knorm;
  bf16_t* att;              // [B][NH*HD]
  int attn_idx, nq, nh, nkv, half, win;
  float eps, scaling;
  int slide;                // the layer's RoPE table: 1 sliding, 0 full
};

// per sequence: the bf16 projection row and its new K/V rows
template <int E>
__global__ void __launch_bounds__(256) k_bd_qkv(BdArgs p) {
  constexpr int HD = 32 * E;
  __shared__ float ks[8][HD];
  const int b = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < p.nq; i += blockDim.x)
    p.qkvg[(size_t)b * p.nq + i] = pb_f2bf(p.y[(size_t)b * p.nq + i]);
  __syncthreads();
  const SeqPtrs sq = p.seq[b];
  const int pos = p.pos[b];
  const size_t per = (size_t)sq.max_ctx * p.nkv * HD;
  unsigned short* kc = sq.kv + (size_t)p.attn_idx * 2 * per;
  unsigned short* vc = kc + per;
  const size_t koff = (size_t)p.nh * HD, voff = koff + (size_t)p.nkv * HD;
  const bf16_t* row = p.qkvg + (size_t)b * p.nq;
  for (int kvh = warp; kvh < p.nkv; kvh += 8) {
    head_norm_rope<E, 0>(row + koff + (size_t)kvh * HD, p.knorm, (p.slide ? sq.rope_cos_s : sq.rope_cos) + (size_t)pos * p.half,
                         (p.slide ? sq.rope_sin_s : sq.rope_sin) + (size_t)pos * p.half, p.half, p.eps, ks[warp]);
#pragma unroll
    for (int j = 0; j < E; j++) {
      const int i = lane * E + j;
      kc[((size_t)pos * p.nkv + kvh) * HD + i] = pb_f2h(ks[warp][i]);
      vc[((size_t)pos * p.nkv + kvh) * HD + i] = pb_f2h(pb_bf2f(row[voff + (size_t)kvh * HD + i]));
    }
    __syncwarp();
  }
}

// CTA (head, sequence): the decode's per-head attention over that sequence's cache
template <int E>
__global__ void __launch_bounds__(256) k_bd_attn(BdArgs p) {
  constexpr int HD = 32 * E;
  extern __shared__ __align__(16) float sl[];     // scores [max_ctx of the longest sequence]
  __shared__ float qv[HD], kv[HD], vv[HD];
  __shared__ float red[8];
  __shared__ float segred[8 * HD];
  const int b = blockIdx.y;
  const SeqPtrs sq = p.seq[b];
  AttnArgs a = {};
  a.qkvg = p.qkvg + (size_t)b * p.nq;
  a.qnorm = p.qnorm;
  a.knorm = p.knorm;
  a.rope_cos = p.slide ? sq.rope_cos_s : sq.rope_cos;
  a.rope_sin = p.slide ? sq.rope_sin_s : sq.rope_sin;
  const size_t per = (size_t)sq.max_ctx * p.nkv * HD;
  a.kc = sq.kv + (size_t)p.attn_idx * 2 * per;
  a.vc = a.kc + per;
  a.out = p.att + (size_t)b * p.nh * HD;
  a.nh = p.nh; a.nkv = p.nkv; a.half = p.half; a.win = p.win; a.max_ctx = sq.max_ctx;
  a.scaling = p.scaling;
  a.eps = p.eps;
  attn_body<E, 0>(a, blockIdx.x, p.pos[b], sl, qv, kv, vv, segred, red);
}

struct BdConvArgs {
  const SeqPtrs* seq;
  const int* pos;
  const float* y;       // [B][3H]
  const float* taps;
  int conv_idx, H;
  int8_t* qx;
  uint16_t* dx;
};

// per sequence: the gated short conv with its own ring (the step's pro_conv),
// the new ring slot, and the quantised output
template <int E, int W>
__global__ void __launch_bounds__(256) k_bd_conv_quant(BdConvArgs p) {
  const int b = blockIdx.x, th = threadIdx.x, H = p.H;
  const int pos = p.pos[b];
  bf16_t* ring = p.seq[b].ring + (size_t)p.conv_idx * W * H;
  const float* yr = p.y + (size_t)b * 3 * H;
  float out[E], bxv[E];
#pragma unroll
  for (int j = 0; j < E; j++) {
    const int i = th * E + j;
    const float bx = pb_bf2f(pb_f2bf(__fmul_rn(pb_bf2f(pb_f2bf(yr[i])), pb_bf2f(pb_f2bf(yr[2 * H + i])))));
    bxv[j] = bx;
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < W; k++) {
      const int pp = pos - (W - 1) + k;
      const float v = k == W - 1 ? bx : pb_bf2f(ring[(size_t)(((pp % W) + W) % W) * H + i]);
      acc = __fadd_rn(acc, __fmul_rn(p.taps[(size_t)i * W + k], v));
    }
    out[j] = pb_bf2f(pb_f2bf(__fmul_rn(pb_bf2f(pb_f2bf(yr[H + i])), pb_bf2f(pb_f2bf(acc)))));
  }
  // the slot of this position held position pos - W, read by no one any more
#pragma unroll
  for (int j = 0; j < E; j++) ring[(size_t)(pos % W) * H + th * E + j] = pb_f2bf(bxv[j]);
  pf_quant_store<E>(out, p.qx + (size_t)b * H, p.dx + (size_t)b * (H / 32), th);
}

}  // namespace
