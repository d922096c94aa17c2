// pb_step.cuh -- device code shared by the per-kernel decode step (pb_model.cu)
// and the persistent decode kernel (pb_decode.cu): argument blocks, the fused
// prologues (embedding, residual add, RMSNorm, gated short conv) and the
// attention body. SYNC selects the CTA barrier: 0 = __syncthreads (a 256-thread
// CTA), 1 = named barrier 1 over the 256 consumer threads of a warp-specialised
// CTA; with SYNC = 1 the activations written earlier in the same launch by
// other CTAs are read through L2 (ld.global.cg), never a possibly stale L1.
#pragma once
#include "pb_common.cuh"

namespace {

constexpr int PRO_PLAIN = 0, PRO_ADDNORM = 1, PRO_EMBED = 2, PRO_CONV = 3, PRO_ATTN = 4;
constexpr int EPI_BF16 = 0, EPI_SILU = 1, EPI_ARGMAX = 2;
constexpr int MAX_CTA = 1024;

// device control block of a state
struct Ctl {
  int token;          // input id of the step; the head writes the greedy id here
  int pos;            // position of the step; the head advances it
  int step;           // greedy step counter (index into ids)
  unsigned counter;   // argmax last-CTA counter
  int* ids;           // optional output: the greedy id of every step
  const int* prompt;  // optional teacher-forced inputs: step i+1 feeds prompt[i+1]
  int n_prompt;
  int _pad;
  float slot_val[MAX_CTA];
  int slot_idx[MAX_CTA];
};

struct StepArgs {
  // weight stream
  const uint4* codes;
  const void* scales;
  int N;
  // prologue
  int pro;
  int K;               // GEMV input length
  int H;               // hidden size (prologue vectors)
  float eps;
  const bf16_t* xin;   // PLAIN: x [K]; ADDNORM: residual [H]; CONV: in_proj output [3H]
  const bf16_t* hin;   // ADDNORM: vector to post-normalise and add (null: none)
  const float* wpost;  // ADDNORM: its norm weight
  const float* wnorm;  // norm giving x from the residual (null: x = residual)
  bf16_t* rout;        // residual written by CTA 0 (null: not written)
  const uint4* emb_codes;   // EMBED: tied table, stream layout
  const void* emb_scales;
  int emb_nch;
  int emb_f32;         // EMBED: scales are fp32 pairs (else fp16 pairs)
  const uint16_t* emb16;    // EMBED: the bf16 table (blob dtype 3) instead, head layout
  bf16_t* ring;        // CONV: [W][H], slot = position mod W
  const float* taps;   // CONV: [H][W]
  int convw;
  const float* segp;   // ATTN: per-head P.V segment partials [NH][8][HD]; xin = q|k|v|gate
  int nh, hd;          // ATTN: heads and head_dim (gate offset = nh*hd + 2*nkv*hd = goff)
  int goff;
  Ctl* ctl;
  // epilogue
  void* y;
  int no_publish;      // ARGMAX: write the logits only (the row-sharded head; a separate argmax publishes)
};

struct AttnArgs {
  const bf16_t* qkvg;      // [NH*HD | NKV*HD | NKV*HD | NH]
  const float* qnorm;      // [HD]
  const float* knorm;      // [HD]
  const float* rope_cos;   // [max_ctx][half]
  const float* rope_sin;
  unsigned short* kc;      // fp16 [max_ctx][NKV][HD]
  unsigned short* vc;
  bf16_t* out;             // [NH*HD] gated attention output
  Ctl* ctl;
  int nh, nkv, half, win, max_ctx;
  float scaling, eps;
  // persistent kernel's split attention: scores/exp [NH][max_ctx], 1/sum [NH],
  // P.V segment partials [NH][8][HD]
  float* scores;
  float* inv;
  float* segp;
};

template <int SYNC>
PB_DEV void csync() {
  if (SYNC) asm volatile("bar.sync 1, 256;" ::: "memory");
  else __syncthreads();
}
template <int SYNC>
PB_DEV unsigned short ldu16(const unsigned short* p) { return SYNC ? __ldcg(p) : *p; }
template <int SYNC>
PB_DEV int ldi(const int* p) { return SYNC ? __ldcg(p) : *p; }

constexpr unsigned PB_WAIT_LIMIT = 1u << 24;   // polls before a wait gives up

// arrival counter of the persistent kernel's grid barrier: wait until `target`
// CTAs have arrived (bounded: PB_WAIT_LIMIT polls, a few seconds). One thread
// per CTA polls with acquire loads and no sleep between them; a sleep, or
// relaxed polls with a fence after the last, measured slower.
PB_DEV bool grid_wait(const unsigned* bar, unsigned target, unsigned limit = PB_WAIT_LIMIT) {
  for (unsigned i = 0; i < limit; i++) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(bar) : "memory");
    if (v >= target) return true;
  }
  return false;
}

// The dependency wait a prologue takes once the loads that do not depend on
// the previous phase (weights of norms, conv taps, ring slots of earlier
// tokens) are in flight. SYNC = 0: the programmatic-launch wait of the
// per-kernel path. SYNC = 1: the persistent kernel's grid barrier (null: the
// launch's first phase, no wait); a wait that gives up raises the abort flag,
// read by the caller after a consumer barrier.
struct GridWait {
  const unsigned* bar;
  unsigned target;
  volatile int* abort;
  int* err;
};
template <int SYNC>
PB_DEV void gw_pass(const GridWait* g) {
  if (!SYNC) {
    pb_grid_wait();
    return;
  }
  if (g) {
    if (threadIdx.x == 0 && !*g->abort && !grid_wait(g->bar, g->target)) {
      *g->abort = 1;
      atomicCAS(g->err, 0, 3);
    }
    csync<1>();
  }
}

// ---------------------------------------------------------------- prologue
// sx (the GEMV input) is stored padded, one spare float per 32, so that lane
// l reading its 32 consecutive values (index 32 l + j) hits bank (l + j) % 32.
PB_DEV int padx(int i) { return i + (i >> 5); }

// The bf16 tied table (blob dtype 3) in its head layout: per row, 16-byte
// granule h*32 + l holds elements l + 32 (8h + m), m = 0..7, so that lane l of
// the head GEMV reads its chain k = l, l+32, ... as 8 conflict-free vector loads.
PB_HD_INL size_t b16_index(int i) { return (size_t)((((i >> 8) * 32 + (i & 31)) << 3) + ((i >> 5) & 7)); }

// element i of row tok of the tied table: bf16(code * scale) from the Q8
// streaming layout (k_dequant_row, lfm3_nanode.cu:138-142), or the bf16
// table's value itself (lfm3_nanode.cu:6062-6070)
PB_DEV float emb_value(const uint4* codes, const void* scales, int nch, int f32s, const uint16_t* e16, int H, int tok,
                       int i) {
  if (e16) return pb_bf2f(e16[(size_t)tok * H + b16_index(i)]);
  const int b = i >> 5, jj = i & 31, c = b >> 6, bb = b & 63, l = bb & 31, half = bb >> 5;
  const size_t seg = (size_t)tok * nch + c;
  const int gi = (half * 2 + (jj >> 4)) * 32 + l;
  const float code = (float)reinterpret_cast<const int8_t*>(codes)[(seg * 128 + gi) * 16 + (jj & 15)];
  const float s = f32s ? reinterpret_cast<const float*>(scales)[(seg * 32 + l) * 2 + half]
                       : pb_h2f(reinterpret_cast<const unsigned short*>(scales)[(seg * 32 + l) * 2 + half]);
  return pb_bf2f(pb_f2bf(__fmul_rn(code, s)));
}

// ---- vector helpers: thread t owns N consecutive elements ---------------
template <int N, int SYNC>
PB_DEV void ld_bf(const bf16_t* p, float (&o)[N]) {
  if (N >= 8) {
#pragma unroll
    for (int v = 0; v < N / 8; v++) {
      const uint4 w = SYNC ? __ldcg(reinterpret_cast<const uint4*>(p) + v) : reinterpret_cast<const uint4*>(p)[v];
      const unsigned ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int k = 0; k < 4; k++) { o[8 * v + 2 * k] = pb_lo2f(ws[k]); o[8 * v + 2 * k + 1] = pb_hi2f(ws[k]); }
    }
  } else if (N == 4) {
    const uint2 w = SYNC ? __ldcg(reinterpret_cast<const uint2*>(p)) : *reinterpret_cast<const uint2*>(p);
    o[0] = pb_lo2f(w.x); o[1] = pb_hi2f(w.x); o[2 % N] = pb_lo2f(w.y); o[3 % N] = pb_hi2f(w.y);
  } else if (N == 2) {
    const unsigned w = SYNC ? __ldcg(reinterpret_cast<const unsigned*>(p)) : *reinterpret_cast<const unsigned*>(p);
    o[0] = pb_lo2f(w); o[1 % N] = pb_hi2f(w);
  } else {
    o[0] = pb_bf2f(ldu16<SYNC>(p));
  }
}
template <int N>
PB_DEV void ld_f32(const float* p, float (&o)[N]) {
  if (N % 4 == 0) {
#pragma unroll
    for (int v = 0; v < N / 4; v++) {
      const float4 w = __ldg(reinterpret_cast<const float4*>(p) + v);
      o[4 * v] = w.x; o[4 * v + 1] = w.y; o[4 * v + 2] = w.z; o[4 * v + 3] = w.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < N; j++) o[j] = __ldg(p + j);
  }
}
template <int N>
PB_DEV void st_bf(bf16_t* p, const float (&v)[N]) {
  if (N >= 8) {
#pragma unroll
    for (int q = 0; q < N / 8; q++) {
      uint4 w;
      w.x = (unsigned)pb_f2bf(v[8 * q]) | ((unsigned)pb_f2bf(v[8 * q + 1]) << 16);
      w.y = (unsigned)pb_f2bf(v[8 * q + 2]) | ((unsigned)pb_f2bf(v[8 * q + 3]) << 16);
      w.z = (unsigned)pb_f2bf(v[8 * q + 4]) | ((unsigned)pb_f2bf(v[8 * q + 5]) << 16);
      w.w = (unsigned)pb_f2bf(v[8 * q + 6]) | ((unsigned)pb_f2bf(v[8 * q + 7]) << 16);
      reinterpret_cast<uint4*>(p)[q] = w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < N; j++) p[j] = pb_f2bf(v[j]);
  }
}

// RMSNorm over the block's H = 256 E values held E per thread (thread t owns
// [E t, E t + E)), in the reference's order (rmsnorm_body,
// lfm3_nanode.cu:383-440): squares summed pairwise, warp shuffle-down tree,
// the 8 warp partials ascending; rs = 1/sqrt(mean + eps) correctly rounded;
// out = bf16(w * bf16(v * rs)) (as floats), w = this thread's E weights.
// `red` (8 floats) must not be in use by a neighbouring call: callers
// alternate two buffers.
template <int E, int SYNC>
__device__ void rms_reg(const float (&v)[E], const float (&wv)[E], float (&out)[E], int H,
                        float eps, float* red) {
  const int t = threadIdx.x;
  float ss[E];
#pragma unroll
  for (int j = 0; j < E; j++) ss[j] = __fmul_rn(v[j], v[j]);
#pragma unroll
  for (int width = E; width > 1; width >>= 1)
#pragma unroll
    for (int i = 0; i < width / 2; i++) ss[i] = __fadd_rn(ss[2 * i], ss[2 * i + 1]);
  const float s = pb_warp_tree(ss[0]);
  if ((t & 31) == 0) red[t >> 5] = s;
  csync<SYNC>();
  float tot = red[0];
#pragma unroll
  for (int i = 1; i < 8; i++) tot = __fadd_rn(tot, red[i]);
  const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(tot, __fdiv_rn(1.0f, (float)H)), eps)));
#pragma unroll
  for (int j = 0; j < E; j++) out[j] = pb_bf2f(pb_f2bf(__fmul_rn(wv[j], pb_bf2f(pb_f2bf(__fmul_rn(v[j], rs))))));
}

// plain GEMV input: K = 256 EK values, EK consecutive per thread
template <int EK, int SYNC>
__device__ void pro_plain(const StepArgs& a, float* sx, const GridWait* gw) {
  // 256 EK values staged: K of them from the input, zeros after it (a
  // one-chunk tensor's padding; K is a multiple of 32, so a thread's EK
  // values are all inside or all past it)
  const int t = threadIdx.x;
  const bf16_t* xin = a.xin;
  gw_pass<SYNC>(gw);
  float x[EK];
  if (t * EK < a.K) {
    ld_bf<EK, SYNC>(xin + (size_t)t * EK, x);
  } else {
#pragma unroll
    for (int j = 0; j < EK; j++) x[j] = 0.0f;
  }
#pragma unroll
  for (int j = 0; j < EK; j++) sx[padx(t * EK + j)] = x[j];
}
// staged length of a GEMV input: K rounded up to whole 2048-code segments
// (the streaming layout; K itself when 2048 divides it)
__host__ __device__ __forceinline__ int pb_kpad(int K) { return (K + 2047) / 2048 * 2048; }

// gated short conv (lfm3_nanode.cu:3790-3818): bx = bf16(B*x) enters the ring
// as the newest slot; y = sum_k taps[i][k] * ring_k (oldest first), one fp32
// chain; out = bf16(C * bf16(y)). The ring slot of position pos held pos - W,
// which no CTA reads any more; CTA 0 writes the new value there.
template <int E, int W, int SYNC>
__device__ void pro_conv(const StepArgs& a, float* sx, const GridWait* gw, int pos) {
  const int t = threadIdx.x, H = a.H;
  const bf16_t* xin = a.xin;
  bf16_t* ring = a.ring;
  float tp[E * W];
  ld_f32<E * W>(a.taps + (size_t)t * E * W, tp);
  // the W-1 older ring slots hold positions of earlier tokens: in the
  // persistent kernel (pos given) they are final before this phase's barrier
  float rg[W - 1][E];
  if (SYNC && pos >= 0) {
#pragma unroll
    for (int k = 0; k < W - 1; k++) {
      const int p = pos - (W - 1) + k;
      ld_bf<E, SYNC>(ring + (size_t)(((p % W) + W) % W) * H + (size_t)t * E, rg[k]);
    }
  }
  gw_pass<SYNC>(gw);
  if (!(SYNC && pos >= 0)) {
    pos = ldi<SYNC>(&a.ctl->pos);
#pragma unroll
    for (int k = 0; k < W - 1; k++) {
      const int p = pos - (W - 1) + k;
      ld_bf<E, SYNC>(ring + (size_t)(((p % W) + W) % W) * H + (size_t)t * E, rg[k]);
    }
  }
  float B[E], C[E], X[E];
  ld_bf<E, SYNC>(xin + (size_t)t * E, B);
  ld_bf<E, SYNC>(xin + H + (size_t)t * E, C);
  ld_bf<E, SYNC>(xin + 2 * H + (size_t)t * E, X);
  float bx[E], y[E];
#pragma unroll
  for (int j = 0; j < E; j++) {
    bx[j] = pb_bf2f(pb_f2bf(__fmul_rn(B[j], X[j])));
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < W; k++)
      acc = __fadd_rn(acc, __fmul_rn(tp[j * W + k], k == W - 1 ? bx[j] : rg[k][j]));
    y[j] = pb_bf2f(pb_f2bf(__fmul_rn(C[j], pb_bf2f(pb_f2bf(acc)))));
    sx[padx(t * E + j)] = y[j];
  }
  if (blockIdx.x == 0) st_bf<E>(ring + (size_t)(pos % W) * H + (size_t)t * E, bx);
}

// residual (embedding row, or xin [+ post-normalised hin]) -> optional rout
// -> optional norm -> x
template <int E, int SYNC>
__device__ void pro_residual(const StepArgs& a, float* sx, float* red, const GridWait* gw) {
  const int t = threadIdx.x, H = a.H;
  const bf16_t* xin = a.xin;
  const bf16_t* hin = a.hin;
  const float* wnorm = a.wnorm;
  bf16_t* rout = a.rout;
  const float eps = a.eps;
  const bool embed = a.pro == PRO_EMBED;
  // norm weights first: they do not depend on the previous phase
  float wp[E], wn[E];
  if (!embed && hin) ld_f32<E>(a.wpost + (size_t)t * E, wp);
  if (wnorm) ld_f32<E>(wnorm + (size_t)t * E, wn);
  gw_pass<SYNC>(gw);
  float R[E];
  if (embed) {
    // the token's row of the tied table
    const int tok = ldi<SYNC>(&a.ctl->token);
#pragma unroll
    for (int j = 0; j < E; j++)
      R[j] = emb_value(a.emb_codes, a.emb_scales, a.emb_nch, a.emb_f32, a.emb16, H, tok, t * E + j);
  } else {
    ld_bf<E, SYNC>(xin + (size_t)t * E, R);
    if (hin) {
      float Hv[E], hn[E];
      ld_bf<E, SYNC>(hin + (size_t)t * E, Hv);
      rms_reg<E, SYNC>(Hv, wp, hn, H, eps, red);
#pragma unroll
      for (int j = 0; j < E; j++) R[j] = pb_bf2f(pb_f2bf(__fadd_rn(R[j], hn[j])));
    }
  }
  if (rout && blockIdx.x == 0) st_bf<E>(rout + (size_t)t * E, R);
  float X[E];
  if (wnorm) rms_reg<E, SYNC>(R, wn, X, H, eps, red + 8);
  else {
#pragma unroll
    for (int j = 0; j < E; j++) X[j] = R[j];
  }
#pragma unroll
  for (int j = 0; j < E; j++) sx[padx(t * E + j)] = X[j];
}

// attention output from the split attention's segment partials: out_d =
// bf16(((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7))) (k_attn_head, lfm3_nanode.cu:594-600),
// then the sigmoid head gate (k_sigmoid_gate, :852-864): bf16(out * 1/(1+e^-g))
template <int EK, int SYNC>
__device__ void pro_attn(const StepArgs& a, float* sx, const GridWait* gw) {
  const int t = threadIdx.x, hd = a.hd;
  gw_pass<SYNC>(gw);
#pragma unroll
  for (int j0 = 0; j0 < EK; j0 += 4) {
    const int i = t * EK + j0, h = i / hd, d = i - h * hd;
    float4 sg[8];
#pragma unroll
    for (int sgi = 0; sgi < 8; sgi++)
      sg[sgi] = __ldcg(reinterpret_cast<const float4*>(a.segp + ((size_t)h * 8 + sgi) * hd + d));
    const float gt = pb_sigmoid(pb_bf2f(ldu16<SYNC>(a.xin + a.goff + h)));
    const float* f = reinterpret_cast<const float*>(sg);
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const float o = __fadd_rn(__fadd_rn(__fadd_rn(f[0 * 4 + k], f[1 * 4 + k]), __fadd_rn(f[2 * 4 + k], f[3 * 4 + k])),
                                __fadd_rn(__fadd_rn(f[4 * 4 + k], f[5 * 4 + k]), __fadd_rn(f[6 * 4 + k], f[7 * 4 + k])));
      sx[padx(i + k)] = pb_bf2f(pb_f2bf(__fmul_rn(pb_bf2f(pb_f2bf(o)), gt)));
    }
  }
}

template <int E, int SYNC>
__device__ void pro_dispatch_conv(const StepArgs& a, float* sx, const GridWait* gw, int pos) {
  switch (a.convw) {
    case 2: pro_conv<E, 2, SYNC>(a, sx, gw, pos); break;
    case 3: pro_conv<E, 3, SYNC>(a, sx, gw, pos); break;
    case 4: pro_conv<E, 4, SYNC>(a, sx, gw, pos); break;
    case 7: pro_conv<E, 7, SYNC>(a, sx, gw, pos); break;
    default: gw_pass<SYNC>(gw); break;   // rejected at load time
  }
}

// Computes the GEMV input x (fp32 values of bf16 numbers) into sx, padded
// (element i at padx(i)). Runs on 256 threads; H = 256 E with E in
// {1, 2, 4, 8, 16}; plain inputs K = 256 EK with EK in {1, 2, 4, 8, 16, 32}.
// `red` holds 16 floats. The dependency wait (gw_pass) is taken inside, after
// the loads that do not need it; pos >= 0 is the step's position when the
// caller knows it (else it is read from the control block). Ends with a CTA
// barrier.
template <int SYNC>
__device__ __noinline__ void step_prologue(const StepArgs& a, float* sx, float* red, const GridWait* gw, int pos) {
  const int pro = a.pro;
  if (pro == PRO_PLAIN) {
    switch (pb_kpad(a.K) >> 8) {
      case 1: pro_plain<1, SYNC>(a, sx, gw); break;
      case 2: pro_plain<2, SYNC>(a, sx, gw); break;
      case 4: pro_plain<4, SYNC>(a, sx, gw); break;
      case 8: pro_plain<8, SYNC>(a, sx, gw); break;
      case 16: pro_plain<16, SYNC>(a, sx, gw); break;
      case 32: pro_plain<32, SYNC>(a, sx, gw); break;
      default: gw_pass<SYNC>(gw); break;
    }
  } else if (pro == PRO_ATTN) {
    switch (a.K >> 8) {
      case 4: pro_attn<4, SYNC>(a, sx, gw); break;
      case 8: pro_attn<8, SYNC>(a, sx, gw); break;
      case 16: pro_attn<16, SYNC>(a, sx, gw); break;
      case 32: pro_attn<32, SYNC>(a, sx, gw); break;
      default: gw_pass<SYNC>(gw); break;
    }
  } else if (pro == PRO_CONV) {
    switch (a.H >> 8) {
      case 1: pro_dispatch_conv<1, SYNC>(a, sx, gw, pos); break;
      case 2: pro_dispatch_conv<2, SYNC>(a, sx, gw, pos); break;
      case 4: pro_dispatch_conv<4, SYNC>(a, sx, gw, pos); break;
      case 8: pro_dispatch_conv<8, SYNC>(a, sx, gw, pos); break;
      case 16: pro_dispatch_conv<16, SYNC>(a, sx, gw, pos); break;
      default: gw_pass<SYNC>(gw); break;
    }
  } else {
    switch (a.H >> 8) {
      case 1: pro_residual<1, SYNC>(a, sx, red, gw); break;
      case 2: pro_residual<2, SYNC>(a, sx, red, gw); break;
      case 4: pro_residual<4, SYNC>(a, sx, red, gw); break;
      case 8: pro_residual<8, SYNC>(a, sx, red, gw); break;
      case 16: pro_residual<16, SYNC>(a, sx, red, gw); break;
      default: gw_pass<SYNC>(gw); break;
    }
  }
  csync<SYNC>();
}

// step_prologue for a kernel specialised to one hidden size (H = 256 EH) and
// conv width W: only those variants are compiled in, and it inlines into its
// caller (no call, no register save area).
template <int SYNC, int EH, int W>
__device__ __forceinline__ void step_prologue_fixed(const StepArgs& a, float* sx, float* red, const GridWait* gw,
                                                    int pos) {
  const int pro = a.pro;
  if (pro == PRO_PLAIN) {
    switch (pb_kpad(a.K) >> 8) {
      case 8: pro_plain<8, SYNC>(a, sx, gw); break;
      case 16: pro_plain<16, SYNC>(a, sx, gw); break;
      case 32: pro_plain<32, SYNC>(a, sx, gw); break;
      default: gw_pass<SYNC>(gw); break;      // other K: the host keeps this kernel off
    }
  } else if (pro == PRO_ATTN) {
    switch (a.K >> 8) {
      case 4: pro_attn<4, SYNC>(a, sx, gw); break;
      case 8: pro_attn<8, SYNC>(a, sx, gw); break;
      case 16: pro_attn<16, SYNC>(a, sx, gw); break;
      default: gw_pass<SYNC>(gw); break;
    }
  } else if (pro == PRO_CONV) {
    pro_conv<EH, W, SYNC>(a, sx, gw, pos);
  } else {
    pro_residual<EH, SYNC>(a, sx, red, gw);
  }
  csync<SYNC>();
}

// ------------------------------------------------------------- attention
// per-head RMSNorm (k_headnorm, lfm3_nanode.cu:460-479) + NeoX RoPE
// (k_rope, :483-498) by one warp; result (fp32 of bf16) into o[HD]
template <int E, int SYNC>
__device__ void head_norm_rope(const bf16_t* __restrict__ x, const float* __restrict__ w,
                               const float* cs, const float* sn, int half, float eps, float* o) {
  const int lane = threadIdx.x & 31;
  constexpr int HD = 32 * E;
  // every load first (activations, weights, rope table): one round trip
  float v[E], ss[E], wv[E], c[E], sv[E];
#pragma unroll
  for (int j = 0; j < E; j++) {
    const int i = lane * E + j;
    v[j] = pb_bf2f(ldu16<SYNC>(x + i));
    wv[j] = __ldg(w + i);
    c[j] = i < half ? __ldg(cs + i) : 0.0f;
    sv[j] = i < half ? __ldg(sn + i) : 0.0f;
  }
#pragma unroll
  for (int j = 0; j < E; j++) ss[j] = __fmul_rn(v[j], v[j]);
#pragma unroll
  for (int width = E; width > 1; width >>= 1)
#pragma unroll
    for (int i = 0; i < width / 2; i++) ss[i] = __fadd_rn(ss[2 * i], ss[2 * i + 1]);
  float s = pb_warp_tree(__fadd_rn(ss[0], 0.0f));
  s = __shfl_sync(0xffffffffu, s, 0);
  const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(s, __fdiv_rn(1.0f, (float)HD)), eps)));
#pragma unroll
  for (int j = 0; j < E; j++) {
    const int i = lane * E + j;
    o[i] = pb_bf2f(pb_f2bf(__fmul_rn(wv[j], pb_bf2f(pb_f2bf(__fmul_rn(v[j], rs))))));
  }
  __syncwarp();
  float lo_n[E], hi_n[E];
#pragma unroll
  for (int j = 0; j < E; j++) {
    const int i = lane * E + j;   // i < HD/2 covers the pairs when i < half
    if (i < half) {
      const float lo = o[i], hi = o[i + HD / 2];
      lo_n[j] = pb_bf2f(pb_f2bf(__fadd_rn(__fmul_rn(lo, c[j]), __fmul_rn(-hi, sv[j]))));
      hi_n[j] = pb_bf2f(pb_f2bf(__fadd_rn(__fmul_rn(hi, c[j]), __fmul_rn(lo, sv[j]))));
    }
  }
  __syncwarp();
#pragma unroll
  for (int j = 0; j < E; j++) {
    const int i = lane * E + j;
    if (i < half) { o[i] = lo_n[j]; o[i + HD / 2] = hi_n[j]; }
  }
  __syncwarp();
}

// k_attn_head (lfm3_nanode.cu:503-602) for q head h over the fp16 cache, with
// the q/k prologue and the sigmoid gate (k_sigmoid_gate, :852-864) fused.
// The current position's k/v are used from shared memory (the CTA of the
// group's first q head also appends them to the cache), so no CTA reads a
// cache row another CTA writes in the same step. sl: scores [max_ctx]. Not
// inlined: the persistent kernel keeps its register budget for the GEMV loop.
template <int E, int SYNC>
__device__ __noinline__ void attn_body(const AttnArgs& a, int h, int pos, float* sl, float* qv, float* kv, float* vv,
                          float* segred, float* red) {
  constexpr int HD = 32 * E;
  const int t = threadIdx.x, lane = t & 31, wid = t >> 5;
  const int grp = a.nh / a.nkv, kvh = h / grp;
  const int npos = pos + 1;
  const int lo = (a.win > 0 && npos > a.win) ? npos - a.win : 0;
  const int np = npos - lo;
  const float* cs = a.rope_cos + (size_t)pos * a.half;
  const float* sn = a.rope_sin + (size_t)pos * a.half;
  const size_t koff = (size_t)a.nh * HD, voff = koff + (size_t)a.nkv * HD, goff = voff + (size_t)a.nkv * HD;
  if (wid == 0) head_norm_rope<E, SYNC>(a.qkvg + (size_t)h * HD, a.qnorm, cs, sn, a.half, a.eps, qv);
  if (wid == 1) {
    head_norm_rope<E, SYNC>(a.qkvg + koff + (size_t)kvh * HD, a.knorm, cs, sn, a.half, a.eps, kv);
#pragma unroll
    for (int j = 0; j < E; j++) {
      const int i = lane * E + j;
      const unsigned short k16 = pb_f2h(kv[i]);
      kv[i] = pb_h2f(k16);
      if (h % grp == 0) a.kc[((size_t)pos * a.nkv + kvh) * HD + i] = k16;
    }
  }
  if (wid == 2) {
#pragma unroll
    for (int j = 0; j < E; j++) {
      const int i = lane * E + j;
      const unsigned short v16 = pb_f2h(pb_bf2f(ldu16<SYNC>(a.qkvg + voff + (size_t)kvh * HD + i)));
      vv[i] = pb_h2f(v16);
      if (h % grp == 0) a.vc[((size_t)pos * a.nkv + kvh) * HD + i] = v16;
    }
  }
  csync<SYNC>();
  // scores: position p by warp (p - lo) % 8, lane chains over its E dims;
  // four positions per pass so that their loads and trees overlap
  float ql[E];
#pragma unroll
  for (int j = 0; j < E; j++) ql[j] = qv[lane * E + j];
  for (int p0 = lo + wid; p0 < npos; p0 += 32) {
    float kl[4][E];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int p = p0 + 8 * u;
      if (p < pos) {
        const unsigned short* kr = a.kc + ((size_t)p * a.nkv + kvh) * HD + lane * E;
#pragma unroll
        for (int j = 0; j < E; j++) kl[u][j] = pb_h2f(ldu16<SYNC>(kr + j));
      } else {
#pragma unroll
        for (int j = 0; j < E; j++) kl[u][j] = kv[lane * E + j];   // p == pos (or past the end)
      }
    }
    float sv[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < E; j++) s = __fadd_rn(s, __fmul_rn(ql[j], kl[u][j]));
      sv[u] = s;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int u = 0; u < 4; u++) sv[u] = __fadd_rn(sv[u], __shfl_down_sync(0xffffffffu, sv[u], o));
    if (lane == 0)
#pragma unroll
      for (int u = 0; u < 4; u++)
        if (p0 + 8 * u < npos) sl[p0 + 8 * u - lo] = __fmul_rn(sv[u], a.scaling);
  }
  csync<SYNC>();
  float mx = -1e30f;
  for (int i = t; i < np; i += 256) mx = fmaxf(mx, sl[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_down_sync(0xffffffffu, mx, o));
  if (lane == 0) red[wid] = mx;
  csync<SYNC>();
  float m = red[0];
#pragma unroll
  for (int i = 1; i < 8; i++) m = fmaxf(m, red[i]);
  csync<SYNC>();
  float sum = 0.0f;
  for (int i = t; i < np; i += 256) {
    const float e = pb_expf(__fadd_rn(sl[i], -m));
    sl[i] = e;
    sum = __fadd_rn(sum, e);
  }
  sum = pb_warp_tree(sum);
  if (lane == 0) red[wid] = sum;
  csync<SYNC>();
  // 8-lane shuffle-down tree: ((r0+r4)+(r2+r6))+((r1+r5)+(r3+r7))
  const float tot = __fadd_rn(__fadd_rn(__fadd_rn(red[0], red[4]), __fadd_rn(red[2], red[6])),
                              __fadd_rn(__fadd_rn(red[1], red[5]), __fadd_rn(red[3], red[7])));
  const float inv = __fdiv_rn(1.0f, tot);
  // P.V: segment = warp, lane owns dims lane*E .. +E; each dim's chain runs
  // over p = seg, seg+8, ... in order, four positions' loads per pass
  float acc[E];
#pragma unroll
  for (int j = 0; j < E; j++) acc[j] = 0.0f;
  for (int p0 = wid; p0 < np; p0 += 32) {
    float vl[4][E], wv[4];
#pragma unroll
    for (int u = 0; u < 4; u++) {
      const int p = p0 + 8 * u, ap = lo + p;
      wv[u] = p < np ? __fmul_rn(sl[p], inv) : 0.0f;
      if (ap < pos) {
        const unsigned short* vr = a.vc + ((size_t)ap * a.nkv + kvh) * HD + lane * E;
#pragma unroll
        for (int j = 0; j < E; j++) vl[u][j] = pb_h2f(ldu16<SYNC>(vr + j));
      } else {
#pragma unroll
        for (int j = 0; j < E; j++) vl[u][j] = vv[lane * E + j];
      }
    }
#pragma unroll
    for (int u = 0; u < 4; u++)
      if (p0 + 8 * u < np)
#pragma unroll
        for (int j = 0; j < E; j++) acc[j] = __fadd_rn(acc[j], __fmul_rn(wv[u], vl[u][j]));
  }
#pragma unroll
  for (int j = 0; j < E; j++) segred[wid * HD + lane * E + j] = acc[j];
  csync<SYNC>();
  if (t < HD) {
    const float* r = segred + t;
    const float o = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[HD]), __fadd_rn(r[2 * HD], r[3 * HD])),
                              __fadd_rn(__fadd_rn(r[4 * HD], r[5 * HD]), __fadd_rn(r[6 * HD], r[7 * HD])));
    const float sg = pb_sigmoid(pb_bf2f(ldu16<SYNC>(a.qkvg + goff + h)));
    a.out[(size_t)h * HD + t] = pb_f2bf(__fmul_rn(pb_bf2f(pb_f2bf(o)), sg));
  }
  csync<SYNC>();   // sl / segred are reused by the caller
}

}  // namespace
