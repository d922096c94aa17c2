/* pb_oracle.c -- CPU restatement of PULSAR-ASM's quantized weight-streaming
 * hot path. TEST INFRASTRUCTURE, NOT PRODUCT: see pb_oracle.h.
 *
 * Reference files (paths relative to the PULSAR-ASM project root):
 *   LFM3 engine      pulsar_arm/asm/lfm3_nanode.cu
 *   Q8_0 activation  pulsar_arm/bonsai2/fwd35_ref.c
 *   Q1_0 host ref    pulsar_arm/bonsai2/pq1_host.c
 *   Q8_K quantizer   pulsar_arm/bonsai2/fwd8.c, pulsar_arm/bonsai2/pq1_parity.c
 *
 * Deterministic replacements for device intrinsics (the CUDA product uses the
 * same ones, so results agree bit for bit):
 *   rsqrtf(v)        -> 1.0f / sqrtf(v), both correctly rounded (the reference's
 *                       MUFU rsqrtf is an approximation with no CPU twin)
 *   expf(x)          -> pbo_expf: Cody-Waite reduction x = n*ln2 + r with a
 *                       two-constant ln2 split, e^r by its degree-7 Taylor
 *                       polynomial in Horner form with fused multiply-adds,
 *                       then an exact scale by 2^n. Max error about 1 ulp.
 *   cosf/sinf(ang)   -> (float)cos((double)ang), (float)sin((double)ang),
 *                       evaluated on the host; the product precomputes the
 *                       same table on the host and uploads it.
 *   argmax ties      -> the lowest index wins.
 */
#include "pb_oracle.h"
#include <math.h>
#include <string.h>
#include <stdlib.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline uint32_t fbits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bitsf(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

int pbo_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ------------------------------------------------------------ scalars ---- */
/* lfm3_nanode.cu:116-121: round to nearest even, inf/nan keep their top bits. */
uint16_t pbo_f2bf(float v) {
  const uint32_t u = fbits(v);
  if (((u >> 23) & 0xffu) == 0xffu) return (uint16_t)(u >> 16);
  return (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
}
float pbo_bf2f(uint16_t h) { return bitsf((uint32_t)h << 16); }

/* IEEE binary16, round to nearest even (the rounding pq1_host.c:386-391 and
 * fwd35_ref.c:55-70 perform). */
uint16_t pbo_f2h(float v) {
  const uint32_t u = fbits(v);
  const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
  const uint32_t a = u & 0x7fffffffu;
  if (a >= 0x7f800000u) return sign | (a > 0x7f800000u ? 0x7e00u : 0x7c00u);
  if (a >= 0x477ff000u) return sign | 0x7c00u;            /* >= 65520 -> inf */
  if (a < 0x38800000u) {                                  /* half subnormal or 0 */
    const float r = rintf(bitsf(a) * 16777216.0f);        /* exact scale by 2^24 */
    return sign | (uint16_t)r;                            /* 1024 -> min normal */
  }
  const uint32_t m = a + 0xfffu + ((a >> 13) & 1u) - (112u << 23);
  return sign | (uint16_t)(m >> 13);
}
/* exact widening, pq1_host.c:14-24 */
float pbo_h2f(uint16_t h) {
  const uint32_t s = (uint32_t)(h & 0x8000u) << 16, e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  if (e == 0) { const float f = (float)m * 5.9604644775390625e-8f; return s ? -f : f; }
  if (e == 31) return bitsf(s | 0x7f800000u | (m << 13));
  return bitsf(s | ((e + 112u) << 23) | (m << 13));
}

/* e^x: x = n*ln2 + r, |r| <= ln2/2 (Cody & Waite, "Software Manual for the
 * Elementary Functions", 1980: argument reduction with ln2 split into a short
 * high part and a low correction); e^r from its Taylor series to r^7 (the
 * truncation error r^8/8! < 6e-9 relative); 2^n applied by exponent
 * arithmetic in at most two exact-or-once-rounded multiplies. */
float pbo_expf(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return INFINITY;
  if (x < -103.97207708399179f) return 0.0f;
  const float n = rintf(x * 1.44269502162933349609375f);
  float r = fmaf(n, -0.693145751953125f, x);
  r = fmaf(n, -1.428606765330187e-06f, r);
  float p = 1.98412701138295233249664306640625e-4f;       /* 1/7! */
  p = fmaf(p, r, 1.38888892251998186111450195312500e-3f);  /* 1/6! */
  p = fmaf(p, r, 8.33333376795053482055664062500000e-3f);  /* 1/5! */
  p = fmaf(p, r, 4.16666679084300994873046875000000e-2f);  /* 1/4! */
  p = fmaf(p, r, 1.66666671633720397949218750000000e-1f);  /* 1/3! */
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int k = (int)n;
  if (k > 127) { p = p * 2.0f; k -= 1; }
  if (k < -126) { p = p * bitsf((uint32_t)(k + 64 + 127) << 23); return p * 5.42101086242752217003726400434970855712890625e-20f; }
  return p * bitsf((uint32_t)(k + 127) << 23);
}

static float pairwise(float* s, int E) {   /* ((s0+s1)+(s2+s3))+... levels */
  for (int w = E; w > 1; w >>= 1)
    for (int i = 0; i < w / 2; i++) s[i] = s[2 * i] + s[2 * i + 1];
  return s[0];
}
static float tree_down(float* v, int n) {  /* __shfl_down_sync tree over n lanes */
  for (int o = n / 2; o > 0; o >>= 1)
    for (int l = 0; l < o; l++) v[l] = v[l] + v[l + o];
  return v[0];
}

/* -------------------------------------------------------- Q8 float path -- */
/* pick(): lfm3_nanode.cu:1763-1768 (KCHUNK 2048 when it divides K, 512 for
 * K == 512, else the whole row). The chunk count fixes the combine order. */
int pbo_q8_kchunk(int K) {
  if (K >= 2048 && K % 2048 == 0) return 2048;
  if (K == 512) return 512;
  return K;
}

/* One (row, chunk): lane l chains blocks b = l, l+32, ... with
 * dot_b = fma(code_j, x_j, dot) over j ascending and acc = fma(s_b, dot_b, acc)
 * (q8_partial<bf16,FMA=true>, lfm3_nanode.cu:270-323), then the shuffle-down
 * tree 16..1 (:326-327). Identical to q8_partial_TLb's 5-bit bit-reversed
 * binary-counter combine (:4045-4123) and to cpuchk_run (:4658-4684). */
static float q8f_chunk(const int8_t* qr, const float* sr, const float* x, int nbc) {
  float v[32];
  for (int l = 0; l < 32; l++) {
    float acc = 0.0f;
    for (int b = l; b < nbc; b += 32) {
      const int8_t* c = qr + (size_t)b * 32;
      const float* xb = x + (size_t)b * 32;
      float dot = 0.0f;
      for (int j = 0; j < 32; j++) dot = fmaf((float)c[j], xb[j], dot);
      acc = fmaf(sr[b], dot, acc);
    }
    v[l] = acc;
  }
  return tree_down(v, 32);
}

/* chunk partials summed ascending from 0 (k_combine_bf / k_combine_f,
 * lfm3_nanode.cu:336-374); the caller rounds to bf16 where the reference does. */
void pbo_q8f_gemm(const int8_t* codes, const float* scales, int N, int K, int T,
                  const uint16_t* x_bf16, float* y) {
  const int KC = pbo_q8_kchunk(K), nch = K / KC, nbc = KC / 32, nb = K / 32;
  float* xf = (float*)malloc((size_t)T * K * sizeof(float));
  for (size_t i = 0; i < (size_t)T * K; i++) xf[i] = pbo_bf2f(x_bf16[i]);
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; n++) {
    const int8_t* qr = codes + (size_t)n * K;
    const float* sr = scales + (size_t)n * nb;
    for (int t = 0; t < T; t++) {
      float acc = 0.0f;
      for (int c = 0; c < nch; c++)
        acc = acc + q8f_chunk(qr + (size_t)c * KC, sr + (size_t)c * nbc,
                              xf + (size_t)t * K + (size_t)c * KC, nbc);
      y[(size_t)t * N + n] = acc;
    }
  }
  free(xf);
}
void pbo_q8f_gemv(const int8_t* codes, const float* scales, int N, int K,
                  const uint16_t* x_bf16, float* y) {
  pbo_q8f_gemm(codes, scales, N, K, 1, x_bf16, y);
}

/* ----------------------------------------------------- Q8_0 integer path -- */
/* fwd35_ref.c:332-343 (the AVX quantize_row_q8_0 form): d = amax/127 stored
 * as fp16; q = rint(x * 127/amax), 0 when amax == 0. */
void pbo_q80_quant_act(const float* x, int K, int8_t* qx, uint16_t* dx_h) {
  for (int b = 0; b < K / 32; b++) {
    float amax = 0.0f;
    for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(x[32 * b + j]));
    const float d = amax / 127.0f;
    dx_h[b] = pbo_f2h(d);
    const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
    for (int j = 0; j < 32; j++) qx[32 * b + j] = (int8_t)rintf(x[32 * b + j] * id);
  }
}
/* exact int32 block dot, then the fold acc += (dw*dx)*(float)isum in block
 * order with no contraction (pattern of pq1_host.c:112-116 and ggml's generic
 * Q8_0 x Q8_0 dot). */
void pbo_q80_gemv(const int8_t* codes, const uint16_t* dw_h, int N, int K,
                  const int8_t* qx, const uint16_t* dx_h, int32_t* isum, float* y) {
  const int nb = K / 32;
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; n++) {
    float acc = 0.0f;
    for (int b = 0; b < nb; b++) {
      const int8_t* c = codes + (size_t)n * K + (size_t)b * 32;
      int32_t s = 0;
      for (int j = 0; j < 32; j++) s += (int32_t)c[j] * (int32_t)qx[32 * b + j];
      if (isum) isum[(size_t)n * nb + b] = s;
      acc = acc + (pbo_h2f(dw_h[(size_t)n * nb + b]) * pbo_h2f(dx_h[b])) * (float)s;
    }
    y[n] = acc;
  }
}

/* ---------------------------------------------------------- Q1_0 x Q8_K -- */
/* pq1_host.c:77-97 (non-ternary build): 18-byte blocks -> 16 sign bytes per
 * 128 weights (LSB-first, bit 1 = +1) and the fp16 scale verbatim. */
void pbo_q1_repack(const uint8_t* q1, int rows, int K, uint32_t* w_bits, uint16_t* w_scales) {
  const int nb = K / 128;
  for (int r = 0; r < rows; r++) {
    const uint8_t* row = q1 + (size_t)r * nb * 18;
    for (int b = 0; b < nb; b++) {
      memcpy(w_bits + (size_t)r * (K / 32) + b * 4, row + b * 18 + 2, 16);
      memcpy(w_scales + (size_t)r * nb + b, row + b * 18, 2);
    }
  }
}
/* Q8_K quantizer: fwd8.c:67-139 as pq1_parity.c:131-148 states it in scalar
 * form (the NEON multiply-add is contracted to one fma by GCC there): amax and
 * the value `mx` at the first index reaching it; iscale = -127/mx;
 * q = min(127, nearest_int(fma(x, iscale, 1.5*2^23))); d = 1/iscale; int16
 * bsums of 16-value groups. An all-zero block is all zero bytes. */
void pbo_q8k_quant(const float* x, int K, uint8_t* xq) {
  for (int b = 0; b < K / 256; b++) {
    const float* xb = x + (size_t)b * 256;
    uint8_t* qb = xq + (size_t)b * 292;
    float amax = 0.0f, mx = 0.0f;
    for (int j = 0; j < 256; j++)
      if (fabsf(xb[j]) > amax) { amax = fabsf(xb[j]); mx = xb[j]; }
    if (!amax) { memset(qb, 0, 292); continue; }
    const float iscale = -127.f / mx;
    int8_t* qs = (int8_t*)(qb + 4);
    for (int j = 0; j < 256; j++) {
      const float v = fmaf(xb[j], iscale, 12582912.f);
      int32_t q = (int32_t)(fbits(v) & 0x007fffffu) - 0x00400000;
      qs[j] = (int8_t)(q < 127 ? q : 127);
    }
    for (int g = 0; g < 16; g++) {
      int s = 0;
      for (int j = 0; j < 16; j++) s += qs[16 * g + j];
      const int16_t s16 = (int16_t)s;
      memcpy(qb + 260 + 2 * g, &s16, 2);
    }
    const float d = 1.0f / iscale;
    memcpy(qb, &d, 4);
  }
}
/* pq1_host.c:14-24 widens -0 to +0 (the only difference from pbo_h2f). */
static float q1_h2f(uint16_t h) { return (h == 0x8000u) ? 0.0f : pbo_h2f(h); }
/* RMS + Q8_K chain of the Q1 engine: fwd8.c:312-317 / pq1_parity.c:124-147:
 * x += r (optional); s = serial double fma sum of squares; sc = 1/sqrtf(float(s/n)
 * + eps); y = (x*sc)*w; then the Q8_K quantizer above. */
void pbo_q1_rms_q8k(float* x, const float* r, const float* w, int n, float eps, float* y,
                    uint8_t* xq) {
  if (r) for (int i = 0; i < n; i++) x[i] = x[i] + r[i];
  double s = 0;
  for (int i = 0; i < n; i++) s = fma((double)x[i], (double)x[i], s);
  const float sc = 1.0f / sqrtf((float)(s / n) + eps);
  for (int i = 0; i < n; i++) y[i] = (x[i] * sc) * w[i];
  if (xq) pbo_q8k_quant(y, n, xq);
}
/* pq1_host.c:99-120: isum = sum(bit ? +q : -q) exact; acc += (ws*db)*(float)isum
 * in group order, no contraction. */
void pbo_q1_gemv(int rows, int K, const uint32_t* w_bits, const uint16_t* w_scales,
                 const uint8_t* xq, int32_t* isum, float* y) {
  const int nb = K / 128;
#pragma omp parallel for schedule(static)
  for (int r = 0; r < rows; r++) {
    const uint32_t* wb = w_bits + (size_t)r * (K / 32);
    float acc = 0.0f;
    for (int b = 0; b < nb; b++) {
      const uint8_t* qb = xq + (size_t)(b >> 1) * 292;
      float db; memcpy(&db, qb, 4);
      const int8_t* qs = (const int8_t*)(qb + 4 + (b & 1) * 128);
      const float ws = q1_h2f(w_scales[(size_t)r * nb + b]);
      const uint32_t* w4 = wb + b * 4;
      int32_t s = 0;
      for (int i = 0; i < 128; i++) s += (((w4[i >> 5] >> (i & 31)) & 1u) ? 1 : -1) * (int32_t)qs[i];
      if (isum) isum[(size_t)r * nb + b] = s;
      acc = acc + (ws * db) * (float)s;
    }
    y[r] = acc;
  }
}

/* ---------------------------------------------------------- layer math --- */
/* rmsnorm_body, lfm3_nanode.cu:383-440, 256 threads with H/256 consecutive
 * elements each: squares summed pairwise, warp shuffle-down tree, 8 warp
 * partials ascending; y = bf16(w * bf16(x*rs)). */
void pbo_rmsnorm(const uint16_t* x, const float* w, uint16_t* y, int H, float eps) {
  const int E = H / 256;
  float part[256], ss[64], wsum[8];
  for (int t = 0; t < 256; t++) {
    for (int j = 0; j < E; j++) { const float v = pbo_bf2f(x[t * E + j]); ss[j] = v * v; }
    part[t] = pairwise(ss, E);
  }
  for (int wi = 0; wi < 8; wi++) wsum[wi] = tree_down(part + 32 * wi, 32);
  float tot = wsum[0];
  for (int i = 1; i < 8; i++) tot = tot + wsum[i];
  const float rs = 1.0f / sqrtf(tot * (1.0f / (float)H) + eps);
  for (int i = 0; i < H; i++) {
    const float r = pbo_bf2f(pbo_f2bf(pbo_bf2f(x[i]) * rs));
    y[i] = pbo_f2bf(w[i] * r);
  }
}
/* k_headnorm, lfm3_nanode.cu:460-479: 32 lanes x hd/32 dims, pairwise then
 * "+ 0", shuffle-down tree, same rounding as rmsnorm. In place. */
void pbo_headnorm(uint16_t* x, const float* w, int nheads, int hd, float eps) {
  const int E = hd / 32;
  for (int h = 0; h < nheads; h++) {
    uint16_t* xr = x + (size_t)h * hd;
    float v32[32], ss[8];
    for (int l = 0; l < 32; l++) {
      for (int j = 0; j < E; j++) { const float v = pbo_bf2f(xr[l * E + j]); ss[j] = v * v; }
      v32[l] = pairwise(ss, E) + 0.0f;
    }
    const float s = tree_down(v32, 32);
    const float rs = 1.0f / sqrtf(s * (1.0f / (float)hd) + eps);
    for (int i = 0; i < hd; i++) {
      const float r = pbo_bf2f(pbo_f2bf(pbo_bf2f(xr[i]) * rs));
      xr[i] = pbo_f2bf(w[i] * r);
    }
  }
}
/* build_invf, lfm3_nanode.cu:3719-3723: the first (int)(partial*hd)/2
 * frequencies follow the full head_dim progression, the rest are 0. */
void pbo_rope_invf(float* invf, float base, int hd, float partial) {
  const int angles = (int)((double)partial * hd) / 2;
  for (int i = 0; i < hd / 2; i++)
    invf[i] = (i < angles) ? 1.0f / powf(base, (float)(2 * i) / (float)hd) : 0.0f;
}
void pbo_rope_cs(const float* invf, int pos, int half, float* c, float* s) {
  for (int i = 0; i < half; i++) {
    const float ang = (float)pos * invf[i];
    c[i] = (float)cos((double)ang);
    s[i] = (float)sin((double)ang);
  }
}
/* k_rope, lfm3_nanode.cu:483-498: NeoX rotate-half on (i, i+hd/2) for
 * i < half, fp32 products, one bf16 round per output. */
void pbo_rope(uint16_t* x, int nheads, int hd, int half, const float* c, const float* s) {
  for (int h = 0; h < nheads; h++) {
    uint16_t* xr = x + (size_t)h * hd;
    for (int i = 0; i < half; i++) {
      const float lo = pbo_bf2f(xr[i]), hi = pbo_bf2f(xr[i + hd / 2]);
      xr[i] = pbo_f2bf(lo * c[i] + (-hi) * s[i]);
      xr[i + hd / 2] = pbo_f2bf(hi * c[i] + lo * s[i]);
    }
  }
}

/* k_attn_head, lfm3_nanode.cu:503-602, over an fp16 cache [ctx][nkv][hd]:
 *  score(p) = (32-lane shuffle-down tree of per-lane chains over hd/32 dims,
 *             ((0 + q0k0) + q1k1) + ...) * scaling
 *  max over the window (order free); e = expf(s - m);
 *  sum = per-thread strided chains (i = tid, tid+256, ...), warp trees, then
 *        the 8-lane shuffle-down tree ((w0+w4)+(w2+w6))+((w1+w5)+(w3+w7));
 *  out_d = pairwise tree over 8 segment chains (p = seg, seg+8, ...) of
 *          (e_p * (1/sum)) * v_p,d, rounded to bf16;
 *  optional sigmoid gate (k_sigmoid_gate, :852-864): bf16(out * 1/(1+e^-g)). */
void pbo_attn_head(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, int kvh,
                   int nkv, int hd, int npos, int win, float scaling, uint16_t gate,
                   int use_gate, uint16_t* out) {
  const int E = hd / 32;
  const int lo = (win > 0 && npos > win) ? npos - win : 0;
  const int np = npos - lo;
  float* sl = (float*)malloc((size_t)np * sizeof(float));
  float qf[256];
  for (int i = 0; i < hd; i++) qf[i] = pbo_bf2f(q[i]);
  for (int p = 0; p < np; p++) {
    const uint16_t* kr = kc + ((size_t)(lo + p) * nkv + kvh) * hd;
    float v32[32];
    for (int l = 0; l < 32; l++) {
      float s = 0.0f;
      for (int j = 0; j < E; j++) s = s + qf[l * E + j] * pbo_h2f(kr[l * E + j]);
      v32[l] = s;
    }
    sl[p] = tree_down(v32, 32) * scaling;
  }
  float m = -1e30f;
  for (int p = 0; p < np; p++) m = fmaxf(m, sl[p]);
  float th[256];
  for (int t = 0; t < 256; t++) th[t] = 0.0f;
  for (int i = 0; i < np; i++) { sl[i] = pbo_expf(sl[i] + (-m)); th[i & 255] = th[i & 255] + sl[i]; }
  float wsum[8];
  for (int w = 0; w < 8; w++) wsum[w] = tree_down(th + 32 * w, 32);
  const float inv = 1.0f / tree_down(wsum, 8);
  float sig = 0.0f;
  if (use_gate) sig = 1.0f / (1.0f + pbo_expf(-pbo_bf2f(gate)));
  for (int d = 0; d < hd; d++) {
    float seg[8];
    for (int sg = 0; sg < 8; sg++) {
      float acc = 0.0f;
      for (int p = sg; p < np; p += 8) {
        const float w = sl[p] * inv;
        acc = acc + w * pbo_h2f(vc[((size_t)(lo + p) * nkv + kvh) * hd + d]);
      }
      seg[sg] = acc;
    }
    uint16_t o = pbo_f2bf(pairwise(seg, 8));
    if (use_gate) o = pbo_f2bf(pbo_bf2f(o) * sig);
    out[d] = o;
  }
  free(sl);
}

/* k_shift_in + k_conv7 (lfm3_nanode.cu:892-911) for any width W: the ring
 * [W][H] (oldest first) shifts by one and takes xin as its newest row; y_i =
 * bf16 of the fp32 chain ((0 + t_i0 r_0i) + t_i1 r_1i) + ... over the taps. */
void pbo_conv_step(uint16_t* ring, const uint16_t* xin, const float* taps, int W, int H, uint16_t* y) {
  for (int k = 0; k + 1 < W; k++) memcpy(ring + (size_t)k * H, ring + (size_t)(k + 1) * H, 2 * (size_t)H);
  memcpy(ring + (size_t)(W - 1) * H, xin, 2 * (size_t)H);
  for (int i = 0; i < H; i++) {
    float acc = 0.0f;
    for (int k = 0; k < W; k++) acc = acc + taps[(size_t)i * W + k] * pbo_bf2f(ring[(size_t)k * H + i]);
    y[i] = pbo_f2bf(acc);
  }
}
/* k_silu_mul_bf (lfm3_nanode.cu:821-829): y = bf16((a * 1/(1+e^-a)) * b) */
void pbo_silu_mul_bf(const uint16_t* a, const uint16_t* b, uint16_t* y, int n) {
  for (int i = 0; i < n; i++) {
    const float av = pbo_bf2f(a[i]);
    const float sg = 1.0f / (1.0f + pbo_expf(-av));
    y[i] = pbo_f2bf((av * sg) * pbo_bf2f(b[i]));
  }
}
/* k_sigmoid_gate (lfm3_nanode.cu:852-859): attn[h][:] = bf16(attn * 1/(1+e^-g_h)) */
void pbo_sigmoid_gate(const uint16_t* g, uint16_t* attn, int nh, int hd) {
  for (int h = 0; h < nh; h++) {
    const float sg = 1.0f / (1.0f + pbo_expf(-pbo_bf2f(g[h])));
    for (int j = 0; j < hd; j++) attn[(size_t)h * hd + j] = pbo_f2bf(pbo_bf2f(attn[(size_t)h * hd + j]) * sg);
  }
}

/* greedy argmax; ties go to the lowest index (the reference's k_argmax,
 * lfm3_nanode.cu:942-964, resolves ties by its reduction tree instead). */
int pbo_argmax(const float* v, int n) {
  int bi = 0;
  for (int i = 1; i < n; i++) if (v[i] > v[bi]) bi = i;
  return bi;
}

/* k_gemv_bf16, lfm3_nanode.cu:3517-3534 (the certified arm's lm_head over the
 * bf16 embedding, blob dtype 3): row n, lane l chains k = l, l+32, ... of
 * s = s + bf16(W[n][k]) * x[k] (product and sum rounded apart), then the
 * shuffle-down tree with rounded adds; the fp32 result is the logit as is. */
void pbo_gemv_bf16(const uint16_t* w, int N, int K, const uint16_t* x_bf16, float* y) {
#pragma omp parallel for schedule(static)
  for (int n = 0; n < N; n++) {
    float v[32];
    const uint16_t* wr = w + (size_t)n * K;
    for (int l = 0; l < 32; l++) {
      float acc = 0.0f;
      for (int k = l; k < K; k += 32) acc = acc + pbo_bf2f(wr[k]) * pbo_bf2f(x_bf16[k]);
      v[l] = acc;
    }
    y[n] = tree_down(v, 32);
  }
}

/* ------------------------------------------------------- decode step ---- */
typedef struct { const int8_t* c; const float* s; int N, K; } q8t;
struct pbo_model {
  pbo_cfg cfg;
  int int_mode;          /* 1: every projection on the Q8_0 integer path */
  int* is_attn;
  q8t (*q)[PBO_NQ8];
  const float* (*f)[PBO_NF32];
  q8t emb;
  const uint16_t* emb16;   /* bf16 tied embedding (dtype 3) instead of emb */
  const float* final_norm;
  float* invf;           /* full-attention layers */
  float* invf_slide;     /* sliding-attention layers */
};
struct pbo_state {
  int n_layers;
  uint16_t** kc; uint16_t** vc; uint16_t** ring;
  uint16_t* x;
};

pbo_model* pbo_model_new(const pbo_cfg* cfg, const int* layer_kind) {
  pbo_model* m = (pbo_model*)calloc(1, sizeof *m);
  m->cfg = *cfg;
  m->is_attn = (int*)malloc(sizeof(int) * cfg->n_layers);      /* 0 conv, 1 full, 2 sliding */
  memcpy(m->is_attn, layer_kind, sizeof(int) * cfg->n_layers);
  m->q = calloc((size_t)cfg->n_layers, sizeof *m->q);
  m->f = calloc((size_t)cfg->n_layers, sizeof *m->f);
  m->invf = (float*)malloc(sizeof(float) * cfg->head_dim / 2);
  pbo_rope_invf(m->invf, cfg->rope_theta, cfg->head_dim, cfg->rope_partial);
  m->invf_slide = (float*)malloc(sizeof(float) * cfg->head_dim / 2);
  pbo_rope_invf(m->invf_slide, cfg->slide_theta, cfg->head_dim, cfg->slide_partial);
  return m;
}
void pbo_model_free(pbo_model* m) {
  if (!m) return;
  free(m->is_attn); free(m->q); free(m->f); free(m->invf); free(m->invf_slide); free(m);
}
void pbo_model_set_q8(pbo_model* m, int layer, int slot, const int8_t* codes,
                      const float* scales, int N, int K) {
  q8t t = {codes, scales, N, K};
  if (layer < 0) m->emb = t; else m->q[layer][slot] = t;
}
void pbo_model_set_emb_bf16(pbo_model* m, const uint16_t* e) { m->emb16 = e; }
void pbo_model_set_f32(pbo_model* m, int layer, int slot, const float* p) {
  if (layer < 0) m->final_norm = p; else m->f[layer][slot] = p;
}
pbo_state* pbo_state_new(const pbo_model* m) {
  const pbo_cfg* c = &m->cfg;
  pbo_state* s = (pbo_state*)calloc(1, sizeof *s);
  s->n_layers = c->n_layers;
  s->kc = calloc((size_t)c->n_layers, sizeof(uint16_t*));
  s->vc = calloc((size_t)c->n_layers, sizeof(uint16_t*));
  s->ring = calloc((size_t)c->n_layers, sizeof(uint16_t*));
  for (int L = 0; L < c->n_layers; L++) {
    if (m->is_attn[L]) {
      const size_t n = (size_t)c->max_ctx * c->n_kv * c->head_dim;
      s->kc[L] = calloc(n, 2); s->vc[L] = calloc(n, 2);
    } else {
      s->ring[L] = calloc((size_t)c->conv_w * c->hidden, 2);
    }
  }
  s->x = calloc((size_t)c->hidden, 2);
  return s;
}
void pbo_state_free(pbo_state* s) {
  if (!s) return;
  for (int L = 0; L < s->n_layers; L++) { free(s->kc[L]); free(s->vc[L]); free(s->ring[L]); }
  free(s->x);
  free(s->kc); free(s->vc); free(s->ring);
  free(s);
}
const uint16_t* pbo_state_kv(const pbo_state* s, int layer, int which) {
  return which ? s->vc[layer] : s->kc[layer];
}
const uint16_t* pbo_state_ring(const pbo_state* s, int layer) { return s->ring[layer]; }

/* the integer path of one projection: x (bf16 values) quantised per 32-block
 * (fwd35_ref.c:332-343), exact int32 block dots, then the fold
 * acc = acc + (dw * dx) * (float)isum in block order (pq1_host.c:112-116
 * pattern); fp32 out */
static void gemv_int(const q8t* t, const uint16_t* x, float* yf) {
  const int K = t->K, nb = K / 32;
  float* xf = (float*)malloc(sizeof(float) * K);
  int8_t* qx = (int8_t*)malloc(K);
  uint16_t* dx = (uint16_t*)malloc(2 * (size_t)nb);
  float* dxf = (float*)malloc(sizeof(float) * nb);
  for (int i = 0; i < K; i++) xf[i] = pbo_bf2f(x[i]);
  pbo_q80_quant_act(xf, K, qx, dx);
  for (int b = 0; b < nb; b++) dxf[b] = pbo_h2f(dx[b]);
#pragma omp parallel for schedule(static)
  for (int n = 0; n < t->N; n++) {
    float acc = 0.0f;
    for (int b = 0; b < nb; b++) {
      const int8_t* cw = t->c + (size_t)n * K + (size_t)b * 32;
      int32_t sum = 0;
      for (int j = 0; j < 32; j++) sum += (int32_t)cw[j] * (int32_t)qx[32 * b + j];
      acc = acc + (t->s[(size_t)n * nb + b] * dxf[b]) * (float)sum;
    }
    yf[n] = acc;
  }
  free(xf); free(qx); free(dx); free(dxf);
}
static int g_int_mode = 0;   /* set for the duration of one pbo_decode call */
static void gemv_bf(const q8t* t, const uint16_t* x, uint16_t* y) {
  float* yf = (float*)malloc(sizeof(float) * t->N);
  if (g_int_mode) gemv_int(t, x, yf);
  else pbo_q8f_gemv(t->c, t->s, t->N, t->K, x, yf);
  for (int i = 0; i < t->N; i++) y[i] = pbo_f2bf(yf[i]);
  free(yf);
}
void pbo_model_set_int(pbo_model* m, int on) { m->int_mode = on; }

/* layer_body, lfm3_nanode.cu:3739-3856 (sandwich norms, conv or attention
 * mixer, SwiGLU FFN), with the conv width and head geometry taken from cfg. */
int pbo_decode(const pbo_model* m, pbo_state* s, int token, int pos, float* logits,
               uint16_t* x_out) {
  const pbo_cfg* c = &m->cfg;
  const int H = c->hidden, F = c->inter, NH = c->n_heads, NKV = c->n_kv, HD = c->head_dim;
  const int W = c->conv_w;
  uint16_t* x = s->x;
  g_int_mode = m->int_mode;
  uint16_t *h1 = malloc(2 * (size_t)H), *h2 = malloc(2 * (size_t)(F > 3 * H ? F : 3 * H));
  uint16_t *h3 = malloc(2 * (size_t)F), *bx = malloc(2 * (size_t)3 * H);
  uint16_t *qb = malloc(2 * (size_t)NH * HD), *kb = malloc(2 * (size_t)NKV * HD);
  uint16_t *vb = malloc(2 * (size_t)NKV * HD), *gb = malloc(2 * (size_t)NH);
  uint16_t *at = malloc(2 * (size_t)NH * HD), *ab = malloc(2 * (size_t)F);
  /* per layer type (lfm3_nanode.cu:3753-3785): full attention rotates
   * (partial * HD)/2 pairs with its own base over every key; sliding attention
   * its own rotation and base over the last slide_window keys */
  const int half_full = (int)((double)c->rope_partial * HD) / 2;
  const int half_slide = (int)((double)c->slide_partial * HD) / 2;
  float* cs = malloc(sizeof(float) * (HD / 2 + 1)); float* sn = malloc(sizeof(float) * (HD / 2 + 1));
  /* embedding row: bf16(code * scale), k_dequant_row (:138-142); a bf16
   * embedding's row as it is (lfm3_nanode.cu:6062-6070) */
  for (int i = 0; i < H; i++)
    x[i] = m->emb16 ? m->emb16[(size_t)token * H + i]
                    : pbo_f2bf((float)m->emb.c[(size_t)token * H + i] * m->emb.s[(size_t)token * (H / 32) + i / 32]);
  for (int L = 0; L < c->n_layers; L++) {
    const q8t* T = m->q[L];
    const float* const* fw = m->f[L];
    pbo_rmsnorm(x, fw[PBO_OPN], h1, H, c->norm_eps);
    if (m->is_attn[L]) {
      gemv_bf(&T[PBO_Q], h1, qb); gemv_bf(&T[PBO_K], h1, kb);
      gemv_bf(&T[PBO_V], h1, vb); gemv_bf(&T[PBO_GATE], h1, gb);
      pbo_headnorm(qb, fw[PBO_QN], NH, HD, c->norm_eps);
      pbo_headnorm(kb, fw[PBO_KN], NKV, HD, c->norm_eps);
      const int slide = m->is_attn[L] == 2;
      const int half = slide ? half_slide : half_full;
      pbo_rope_cs(slide ? m->invf_slide : m->invf, pos, half, cs, sn);
      pbo_rope(qb, NH, HD, half, cs, sn);
      pbo_rope(kb, NKV, HD, half, cs, sn);
      for (int i = 0; i < NKV * HD; i++) {
        s->kc[L][(size_t)pos * NKV * HD + i] = pbo_f2h(pbo_bf2f(kb[i]));
        s->vc[L][(size_t)pos * NKV * HD + i] = pbo_f2h(pbo_bf2f(vb[i]));
      }
      const float scaling = 1.0f / sqrtf((float)HD);
      for (int h = 0; h < NH; h++)
        pbo_attn_head(qb + (size_t)h * HD, s->kc[L], s->vc[L], h / (NH / NKV), NKV, HD, pos + 1,
                      slide ? c->slide_window : c->sliding_window, scaling, gb[h], 1, at + (size_t)h * HD);
      gemv_bf(&T[PBO_O], at, h2);
    } else {
      gemv_bf(&T[PBO_IN], h1, bx);
      for (int i = 0; i < H; i++)                       /* B * x, k_mul_bf (:811-815) */
        h3[i] = pbo_f2bf(pbo_bf2f(bx[i]) * pbo_bf2f(bx[2 * H + i]));
      pbo_conv_step(s->ring[L], h3, fw[PBO_TAPS], W, H, h3);   /* h3 <- conv output */
      for (int i = 0; i < H; i++)                       /* C * y */
        h3[i] = pbo_f2bf(pbo_bf2f(bx[H + i]) * pbo_bf2f(h3[i]));
      gemv_bf(&T[PBO_OUT], h3, h2);
    }
    pbo_rmsnorm(h2, fw[PBO_POSTOPN], h3, H, c->norm_eps);
    for (int i = 0; i < H; i++) x[i] = pbo_f2bf(pbo_bf2f(x[i]) + pbo_bf2f(h3[i]));
    pbo_rmsnorm(x, fw[PBO_FFNN], h1, H, c->norm_eps);
    gemv_bf(&T[PBO_W1], h1, ab);
    gemv_bf(&T[PBO_W3], h1, h3);
    for (int i = 0; i < F; i++) {                       /* k_silu_mul_bf (:821-829) */
      const float a = pbo_bf2f(ab[i]);
      const float sg = 1.0f / (1.0f + pbo_expf(-a));
      ab[i] = pbo_f2bf((a * sg) * pbo_bf2f(h3[i]));
    }
    gemv_bf(&T[PBO_W2], ab, h2);
    pbo_rmsnorm(h2, fw[PBO_POSTFFNN], h3, H, c->norm_eps);
    for (int i = 0; i < H; i++) x[i] = pbo_f2bf(pbo_bf2f(x[i]) + pbo_bf2f(h3[i]));
  }
  /* embedding_norm, then the tied head in fp32 (gemv_f + k_combine_f) */
  pbo_rmsnorm(x, m->final_norm, h1, H, c->norm_eps);
  float* lg = logits ? logits : (float*)malloc(sizeof(float) * c->vocab);
  if (m->emb16) {
    pbo_gemv_bf16(m->emb16, c->vocab, H, h1, lg);     /* lm_head_bf16 in either mode (:5172-5175) */
  } else if (m->int_mode) {
    const q8t head = {m->emb.c, m->emb.s, c->vocab, H};
    gemv_int(&head, h1, lg);
  } else {
    pbo_q8f_gemv(m->emb.c, m->emb.s, c->vocab, H, h1, lg);
  }
  const int id = pbo_argmax(lg, c->vocab);
  if (x_out) memcpy(x_out, x, 2 * (size_t)H);
  if (!logits) free(lg);
  free(h1); free(h2); free(h3); free(bx); free(qb); free(kb); free(vb); free(gb); free(at); free(ab);
  free(cs); free(sn);
  return id;
}

/* ================================================================ Bonsai ====
 * The Q1_0 decode step of pulsar_arm/bonsai2/fwd8.c (Qwen3-style dense GQA
 * layer, head_dim 128). Departure: expf -> pbo_expf (above), as on the device. */

/* fwd8.c:312-317: s = serial double sum of x*x (the products are exact in
 * double, so a contracted fma gives the same value); sc = 1/sqrtf(float(s/n) +
 * 1e-6); y = (x*sc)*w. In place when y == x. */
void pbo_bs_rms(const float* x, const float* w, int n, float* y) {
  double s = 0;
  for (int i = 0; i < n; i++) s = s + (double)x[i] * (double)x[i];
  const float sc = 1.0f / sqrtf((float)(s / n) + 1e-6f);
  for (int i = 0; i < n; i++) y[i] = (x[i] * sc) * w[i];
}

/* fwd8.c:322-358: the YaRN correction range and the 64 (cos, sin) pairs of one
 * position, the contraction of gcc's default build written out: msc =
 * fma(0.1, ln factor, 1), th = fma(ti, 1 - ramp, te*ramp). */
static float bs_corr_dim(int n_ctx, float rot, float base) {
  return 128 * logf(n_ctx / (rot * 2 * (float)M_PI)) / (2 * logf(base));
}
void pbo_bs_rope_table(int pos, float factor, int orig_ctx, float base, float* c, float* s) {
  const float st = floorf(bs_corr_dim(orig_ctx, 32.0f, base));
  const float en = ceilf(bs_corr_dim(orig_ctx, 1.0f, base));
  const float c0 = st > 0 ? st : 0, c1 = en < 127 ? en : 127;
  const float fs = 1.0f / factor, msc = fmaf(0.1f, logf(factor), 1.0f);
  const float tscale = powf(base, -2.0f / 128.0f);
  float theta = (float)pos;
  for (int j = 0; j < 64; j++, theta *= tscale) {
    const float y = (j - c0) / fmaxf(0.001f, c1 - c0);
    const float ramp = 1.0f - fminf(1.0f, fmaxf(0.0f, y));
    const float ti = fs * theta, te = theta;
    const float th = fmaf(ti, 1 - ramp, te * ramp);
    c[j] = cosf(th) * msc;
    s[j] = sinf(th) * msc;
  }
}
/* fwd8.c:359-369 on NEOX pairs (j, j+64), contracted as gcc emits it
 * (fmul; fnmsub; fmul; fmadd): x[j] = fma(a, c, -(b*s)), x[j+64] = fma(a, s, b*c) */
void pbo_bs_rope(float* x, int heads, const float* c, const float* s) {
  for (int h = 0; h < heads; h++) {
    float* xh = x + (size_t)h * 128;
    for (int j = 0; j < 64; j++) {
      const float a = xh[j], b = xh[j + 64];
      xh[j] = fmaf(a, c[j], -(b * s[j]));
      xh[j + 64] = fmaf(a, s[j], b * c[j]);
    }
  }
}

/* pq1_host.c:404-434: one query head over positions 0..T-1 of its kv head with
 * f16 K/V rows [T][128], the fork's flash-attention decode order: Q rounded to
 * f16; q.k as 16 fma chains (chain c = elements 16j+c) reduced
 * ((a_l + a_8+l) + (a_4+l + a_12+l)), ((r0 + r1) + (r2 + r3)); s *= scale;
 * online softmax with the accumulator rounded to f16 after every update. */
void pbo_bs_fa16_head(const float* q, const uint16_t* K, const uint16_t* V, int T, float scale,
                      float* out) {
  float qh[128], vkq[128];
  for (int i = 0; i < 128; i++) { qh[i] = pbo_h2f(pbo_f2h(q[i])); vkq[i] = 0.0f; }
  float S = 0.0f, M = -INFINITY;
  for (int t = 0; t < T; t++) {
    const uint16_t *k = K + (size_t)t * 128, *v = V + (size_t)t * 128;
    float a[16];
    for (int c = 0; c < 16; c++) a[c] = 0.0f;
    for (int j = 0; j < 8; j++)
      for (int c = 0; c < 16; c++) a[c] = fmaf(pbo_h2f(k[16 * j + c]), qh[16 * j + c], a[c]);
    float r[4];
    for (int l = 0; l < 4; l++) r[l] = (a[l] + a[8 + l]) + (a[4 + l] + a[12 + l]);
    float sc = ((r[0] + r[1]) + (r[2] + r[3])) * scale;
    float ms = 1.0f, vs = 1.0f;
    const float Mold = M;
    if (sc > M) {
      M = sc;
      ms = pbo_expf(Mold - M);
      for (int d = 0; d < 128; d++) vkq[d] = pbo_h2f(pbo_f2h(vkq[d] * ms));
    } else {
      vs = pbo_expf(sc - M);
    }
    for (int d = 0; d < 128; d++) vkq[d] = pbo_h2f(pbo_f2h(fmaf(pbo_h2f(v[d]), vs, vkq[d])));
    S = fmaf(S, ms, vs);
  }
  const float si = S == 0.0f ? 0.0f : 1.0f / S;
  for (int d = 0; d < 128; d++) out[d] = vkq[d] * si;
}

/* pq1_host.c:196-227: lu = (g * (1 / (1 + e^-g))) * lu */
void pbo_bs_silu_mul(float* lu, const float* lg, int n) {
  for (int i = 0; i < n; i++) lu[i] = (lg[i] * (1.0f / (1.0f + pbo_expf(-lg[i])))) * lu[i];
}

/* ---- the whole step --------------------------------------------------------- */
typedef struct { uint32_t* bits; uint16_t* scales; int rows, K; } q1t;
struct pbo_bs_model {
  pbo_bs_cfg cfg;
  q1t (*q)[PBO_BS_NQ1];
  const float* (*f)[PBO_BS_NF32];
  q1t emb, head;
  const float* out_norm;
};
struct pbo_bs_state {
  int n_layers;
  uint16_t **kc, **vc;   /* [layer] -> [n_kv][max_ctx][128] f16 */
  float* x;
  int tq;                /* 0: f16 cache; 3, 4, 43: TurboQuant (pbo_bs_state_new_tq) */
  uint32_t **tkc, **tvc; /* [layer] -> codes [n_kv][max_ctx][CW] */
  float **tks, **tvs;    /* [layer] -> scales [n_kv][max_ctx] */
};
pbo_bs_model* pbo_bs_model_new(const pbo_bs_cfg* cfg) {
  pbo_bs_model* m = (pbo_bs_model*)calloc(1, sizeof *m);
  m->cfg = *cfg;
  m->q = calloc((size_t)cfg->n_layers, sizeof *m->q);
  m->f = calloc((size_t)cfg->n_layers, sizeof *m->f);
  return m;
}
static void q1t_free(q1t* t) { free(t->bits); free(t->scales); t->bits = NULL; t->scales = NULL; }
void pbo_bs_model_free(pbo_bs_model* m) {
  if (!m) return;
  for (int L = 0; L < m->cfg.n_layers; L++)
    for (int j = 0; j < PBO_BS_NQ1; j++) q1t_free(&m->q[L][j]);
  q1t_free(&m->emb); q1t_free(&m->head);
  free(m->q); free(m->f); free(m);
}
/* layer -1: slot 0 = token_embd, slot 1 = output.weight (absent: tied) */
void pbo_bs_model_set_q1(pbo_bs_model* m, int layer, int slot, const uint8_t* blocks, int rows, int K) {
  q1t t = {malloc((size_t)rows * (K / 32) * 4), malloc((size_t)rows * (K / 128) * 2), rows, K};
  pbo_q1_repack(blocks, rows, K, t.bits, t.scales);
  q1t* d = layer < 0 ? (slot == 0 ? &m->emb : &m->head) : &m->q[layer][slot];
  q1t_free(d);
  *d = t;
}
/* layer -1: the output norm */
void pbo_bs_model_set_f32(pbo_bs_model* m, int layer, int slot, const float* p) {
  if (layer < 0) m->out_norm = p; else m->f[layer][slot] = p;
}
pbo_bs_state* pbo_bs_state_new(const pbo_bs_model* m) {
  const pbo_bs_cfg* c = &m->cfg;
  pbo_bs_state* s = (pbo_bs_state*)calloc(1, sizeof *s);
  s->n_layers = c->n_layers;
  s->kc = calloc((size_t)c->n_layers, sizeof(uint16_t*));
  s->vc = calloc((size_t)c->n_layers, sizeof(uint16_t*));
  for (int L = 0; L < c->n_layers; L++) {
    s->kc[L] = calloc((size_t)c->n_kv * c->max_ctx * 128, 2);
    s->vc[L] = calloc((size_t)c->n_kv * c->max_ctx * 128, 2);
  }
  s->x = calloc((size_t)c->hidden, 4);
  return s;
}
/* a state whose K/V cache is TurboQuant-coded (bits 3, 4 or 43, pq1_fwd8_glue.c:
 * 211-232); needs n_heads = 4 n_kv */
pbo_bs_state* pbo_bs_state_new_tq(const pbo_bs_model* m, int bits) {
  pbo_bs_state* s = pbo_bs_state_new(m);
  const pbo_bs_cfg* c = &m->cfg;
  const int bk = bits == 43 ? 4 : bits, bv = bits == 43 ? 3 : bits;
  s->tq = bits;
  s->tkc = calloc((size_t)c->n_layers, sizeof(uint32_t*));
  s->tvc = calloc((size_t)c->n_layers, sizeof(uint32_t*));
  s->tks = calloc((size_t)c->n_layers, sizeof(float*));
  s->tvs = calloc((size_t)c->n_layers, sizeof(float*));
  for (int L = 0; L < c->n_layers; L++) {
    s->tkc[L] = calloc((size_t)c->n_kv * c->max_ctx * (bk == 3 ? 12 : 16), 4);
    s->tvc[L] = calloc((size_t)c->n_kv * c->max_ctx * (bv == 3 ? 12 : 16), 4);
    s->tks[L] = calloc((size_t)c->n_kv * c->max_ctx, 4);
    s->tvs[L] = calloc((size_t)c->n_kv * c->max_ctx, 4);
  }
  return s;
}
/* a TurboQuant state's codes of positions < n recoded from its f16 rows (for
 * a cache loaded with pbo_bs_state_kv's arrays) */
void pbo_bs_state_tq_recode(pbo_bs_state* s, const pbo_bs_model* m, int n) {
  if (!s->tq) return;
  const pbo_bs_cfg* c = &m->cfg;
  const int bk = s->tq == 43 ? 4 : s->tq, bv = s->tq == 43 ? 3 : s->tq;
  const int cwk = bk == 3 ? 12 : 16, cwv = bv == 3 ? 12 : 16;
  for (int L = 0; L < c->n_layers; L++)
    for (int kh = 0; kh < c->n_kv; kh++)
      for (int t = 0; t < n; t++) {
        const size_t r = (size_t)kh * c->max_ctx + t;
        pbo_tq_row(s->kc[L] + r * 128, bk, s->tkc[L] + r * cwk, s->tks[L] + r);
        pbo_tq_row(s->vc[L] + r * 128, bv, s->tvc[L] + r * cwv, s->tvs[L] + r);
      }
}
void pbo_bs_state_free(pbo_bs_state* s) {
  if (!s) return;
  if (s->tq) {
    for (int L = 0; L < s->n_layers; L++) { free(s->tkc[L]); free(s->tvc[L]); free(s->tks[L]); free(s->tvs[L]); }
    free(s->tkc); free(s->tvc); free(s->tks); free(s->tvs);
  }
  for (int L = 0; L < s->n_layers; L++) { free(s->kc[L]); free(s->vc[L]); }
  free(s->kc); free(s->vc); free(s->x); free(s);
}
const uint16_t* pbo_bs_state_kv(const pbo_bs_state* s, int layer, int which) {
  return which ? s->vc[layer] : s->kc[layer];
}
/* gemvP (fwd8.c:288-293): Q8_K of x, then the Q1 GEMV */
static void bs_gemv(const q1t* t, const float* x, uint8_t* xq, float* y) {
  pbo_q8k_quant(x, t->K, xq);
  pbo_q1_gemv(t->rows, t->K, t->bits, t->scales, xq, NULL, y);
}
/* embed (fwd8.c:438-452, Q1_0 branch): x = bit ? sc : -sc, sc the widened
 * fp16 scale with -0 read as +0 (fwd8.c:265-272) */
static void bs_embed(const q1t* e, int id, float* x) {
  const int ng = e->K / 128;
  for (int g = 0; g < ng; g++) {
    const uint16_t h = e->scales[(size_t)id * ng + g];
    const float sc = h == 0x8000u ? 0.0f : pbo_h2f(h);
    for (int j = 0; j < 128; j++) {
      const uint32_t w = e->bits[(size_t)id * (e->K / 32) + g * 4 + (j >> 5)];
      x[g * 128 + j] = ((w >> (j & 31)) & 1u) ? sc : -sc;
    }
  }
}
/* fwd8.c:812-883 with attn_cpu (:529-647, the PQ1 f16 branch): one token at
 * position pos. x_in (fp32 [hidden]) replaces the embedding when non-NULL
 * (pq1_token_fused's contract); logits (fp32 [vocab]) and x_out (the final
 * residual) are optional. Returns the greedy id (fwd8.c:465-469: first max). */
int pbo_bs_decode(const pbo_bs_model* m, pbo_bs_state* s, int token, int pos, const float* x_in,
                  float* logits, float* x_out) {
  const pbo_bs_cfg* c = &m->cfg;
  const int H = c->hidden, F = c->inter, NH = c->n_heads, NKV = c->n_kv;
  const int QD = NH * 128, KD = NKV * 128, G = NH / NKV;
  const int KMAX = (F > QD ? F : QD) > H ? (F > QD ? F : QD) : H;
  float* x = s->x;
  float *xn = malloc(4 * (size_t)H), *qf = malloc(4 * (size_t)QD), *kf = malloc(4 * (size_t)KD);
  float *vf = malloc(4 * (size_t)KD), *at = malloc(4 * (size_t)QD), *ao = malloc(4 * (size_t)H);
  float *lg = malloc(4 * (size_t)F), *lu = malloc(4 * (size_t)F);
  uint8_t* xq = malloc((size_t)(KMAX / 256) * 292);
  float rc[64], rs[64];
  pbo_bs_rope_table(pos, c->rope_factor, c->rope_orig_ctx, c->rope_base, rc, rs);
  if (x_in) memcpy(x, x_in, 4 * (size_t)H);
  else bs_embed(&m->emb, token, x);
  for (int L = 0; L < c->n_layers; L++) {
    const q1t* T = m->q[L];
    const float* const* fw = m->f[L];
    pbo_bs_rms(x, fw[PBO_BS_ATTN_NORM], H, xn);
    pbo_q8k_quant(xn, H, xq);
    pbo_q1_gemv(QD, H, T[PBO_BS_Q].bits, T[PBO_BS_Q].scales, xq, NULL, qf);
    pbo_q1_gemv(KD, H, T[PBO_BS_K].bits, T[PBO_BS_K].scales, xq, NULL, kf);
    pbo_q1_gemv(KD, H, T[PBO_BS_V].bits, T[PBO_BS_V].scales, xq, NULL, vf);
    for (int h = 0; h < NH; h++) pbo_bs_rms(qf + h * 128, fw[PBO_BS_Q_NORM], 128, qf + h * 128);
    for (int h = 0; h < NKV; h++) pbo_bs_rms(kf + h * 128, fw[PBO_BS_K_NORM], 128, kf + h * 128);
    pbo_bs_rope(qf, NH, rc, rs);
    pbo_bs_rope(kf, NKV, rc, rs);
    for (int kh = 0; kh < NKV; kh++)
      for (int d = 0; d < 128; d++) {
        const size_t o = ((size_t)kh * c->max_ctx + pos) * 128 + d;
        s->kc[L][o] = pbo_f2h(kf[kh * 128 + d]);
        s->vc[L][o] = pbo_f2h(vf[kh * 128 + d]);
      }
    if (s->tq) {   /* the f16 rows of pos, coded (pq1_tq_store), then the TurboQuant attention */
      const int bk = s->tq == 43 ? 4 : s->tq, bv = s->tq == 43 ? 3 : s->tq;
      const int cwk = bk == 3 ? 12 : 16, cwv = bv == 3 ? 12 : 16;
      for (int kh = 0; kh < NKV; kh++) {
        const size_t r = (size_t)kh * c->max_ctx + pos;
        pbo_tq_row(s->kc[L] + r * 128, bk, s->tkc[L] + r * cwk, s->tks[L] + r);
        pbo_tq_row(s->vc[L] + r * 128, bv, s->tvc[L] + r * cwv, s->tvs[L] + r);
      }
      for (int kh = 0; kh < NKV; kh++) {
        const size_t r = (size_t)kh * c->max_ctx;
        pbo_tq_attn(qf + (size_t)kh * 4 * 128, bk, bv, s->tkc[L] + r * cwk, s->tks[L] + r, s->tvc[L] + r * cwv,
                    s->tvs[L] + r, pos + 1, at + (size_t)kh * 4 * 128);
      }
    } else {
      for (int h = 0; h < NH; h++) {
        const size_t base = (size_t)(h / G) * c->max_ctx * 128;
        pbo_bs_fa16_head(qf + h * 128, s->kc[L] + base, s->vc[L] + base, pos + 1, c->attn_scale,
                         at + h * 128);
      }
    }
    bs_gemv(&T[PBO_BS_O], at, xq, ao);
    for (int i = 0; i < H; i++) x[i] = x[i] + ao[i];
    pbo_bs_rms(x, fw[PBO_BS_FFN_NORM], H, xn);
    pbo_q8k_quant(xn, H, xq);
    pbo_q1_gemv(F, H, T[PBO_BS_GATE].bits, T[PBO_BS_GATE].scales, xq, NULL, lg);
    pbo_q1_gemv(F, H, T[PBO_BS_UP].bits, T[PBO_BS_UP].scales, xq, NULL, lu);
    pbo_bs_silu_mul(lu, lg, F);
    bs_gemv(&T[PBO_BS_DOWN], lu, xq, ao);
    for (int i = 0; i < H; i++) x[i] = x[i] + ao[i];
  }
  pbo_bs_rms(x, m->out_norm, H, xn);
  const q1t* hd = m->head.bits ? &m->head : &m->emb;
  float* out = logits ? logits : (float*)malloc(sizeof(float) * c->vocab);
  bs_gemv(hd, xn, xq, out);
  const int id = pbo_argmax(out, c->vocab);
  if (x_out) memcpy(x_out, x, 4 * (size_t)H);
  if (!logits) free(out);
  free(xn); free(qf); free(kf); free(vf); free(at); free(ao); free(lg); free(lu); free(xq);
  return id;
}

/* ---- sampler ------------------------------------------------------------------
 * sample_topkpp + frand01, pulsar_arm/bonsai2/fwd8.c:465-521. The reference
 * keeps a descending insertion list of at most k entries; a later value equal
 * to an entry goes after it and a full list drops it, so the list is the
 * first k of all (value, index) pairs ordered by value descending, then index
 * ascending. That order is produced here by a sort. */
typedef struct { float v; int i; } pbo_vi;
static int pbo_vi_cmp(const void* pa, const void* pb) {
  const pbo_vi* a = (const pbo_vi*)pa;
  const pbo_vi* b = (const pbo_vi*)pb;
  if (a->v > b->v) return -1;
  if (a->v < b->v) return 1;
  return (a->i > b->i) - (a->i < b->i);
}
int pbo_sample_topkpp(const float* lg, int n, float temp, float topp, int topk, float minp, uint64_t* rs,
                      int libm_exp) {
  float (*ex)(float) = libm_exp ? expf : pbo_expf;
  for (int i = 0; i < n; i++)
    if (lg[i] != lg[i]) return -1;
  if (temp <= 0.0f) return pbo_argmax(lg, n);
  int k = (topk <= 0 || topk > 1024) ? 1024 : topk;
  if (k > n) k = n;
  pbo_vi* all = malloc(sizeof(pbo_vi) * (size_t)n);
  for (int i = 0; i < n; i++) { all[i].v = lg[i]; all[i].i = i; }
  qsort(all, (size_t)n, sizeof(pbo_vi), pbo_vi_cmp);
  const float mx = all[0].v;
  int m = k;
  if (minp > 0.0f) {   /* min-p on the raw logits */
    const float thr = mx + logf(minp);
    while (m > 1 && all[m - 1].v < thr) m--;
  }
  double es = 0.0;     /* top-p on the raw logits */
  for (int j = 0; j < m; j++) es += (double)ex(all[j].v - mx);
  double acc = 0.0;
  int keep = m;
  for (int j = 0; j < m; j++) {
    acc += (double)ex(all[j].v - mx) / es;
    if (acc >= (double)topp) { keep = j + 1; break; }
  }
  double es2 = 0.0;    /* temperature last, softmax, draw */
  for (int j = 0; j < keep; j++) es2 += (double)ex((all[j].v - mx) / temp);
  *rs = *rs * 6364136223846793005ull + 1442695040888963407ull;
  const float r01 = (float)((double)(*rs >> 11) * (1.0 / 9007199254740992.0));
  const double r = (double)r01 * es2;
  double a2 = 0.0;
  int id = all[keep - 1].i;
  for (int j = 0; j < keep; j++) {
    a2 += (double)ex((all[j].v - mx) / temp);
    if (r < a2 || j == keep - 1) { id = all[j].i; break; }
  }
  free(all);
  return id;
}

/* ---- low-bit (Q4 / Q5) GEMV --------------------------------------------------
 * pulsar_arm/asm/lfm3_qlow.cuh:20-113. Per row r (tile r/32, lane r%32): K is
 * cut into KS slices (2, or 4 from K = 4096, lfm3_nanode.cu:1899); per slice
 * y = 0 and, group by group in order, the codes q of the group become
 * f = 1 + q/128, four fma chains a_b run over weights b, b+4, ..., b+28,
 * acc = (a0 + a1) + (a2 + a3), sx = the group's x summed in order from 0,
 * y = fma(d', acc - sx, fma(mn, sx, y)); out = bf16(((0 + y_0) + y_1) ...)
 * (k_qlow_combine, :104-110; its rounding has no inf / NaN case). */
static inline uint32_t qlow_code(const uint8_t* grp, int bits, int lane, int k) {
  /* grp: the (tile, group) record; lane's uint4 at grp + 16*lane; weight k =
   * 8i + 4hf + b sits in word i, byte b, nibble hf */
  const int i = k >> 3, hf = (k >> 2) & 1, b = k & 3;
  const uint8_t byte = grp[16 * lane + 4 * i + b];
  uint32_t q = hf ? (uint32_t)(byte >> 4) : (uint32_t)(byte & 15u);
  if (bits == 5) {
    const uint8_t* pl = grp + 512 + 4 * lane;   /* the lane's high-bit plane word */
    const int p = 2 * i + hf;                   /* quad; bit 8b + p of the word */
    const uint32_t word = (uint32_t)pl[0] | (uint32_t)pl[1] << 8 | (uint32_t)pl[2] << 16 | (uint32_t)pl[3] << 24;
    q |= ((word >> (8 * b + p)) & 1u) << 4;
  }
  return q;
}
void pbo_qlow_gemv(const uint8_t* codes, const uint16_t* scales, int bits, int N, int K, int T,
                   const uint16_t* x, uint16_t* y) {
  const int G = K / 32, KS = K >= 4096 ? 4 : 2, GL = G / KS;
  const size_t rec = bits == 5 ? 640 : 512;   /* bytes per (tile, group) */
  float* xf = malloc(sizeof(float) * (size_t)K);
  float* sx = malloc(sizeof(float) * (size_t)G);
  for (int t = 0; t < T; t++) {
    for (int k = 0; k < K; k++) xf[k] = pbo_bf2f(x[(size_t)t * K + k]);
    for (int g = 0; g < G; g++) {
      float s = 0.0f;
      for (int k = 0; k < 32; k++) s = s + xf[g * 32 + k];
      sx[g] = s;
    }
#pragma omp parallel for schedule(static)
    for (int r = 0; r < N; r++) {
      const int tile = r / 32, lane = r % 32;
      float out = 0.0f;
      for (int sl = 0; sl < KS; sl++) {
        float yv = 0.0f;
        for (int g = sl * GL; g < (sl + 1) * GL; g++) {
          const uint8_t* grp = codes + ((size_t)tile * G + g) * rec;
          float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          for (int k = 0; k < 32; k++) {   /* chain b = k % 4, in k order */
            const uint32_t q = qlow_code(grp, bits, lane, k);
            const float f = bitsf(0x3F800000u | (q << 16));   /* 1 + q/128 */
            a[k & 3] = fmaf(f, xf[g * 32 + k], a[k & 3]);
          }
          const float acc = (a[0] + a[1]) + (a[2] + a[3]);
          const size_t si = (((size_t)tile * G + g) * 32 + lane) * 2;
          const float dp = pbo_h2f(scales[si]), mn = pbo_h2f(scales[si + 1]);
          yv = fmaf(dp, acc - sx[g], fmaf(mn, sx[g], yv));
        }
        out = out + yv;
      }
      const uint32_t u = fbits(out);
      y[(size_t)t * N + r] = (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
    }
  }
  free(xf);
  free(sx);
}

/* ---- TurboQuant K/V cache ----------------------------------------------------
 * pulsar_arm/bonsai2/pq1_swar_sm53.cu:3264-3990 (Zandieh et al., TurboQuant,
 * the MSE variant): a 128-value row x is rotated, y = H D x (H the Sylvester
 * Hadamard matrix, unnormalised, D the fixed sign pattern below), each
 * coordinate of y / |x| is replaced by the index of its Lloyd-Max level for
 * the sphere marginal at d = 128 (sign + magnitude), and the row keeps
 * s = |x| / |c|. The codebook, its thresholds and D define the stored format
 * and are the reference's (:3282-3288). The warp orders of the reference's
 * kernels are emulated: lane l holds elements 4l..4l+3; a butterfly over lanes
 * is the xor-shuffle loop the kernels run. */
static const float TQC3[4] = {0.24444127f, 0.75336427f, 1.33664119f, 2.13151002f};
static const float TQT3[3] = {0.49890277f, 1.04500270f, 1.73407555f};
static const float TQC4[8] = {0.12788960f, 0.38643676f, 0.65370631f, 0.93720949f,
                              1.24789774f, 1.60447431f, 2.04605246f, 2.68896675f};
static const float TQT4[7] = {0.25716320f, 0.52007151f, 0.79545790f, 1.09255362f,
                              1.42618608f, 1.82526338f, 2.36750960f};
static const uint32_t TQD[4] = {0xb5297a4du, 0x68e31da4u, 0x1b56c4e9u, 0xf3c2a581u};

static float tq_dsign(float v, int j) { return (TQD[j >> 5] >> (j & 31)) & 1u ? -v : v; }
static float tq_cent(int bits, int v) {   /* signed level of code v */
  const float m = bits == 3 ? TQC3[v & 3] : TQC4[v & 7];
  return (v >> (bits - 1)) & 1 ? -m : m;
}
/* xs[128] (lane l holds 4l..4l+3) <- H xs: the pairs within a lane, then the
 * xor butterflies over lanes m = 1, 2, ..., 16 (:3297-3307) */
static void tq_fwht(float* xs) {
  for (int l = 0; l < 32; l++) {
    float* x = xs + 4 * l;
    const float a = x[0] + x[1], b = x[0] - x[1], c = x[2] + x[3], d = x[2] - x[3];
    x[0] = a + c; x[1] = b + d; x[2] = a - c; x[3] = b - d;
  }
  for (int m = 1; m < 32; m <<= 1) {
    float y[128];
    for (int l = 0; l < 32; l++)
      for (int i = 0; i < 4; i++) {
        const float own = xs[4 * l + i], p = xs[4 * (l ^ m) + i];
        y[4 * l + i] = (l & m) ? p - own : own + p;
      }
    memcpy(xs, y, sizeof y);
  }
}
/* the xor-shuffle sum of one value per lane (o = 16, 8, 4, 2, 1); every lane
 * ends with the same total, returned */
static float tq_xor_sum(const float* v) {
  float a[32];
  memcpy(a, v, sizeof a);
  for (int o = 16; o; o >>= 1) {
    float b[32];
    for (int l = 0; l < 32; l++) b[l] = a[l] + a[l ^ o];
    memcpy(a, b, sizeof a);
  }
  return a[0];
}
/* pq1_tq_row (:3312-3366) */
void pbo_tq_row(const uint16_t* row, int bits, uint32_t* cw, float* scale) {
  float x[128], n2l[32], c2l[32];
  int v[128];
  for (int l = 0; l < 32; l++) {
    float n2 = 0.0f;
    for (int i = 0; i < 4; i++) {
      const float e = pbo_h2f(row[4 * l + i]);
      n2 = fmaf(e, e, n2);
      x[4 * l + i] = tq_dsign(e, 4 * l + i);
    }
    n2l[l] = n2;
  }
  const float n2 = tq_xor_sum(n2l);
  tq_fwht(x);
  const float nrm = sqrtf(n2), inv = nrm > 0.0f ? 1.0f / nrm : 0.0f;
  for (int l = 0; l < 32; l++) {
    float c2 = 0.0f;
    for (int i = 0; i < 4; i++) {
      const float z = x[4 * l + i] * inv, a = fabsf(z);
      int m = 0;
      if (bits == 3) m = (a > TQT3[0]) + (a > TQT3[1]) + (a > TQT3[2]);
      else for (int k = 0; k < 7; k++) m += a > TQT4[k];
      const float c = bits == 3 ? TQC3[m] : TQC4[m];
      c2 = fmaf(c, c, c2);
      v[4 * l + i] = m | ((z < 0.0f) << (bits - 1));
    }
    c2l[l] = c2;
  }
  const float c2 = tq_xor_sum(c2l);
  if (bits == 3) {   /* 8 words of 2-bit magnitudes (16 per word), 4 words of sign bits */
    for (int k = 0; k < 12; k++) cw[k] = 0u;
    for (int j = 0; j < 128; j++) {
      cw[j >> 4] |= (uint32_t)(v[j] & 3) << (2 * (j & 15));
      cw[8 + (j >> 5)] |= (uint32_t)(v[j] >> 2) << (j & 31);
    }
  } else {           /* 16 words of nibbles (magnitude | sign << 3) */
    for (int k = 0; k < 16; k++) cw[k] = 0u;
    for (int j = 0; j < 128; j++) cw[j >> 3] |= (uint32_t)v[j] << (4 * (j & 7));
  }
  *scale = c2 > 0.0f ? nrm * (1.0f / sqrtf(c2)) : 0.0f;
}
static int tq_code(const uint32_t* cw, int bits, int j) {
  if (bits == 3) return (int)((cw[j >> 4] >> (2 * (j & 15))) & 3u) | (int)(((cw[8 + (j >> 5)] >> (j & 31)) & 1u) << 2);
  return (int)((cw[j >> 3] >> (4 * (j & 7))) & 15u);
}
/* pq1_tq_qk2 / pq1_tq_sm / pq1_tq_pv2 / pq1_tq_out (:3447-3714, the long
 * chain; the short pair, :3722-3905, is the same arithmetic) */
void pbo_tq_attn(const float* q, int bk, int bv, const uint32_t* kcode, const float* ksc, const uint32_t* vcode,
                 const float* vsc, int T, float* atto) {
  const int cwk = bk == 3 ? 12 : 16, cwv = bv == 3 ? 12 : 16;
  float qr[4][128];
  for (int h = 0; h < 4; h++) {   /* R q with R's 1/sqrt(128) and the score scale: 2^-7 */
    float x[128];
    for (int j = 0; j < 128; j++) x[j] = tq_dsign(q[h * 128 + j], j);
    tq_fwht(x);
    for (int j = 0; j < 128; j++) qr[h][j] = x[j] * 0.0078125f;
  }
  float* sc = malloc(sizeof(float) * 4 * (size_t)T);
  for (int t = 0; t < T; t++) {   /* scores: a + fl(q_r c) over j in order, then the row scale */
    const uint32_t* cw = kcode + (size_t)t * cwk;
    for (int h = 0; h < 4; h++) {
      float a = 0.0f;
      for (int j = 0; j < 128; j++) a = a + qr[h][j] * tq_cent(bk, tq_code(cw, bk, j));
      sc[h * T + t] = a * ksc[t];
    }
  }
  float inv[4];
  for (int h = 0; h < 4; h++) {   /* 256 threads: strided per-thread max and sum, warp xor tree, 8 warps in order */
    float* s = sc + (size_t)h * T;
    float tm[256], ts[256], wm[8], wsum[8];
    for (int th = 0; th < 256; th++) {
      float m = -INFINITY;
      for (int t = th; t < T; t += 256) m = fmaxf(m, s[t]);
      tm[th] = m;
    }
    for (int w = 0; w < 8; w++) {
      float a[32];
      memcpy(a, tm + 32 * w, sizeof a);
      for (int o = 16; o; o >>= 1) {
        float b[32];
        for (int l = 0; l < 32; l++) b[l] = fmaxf(a[l], a[l ^ o]);
        memcpy(a, b, sizeof a);
      }
      wm[w] = a[0];
    }
    float m = wm[0];
    for (int k = 1; k < 8; k++) m = fmaxf(m, wm[k]);
    for (int th = 0; th < 256; th++) {
      float sum = 0.0f;
      for (int t = th; t < T; t += 256) { const float p = pbo_expf(s[t] - m); s[t] = p; sum += p; }
      ts[th] = sum;
    }
    for (int w = 0; w < 8; w++) wsum[w] = tq_xor_sum(ts + 32 * w);
    float z = 0.0f;
    for (int k = 0; k < 8; k++) z += wsum[k];
    inv[h] = 1.0f / z;
  }
  const int nc = (T + 255) / 256;   /* P.V in the rotated domain, 256-position chunks */
  float acc[4][128];
  for (int h = 0; h < 4; h++) for (int d = 0; d < 128; d++) acc[h][d] = 0.0f;
  for (int c = 0; c < nc; c++) {
    const int t0 = c * 256, n = T - t0 < 256 ? T - t0 : 256;
    float part[4][4][128];   /* [warp][head][dim]: warp w takes positions w, w+4, ... of the chunk */
    for (int w = 0; w < 4; w++)
      for (int h = 0; h < 4; h++) {
        for (int d = 0; d < 128; d++) part[w][h][d] = 0.0f;
        for (int t = w; t < n; t += 4) {
          const float g = sc[h * T + t0 + t] * vsc[t0 + t];
          const uint32_t* cw = vcode + (size_t)(t0 + t) * cwv;
          for (int d = 0; d < 128; d++) part[w][h][d] = fmaf(g, tq_cent(bv, tq_code(cw, bv, d)), part[w][h][d]);
        }
      }
    for (int h = 0; h < 4; h++)
      for (int d = 0; d < 128; d++) {
        const float cs = ((part[0][h][d] + part[1][h][d]) + part[2][h][d]) + part[3][h][d];
        acc[h][d] = acc[h][d] + cs;
      }
  }
  for (int h = 0; h < 4; h++) {   /* R^T: H, the 1/sqrt(128), 1/sum, then D */
    float x[128];
    memcpy(x, acc[h], sizeof x);
    tq_fwht(x);
    const float k = inv[h] * 0.0883883476f;
    for (int j = 0; j < 128; j++) atto[h * 128 + j] = tq_dsign(x[j] * k, j);
  }
  free(sc);
}
