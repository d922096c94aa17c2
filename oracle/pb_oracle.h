/* pb_oracle.h -- CPU restatement of PULSAR-ASM's quantized weight-streaming
 * hot path. TEST INFRASTRUCTURE ONLY: this library is the checker that the
 * CUDA product is compared against. Only tests/, __graft_entry__.smoke() and
 * bench.py's CPU-baseline arm may load it; the product never links it.
 *
 * Every function names the reference file:line whose arithmetic it restates
 * (paths are relative to the PULSAR-ASM project root). Built with
 * -ffp-contract=off so every fmaf() below is the one written and no other
 * multiply/add pair is fused, as the reference's own host code insists
 * (.auto/lfm3/q8_gemv_cpu.c:10-16).
 *
 * Where the reference uses device intrinsics that have no bit-identical CPU
 * counterpart (rsqrtf, expf, cosf/sinf on the GPU), this oracle and the CUDA
 * product both use the deterministic replacements listed in pb_oracle.c's
 * header comment, so the two agree bit for bit.
 */
#ifndef PB_ORACLE_H
#define PB_ORACLE_H
#include <stdint.h>
#include <stddef.h>
#ifdef __cplusplus
extern "C" {
#endif

/* ---- scalar numerics ---------------------------------------------------- */
uint16_t pbo_f2bf(float v);          /* lfm3_nanode.cu:116-121 (RNE, inf/nan pass-through) */
float pbo_bf2f(uint16_t h);
uint16_t pbo_f2h(float v);           /* IEEE binary16, round to nearest even */
float pbo_h2f(uint16_t h);           /* exact widening (pq1_host.c:14-24) */
float pbo_expf(float x);             /* Cody-Waite + degree-7 Taylor, see pb_oracle.c */

/* ---- Q8 float path (LFM3 REF_FLOAT): bf16 x, fp32 FMA, reference tree ---- */
int pbo_q8_kchunk(int K);            /* pick(): lfm3_nanode.cu:1763-1768 */
/* y[n] = ((0 + p_0) + p_1) + ... over K-chunks; p_c = 32-leaf shuffle tree of
 * lane chains (lfm3_nanode.cu:222-343). scales are fp32 (fp16 callers widen). */
void pbo_q8f_gemv(const int8_t* codes, const float* scales, int N, int K,
                  const uint16_t* x_bf16, float* y);
/* T positions, position-major x [T][K], y [T][N] (pf_gemv_T values). */
void pbo_q8f_gemm(const int8_t* codes, const float* scales, int N, int K, int T,
                  const uint16_t* x_bf16, float* y);

/* ---- Q8_0 x Q8_0 integer path --------------------------------------------- */
/* Activation quantizer per 32-block (fwd35_ref.c:332-343). */
void pbo_q80_quant_act(const float* x, int K, int8_t* qx, uint16_t* dx_h);
/* isum[n][b] exact int32; y[n] = sum_b (dw*dx)*(float)isum in block order. */
void pbo_q80_gemv(const int8_t* codes, const uint16_t* dw_h, int N, int K,
                  const int8_t* qx, const uint16_t* dx_h, int32_t* isum, float* y);

/* ---- Q1_0 x Q8_K ---------------------------------------------------------- */
void pbo_q1_repack(const uint8_t* q1, int rows, int K, uint32_t* w_bits, uint16_t* w_scales);
void pbo_q8k_quant(const float* x, int K, uint8_t* xq);  /* 292 B per 256 values */
void pbo_q1_rms_q8k(float* x, const float* r, const float* w, int n, float eps, float* y,
                    uint8_t* xq);
void pbo_q1_gemv(int rows, int K, const uint32_t* w_bits, const uint16_t* w_scales,
                 const uint8_t* xq, int32_t* isum, float* y);

/* ---- layer pieces (bf16 activations stored as uint16) --------------------- */
void pbo_rmsnorm(const uint16_t* x, const float* w, uint16_t* y, int H, float eps);
void pbo_headnorm(uint16_t* x, const float* w, int nheads, int hd, float eps);
void pbo_rope_invf(float* invf, float base, int hd, float partial);
void pbo_rope_cs(const float* invf, int pos, int half, float* c, float* s);
void pbo_rope(uint16_t* x, int nheads, int hd, int half, const float* c, const float* s);
void pbo_attn_head(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, int kvh,
                   int nkv, int hd, int npos, int win, float scaling, uint16_t gate,
                   int use_gate, uint16_t* out);
int pbo_argmax(const float* v, int n);
void pbo_conv_step(uint16_t* ring, const uint16_t* xin, const float* taps, int W, int H, uint16_t* y);
void pbo_silu_mul_bf(const uint16_t* a, const uint16_t* b, uint16_t* y, int n);
void pbo_sigmoid_gate(const uint16_t* g, uint16_t* attn, int nh, int hd);

/* ---- whole LFM3-style decode step ----------------------------------------- */
typedef struct {
  int hidden, inter, n_layers, n_heads, n_kv, head_dim, vocab, conv_w, max_ctx;
  int sliding_window;          /* full-attention layers' window; 0 = every key */
  float rope_theta, rope_partial, norm_eps;
  /* sliding-attention layers (layer kind 2): their window and RoPE */
  int slide_window;
  float slide_theta, slide_partial;
} pbo_cfg;

enum {  /* tensor slots per layer */
  PBO_Q = 0, PBO_K, PBO_V, PBO_GATE, PBO_O, PBO_IN, PBO_OUT, PBO_W1, PBO_W3, PBO_W2,
  PBO_NQ8
};
enum {  /* fp32 slots per layer */
  PBO_OPN = 0, PBO_POSTOPN, PBO_FFNN, PBO_POSTFFNN, PBO_QN, PBO_KN, PBO_TAPS, PBO_NF32
};

typedef struct pbo_model pbo_model;
typedef struct pbo_state pbo_state;

/* layer_kind per layer: 0 gated short conv, 1 full attention, 2 sliding attention */
pbo_model* pbo_model_new(const pbo_cfg* cfg, const int* layer_kind);
void pbo_model_free(pbo_model* m);
void pbo_model_set_q8(pbo_model* m, int layer, int slot, const int8_t* codes,
                      const float* scales, int N, int K);
void pbo_model_set_f32(pbo_model* m, int layer, int slot, const float* p);
/* 1: every projection (and the head) on the Q8_0 integer path: activations
 * quantised per 32-block, exact block dots, in-order fp32 fold (the chunked
 * prefill's tensor-core form); 0: the reference's float path (default) */
void pbo_model_set_int(pbo_model* m, int on);
/* layer -1: the tied embedding / head (Q8) and the final norm (fp32). */
/* the tied embedding as bf16 (blob dtype 3): the embedding row is copied and
 * the head is k_gemv_bf16 (lfm3_nanode.cu:3517-3534) */
void pbo_model_set_emb_bf16(pbo_model* m, const uint16_t* e);
void pbo_gemv_bf16(const uint16_t* w, int N, int K, const uint16_t* x_bf16, float* y);
pbo_state* pbo_state_new(const pbo_model* m);
void pbo_state_free(pbo_state* s);
/* one token at position pos; returns the greedy id. logits (fp32 [vocab])
 * and the final residual x (bf16 [hidden]) are optional outputs. */
int pbo_decode(const pbo_model* m, pbo_state* s, int token, int pos, float* logits,
               uint16_t* x_out);
/* expose state for checks: K/V cache row (fp16) and conv ring (bf16) */
const uint16_t* pbo_state_kv(const pbo_state* s, int layer, int which);
const uint16_t* pbo_state_ring(const pbo_state* s, int layer);

/* ---- Bonsai-8B-shaped Q1_0 decode step (fwd8.c), head_dim 128 ------------- */
void pbo_bs_rms(const float* x, const float* w, int n, float* y);          /* fwd8.c:312-317 */
void pbo_bs_rope_table(int pos, float factor, int orig_ctx, float base, float* c, float* s);
void pbo_bs_rope(float* x, int heads, const float* c, const float* s);    /* fwd8.c:359-369 */
void pbo_bs_fa16_head(const float* q, const uint16_t* K, const uint16_t* V, int T, float scale,
                      float* out);                                         /* pq1_host.c:404-434 */
void pbo_bs_silu_mul(float* lu, const float* lg, int n);                   /* pq1_host.c:196-227 */

typedef struct {
  int hidden, inter, n_layers, n_heads, n_kv, vocab, max_ctx;
  float rope_factor;   /* YaRN factor (fwd8.c:51: 4) */
  int rope_orig_ctx;   /* YaRN original context (fwd8.c:56: 16384 for the 8B) */
  float rope_base;     /* fwd8.c:57: 1e6 for the 8B */
  float attn_scale;    /* fwd8.c:566: 0.0883883476 = 1/sqrt(128) */
} pbo_bs_cfg;
enum { PBO_BS_Q = 0, PBO_BS_K, PBO_BS_V, PBO_BS_O, PBO_BS_GATE, PBO_BS_UP, PBO_BS_DOWN, PBO_BS_NQ1 };
enum { PBO_BS_ATTN_NORM = 0, PBO_BS_FFN_NORM, PBO_BS_Q_NORM, PBO_BS_K_NORM, PBO_BS_NF32 };
typedef struct pbo_bs_model pbo_bs_model;
typedef struct pbo_bs_state pbo_bs_state;
pbo_bs_model* pbo_bs_model_new(const pbo_bs_cfg* cfg);
void pbo_bs_model_free(pbo_bs_model* m);
/* Q1_0 18-byte blocks [rows][K/128]; layer -1: slot 0 token_embd, slot 1 output.weight */
void pbo_bs_model_set_q1(pbo_bs_model* m, int layer, int slot, const uint8_t* blocks, int rows, int K);
/* fp32 norm weights (kept by pointer); layer -1: output_norm */
void pbo_bs_model_set_f32(pbo_bs_model* m, int layer, int slot, const float* p);
pbo_bs_state* pbo_bs_state_new(const pbo_bs_model* m);
/* the same with a TurboQuant K/V cache (bits 3, 4 or 43; n_heads = 4 n_kv):
 * each position's f16 K/V rows are coded at their store, and attention runs
 * over the codes (pbo_tq_attn) */
pbo_bs_state* pbo_bs_state_new_tq(const pbo_bs_model* m, int bits);
void pbo_bs_state_tq_recode(pbo_bs_state* s, const pbo_bs_model* m, int n);
void pbo_bs_state_free(pbo_bs_state* s);
const uint16_t* pbo_bs_state_kv(const pbo_bs_state* s, int layer, int which);
int pbo_bs_decode(const pbo_bs_model* m, pbo_bs_state* s, int token, int pos, const float* x_in,
                  float* logits, float* x_out);

/* the low-bit GEMV (lfm3_qlow.cuh: k_qlow + k_qlow_combine, launched by
 * qlow_gemv, lfm3_nanode.cu:1894-1915): codes / scales in the exporter's
 * tiled payload, bits 4 or 5; T positions x [T][K] bf16 -> y [T][N] bf16 */
void pbo_qlow_gemv(const uint8_t* codes, const uint16_t* scales, int bits, int N, int K, int T,
                   const uint16_t* x, uint16_t* y);

/* TurboQuant K/V cache (pulsar_arm/bonsai2/pq1_swar_sm53.cu:3264-3990): bits
 * 3 or 4 per coordinate; a row is CW = 12 (3-bit) or 16 (4-bit) code words and
 * one f32 scale. pbo_tq_row encodes one f16 row of 128 values. pbo_tq_attn is
 * the attention of the 4 query heads of one KV head (post-rope fp32 q [4][128])
 * over positions 0..T-1 of a TurboQuant cache (codes [ctx][CW], scales [ctx])
 * into atto [4][128]. rsqrtf -> 1/sqrt and expf -> pbo_expf, as everywhere. */
void pbo_tq_row(const uint16_t* row, int bits, uint32_t* cw, float* scale);
void pbo_tq_attn(const float* q, int bk, int bv, const uint32_t* kcode, const float* ksc, const uint32_t* vcode,
                 const float* vsc, int T, float* atto);

/* sample_topkpp + frand01 (fwd8.c:465-521): top-k (k <= 1024; <= 0 means
 * 1024), min-p and top-p on the raw logits, temperature last, softmax draw
 * from the LCG state *rs (advanced only when temp > 0). libm_exp selects the
 * C library's expf (the reference's) instead of pbo_expf (the device's).
 * Rows holding a NaN return -1. */
int pbo_sample_topkpp(const float* lg, int n, float temp, float topp, int topk, float minp, uint64_t* rs,
                      int libm_exp);

int pbo_threads(void);

#ifdef __cplusplus
}
#endif
#endif
