// pb_model.cu -- the LFM3-style backbone on sm_100a: .lfm3q8 loader, fused
// decode-step kernels, whole-token CUDA graphs and the model C ABI.
//
// One decode token (layer_body, lfm3_nanode.cu:3739-3856, for every layer;
// then the embedding norm, the tied head and greedy argmax) runs as 4 kernels
// per conv layer, 5 per attention layer and 1 for the head. Everything that is
// not a weight stream is fused into the GEMV that consumes it:
//   [embed | residual add + post-norm] + operator_norm -> in_proj / q|k|v|gate
//   headnorm + RoPE + fp16 KV append + attention + sigmoid gate   (k_attn)
//   B*x, conv ring, taps, C*y                                      -> out_proj
//   post_operator_norm + residual add + ffn_norm                   -> w1|w3
//   SiLU(w1)*w3 in the w1|w3 epilogue (their rows are interleaved)
//   post_ffn_norm + residual add + embedding_norm -> head -> argmax -> next id
// Each fused prologue is computed redundantly by every CTA (it is a few KB of
// L2 reads) so that no extra grid-wide dependency is needed. Kernels launch
// with programmatic dependent launch: a kernel starts while its predecessor
// drains, bulk-prefetches its own weight slice into L2, and only then waits
// for the predecessor's results (griddepcontrol.wait).
#include "pb_common.cuh"
#include "pb_internal.h"
#include "pb_json.h"
#include "pb_step.cuh"
#include "pb_decode.cuh"
#include "pb_prefill.cuh"
#include <zlib.h>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>
#include <algorithm>
#include <mutex>
#include <dlfcn.h>
#include <nccl.h>   // types only: the library resolves NCCL at run time

namespace {

// ------------------------------------------------------------ step GEMV
// The streaming GEMV of pb_q8.cu (same granule layout, same leaf chains and
// trees) with a fused prologue and epilogue. CTA b owns a contiguous range of
// row blocks, prefetches that slice of codes and scales into L2 before it
// waits on its predecessor, then streams it.
template <bool F32S>
struct SPair;
template <>
struct SPair<false> {
  static PB_DEV void load(const void* base, size_t idx, float& lo, float& hi) {
    const unsigned w = pb_ldg_stream32(reinterpret_cast<const unsigned*>(base) + idx);
    lo = pb_h2f((unsigned short)(w & 0xffffu));
    hi = pb_h2f((unsigned short)(w >> 16));
  }
  static constexpr int BYTES = 4;
};
template <>
struct SPair<true> {
  static PB_DEV void load(const void* base, size_t idx, float& lo, float& hi) {
    const uint2 w = pb_ldg_stream64(reinterpret_cast<const uint2*>(base) + idx);
    lo = __uint_as_float(w.x);
    hi = __uint_as_float(w.y);
  }
  static constexpr int BYTES = 8;
};

PB_DEV float s_dot16(const uint4 g, const float* xr, float dot) {
  const unsigned ws[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const unsigned ub = ws[k] ^ 0x80808080u;
#pragma unroll
    for (int j = 0; j < 4; j++) dot = __fmaf_rn(pb_code(ub, j), xr[4 * k + j], dot);
  }
  return dot;
}
PB_DEV void s_dots(const uint4 (&q)[4], const float (&xr)[64], float& d0, float& d1) {
  d0 = s_dot16(q[0], xr, 0.0f);
  d0 = s_dot16(q[1], xr + 16, d0);
  d1 = s_dot16(q[2], xr + 32, 0.0f);
  d1 = s_dot16(q[3], xr + 48, d1);
}
// one-chunk rows (K not a multiple of 2048): lane l's chain over blocks l,
// l+32, l+64, ... runs on across the row's segments, then one tree; p holds
// (dot_lo, dot_hi, s_lo, s_hi) per segment and lane
template <int NCH>
PB_DEV float s_one_chain(const float4* p, int lane) {
  float acc = 0.0f;
#pragma unroll
  for (int c = 0; c < NCH; c++) {
    const float4 v = p[c * 32 + lane];
    acc = __fmaf_rn(v.z, v.x, acc);
    acc = __fmaf_rn(v.w, v.y, acc);
  }
  return pb_warp_tree(acc);
}
PB_DEV float s_leaf(const uint4 (&q)[4], float slo, float shi, const float (&xr)[64]) {
  float d0 = s_dot16(q[0], xr, 0.0f);
  d0 = s_dot16(q[1], xr + 16, d0);
  const float acc = __fmaf_rn(slo, d0, 0.0f);
  float d1 = s_dot16(q[2], xr + 32, 0.0f);
  d1 = s_dot16(q[3], xr + 48, d1);
  return __fmaf_rn(shi, d1, acc);
}

PB_DEV void l2_prefetch(const void* p, size_t bytes) {
  const char* c = reinterpret_cast<const char*>(p);
  // 16-byte aligned start and size for cp.async.bulk.prefetch
  const uintptr_t a0 = ((uintptr_t)c + 15) & ~(uintptr_t)15;
  const uintptr_t a1 = ((uintptr_t)c + bytes) & ~(uintptr_t)15;
  for (uintptr_t a = a0; a < a1; a += 32768) {
    const unsigned n = (unsigned)((a1 - a) < 32768 ? (a1 - a) : 32768);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(n) : "memory");
  }
}

// greedy argmax of the logits a CTA wrote, ties to the lowest index: per-thread
// best -> warp -> CTA slot; the last CTA to finish reduces the slots and
// publishes the id (and the step's bookkeeping)
PB_DEV void step_argmax_publish(const StepArgs& a, float bv, int bi, float* bestv, int* besti) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_down_sync(0xffffffffu, bv, o);
    const int oi = __shfl_down_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  if (lane == 0) { bestv[warp] = bv; besti[warp] = bi; }
  __syncthreads();
  __shared__ int am_last;
  if (threadIdx.x == 0) {
    float b = bestv[0]; int ix = besti[0];
    for (int w = 1; w < 8; w++)
      if (bestv[w] > b || (bestv[w] == b && besti[w] < ix)) { b = bestv[w]; ix = besti[w]; }
    a.ctl->slot_val[blockIdx.x] = b;
    a.ctl->slot_idx[blockIdx.x] = ix;
    __threadfence();
    const unsigned prev = atomicAdd(&a.ctl->counter, 1u);
    am_last = prev == gridDim.x - 1;
  }
  __syncthreads();
  if (am_last && threadIdx.x == 0) {
    __threadfence();
    volatile float* sv = a.ctl->slot_val;
    volatile int* si = a.ctl->slot_idx;
    float b = sv[0]; int ix = si[0];
    for (int k = 1; k < (int)gridDim.x; k++) {
      const float ov = sv[k]; const int oi = si[k];
      if (ov > b || (ov == b && oi < ix)) { b = ov; ix = oi; }
    }
    const int step = a.ctl->step;
    a.ctl->token = (step + 1 < a.ctl->n_prompt) ? a.ctl->prompt[step + 1] : ix;
    if (a.ctl->ids) a.ctl->ids[step] = ix;
    a.ctl->step = step + 1;
    a.ctl->pos += 1;
    a.ctl->counter = 0;
  }
}

template <int NCH, bool F32S, int EPI, bool ONE>
__global__ void __launch_bounds__(256, 2) k_step(StepArgs a) {
  constexpr int U = 2, G = 8 / NCH, RB = G * U;
  static_assert(!ONE || (NCH > 1 && RB <= 8 && EPI == EPI_BF16), "one-chunk rows: a warp per row, bf16 out");
  extern __shared__ __align__(16) float smem[];
  float* sx = smem;                          // padded K + K/32 (padded)
  __shared__ float red[16];
  __shared__ float part[2][RB][NCH];
  __shared__ float4 partq[ONE ? 2 : 1][ONE ? RB : 1][ONE ? NCH * 32 : 1];
  __shared__ float bestv[8];
  __shared__ int besti[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = warp % NCH, g = warp / NCH;
  const int nrb = (a.N + RB - 1) / RB;
  const int rb0 = (int)(((long long)blockIdx.x * nrb) / gridDim.x);
  const int rb1 = (int)(((long long)(blockIdx.x + 1) * nrb) / gridDim.x);
  if (threadIdx.x == 0 && rb1 > rb0) {
    const int r0 = rb0 * RB, r1 = min(rb1 * RB, a.N);
    l2_prefetch(reinterpret_cast<const char*>(a.codes) + (size_t)r0 * NCH * 2048, (size_t)(r1 - r0) * NCH * 2048);
    l2_prefetch(reinterpret_cast<const char*>(a.scales) + (size_t)r0 * NCH * 32 * SPair<F32S>::BYTES,
                (size_t)(r1 - r0) * NCH * 32 * SPair<F32S>::BYTES);
  }
  pb_grid_launch_dependents();
  step_prologue<0>(a, sx, red, nullptr, -1);   // takes the dependency wait after its constant loads
  float xr[64];
  {
    const float* x0 = sx + (c * 64 + lane) * 33;          // block c*64 + lane, padded
    const float* x1 = sx + (c * 64 + 32 + lane) * 33;     // block c*64 + 32 + lane
#pragma unroll
    for (int j = 0; j < 32; j++) { xr[j] = x0[j]; xr[32 + j] = x1[j]; }
  }
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  int it = 0;
  for (int rb = rb0; rb < rb1; rb++, it ^= 1) {
    const int row0 = rb * RB + g * U;
    uint4 q[U][4];
    float slo[U], shi[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const int row = row0 + u;
      if (row < a.N) {
        const size_t seg = (size_t)row * NCH + c;
        const uint4* base = a.codes + seg * 128 + lane;
#pragma unroll
        for (int h = 0; h < 4; h++) q[u][h] = pb_ldg_stream(base + 32 * h);
        SPair<F32S>::load(a.scales, seg * 32 + lane, slo[u], shi[u]);
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
        s_dots(q[u], xr, d0, d1);
        partq[it][g * U + u][c * 32 + lane] = make_float4(d0, d1, slo[u], shi[u]);
      }
      __syncthreads();
      if (warp < RB) {
        const int row = rb * RB + warp;
        const float v = s_one_chain<NCH>(&partq[it][warp][0], lane);
        if (lane == 0 && row < a.N) reinterpret_cast<bf16_t*>(a.y)[row] = pb_f2bf(__fadd_rn(0.0f, v));
      }
    } else {
      float v[U];
#pragma unroll
      for (int u = 0; u < U; u++) v[u] = pb_warp_tree(s_leaf(q[u], slo[u], shi[u], xr));
      if (NCH == 1) {
        if (lane == 0) {
          if (EPI == EPI_SILU) {
            // rows 2i (w1) and 2i+1 (w3): k_silu_mul_bf, lfm3_nanode.cu:821-829
            if (row0 + 1 < a.N) {
              const float av = pb_bf2f(pb_f2bf(__fadd_rn(0.0f, v[0])));
              const float bw = pb_bf2f(pb_f2bf(__fadd_rn(0.0f, v[1])));
              reinterpret_cast<bf16_t*>(a.y)[row0 >> 1] =
                  pb_f2bf(__fmul_rn(__fmul_rn(av, pb_sigmoid(av)), bw));
            }
          } else {
#pragma unroll
            for (int u = 0; u < U; u++) {
              const int row = row0 + u;
              if (row < a.N) {
                const float o = __fadd_rn(0.0f, v[u]);
                if (EPI == EPI_ARGMAX) {
                  reinterpret_cast<float*>(a.y)[row] = o;
                  if (o > bv || (o == bv && row < bi)) { bv = o; bi = row; }
                } else {
                  reinterpret_cast<bf16_t*>(a.y)[row] = pb_f2bf(o);
                }
              }
            }
          }
        }
      } else {
        if (lane == 0)
#pragma unroll
          for (int u = 0; u < U; u++) part[it][g * U + u][c] = v[u];
        __syncthreads();
        if (threadIdx.x < RB) {
          const int row = rb * RB + threadIdx.x;
          float acc = 0.0f;
#pragma unroll
          for (int cc = 0; cc < NCH; cc++) acc = __fadd_rn(acc, part[it][threadIdx.x][cc]);
          if (EPI == EPI_SILU) {
            if ((threadIdx.x & 1) == 0 && row + 1 < a.N) {
              float acc1 = 0.0f;
#pragma unroll
              for (int cc = 0; cc < NCH; cc++) acc1 = __fadd_rn(acc1, part[it][threadIdx.x + 1][cc]);
              const float av = pb_bf2f(pb_f2bf(acc)), bw = pb_bf2f(pb_f2bf(acc1));
              reinterpret_cast<bf16_t*>(a.y)[row >> 1] = pb_f2bf(__fmul_rn(__fmul_rn(av, pb_sigmoid(av)), bw));
            }
          } else if (row < a.N) {
            if (EPI == EPI_ARGMAX) {
              reinterpret_cast<float*>(a.y)[row] = acc;
              if (acc > bv || (acc == bv && row < bi)) { bv = acc; bi = row; }
            } else {
              reinterpret_cast<bf16_t*>(a.y)[row] = pb_f2bf(acc);
            }
          }
        }
      }
    }
  }
  if (EPI == EPI_ARGMAX && !a.no_publish) step_argmax_publish(a, bv, bi, bestv, besti);
}

// the head over the bf16 tied table (blob dtype 3): the same prologue as
// k_step, then k_gemv_bf16 (lfm3_nanode.cu:3517-3534) per row -- lane l chains
// s = s + bf16(W[k]) * x[k] over k = l, l+32, ... -- the shuffle-down tree, and
// the fp32 logit as is; then the greedy argmax. a.codes: the table in the head
// layout (b16_index); KG = K / 256.
template <int KG>
__global__ void __launch_bounds__(256, 2) k_step16(StepArgs a) {
  constexpr int K = KG * 256;
  extern __shared__ __align__(16) float smem[];
  float* sx = smem;
  __shared__ float red[16];
  __shared__ float bestv[8];
  __shared__ int besti[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pb_grid_launch_dependents();
  step_prologue<0>(a, sx, red, nullptr, -1);
  float xr[K / 32];
#pragma unroll
  for (int m = 0; m < K / 32; m++) xr[m] = sx[padx(lane + 32 * m)];
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  const uint16_t* w = reinterpret_cast<const uint16_t*>(a.codes);
  for (int row = blockIdx.x * 8 + warp; row < a.N; row += gridDim.x * 8) {
    const uint4* g = reinterpret_cast<const uint4*>(w + (size_t)row * K) + lane;
    float acc = 0.0f;
#pragma unroll
    for (int h = 0; h < KG; h++) {
      const uint4 q = pb_ldg_stream(g + 32 * h);
      const unsigned ws[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int i = 0; i < 4; i++) {
        acc = __fadd_rn(acc, __fmul_rn(pb_lo2f(ws[i]), xr[8 * h + 2 * i]));
        acc = __fadd_rn(acc, __fmul_rn(pb_hi2f(ws[i]), xr[8 * h + 2 * i + 1]));
      }
    }
    const float v = pb_warp_tree(acc);
    if (lane == 0) {
      reinterpret_cast<float*>(a.y)[row] = v;
      if (v > bv || (v == bv && row < bi)) { bv = v; bi = row; }
    }
  }
  if (!a.no_publish) step_argmax_publish(a, bv, bi, bestv, besti);
}

// ------------------------------------------------------------- attention
template <int E>
__global__ void __launch_bounds__(256) k_attn(AttnArgs a) {
  constexpr int HD = 32 * E;
  extern __shared__ __align__(16) float sl[];     // scores [max_ctx]
  __shared__ float qv[HD], kv[HD], vv[HD];
  __shared__ float red[8];
  __shared__ float segred[8 * HD];
  pb_grid_launch_dependents();
  pb_grid_wait();
  attn_body<E, 0>(a, blockIdx.x, a.ctl->pos, sl, qv, kv, vv, segred, red);
}

// residual tail for the standalone layer step: x = R + bf16(rms(h, w))
__global__ void __launch_bounds__(256) k_tail(StepArgs a) {
  extern __shared__ __align__(16) float smem[];
  __shared__ float red[16];
  pb_grid_launch_dependents();
  step_prologue<0>(a, smem, red, nullptr, -1);
}

// ----------------------------------------------------------- host model
struct Layer {
  bool attn = false;
  bool slide = false;    // sliding-window attention layer
  pb_q8 first;           // q|k|v|gate or in_proj
  pb_q8 mix;             // o_proj or out_proj
  pb_q8 w13;             // w1 row i at 2i, w3 row i at 2i+1
  pb_q8 w2;
  float* op_norm = nullptr; float* post_op_norm = nullptr;
  float* ffn_norm = nullptr; float* post_ffn_norm = nullptr;
  float* q_norm = nullptr; float* k_norm = nullptr;
  float* taps = nullptr;
  int attn_idx = -1, conv_idx = -1;
};

struct Tensor {
  std::string name;
  int dtype = -1;
  std::vector<long long> ne;
  size_t off = 0, nc = 0, ns = 0;
  uint32_t crc = 0;
};

}  // namespace

struct pb_model {
  int device = 0;
  // per-tensor mode (a model holding Q4 / Q5 records, blob dtypes 6 / 7): every
  // 2-D Q8 / Q4 / Q5 tensor on the device by itself for pb_model_gemv, as the
  // reference's gemv() dispatches by record (lfm3_nanode.cu:1916-1922); the
  // fused decode paths decline such a model
  bool per_tensor = false;
  std::vector<pb_q8*> pt_q8;      // [tensor id], null where not a Q8 record
  std::vector<pb_qlow*> pt_qlow;  // [tensor id], null where not a Q4 / Q5 record
  int H = 0, F = 0, L = 0, NH = 0, NKV = 0, HD = 0, V = 0, W = 3, n_attn = 0, win = 0;
  float theta = 1e6f, partial = 1.0f, eps = 1e-5f;
  // sliding-attention layers (lfm3_nanode.cu:3753-3785, :5402-5420): their
  // own RoPE base and rotated share, over the last win_s keys
  float theta_s = 1e4f, partial_s = 1.0f;
  int win_s = 256;
  bool any_slide = false;
  int sdt = PB_DT_F16;
  std::vector<Layer> layers;
  pb_q8 head;                // the tied table (Q8); N, K also describe a bf16 table
  uint16_t* head16 = nullptr;   // the tied table as bf16 (blob dtype 3), head layout (b16_index)
  float* final_norm = nullptr;
  char* arena = nullptr;
  size_t arena_bytes = 0;
  std::vector<Tensor> table;
  std::vector<float> invf;        // full-attention layers
  std::vector<float> invf_s;      // sliding-attention layers
  uint64_t weight_bytes = 0;
  bool decode_ok = true;     // every decode tensor in the streaming layout
  // tensor-core copies of every projection for the chunked prefill (built on first use)
  char* tc_arena = nullptr;
  std::vector<pb_q8> tc;     // per layer: first, mix, w13, w2; then the head
};

struct pb_state {
  pb_model* m = nullptr;
  int max_ctx = 0;
  unsigned short* kv = nullptr;   // [n_attn][2][max_ctx][NKV][HD]
  bf16_t* ring = nullptr;         // [n_conv][W][H]
  float* rope_cos = nullptr;      // [max_ctx][half] of the full-attention layers
  float* rope_sin = nullptr;
  float* rope_cos_s = nullptr;    // [max_ctx][half_s] of the sliding-attention layers
  float* rope_sin_s = nullptr;
  bf16_t* res[3] = {nullptr, nullptr, nullptr};
  bf16_t* h_first = nullptr;      // q|k|v|gate or in_proj output
  bf16_t* h_attn = nullptr;
  bf16_t* h_mix = nullptr;
  bf16_t* h_u = nullptr;
  bf16_t* h_w2 = nullptr;
  float* logits = nullptr;
  Ctl* ctl = nullptr;
  Ctl* h_ctl = nullptr;           // pinned host mirror for token/pos uploads, then one
                                  // pinned int for the decode kernel's error word
  char* mem = nullptr;
  size_t mem_bytes = 0;
  // persistent decode kernel: phase table, arrival counter, error word
  DPhase* d_phases = nullptr;
  // tagged activations of the persistent kernel (bf16 value | 16-bit phase tag)
  uint32_t* t_first = nullptr;    // q|k|v|gate or in_proj output
  uint32_t* t_attn = nullptr;     // gated attention output
  uint32_t* t_mix = nullptr;      // o_proj / out_proj output
  uint32_t* t_u = nullptr;        // SwiGLU output
  uint32_t* t_w2 = nullptr;       // w2 output
  unsigned long long* t_scores = nullptr;   // [NH][max_ctx] attention scores (phase << 32 | fp32 bits)
  size_t tag_bytes = 0;           // the six buffers, contiguous from t_first
  unsigned qbase = 0;             // sequence number of the next launch's first phase
  size_t res_smem_off = 0;
  char* d_sched = nullptr;         // weight-stream schedule: GemvSched [CTA][ngemv], spt [CTA], StageDesc [CTA][spt_max]
  int ngemv = 0, spt_max = 0;
  size_t sched_bytes = 0, spt_off = 0, map_off = 0, sched_smem_off = 0;
  int nphase = 0;
  unsigned* d_bar = nullptr;
  int* d_err = nullptr;
  int xregion = 0, ds = 0;
  size_t dsmem = 0;
  bool decode_checked = false;     // the kernel's shared-memory attribute set and its fit checked for dsmem
  bool persistent = true;
  unsigned long long* d_trace = nullptr;   // PB_DECODE_TRACE=1: phase timing marks
  float* att_scores = nullptr;   // split attention: [NH][max_ctx] scores, then e
  float* att_inv = nullptr;      // [NH] 1/sum
  float* att_segp = nullptr;     // [NH][8][HD] P.V segment partials
  int pv_per_warp = 0;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  cudaStream_t graph_stream = nullptr;
  int graph_res = 0;              // residual buffer holding the final residual
  uint64_t graph_launches = 0;    // kernels per graph replay
  // chunked prefill buffers (allocated on first use, for up to pf_cap positions)
  char* pf_mem = nullptr;
  int pf_cap = 0;
  bf16_t* pf_R = nullptr;         // [T][H] residual
  int8_t* pf_qx = nullptr;        // [T][Kmax] quantised projection input
  uint16_t* pf_dx = nullptr;      // [T][Kmax/32]
  float* pf_y = nullptr;          // [T][Nmax] projection output
  bf16_t* pf_qkvg = nullptr;      // [T][q|k|v|gate]
  bf16_t* pf_att = nullptr;       // [T][NH*HD] gated attention output
  float* pf_logits = nullptr;     // [T][V]
  int* pf_tok = nullptr;          // [T]
  bf16_t* pf_R2 = nullptr;        // [T][H] x of the bf16 head (a dtype-3 table)
  // row sharding over tp_world ranks (pb_state_shard): every GEMV computes its
  // rank's rows, an in-place NCCL all-gather completes the output vector
  int tp_rank = 0, tp_world = 1;
  ncclComm_t comm = nullptr;
};

namespace {

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

int half_rot(const pb_model* m) { return (int)((double)m->partial * m->HD) / 2; }
int half_rot_s(const pb_model* m) { return (int)((double)m->partial_s * m->HD) / 2; }
// per attention layer: rotated pairs, key window, RoPE tables
int layer_half(const pb_model* m, int L) { return m->layers[L].slide ? half_rot_s(m) : half_rot(m); }
int layer_win(const pb_model* m, int L) { return m->layers[L].slide ? m->win_s : m->win; }
const float* layer_cos(const pb_state* s, int L) { return s->m->layers[L].slide ? s->rope_cos_s : s->rope_cos; }
const float* layer_sin(const pb_state* s, int L) { return s->m->layers[L].slide ? s->rope_sin_s : s->rope_sin; }
// the longest attention span any layer of the model reads at max_ctx
int max_span(const pb_model* m, int max_ctx) {
  int span = 0;
  for (int L = 0; L < m->L; L++)
    if (m->layers[L].attn) {
      const int w = layer_win(m, L);
      span = std::max(span, (w > 0 && w < max_ctx) ? w : max_ctx);
    }
  return span > 0 ? span : 1;
}

// ---- launches ---------------------------------------------------------------
size_t step_smem(int K, int H) {
  const int kp = pb_kpad(K);
  return (size_t)(kp + kp / 32 + 2 * H) * sizeof(float);
}

template <int NCH, bool F32S, int EPI, bool ONE = false>
int launch_step_t(const StepArgs& a, cudaStream_t st, bool pdl) {
  const size_t smem = step_smem(a.K, a.H);
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(k_step<NCH, F32S, EPI, ONE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
    set = true;
  }
  if (smem > 96 * 1024) return pb_set_error(PB_ENOTSUP, "step: K=%d H=%d needs too much shared memory", a.K, a.H);
  constexpr int RB = (8 / NCH) * 2;
  const int nrb = (a.N + RB - 1) / RB;
  int grid = pb_num_sms();
  if (grid > nrb) grid = nrb;
  if (EPI == EPI_ARGMAX && grid > MAX_CTA) grid = MAX_CTA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_step<NCH, F32S, EPI, ONE>, a);
  if (e != cudaSuccess) return pb_set_error(PB_ECUDA, "launch k_step: %s", cudaGetErrorString(e));
  pb_count_launch();
  return PB_OK;
}

template <bool F32S, int EPI>
int launch_step_n(int nch, int one, const StepArgs& a, cudaStream_t st, bool pdl) {
  if (one && nch > 1) {
    if (EPI != EPI_BF16) return pb_set_error(PB_ENOTSUP, "step: one-chunk rows (K %d) feed a bf16 output only", a.K);
    switch (nch) {
      case 2: return launch_step_t<2, F32S, EPI_BF16, true>(a, st, pdl);
      case 4: return launch_step_t<4, F32S, EPI_BF16, true>(a, st, pdl);
      case 8: return launch_step_t<8, F32S, EPI_BF16, true>(a, st, pdl);
    }
    return pb_set_error(PB_ENOTSUP, "step: %d chunks", nch);
  }
  switch (nch) {
    case 1: return launch_step_t<1, F32S, EPI>(a, st, pdl);
    case 2: return launch_step_t<2, F32S, EPI>(a, st, pdl);
    case 4: return launch_step_t<4, F32S, EPI>(a, st, pdl);
    case 8: return launch_step_t<8, F32S, EPI>(a, st, pdl);
  }
  return pb_set_error(PB_ENOTSUP, "step: %d chunks", nch);
}

template <int KG>
int launch_step16_t(const StepArgs& a, cudaStream_t st, bool pdl) {
  const size_t smem = step_smem(a.K, a.H);
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(k_step16<KG>, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
    set = true;
  }
  int grid = 2 * pb_num_sms();
  if (grid > (a.N + 7) / 8) grid = (a.N + 7) / 8;
  if (grid > MAX_CTA) grid = MAX_CTA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_step16<KG>, a);
  if (e != cudaSuccess) return pb_set_error(PB_ECUDA, "launch k_step16: %s", cudaGetErrorString(e));
  pb_count_launch();
  return PB_OK;
}

int launch_step(const pb_q8& w, int epi, StepArgs a, cudaStream_t st, bool pdl) {
  a.codes = reinterpret_cast<const uint4*>(w.codes);
  a.scales = w.scales;
  a.N = w.N;
  a.K = w.K;
  if (w.layout == PB_Q8_B16) {
    if (epi != EPI_ARGMAX) return pb_set_error(PB_ENOTSUP, "step: the bf16 table is the head only");
    switch (w.K) {
      case 256: return launch_step16_t<1>(a, st, pdl);
      case 512: return launch_step16_t<2>(a, st, pdl);
      case 1024: return launch_step16_t<4>(a, st, pdl);
      case 2048: return launch_step16_t<8>(a, st, pdl);
      case 4096: return launch_step16_t<16>(a, st, pdl);
    }
    return pb_set_error(PB_ENOTSUP, "step: bf16 head with K=%d", w.K);
  }
  const bool f = w.sdt == PB_DT_F32;
  if (epi == EPI_BF16) return f ? launch_step_n<true, EPI_BF16>(w.nch, w.one, a, st, pdl) : launch_step_n<false, EPI_BF16>(w.nch, w.one, a, st, pdl);
  if (epi == EPI_SILU) return f ? launch_step_n<true, EPI_SILU>(w.nch, w.one, a, st, pdl) : launch_step_n<false, EPI_SILU>(w.nch, w.one, a, st, pdl);
  return f ? launch_step_n<true, EPI_ARGMAX>(w.nch, w.one, a, st, pdl) : launch_step_n<false, EPI_ARGMAX>(w.nch, w.one, a, st, pdl);
}

int launch_attn(const pb_model* m, pb_state* s, int layer, cudaStream_t st, bool pdl) {
  const Layer& Ly = m->layers[layer];
  AttnArgs a;
  a.qkvg = s->h_first;
  a.qnorm = Ly.q_norm;
  a.knorm = Ly.k_norm;
  a.rope_cos = layer_cos(s, layer);
  a.rope_sin = layer_sin(s, layer);
  const size_t per = (size_t)s->max_ctx * m->NKV * m->HD;
  a.kc = s->kv + (size_t)Ly.attn_idx * 2 * per;
  a.vc = a.kc + per;
  a.out = s->h_attn;
  a.ctl = s->ctl;
  a.nh = m->NH; a.nkv = m->NKV; a.half = layer_half(m, layer); a.win = layer_win(m, layer);
  a.max_ctx = s->max_ctx;
  a.scaling = 1.0f / sqrtf((float)m->HD);
  a.eps = m->eps;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(m->NH);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = (size_t)s->max_ctx * sizeof(float);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e;
  switch (m->HD) {
    case 32: cudaFuncSetAttribute(k_attn<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
             e = cudaLaunchKernelEx(&cfg, k_attn<1>, a); break;
    case 64: cudaFuncSetAttribute(k_attn<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
             e = cudaLaunchKernelEx(&cfg, k_attn<2>, a); break;
    case 128: cudaFuncSetAttribute(k_attn<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
              e = cudaLaunchKernelEx(&cfg, k_attn<4>, a); break;
    default: return pb_set_error(PB_ENOTSUP, "attention head_dim %d", m->HD);
  }
  if (e != cudaSuccess) return pb_set_error(PB_ECUDA, "launch k_attn: %s", cudaGetErrorString(e));
  pb_count_launch();
  return PB_OK;
}

// ---- row sharding --------------------------------------------------------
// NCCL is resolved at run time from the libnccl.so.2 already in the process
// (the one torch.distributed loaded) or, failing that, the system one; the
// library itself links only libcudart and libz.
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};
NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.all_gather && api.comm_destroy && api.error_string;
  });
  return api;
}

// the greedy id of the full (gathered) logits, ties to the lowest index; the
// control block advances as the unsharded head's epilogue advances it
__global__ void __launch_bounds__(1024) k_tp_argmax(const float* __restrict__ lg, int V, Ctl* ctl) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float b = -INFINITY;
  int ix = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = lg[i];
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
    for (int w = 1; w < 32; w++)
      if (bv[w] > bv[0] || (bv[w] == bv[0] && bi[w] < bi[0])) { bv[0] = bv[w]; bi[0] = bi[w]; }
    const int id = bi[0];
    const int step = ctl->step;
    ctl->token = (step + 1 < ctl->n_prompt) ? ctl->prompt[step + 1] : id;
    if (ctl->ids) ctl->ids[step] = id;
    ctl->step = step + 1;
    ctl->pos += 1;
  }
}

// one GEMV of the step: the whole tensor, or this rank's rows followed by the
// in-place all-gather of the output (bf16 rows, bf16 SiLU pairs, fp32 logits)
int launch_gemv(pb_state* s, const pb_q8& w, int epi, StepArgs a, cudaStream_t st, bool pdl, uint64_t& nk) {
  if (s->tp_world <= 1) {
    const int rc = launch_step(w, epi, a, st, pdl);
    if (!rc) nk++;
    return rc;
  }
  const int world = s->tp_world, r = s->tp_rank, rows = w.N / world, r0 = r * rows;
  pb_q8 part = w;
  part.N = rows;
  part.owner = false;
  part.codes = w.codes + (size_t)r0 * (w.layout == PB_Q8_B16 ? (size_t)w.K * 2 : (size_t)w.nch * 2048);
  if (w.layout != PB_Q8_B16)
    part.scales = static_cast<char*>(w.scales) + (size_t)r0 * w.nch * 32 * (w.sdt == PB_DT_F32 ? 8 : 4);
  size_t elem = 2, per_rank = rows, first = r0;
  if (epi == EPI_SILU) { per_rank = rows / 2; first = r0 / 2; }
  else if (epi == EPI_ARGMAX) { elem = 4; a.no_publish = 1; }
  char* full = static_cast<char*>(a.y);
  a.y = full + first * elem;
  int rc = launch_step(part, epi, a, st, pdl);
  if (rc) return rc;
  nk++;
  const ncclResult_t nr = nccl().all_gather(full + (size_t)r * per_rank * elem, full, per_rank * elem, ncclUint8,
                                            s->comm, st);
  if (nr != ncclSuccess) return pb_set_error(PB_ECUDA, "ncclAllGather: %s", nccl().error_string(nr));
  nk++;
  return PB_OK;
}

StepArgs base_args(const pb_model* m, pb_state* s) {
  StepArgs a = {};
  a.H = m->H;
  a.eps = m->eps;
  a.ctl = s->ctl;
  a.convw = m->W;
  return a;
}

// Enqueue one layer. `cur` is the residual buffer index holding x on entry;
// on exit it names the buffer holding the layer's pre-FFN residual (the
// post-FFN add is folded into whoever consumes h_w2 next).
// first_mode: PRO_EMBED (layer 0 of a token), PRO_ADDNORM with hin = h_w2
// (layer L > 0 of a token) or PRO_ADDNORM with hin = null (standalone step).
int enqueue_layer(const pb_model* m, pb_state* s, int L, int& cur, int first_mode, bool add_prev,
                  const bf16_t* x_in, cudaStream_t st, bool pdl, uint64_t& nk) {
  const Layer& Ly = m->layers[L];
  int rc;
  StepArgs a = base_args(m, s);
  a.pro = first_mode;
  a.wnorm = Ly.op_norm;
  a.y = s->h_first;
  if (first_mode == PRO_EMBED) {
    a.emb_codes = reinterpret_cast<const uint4*>(m->head.codes);
    a.emb_scales = m->head.scales;
    a.emb_nch = m->head.nch;
    a.emb_f32 = m->head.sdt == PB_DT_F32;
    a.emb16 = m->head.layout == PB_Q8_B16 ? m->head16 : nullptr;
    a.rout = s->res[cur];
  } else {
    a.xin = x_in ? x_in : s->res[cur];
    if (add_prev) {
      a.hin = s->h_w2;
      a.wpost = m->layers[L - 1].post_ffn_norm;
      a.rout = s->res[cur ^ 1];
      cur ^= 1;
    }
  }
  if ((rc = launch_gemv(s, Ly.first, EPI_BF16, a, st, pdl, nk))) return rc;
  if (Ly.attn) {
    if ((rc = launch_attn(m, s, L, st, pdl))) return rc;
    nk++;
    StepArgs b = base_args(m, s);
    b.pro = PRO_PLAIN;
    b.xin = s->h_attn;
    b.y = s->h_mix;
    if ((rc = launch_gemv(s, Ly.mix, EPI_BF16, b, st, pdl, nk))) return rc;
  } else {
    StepArgs b = base_args(m, s);
    b.pro = PRO_CONV;
    b.xin = s->h_first;
    b.ring = s->ring + (size_t)Ly.conv_idx * m->W * m->H;
    b.taps = Ly.taps;
    b.y = s->h_mix;
    if ((rc = launch_gemv(s, Ly.mix, EPI_BF16, b, st, pdl, nk))) return rc;
  }
  // post_operator_norm + residual + ffn_norm -> w1|w3 (+ SiLU*mul)
  StepArgs c = base_args(m, s);
  c.pro = PRO_ADDNORM;
  c.xin = (first_mode != PRO_EMBED && !add_prev && x_in) ? x_in : s->res[cur];
  c.hin = s->h_mix;
  c.wpost = Ly.post_op_norm;
  c.wnorm = Ly.ffn_norm;
  c.rout = s->res[cur ^ 1];
  cur ^= 1;
  c.y = s->h_u;
  if ((rc = launch_gemv(s, Ly.w13, EPI_SILU, c, st, pdl, nk))) return rc;
  StepArgs d = base_args(m, s);
  d.pro = PRO_PLAIN;
  d.xin = s->h_u;
  d.y = s->h_w2;
  if ((rc = launch_gemv(s, Ly.w2, EPI_BF16, d, st, pdl, nk))) return rc;
  return PB_OK;
}

int enqueue_token(const pb_model* m, pb_state* s, cudaStream_t st, bool pdl, int& final_res, uint64_t& nk) {
  int cur = 0;
  int rc;
  for (int L = 0; L < m->L; L++) {
    if ((rc = enqueue_layer(m, s, L, cur, L == 0 ? PRO_EMBED : PRO_ADDNORM, L > 0, nullptr, st, pdl, nk))) return rc;
  }
  StepArgs h = base_args(m, s);
  h.pro = PRO_ADDNORM;
  h.xin = s->res[cur];
  h.hin = s->h_w2;
  h.wpost = m->layers[m->L - 1].post_ffn_norm;
  h.wnorm = m->final_norm;
  h.rout = s->res[cur ^ 1];
  final_res = cur ^ 1;
  h.y = s->logits;
  if ((rc = launch_gemv(s, m->head, EPI_ARGMAX, h, st, pdl, nk))) return rc;
  if (s->tp_world > 1) {
    k_tp_argmax<<<1, 1024, 0, st>>>(s->logits, m->V, s->ctl);
    PB_LAUNCHED("k_tp_argmax");
    nk++;
  }
  return PB_OK;
}

int build_graph(pb_state* s) {
  if (s->exec) return PB_OK;
  pb_model* m = s->m;
  if (!s->graph_stream) PB_TRY_CUDA(cudaStreamCreateWithFlags(&s->graph_stream, cudaStreamNonBlocking));
  cudaStream_t st = s->graph_stream;
  PB_TRY_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  uint64_t nk = 0;
  int fr = 0;
  pb_set_capturing(true);     // captured launches are counted when the graph runs
  int rc = enqueue_token(m, s, st, true, fr, nk);
  pb_set_capturing(false);
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamEndCapture(st, &g);
  if (rc) { if (g) cudaGraphDestroy(g); return rc; }
  if (e != cudaSuccess) return pb_set_error(PB_ECUDA, "graph capture: %s", cudaGetErrorString(e));
  cudaGraphExec_t ex = nullptr;
  e = cudaGraphInstantiate(&ex, g, 0);
  if (e != cudaSuccess) { cudaGraphDestroy(g); return pb_set_error(PB_ECUDA, "graph instantiate: %s", cudaGetErrorString(e)); }
  s->graph = g;
  s->exec = ex;
  s->graph_res = fr;
  s->graph_launches = nk;
  return PB_OK;
}

// ---- persistent decode ---------------------------------------------------
// The persistent kernel is compiled for the shapes listed here: hidden 2048
// with head_dim 64 and conv width 3 (the LFM3 2B-class backbone) or head_dim
// 128 and conv width 7 (the reference engine's own model, lfm3_nanode.cu:76-
// 101); other models decode on the per-kernel CUDA-graph path, with the same
// results.
bool persistent_shape(const pb_model* m) {
  if (m->H != 2048 || !((m->HD == 64 && m->W == 3) || (m->HD == 128 && m->W == 7))) return false;
  // PRO_PLAIN inputs (w2: K = F; o_proj: K = NH*HD) stage 256*{8,16,32}
  // values (K padded to whole segments); the P.V phase runs on 4 NH CTAs
  const int kf = pb_kpad(m->F) >> 8, ka = pb_kpad(m->NH * m->HD) >> 8;
  return (kf == 8 || kf == 16 || kf == 32) && (ka == 8 || ka == 16 || ka == 32) && 4 * m->NH <= pb_num_sms();
}

// shapes the integer-path chunk kernels (prefill, batched decode) are compiled
// for: hidden 2048, head_dim 64 with conv width 3 or head_dim 128 with conv
// width 7, the attention output 2048 wide, F a multiple of 32 up to 8192
bool chunk_shape(const pb_model* m) {
  return m->H == 2048 && ((m->HD == 64 && m->W == 3) || (m->HD == 128 && m->W == 7)) && m->F % 32 == 0 &&
         m->F <= 8192 && m->F % 256 == 0 && m->NH * m->HD == 2048;
}

AttnArgs attn_args(const pb_model* m, pb_state* s, int layer) {
  const Layer& Ly = m->layers[layer];
  AttnArgs a;
  a.qkvg = s->h_first;
  a.qnorm = Ly.q_norm;
  a.knorm = Ly.k_norm;
  a.rope_cos = layer_cos(s, layer);
  a.rope_sin = layer_sin(s, layer);
  const size_t per = (size_t)s->max_ctx * m->NKV * m->HD;
  a.kc = s->kv + (size_t)Ly.attn_idx * 2 * per;
  a.vc = a.kc + per;
  a.out = s->h_attn;
  a.ctl = s->ctl;
  a.nh = m->NH; a.nkv = m->NKV; a.half = layer_half(m, layer); a.win = layer_win(m, layer);
  a.max_ctx = s->max_ctx;
  a.scaling = 1.0f / sqrtf((float)m->HD);
  a.eps = m->eps;
  a.scores = s->att_scores;
  a.inv = s->att_inv;
  a.segp = s->att_segp;
  return a;
}

DPhase dgemv(const pb_model* m, const pb_q8& w, int pro, int epi, const uint32_t* tin, uint32_t* tout) {
  DPhase ph = {};
  ph.kind = PH_GEMV;
  ph.pro = pro;
  ph.epi = epi;
  ph.N = w.N;
  ph.K = w.K;
  ph.nch = w.nch;
  ph.one = w.one && w.nch > 1;
  ph.b16 = w.layout == PB_Q8_B16;
  ph.H = m->H;
  ph.eps = m->eps;
  ph.tin = tin;
  ph.tout = tout;
  return ph;
}

// The token as a phase list (the same arithmetic, in the same order, as
// enqueue_token): per layer the first GEMV (embedding or residual add +
// post-norm + operator_norm), attention (one phase) or nothing, the mixer
// GEMV (conv prologue or the attention output), w1|w3 (residual add +
// post-norm + ffn_norm; SwiGLU epilogue), w2; then the head (residual add +
// post-norm + embedding_norm; logits and per-CTA argmax). Every phase reads
// the previous phase's tagged output.
int build_phases(pb_state* s) {
  if (s->d_phases) return PB_OK;
  pb_model* m = s->m;
  std::vector<DPhase> ph;
  for (int L = 0; L < m->L; L++) {
    const Layer& Ly = m->layers[L];
    DPhase a = dgemv(m, Ly.first, L == 0 ? PRO_EMBED : PRO_ADDNORM, EPI_BF16, s->t_w2, s->t_first);
    a.wnorm = Ly.op_norm;
    if (L == 0) {
      a.tin = nullptr;
      a.emb_codes = reinterpret_cast<const uint4*>(m->head.codes);
      a.emb_scales = m->head.scales;
      a.emb_nch = m->head.nch;
      a.emb_f32 = m->head.sdt == PB_DT_F32;
      a.emb16 = m->head.layout == PB_Q8_B16 ? m->head16 : nullptr;
    } else {
      a.wpost = m->layers[L - 1].post_ffn_norm;
    }
    ph.push_back(a);
    if (Ly.attn) {
      DPhase sc = {};
      sc.kind = PH_SCORE;
      sc.tin = s->t_first;
      sc.tsc = s->t_scores;
      sc.at = attn_args(m, s, L);
      ph.push_back(sc);
      DPhase pv = sc;
      pv.kind = PH_PV;
      pv.tout = s->t_attn;
      ph.push_back(pv);
      ph.push_back(dgemv(m, Ly.mix, PRO_PLAIN, EPI_BF16, s->t_attn, s->t_mix));
    } else {
      DPhase b = dgemv(m, Ly.mix, PRO_CONV, EPI_BF16, s->t_first, s->t_mix);
      b.ring = s->ring + (size_t)Ly.conv_idx * m->W * m->H;
      b.taps = Ly.taps;
      ph.push_back(b);
    }
    DPhase c = dgemv(m, Ly.w13, PRO_ADDNORM, EPI_SILU, s->t_mix, s->t_u);
    c.wpost = Ly.post_op_norm;
    c.wnorm = Ly.ffn_norm;
    ph.push_back(c);
    ph.push_back(dgemv(m, Ly.w2, PRO_PLAIN, EPI_BF16, s->t_u, s->t_w2));
  }
  DPhase h = dgemv(m, m->head, PRO_ADDNORM, EPI_ARGMAX, s->t_w2, nullptr);
  h.wpost = m->layers[m->L - 1].post_ffn_norm;
  h.wnorm = m->final_norm;
  h.rout = s->res[0];
  h.fout = s->logits;
  h.at.ctl = s->ctl;
  s->graph_res = 0;
  ph.push_back(h);
  // shared-memory plan: the activation region holds a GEMV phase's padded
  // input, then its row values (at most ceil(row blocks / CTAs) stages of 16
  // chunk values per CTA); the score phase's q and k per warp; the P.V
  // phase's V chunk (32 KB), scores, partials, current v row and gate
  const int span = max_span(m, s->max_ctx);
  const int dq = m->HD / 4;
  int xr = std::max(DWARPS * 2 * m->HD, 32768 / 4 + ((span + 3) & ~3) + 9 * dq + 4);
  const int G = pb_num_sms();
  for (auto& p : ph)
    if (p.kind == PH_GEMV) {
      const int RB = DSEGS / p.nch;
      const int nrb = (p.N + RB - 1) / RB;
      const int kp = pb_kpad(p.K);
      p.rowoff = (kp + kp / 32 + 3) & ~3;
      // row values: one float per (row, segment); one-chunk rows park four
      // per (row, segment, lane)
      xr = std::max(xr, p.rowoff + ((nrb + G - 1) / G) * DSEGS * (p.one ? 128 : 1));
    }
  // weight-stream schedule: per CTA and GEMV its rows and first stage within
  // the token, and one descriptor per stage
  int ngemv = 0;
  for (auto& p : ph)
    if (p.kind == PH_GEMV) p.gidx = ngemv++;
  std::vector<GemvSched> sched((size_t)G * ngemv);
  std::vector<int> spt(G, 0);
  std::vector<std::vector<StageDesc>> sdesc(G);
  const size_t q8s = m->sdt == PB_DT_F32 ? 8 : 4;   // bytes per scale pair
  std::vector<const pb_q8*> wts;   // the GEMV phases' tensors, in phase order
  for (int L = 0; L < m->L; L++) {
    const Layer& Ly = m->layers[L];
    wts.push_back(&Ly.first); wts.push_back(&Ly.mix); wts.push_back(&Ly.w13); wts.push_back(&Ly.w2);
  }
  wts.push_back(&m->head);
  for (int b = 0; b < G; b++) {
    int base = 0, k = 0;
    for (auto& p : ph) {
      if (p.kind != PH_GEMV) continue;
      const pb_q8& w = *wts[k++];
      const int RB = DSEGS / p.nch;
      const int nrb = (p.N + RB - 1) / RB;
      const int rb0 = (int)(((long long)b * nrb) / G), rb1 = (int)(((long long)(b + 1) * nrb) / G);
      GemvSched& g = sched[(size_t)b * ngemv + p.gidx];
      g.codes = reinterpret_cast<const char*>(w.codes);
      g.scales = reinterpret_cast<const char*>(p.b16 ? w.codes : w.scales);   // (a bf16 table has none)
      g.r0 = rb0 * RB;
      g.r1 = std::min(rb1 * RB, p.N);
      g.base = base;
      g.nch = p.nch;
      for (int kb = rb0; kb < rb1; kb++) {
        const int r = kb * RB, nr = std::min(RB, p.N - r);
        StageDesc sd;
        sd.codes16 = (unsigned)(((size_t)(g.codes - m->arena) + (size_t)r * p.nch * 2048) / 16);
        sd.scales16 = (unsigned)(((size_t)(g.scales - m->arena) + (size_t)r * p.nch * 32 * q8s) / 16);
        sd.bc = (unsigned)(nr * p.nch * 2048);
        sd.bs = p.b16 ? 0u : (unsigned)(nr * p.nch * 32 * q8s);
        sdesc[b].push_back(sd);
      }
      base += rb1 - rb0;
    }
    spt[b] = base;
  }
  int spt_max = 1;
  for (int b = 0; b < G; b++) spt_max = std::max(spt_max, spt[b]);
  if (m->arena_bytes / 16 > 0xffffffffull || ngemv > 65535 || spt_max > 4096)
    return pb_set_error(PB_ENOTSUP, "persistent decode: %d GEMVs, %d stages per token", ngemv, spt_max);
  int dev = 0;
  cudaGetDevice(&dev);
  int optin = 0;
  cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const size_t stage = m->sdt == PB_DT_F32 ? DGeo<true>::STAGE : DGeo<false>::STAGE;
  const size_t static_est = 1024;
  const size_t xb = (size_t)((xr + 1) & ~1) * 4;
  const size_t resb = ((size_t)m->H * 2 + 15) & ~(size_t)15;
  const size_t tab = (size_t)ngemv * sizeof(GemvSched) + (size_t)spt_max * sizeof(StageDesc);
  long avail = (long)optin - (long)static_est - ISSUE_BYTES - (long)xb - MAX_DS * 8 - 16 - (long)resb - (long)tab;
  int ds = (int)std::min<long>(6, avail / (long)stage);
  if (ds < 2) return pb_set_error(PB_ENOTSUP, "persistent decode: shared memory for %d ring stages", ds);
  s->ds = ds;
  s->xregion = xr;
  s->ngemv = ngemv;
  s->spt_max = spt_max;
  // dynamic shared memory: issue context, ring, activation region, mbarriers,
  // residual copy, schedule, stage descriptors
  const size_t res_off = (ISSUE_BYTES + (size_t)ds * stage + xb + (size_t)ds * 8 + 15) & ~(size_t)15;
  const size_t sched_off = res_off + resb;
  s->res_smem_off = res_off;
  s->dsmem = sched_off + tab;
  s->decode_checked = false;
  {
    // one device buffer: schedule [G][ngemv], spt [G], map [G][spt_max]
    const size_t sb = sched.size() * sizeof(GemvSched);
    s->spt_off = sb;
    const size_t mo = (sb + (size_t)G * 4 + 15) & ~(size_t)15;
    s->sched_bytes = mo + (size_t)G * spt_max * sizeof(StageDesc);
    std::vector<char> host(s->sched_bytes, 0);
    memcpy(host.data(), sched.data(), sb);
    memcpy(host.data() + sb, spt.data(), (size_t)G * 4);
    for (int b = 0; b < G; b++)
      if (!sdesc[b].empty())
        memcpy(host.data() + mo + (size_t)b * spt_max * sizeof(StageDesc), sdesc[b].data(),
               sdesc[b].size() * sizeof(StageDesc));
    if (cudaMalloc(&s->d_sched, s->sched_bytes) != cudaSuccess) {
      cudaGetLastError();
      s->d_sched = nullptr;
      return pb_set_error(PB_ENOMEM, "persistent decode: schedule");
    }
    PB_TRY_CUDA(cudaMemcpy(s->d_sched, host.data(), s->sched_bytes, cudaMemcpyHostToDevice));
    s->map_off = mo;
  }
  s->sched_smem_off = sched_off;
  s->nphase = (int)ph.size();
  if (getenv("PB_DECODE_TRACE") && !s->d_trace) {
    if (cudaMalloc(&s->d_trace, (size_t)pb_num_sms() * ph.size() * 8 * 8) != cudaSuccess) {
      cudaGetLastError();
      s->d_trace = nullptr;
    }
  }
  if (cudaMalloc(&s->d_phases, ph.size() * sizeof(DPhase)) != cudaSuccess) {
    cudaGetLastError();
    s->d_phases = nullptr;
    return pb_set_error(PB_ENOMEM, "persistent decode: phase table");
  }
  PB_TRY_CUDA(cudaMemcpy(s->d_phases, ph.data(), ph.size() * sizeof(DPhase), cudaMemcpyHostToDevice));
  return PB_OK;
}

template <bool F32S, int E, int EH, int W, bool EXT>
int launch_decode_t(pb_state* s, int ntok, cudaStream_t st) {
  DecodeArgs d;
  d.phases = s->d_phases;
  d.nphase = s->nphase;
  d.ntok = ntok;
  d.qbase = s->qbase;
  d.ctl = s->ctl;
  d.bar = s->d_bar;
  d.err = s->d_err;
  d.xregion = s->xregion;
  d.nh = s->m->NH;
  d.ds = s->ds;
  d.trace = s->d_trace;
  d.sched = reinterpret_cast<const GemvSched*>(s->d_sched);
  d.spt = reinterpret_cast<const int*>(s->d_sched + s->spt_off);
  d.sdesc = reinterpret_cast<const StageDesc*>(s->d_sched + s->map_off);
  d.arena = s->m->arena;
  d.ngemv = s->ngemv;
  d.spt_max = s->spt_max;
  d.sched_off = (int)s->sched_smem_off;
  d.desc_off = (int)(s->sched_smem_off + (size_t)s->ngemv * sizeof(GemvSched));
  d.res_off = (int)s->res_smem_off;
  if (!s->decode_checked) {   // once per state and schedule, not per launch
    // the attribute belongs to the kernel on a device, shared by every state
    // there: only ever raise it, to the largest shared memory any state needs
    static std::mutex mu;
    static size_t attr_max[64] = {};
    int dev = 0;
    PB_TRY_CUDA(cudaGetDevice(&dev));
    {
      std::lock_guard<std::mutex> lk(mu);
      if (dev < 0 || dev >= 64 || s->dsmem > attr_max[dev]) {
        PB_TRY_CUDA(cudaFuncSetAttribute(k_decode<F32S, E, EH, W, EXT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)s->dsmem));
        if (dev >= 0 && dev < 64) attr_max[dev] = s->dsmem;
      }
    }
    int per_sm = 0;
    PB_TRY_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_decode<F32S, E, EH, W, EXT>, DTHREADS, s->dsmem));
    if (per_sm < 1) return pb_set_error(PB_ENOTSUP, "persistent decode does not fit on an SM");
    s->decode_checked = true;
  }
  const int grid = pb_num_sms();
  if (grid > MAX_CTA || grid < s->m->NH) return pb_set_error(PB_ENOTSUP, "persistent decode grid %d", grid);
  PB_TRY_CUDA(cudaMemsetAsync(s->d_bar, 0, sizeof(unsigned), st));
  if (s->d_trace) PB_TRY_CUDA(cudaMemsetAsync(s->d_trace, 0, (size_t)pb_num_sms() * s->nphase * 8 * 8, st));
  void* args[] = {&d};
  cudaError_t e = cudaLaunchCooperativeKernel((const void*)k_decode<F32S, E, EH, W, EXT>, dim3(grid), dim3(DTHREADS), args,
                                              s->dsmem, st);
  // the tags of the next launch continue after this one's, whether or not it
  // ran to the end (a launch that gave up leaves words of its own tag range)
  s->qbase += (unsigned)ntok * (unsigned)s->nphase;
  if (e != cudaSuccess) return pb_set_error(PB_ECUDA, "launch k_decode: %s", cudaGetErrorString(e));
  pb_count_launch();
  return PB_OK;
}

// a model with one-chunk rows (K not a multiple of 2048) or the bf16 head
bool model_ext(const pb_model* m) {
  if (m->head.layout == PB_Q8_B16) return true;
  for (const auto& Ly : m->layers)
    if ((Ly.first.one && Ly.first.nch > 1) || (Ly.mix.one && Ly.mix.nch > 1) || (Ly.w13.one && Ly.w13.nch > 1) ||
        (Ly.w2.one && Ly.w2.nch > 1))
      return true;
  return false;
}

int launch_decode(pb_state* s, int ntok, cudaStream_t st) {
  int rc = build_phases(s);
  if (rc) return rc;
  const bool f = s->m->sdt == PB_DT_F32;
  if (persistent_shape(s->m)) {
    if (s->m->HD == 128)
      return f ? launch_decode_t<true, 4, 8, 7, true>(s, ntok, st) : launch_decode_t<false, 4, 8, 7, true>(s, ntok, st);
    if (model_ext(s->m))
      return f ? launch_decode_t<true, 2, 8, 3, true>(s, ntok, st) : launch_decode_t<false, 2, 8, 3, true>(s, ntok, st);
    return f ? launch_decode_t<true, 2, 8, 3, false>(s, ntok, st) : launch_decode_t<false, 2, 8, 3, false>(s, ntok, st);
  }
  return pb_set_error(PB_ENOTSUP, "persistent decode: shape not compiled");
}

// the kernel's error word (a bounded wait gave up); clears it
int check_decode_error(pb_state* s, cudaStream_t st) {
  int* he = reinterpret_cast<int*>(s->h_ctl + 1);   // pinned: the copy stays asynchronous
  PB_TRY_CUDA(cudaMemcpyAsync(he, s->d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
  PB_TRY_CUDA(cudaStreamSynchronize(st));
  const int e = *he;
  if (e) {
    cudaMemsetAsync(s->d_err, 0, sizeof(int), st);
    return pb_set_error(PB_ECUDA, "decode kernel: a bounded wait gave up (code %d)", e);
  }
  return PB_OK;
}

// ---- loader -----------------------------------------------------------------
int read_all(FILE* f, void* dst, size_t n) {
  return fread(dst, 1, n, f) == n ? PB_OK : PB_EIO;
}

const Tensor* find(const pb_model* m, const std::string& name) {
  for (auto& t : m->table) if (t.name == name) return &t;
  return nullptr;
}

std::string lname(int L, const char* suf) {
  char b[160];
  snprintf(b, sizeof b, "lfm.model.layers.%d.%s", L, suf);
  return b;
}

}  // namespace

// ============================================================== C ABI
extern "C" int pb_open(const char* path, int device, pb_model** out) {
  if (!path || !out) return pb_set_error(PB_EINVAL, "pb_open: null argument");
  *out = nullptr;
  FILE* f = fopen(path, "rb");
  if (!f) return pb_set_error(PB_EIO, "pb_open: cannot open %s", path);
  char magic[8];
  uint32_t hl = 0;
  if (fread(magic, 1, 8, f) != 8 || memcmp(magic, "LFM3Q8\x01\x00", 8) != 0) {
    fclose(f);
    return pb_set_error(PB_EFORMAT, "pb_open: bad magic in %s", path);
  }
  if (fread(&hl, 4, 1, f) != 1 || hl == 0 || hl > (1u << 30)) {
    fclose(f);
    return pb_set_error(PB_EFORMAT, "pb_open: bad header length");
  }
  std::string js(hl, '\0');
  if (read_all(f, &js[0], hl)) { fclose(f); return pb_set_error(PB_EIO, "pb_open: short header"); }
  const size_t base = 8 + 4 + (size_t)hl;
  pbjson::Value root;
  pbjson::Parser P(js.data(), js.size());
  if (!P.parse(root) || root.kind != pbjson::Value::OBJ) {
    fclose(f);
    return pb_set_error(PB_EFORMAT, "pb_open: header JSON: %s", P.error());
  }
  const pbjson::Value* cfg = root.get("cfg");
  const pbjson::Value* table = root.get("table");
  if (!cfg || cfg->kind != pbjson::Value::OBJ || !table || table->kind != pbjson::Value::ARR) {
    fclose(f);
    return pb_set_error(PB_EFORMAT, "pb_open: header lacks cfg/table");
  }
  pb_model* m = new pb_model();
  m->device = device;
  auto cint = [&](const char* k, long long d) { const pbjson::Value* v = cfg->get(k); return v ? v->as_int(d) : d; };
  auto cnum = [&](const char* k, double d) { const pbjson::Value* v = cfg->get(k); return v ? v->as_num(d) : d; };
  m->H = (int)cint("hidden_size", 0);
  m->F = (int)cint("intermediate_size", cint("block_ff_dim", 0));
  m->L = (int)cint("num_hidden_layers", 0);
  m->NH = (int)cint("num_attention_heads", 0);
  m->NKV = (int)cint("num_key_value_heads", m->NH);
  m->HD = (int)cint("head_dim", m->NH ? m->H / m->NH : 0);
  m->V = (int)cint("vocab_size", 0);
  m->W = (int)cint("conv_L_cache", 3);
  m->win = (int)cint("sliding_window_decode", 0);
  m->theta = (float)cnum("rope_theta", 1e6);
  m->partial = (float)cnum("partial_rotary_factor", 1.0);
  m->eps = (float)cnum("norm_eps", 1e-5);
  // sliding-attention layers: window and RoPE of their own (top-level keys,
  // or the per-type rope_parameters object of the HF config)
  m->win_s = (int)cint("sliding_window", 256);
  m->theta_s = (float)cnum("sliding_rope_theta", 1e4);
  m->partial_s = (float)cnum("sliding_partial_rotary_factor", 1.0);
  if (const pbjson::Value* rp = cfg->get("rope_parameters")) {
    if (rp->kind == pbjson::Value::OBJ) {
      if (const pbjson::Value* fa = rp->get("full_attention")) {
        if (const pbjson::Value* v = fa->get("rope_theta")) m->theta = (float)v->as_num(m->theta);
        if (const pbjson::Value* v = fa->get("partial_rotary_factor")) m->partial = (float)v->as_num(m->partial);
      }
      if (const pbjson::Value* sa = rp->get("sliding_attention")) {
        if (const pbjson::Value* v = sa->get("rope_theta")) m->theta_s = (float)v->as_num(m->theta_s);
        if (const pbjson::Value* v = sa->get("partial_rotary_factor")) m->partial_s = (float)v->as_num(m->partial_s);
      }
    }
  }
  const pbjson::Value* lt = cfg->get("layer_types");
  auto bad = [&](int code, const char* msg) { fclose(f); delete m; return pb_set_error(code, "pb_open: %s", msg); };
  if (m->H <= 0 || m->F <= 0 || m->L <= 0 || m->NH <= 0 || m->NKV <= 0 || m->HD <= 0 || m->V <= 0 || m->W <= 0)
    return bad(PB_EFORMAT, "cfg lacks a positive hidden/intermediate/layers/heads/vocab/conv size");
  if (!lt || lt->kind != pbjson::Value::ARR || (int)lt->arr.size() != m->L)
    return bad(PB_EFORMAT, "cfg.layer_types must list every layer");
  if (m->NH % m->NKV) return bad(PB_EFORMAT, "heads not a multiple of kv heads");
  if (m->H % 256 || m->H > 4096) return bad(PB_ENOTSUP, "hidden size must be a multiple of 256 up to 4096");
  // table
  for (auto& rv : table->arr) {
    Tensor t;
    const pbjson::Value* nm = rv.get("name");
    const pbjson::Value* ne = rv.get("ne");
    if (!nm || nm->kind != pbjson::Value::STR || !ne || ne->kind != pbjson::Value::ARR)
      return bad(PB_EFORMAT, "record without name/ne");
    t.name = nm->str;
    for (auto& d : ne->arr) t.ne.push_back(d.as_int(-1));
    const pbjson::Value *dt = rv.get("dtype"), *of = rv.get("off"), *nc = rv.get("ncodes"), *ns = rv.get("nscales"), *cr = rv.get("crc");
    if (!dt || !of || !nc || !cr) return bad(PB_EFORMAT, "record lacks dtype/off/ncodes/crc");
    t.dtype = (int)dt->as_int(-1);
    t.off = (size_t)of->as_int(0);
    t.nc = (size_t)nc->as_int(0);
    t.ns = ns ? (size_t)ns->as_int(0) : 0;
    t.crc = (uint32_t)cr->as_int(0);
    if (t.dtype == 1 || t.dtype == 8) {
      if (t.ne.size() != 2 || t.ne[0] <= 0 || t.ne[1] <= 0 || t.ne[1] % 32)
        return bad(PB_EFORMAT, ("Q8 tensor with bad shape: " + t.name).c_str());
      const size_t want_s = (size_t)t.ne[0] * (t.ne[1] / 32) * (t.dtype == 1 ? 4 : 2);
      if (t.nc != (size_t)t.ne[0] * t.ne[1] || t.ns != want_s)
        return bad(PB_EFORMAT, ("Q8 tensor with inconsistent sizes: " + t.name).c_str());
    } else if (t.dtype == 2) {
      size_t n = 1;
      for (auto d : t.ne) n *= (size_t)d;
      if (t.nc != n * 4) return bad(PB_EFORMAT, ("f32 tensor with inconsistent size: " + t.name).c_str());
    } else if (t.dtype == 3) {
      // bf16 payload, verbatim (export_lfm3_q8.py:96-110): ncodes = N K 2, nscales = 0
      if (t.ne.size() != 2 || t.ne[0] <= 0 || t.ne[1] <= 0 || t.ne[1] % 256 ||
          t.nc != (size_t)t.ne[0] * t.ne[1] * 2 || t.ns != 0)
        return bad(PB_EFORMAT, ("bf16 tensor with inconsistent sizes: " + t.name).c_str());
    } else if (t.dtype == 6 || t.dtype == 7) {
      // low-bit Q4 / Q5 payload, pre-tiled by the exporter (lfm3_nanode.cu:1494-1501)
      if (t.ne.size() != 2 || t.ne[0] <= 0 || t.ne[1] <= 0 || t.ne[0] % 32 || t.ne[1] % 256 ||
          t.nc != (size_t)t.ne[0] * t.ne[1] / 32 * (t.dtype == 6 ? 16 : 20) ||
          t.ns != (size_t)t.ne[0] * t.ne[1] / 32 * 4)
        return bad(PB_EFORMAT, ("bad low-bit record: " + t.name).c_str());
    } else {
      return bad(PB_ENOTSUP, ("tensor dtype not supported by this build: " + t.name).c_str());
    }
    m->table.push_back(t);
  }
  // layer types and per-layer tensors
  m->layers.resize(m->L);
  int sdt = -1;
  auto q8shape = [&](const std::string& n, int& N, int& K) -> const Tensor* {
    const Tensor* t = find(m, n);
    if (!t || (t->dtype != 1 && t->dtype != 8)) return nullptr;
    N = (int)t->ne[0]; K = (int)t->ne[1];
    const int d = t->dtype == 1 ? PB_DT_F32 : PB_DT_F16;
    if (sdt < 0) sdt = d;
    else if (sdt != d) return nullptr;
    return t;
  };
  int n_attn = 0, n_conv = 0;
  for (int L = 0; L < m->L; L++) {
    const pbjson::Value& v = lt->arr[L];
    if (v.kind != pbjson::Value::STR) return bad(PB_EFORMAT, "layer_types entries must be strings");
    m->layers[L].attn = v.str != "conv";
    m->layers[L].slide = v.str == "sliding_attention";
    m->any_slide = m->any_slide || m->layers[L].slide;
    if (m->layers[L].attn) m->layers[L].attn_idx = n_attn++;
    else m->layers[L].conv_idx = n_conv++;
  }
  m->n_attn = n_attn;
  bool lowbit = false;
  for (auto& t : m->table) lowbit = lowbit || t.dtype == 6 || t.dtype == 7;
  if (lowbit) {   // per-tensor mode: every projection on the device by itself
    m->per_tensor = true;
    m->decode_ok = false;
    std::vector<char> buf;
    auto read_tensor = [&](const Tensor& t) -> int {
      buf.resize(t.nc + t.ns);
      if (fseeko(f, (off_t)(base + t.off), SEEK_SET) != 0 || read_all(f, buf.data(), buf.size()))
        return pb_set_error(PB_EIO, "pb_open: short read in %s", t.name.c_str());
      const uint32_t c = (uint32_t)crc32(0L, reinterpret_cast<const Bytef*>(buf.data()), (uInt)buf.size());
      if (c != t.crc) return pb_set_error(PB_ECRC, "pb_open: CRC mismatch in %s", t.name.c_str());
      return PB_OK;
    };
    int rc = PB_OK;
    if (device < 0) {   // validate only
      for (auto& t : m->table)
        if ((rc = read_tensor(t)) != PB_OK) break;
      fclose(f);
      delete m;
      return rc;
    }
    if (cudaSetDevice(device) != cudaSuccess) {
      cudaGetLastError();
      return bad(PB_ECUDA, "cudaSetDevice failed");
    }
    m->pt_q8.assign(m->table.size(), nullptr);
    m->pt_qlow.assign(m->table.size(), nullptr);
    for (size_t i = 0; rc == PB_OK && i < m->table.size(); i++) {
      const Tensor& t = m->table[i];
      if (t.dtype != 1 && t.dtype != 8 && t.dtype != 6 && t.dtype != 7) continue;
      if ((rc = read_tensor(t)) != PB_OK) break;
      const int N = (int)t.ne[0], K = (int)t.ne[1];
      if (t.dtype == 6 || t.dtype == 7)
        rc = pb_qlow_pack(buf.data(), buf.data() + t.nc, t.dtype == 6 ? 4 : 5, N, K, 0, nullptr, &m->pt_qlow[i]);
      else
        rc = pb_q8_pack(reinterpret_cast<const int8_t*>(buf.data()), buf.data() + t.nc,
                        t.dtype == 1 ? PB_DT_F32 : PB_DT_F16, N, K, 0, nullptr, &m->pt_q8[i]);
      m->weight_bytes += t.nc + t.ns;
    }
    fclose(f);
    if (rc != PB_OK) { pb_close(m); return rc; }
    *out = m;
    return PB_OK;
  }
  // arena plan
  struct Piece { std::string name; pb_q8* dst; int rmul, radd; };
  std::vector<Piece> q8pieces;
  struct FPiece { std::string name; float** dst; size_t n; };
  std::vector<FPiece> fpieces;
  size_t need = 0;
  auto plan_q8 = [&](pb_q8& w, int N, int K) {
    w.N = N; w.K = K; w.owner = false;
    const int nch = pb_q8_stream_chunks(K, &w.one);
    w.layout = nch ? PB_Q8_STREAM : PB_Q8_ROWMAJOR;
    w.nch = nch ? nch : 1;
    need += align256(pb_q8_code_bytes(N, K));
    need += align256(pb_q8_layout_scale_bytes(N, K, PB_DT_F32));   // room for fp32 scales
    if (w.layout != PB_Q8_STREAM) m->decode_ok = false;
  };
  const int H = m->H, F = m->F, NH = m->NH, NKV = m->NKV, HD = m->HD, W = m->W;
  for (int L = 0; L < m->L; L++) {
    Layer& Ly = m->layers[L];
    int N, K;
    if (Ly.attn) {
      const char* nm[4] = {"self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                           "self_attn.gate_proj.weight"};
      const int want[4] = {NH * HD, NKV * HD, NKV * HD, NH};
      int off = 0;
      for (int i = 0; i < 4; i++) {
        if (!q8shape(lname(L, nm[i]), N, K) || N != want[i] || K != H) return bad(PB_EFORMAT, (lname(L, nm[i]) + " missing or misshapen").c_str());
      }
      plan_q8(Ly.first, NH * HD + 2 * NKV * HD + NH, H);
      for (int i = 0; i < 4; i++) { q8pieces.push_back({lname(L, nm[i]), &Ly.first, 1, off}); off += want[i]; }
      if (!q8shape(lname(L, "self_attn.o_proj.weight"), N, K) || N != H || K != NH * HD) return bad(PB_EFORMAT, "o_proj missing or misshapen");
      plan_q8(Ly.mix, H, NH * HD);
      q8pieces.push_back({lname(L, "self_attn.o_proj.weight"), &Ly.mix, 1, 0});
      fpieces.push_back({lname(L, "self_attn.q_norm.weight"), &Ly.q_norm, (size_t)HD});
      fpieces.push_back({lname(L, "self_attn.k_norm.weight"), &Ly.k_norm, (size_t)HD});
    } else {
      if (!q8shape(lname(L, "conv.in_proj.weight"), N, K) || N != 3 * H || K != H) return bad(PB_EFORMAT, "in_proj missing or misshapen");
      plan_q8(Ly.first, 3 * H, H);
      q8pieces.push_back({lname(L, "conv.in_proj.weight"), &Ly.first, 1, 0});
      if (!q8shape(lname(L, "conv.out_proj.weight"), N, K) || N != H || K != H) return bad(PB_EFORMAT, "out_proj missing or misshapen");
      plan_q8(Ly.mix, H, H);
      q8pieces.push_back({lname(L, "conv.out_proj.weight"), &Ly.mix, 1, 0});
      fpieces.push_back({lname(L, "conv.conv.weight"), &Ly.taps, (size_t)H * W});
    }
    if (!q8shape(lname(L, "feed_forward.w1.weight"), N, K) || N != F || K != H) return bad(PB_EFORMAT, "w1 missing or misshapen");
    if (!q8shape(lname(L, "feed_forward.w3.weight"), N, K) || N != F || K != H) return bad(PB_EFORMAT, "w3 missing or misshapen");
    plan_q8(Ly.w13, 2 * F, H);
    q8pieces.push_back({lname(L, "feed_forward.w1.weight"), &Ly.w13, 2, 0});
    q8pieces.push_back({lname(L, "feed_forward.w3.weight"), &Ly.w13, 2, 1});
    if (!q8shape(lname(L, "feed_forward.w2.weight"), N, K) || N != H || K != F) return bad(PB_EFORMAT, "w2 missing or misshapen");
    plan_q8(Ly.w2, H, F);
    q8pieces.push_back({lname(L, "feed_forward.w2.weight"), &Ly.w2, 1, 0});
    fpieces.push_back({lname(L, "operator_norm.weight"), &Ly.op_norm, (size_t)H});
    fpieces.push_back({lname(L, "post_operator_norm.weight"), &Ly.post_op_norm, (size_t)H});
    fpieces.push_back({lname(L, "ffn_norm.weight"), &Ly.ffn_norm, (size_t)H});
    fpieces.push_back({lname(L, "post_ffn_norm.weight"), &Ly.post_ffn_norm, (size_t)H});
  }
  bool emb16 = false;
  {
    int N, K;
    const Tensor* et = find(m, "lfm.model.embed_tokens.weight");
    if (et && et->dtype == 3) {
      // the certified arm's bf16 table (lfm3_nanode.cu:3505-3534): embedding
      // rows copied, the head as k_gemv_bf16
      if (et->ne[0] != m->V || et->ne[1] != H) return bad(PB_EFORMAT, "embed_tokens misshapen");
      emb16 = true;
      m->head.N = m->V; m->head.K = H; m->head.owner = false;
      need += align256(et->nc);
    } else {
      if (!q8shape("lfm.model.embed_tokens.weight", N, K) || N != m->V || K != H) return bad(PB_EFORMAT, "embed_tokens missing or misshapen");
      plan_q8(m->head, m->V, H);
      q8pieces.push_back({"lfm.model.embed_tokens.weight", &m->head, 1, 0});
    }
    fpieces.push_back({"lfm.model.embedding_norm.weight", &m->final_norm, (size_t)H});
  }
  for (auto& fp : fpieces) {
    const Tensor* t = find(m, fp.name);
    if (!t || t->dtype != 2 || t->nc != fp.n * 4) return bad(PB_EFORMAT, (fp.name + " missing or misshapen").c_str());
    need += align256(fp.n * 4);
  }
  m->sdt = sdt < 0 ? PB_DT_F16 : sdt;
  if (device < 0) {
    // validate only: every payload's size and CRC, no GPU touched
    std::vector<char> buf;
    for (auto& t : m->table) {
      buf.resize(t.nc + t.ns);
      if (fseeko(f, (off_t)(base + t.off), SEEK_SET) != 0 || read_all(f, buf.data(), buf.size()))
        return bad(PB_EIO, ("short read in " + t.name).c_str());
      const uint32_t c = (uint32_t)crc32(0L, reinterpret_cast<const Bytef*>(buf.data()), (uInt)buf.size());
      if (c != t.crc) return bad(PB_ECRC, ("CRC mismatch in " + t.name).c_str());
    }
    fclose(f);
    delete m;
    return PB_OK;
  }
  if (cudaSetDevice(device) != cudaSuccess) {
    cudaGetLastError();
    return bad(PB_ECUDA, "cudaSetDevice failed");
  }
  // allocate
  if (cudaMalloc(&m->arena, need) != cudaSuccess) {
    cudaGetLastError();
    return bad(PB_ENOMEM, "cannot allocate the weight arena");
  }
  m->arena_bytes = need;
  size_t cursor = 0;
  std::vector<pb_q8*> assigned;
  auto assign = [&](pb_q8* w) {
    for (auto* p : assigned) if (p == w) return;
    w->sdt = m->sdt;
    w->codes = reinterpret_cast<int8_t*>(m->arena + cursor);
    cursor += align256(pb_q8_code_bytes(w->N, w->K));
    w->scales = m->arena + cursor;
    cursor += align256(pb_q8_layout_scale_bytes(w->N, w->K, PB_DT_F32));
    assigned.push_back(w);
  };
  for (auto& p : q8pieces) assign(p.dst);
  if (emb16) {
    m->head16 = reinterpret_cast<uint16_t*>(m->arena + cursor);
    cursor += align256((size_t)m->V * H * 2);
    m->head.layout = PB_Q8_B16;
    m->head.codes = reinterpret_cast<int8_t*>(m->head16);
    m->head.scales = nullptr;
    m->head.nch = H >= 1024 ? H / 1024 : 1;   // 2048-byte segments per row (the persistent kernel takes H 2048)
  }
  for (auto& fp : fpieces) {
    *fp.dst = reinterpret_cast<float*>(m->arena + cursor);
    cursor += align256(fp.n * 4);
  }
  // stream the payloads: read, CRC, upload, pack
  size_t maxb = 0;
  for (auto& t : m->table) maxb = std::max(maxb, t.nc + t.ns);
  char* host = nullptr;
  char* stage = nullptr;
  cudaStream_t st = nullptr;
  int rc = PB_OK;
  if (cudaMallocHost(&host, maxb) != cudaSuccess || cudaMalloc(&stage, maxb) != cudaSuccess ||
      cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) {
    cudaGetLastError();
    rc = pb_set_error(PB_ENOMEM, "pb_open: staging buffers");
  }
  auto load = [&](const Tensor* t) -> int {
    if (fseeko(f, (off_t)(base + t->off), SEEK_SET) != 0) return pb_set_error(PB_EIO, "seek %s", t->name.c_str());
    if (cudaStreamSynchronize(st) != cudaSuccess) return pb_set_error(PB_ECUDA, "upload sync");
    if (read_all(f, host, t->nc + t->ns)) return pb_set_error(PB_EIO, "short read in %s", t->name.c_str());
    const uint32_t c = (uint32_t)crc32(0L, reinterpret_cast<const Bytef*>(host), (uInt)(t->nc + t->ns));
    if (c != t->crc) return pb_set_error(PB_ECRC, "CRC mismatch in %s: file %08x, table %08x", t->name.c_str(), c, t->crc);
    PB_TRY_CUDA(cudaMemcpyAsync(stage, host, t->nc + t->ns, cudaMemcpyHostToDevice, st));
    return PB_OK;
  };
  for (size_t i = 0; rc == PB_OK && i < q8pieces.size(); i++) {
    const Tensor* t = find(m, q8pieces[i].name);
    if ((rc = load(t)) != PB_OK) break;
    rc = pb_q8_pack_into(q8pieces[i].dst, reinterpret_cast<int8_t*>(stage), stage + t->nc, st,
                         (int)t->ne[0], q8pieces[i].rmul, q8pieces[i].radd);
    m->weight_bytes += t->nc + (size_t)t->ne[0] * (t->ne[1] / 32) * (m->sdt == PB_DT_F32 ? 4 : 2);
  }
  if (rc == PB_OK && emb16) {
    const Tensor* t = find(m, "lfm.model.embed_tokens.weight");
    if ((rc = load(t)) == PB_OK) {
      rc = pb_b16_pack(reinterpret_cast<const uint16_t*>(stage), m->head16, m->V, H, st);
      m->weight_bytes += t->nc;
    }
  }
  for (size_t i = 0; rc == PB_OK && i < fpieces.size(); i++) {
    const Tensor* t = find(m, fpieces[i].name);
    if ((rc = load(t)) != PB_OK) break;
    if (cudaMemcpyAsync(*fpieces[i].dst, stage, t->nc, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
      rc = pb_set_error(PB_ECUDA, "upload %s", t->name.c_str());
    m->weight_bytes += t->nc;
  }
  if (rc == PB_OK && cudaStreamSynchronize(st) != cudaSuccess)
    rc = pb_set_error(PB_ECUDA, "pb_open: %s", cudaGetErrorString(cudaGetLastError()));
  if (host) cudaFreeHost(host);
  if (stage) cudaFree(stage);
  if (st) cudaStreamDestroy(st);
  fclose(f);
  if (rc != PB_OK) { cudaFree(m->arena); delete m; return rc; }
  // build_invf (lfm3_nanode.cu:3719-3723) for each attention layer type
  auto invf = [&](std::vector<float>& out, float base, float partial) {
    out.resize(m->HD / 2);
    const int angles = (int)((double)partial * m->HD) / 2;
    for (int i = 0; i < m->HD / 2; i++)
      out[i] = (i < angles) ? 1.0f / powf(base, (float)(2 * i) / (float)m->HD) : 0.0f;
  };
  invf(m->invf, m->theta, m->partial);
  invf(m->invf_s, m->theta_s, m->partial_s);
  *out = m;
  return PB_OK;
}

extern "C" int pb_close(pb_model* m) {
  if (!m) return PB_OK;
  for (auto* q : m->pt_q8) pb_q8_free(q);
  for (auto* q : m->pt_qlow) pb_qlow_free(q);
  cudaFree(m->arena);
  cudaFree(m->tc_arena);
  delete m;
  return PB_OK;
}

extern "C" int pb_model_get_info(const pb_model* m, pb_model_info* info) {
  if (!m || !info) return pb_set_error(PB_EINVAL, "pb_model_get_info: null argument");
  info->hidden = m->H; info->inter = m->F; info->n_layers = m->L; info->n_heads = m->NH;
  info->n_kv = m->NKV; info->head_dim = m->HD; info->vocab = m->V; info->conv_w = m->W;
  info->n_attn = m->n_attn; info->sliding_window = m->win;
  info->rope_theta = m->theta; info->rope_partial = m->partial; info->norm_eps = m->eps;
  info->weight_bytes = m->weight_bytes;
  return PB_OK;
}

extern "C" int pb_tensor_id(const pb_model* m, const char* name) {
  if (!m || !name) return pb_set_error(PB_EINVAL, "pb_tensor_id: null argument");
  for (size_t i = 0; i < m->table.size(); i++)
    if (m->table[i].name == name) return (int)i;
  return pb_set_error(PB_EINVAL, "pb_tensor_id: no tensor %s", name);
}

extern "C" int pb_model_gemv(pb_model* m, int tensor_id, const uint16_t* d_x, uint16_t* d_y, void* stream) {
  if (!m || !d_x || !d_y) return pb_set_error(PB_EINVAL, "pb_model_gemv: null argument");
  if (!m->per_tensor)
    return pb_set_error(PB_ENOTSUP, "pb_model_gemv: the model's projections are fused for decoding "
                                    "(per-tensor GEMVs are for models holding Q4 / Q5 records)");
  if (tensor_id < 0 || tensor_id >= (int)m->table.size())
    return pb_set_error(PB_EINVAL, "pb_model_gemv: tensor id %d", tensor_id);
  PB_TRY_CUDA(cudaSetDevice(m->device));
  if (m->pt_qlow[tensor_id]) return pb_qlow_gemv(m->pt_qlow[tensor_id], d_x, d_y, stream);
  if (m->pt_q8[tensor_id]) return pb_q8_gemv(m->pt_q8[tensor_id], d_x, d_y, PB_DT_BF16, stream);
  return pb_set_error(PB_EINVAL, "pb_model_gemv: %s is not a Q8 / Q4 / Q5 matrix", m->table[tensor_id].name.c_str());
}

extern "C" int pb_state_create(pb_model* m, int max_ctx, pb_state** out) {
  if (!m || !out || max_ctx <= 0) return pb_set_error(PB_EINVAL, "pb_state_create: bad argument");
  *out = nullptr;
  if (m->per_tensor) return pb_set_error(PB_ENOTSUP, "pb_state_create: a model holding Q4 / Q5 records runs per-tensor GEMVs only (pb_model_gemv)");
  if (!m->decode_ok) return pb_set_error(PB_ENOTSUP, "decode needs every matrix in the streaming layout (K up to 16384)");
  if ((size_t)max_ctx * 4 > 160 * 1024) return pb_set_error(PB_ENOTSUP, "max_ctx %d too large", max_ctx);
  PB_TRY_CUDA(cudaSetDevice(m->device));
  pb_state* s = new pb_state();
  s->m = m;
  s->max_ctx = max_ctx;
  {
    const char* mode = getenv("PB_DECODE_MODE");   // "graph": the per-kernel CUDA-graph path
    s->persistent = !(mode && strcmp(mode, "graph") == 0);
    // the persistent softmax holds a head's scores in registers (64 per lane)
    if (max_span(m, max_ctx) > 2048 || !persistent_shape(m)) s->persistent = false;
  }
  const int H = m->H, n_conv = m->L - m->n_attn, half = half_rot(m), half_s = half_rot_s(m);
  const size_t kvb = (size_t)m->n_attn * 2 * max_ctx * m->NKV * m->HD * 2;
  const size_t ringb = (size_t)n_conv * m->W * H * 2;
  const size_t ropeb = (size_t)max_ctx * (half > 0 ? half : 1) * 4;
  const size_t ropeb_s = m->any_slide ? (size_t)max_ctx * (half_s > 0 ? half_s : 1) * 4 : 0;
  const size_t firstn = std::max((size_t)3 * H, (size_t)m->NH * m->HD + 2 * (size_t)m->NKV * m->HD + m->NH);
  size_t sizes[] = {kvb, ringb, ropeb, ropeb, (size_t)H * 2, (size_t)H * 2, (size_t)H * 2, firstn * 2,
                    (size_t)m->NH * m->HD * 2, (size_t)H * 2, (size_t)m->F * 2, (size_t)H * 2,
                    (size_t)m->V * 4, sizeof(Ctl), 256, 256, (size_t)m->NH * max_ctx * 4, (size_t)m->NH * 4,
                    (size_t)m->NH * 8 * m->HD * 4,
                    firstn * 4, (size_t)m->NH * m->HD * 4, (size_t)H * 4, (size_t)m->F * 4, (size_t)H * 4,
                    (size_t)m->NH * max_ctx * 8, ropeb_s, ropeb_s};
  size_t tot = 0;
  for (size_t x : sizes) tot += align256(x);
  if (cudaMalloc(&s->mem, tot) != cudaSuccess) { cudaGetLastError(); delete s; return pb_set_error(PB_ENOMEM, "pb_state_create: %zu bytes", tot); }
  s->mem_bytes = tot;
  char* p = s->mem;
  void** slots[] = {(void**)&s->kv, (void**)&s->ring, (void**)&s->rope_cos, (void**)&s->rope_sin,
                    (void**)&s->res[0], (void**)&s->res[1], (void**)&s->res[2], (void**)&s->h_first,
                    (void**)&s->h_attn, (void**)&s->h_mix, (void**)&s->h_u, (void**)&s->h_w2,
                    (void**)&s->logits, (void**)&s->ctl, (void**)&s->d_bar, (void**)&s->d_err,
                    (void**)&s->att_scores, (void**)&s->att_inv, (void**)&s->att_segp,
                    (void**)&s->t_first, (void**)&s->t_attn, (void**)&s->t_mix, (void**)&s->t_u, (void**)&s->t_w2,
                    (void**)&s->t_scores, (void**)&s->rope_cos_s, (void**)&s->rope_sin_s};
  for (size_t i = 0; i < sizeof(sizes) / sizeof(sizes[0]); i++) { *slots[i] = p; p += align256(sizes[i]); }
  s->tag_bytes = (size_t)((char*)s->t_scores - (char*)s->t_first) + align256((size_t)m->NH * max_ctx * 8);
  if (cudaMallocHost(&s->h_ctl, sizeof(Ctl) + 16) != cudaSuccess) {
    cudaGetLastError(); cudaFree(s->mem); delete s;
    return pb_set_error(PB_ENOMEM, "pb_state_create: pinned control block");
  }
  // RoPE tables on the host, one per attention layer type: angle (float)pos *
  // invf[i] in fp32 (lfm3_nanode.cu:492), cos/sin evaluated in double and
  // rounded once to float
  auto table = [&](const std::vector<float>& invf, int hf, float* dc, float* dsn) -> bool {
    std::vector<float> hc((size_t)max_ctx * (hf > 0 ? hf : 1)), hs(hc.size());
    for (int pos = 0; pos < max_ctx; pos++)
      for (int i = 0; i < hf; i++) {
        const float ang = (float)pos * invf[i];
        hc[(size_t)pos * hf + i] = (float)cos((double)ang);
        hs[(size_t)pos * hf + i] = (float)sin((double)ang);
      }
    return cudaMemcpy(dc, hc.data(), hc.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess &&
           cudaMemcpy(dsn, hs.data(), hs.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess;
  };
  bool rope_ok = table(m->invf, half, s->rope_cos, s->rope_sin);
  if (m->any_slide) rope_ok = rope_ok && table(m->invf_s, half_s, s->rope_cos_s, s->rope_sin_s);
  else { s->rope_cos_s = s->rope_cos; s->rope_sin_s = s->rope_sin; }
  if (!rope_ok) {
    cudaFreeHost(s->h_ctl); cudaFree(s->mem); delete s;
    return pb_set_error(PB_ECUDA, "pb_state_create: rope upload");
  }
  int rc = pb_state_reset(s, nullptr);
  if (rc == PB_OK && cudaDeviceSynchronize() != cudaSuccess) rc = pb_set_error(PB_ECUDA, "pb_state_create: sync");
  if (rc) { cudaFreeHost(s->h_ctl); cudaFree(s->mem); delete s; return rc; }
  *out = s;
  return PB_OK;
}

extern "C" int pb_state_destroy(pb_state* s) {
  if (!s) return PB_OK;
  // the graph holds the communicator's captured collectives: release it first,
  // or the communicator's destruction waits for it forever
  if (s->exec) cudaGraphExecDestroy(s->exec);
  if (s->graph) cudaGraphDestroy(s->graph);
  s->exec = nullptr;
  s->graph = nullptr;
  if (s->comm) {
    cudaDeviceSynchronize();
    nccl().comm_destroy(s->comm);
  }
  if (s->d_phases) cudaFree(s->d_phases);
  if (s->d_sched) cudaFree(s->d_sched);
  if (s->d_trace) cudaFree(s->d_trace);
  if (s->graph_stream) cudaStreamDestroy(s->graph_stream);
  cudaFreeHost(s->h_ctl);
  cudaFree(s->mem);
  cudaFree(s->pf_mem);
  delete s;
  return PB_OK;
}

extern "C" int pb_state_reset(pb_state* s, void* stream) {
  if (!s) return pb_set_error(PB_EINVAL, "pb_state_reset: null state");
  cudaStream_t st = (cudaStream_t)stream;
  const pb_model* m = s->m;
  const size_t kvb = (size_t)m->n_attn * 2 * s->max_ctx * m->NKV * m->HD * 2;
  const size_t ringb = (size_t)(m->L - m->n_attn) * m->W * m->H * 2;
  if (kvb) PB_TRY_CUDA(cudaMemsetAsync(s->kv, 0, kvb, st));
  if (ringb) PB_TRY_CUDA(cudaMemsetAsync(s->ring, 0, ringb, st));
  PB_TRY_CUDA(cudaMemsetAsync(s->ctl, 0, sizeof(Ctl), st));
  PB_TRY_CUDA(cudaMemsetAsync(s->d_err, 0, sizeof(int), st));
  // tagged activations: tag 0xffff, which no phase of the next 65535 carries
  // (scores: 0xffffffff)
  PB_TRY_CUDA(cudaMemsetAsync(s->t_first, 0xff, s->tag_bytes, st));
  s->qbase = 0;
  return PB_OK;
}

static int set_ctl(pb_state* s, int token, int pos, int* ids, cudaStream_t st,
                   const int* prompt = nullptr, int n_prompt = 0) {
  // the previous upload from this pinned block must have landed first
  PB_TRY_CUDA(cudaStreamSynchronize(st));
  s->h_ctl->token = token;
  s->h_ctl->pos = pos;
  s->h_ctl->step = 0;
  s->h_ctl->counter = 0;
  s->h_ctl->ids = ids;
  s->h_ctl->prompt = prompt;
  s->h_ctl->n_prompt = n_prompt;
  PB_TRY_CUDA(cudaMemcpyAsync(s->ctl, s->h_ctl, offsetof(Ctl, slot_val), cudaMemcpyHostToDevice, st));
  return PB_OK;
}

extern "C" int pb_layer_step(pb_model* m, pb_state* s, int layer, int pos, uint16_t* d_x, void* stream) {
  if (!m || !s || !d_x || layer < 0 || layer >= m->L || pos < 0 || pos >= s->max_ctx)
    return pb_set_error(PB_EINVAL, "pb_layer_step: bad argument");
  cudaStream_t st = (cudaStream_t)stream;
  int rc = set_ctl(s, 0, pos, nullptr, st);
  if (rc) return rc;
  // residual in d_x; the layer writes its pre-FFN residual into res[1] (cur
  // flips 0 -> 1) and the tail adds the FFN branch back into d_x
  int cur = 0;
  uint64_t nk = 0;
  if ((rc = enqueue_layer(m, s, layer, cur, PRO_ADDNORM, false, d_x, st, false, nk))) return rc;
  StepArgs a = base_args(m, s);
  a.pro = PRO_ADDNORM;
  a.xin = s->res[cur];
  a.hin = s->h_w2;
  a.wpost = m->layers[layer].post_ffn_norm;
  a.wnorm = nullptr;
  a.rout = d_x;
  a.K = m->H;
  k_tail<<<1, 256, step_smem(m->H, m->H), st>>>(a);
  PB_LAUNCHED("k_tail");
  return PB_OK;
}

extern "C" int pb_decode_token(pb_model* m, pb_state* s, int token, int pos, int* h_out_id,
                               float* d_logits, void* stream) {
  if (!m || !s || token < 0 || token >= m->V || pos < 0 || pos >= s->max_ctx)
    return pb_set_error(PB_EINVAL, "pb_decode_token: bad argument");
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
  if (s->persistent) {
    if ((rc = build_phases(s))) return rc;
    if ((rc = set_ctl(s, token, pos, nullptr, st))) return rc;
    if ((rc = launch_decode(s, 1, st))) return rc;
  } else {
    if ((rc = build_graph(s))) return rc;
    if ((rc = set_ctl(s, token, pos, nullptr, st))) return rc;
    PB_TRY_CUDA(cudaGraphLaunch(s->exec, st));
    pb_count_launch(s->graph_launches);
  }
  if (d_logits) PB_TRY_CUDA(cudaMemcpyAsync(d_logits, s->logits, (size_t)m->V * 4, cudaMemcpyDeviceToDevice, st));
  if (h_out_id) {
    PB_TRY_CUDA(cudaMemcpyAsync(&s->h_ctl->token, &s->ctl->token, sizeof(int), cudaMemcpyDeviceToHost, st));
    if (s->persistent) {
      if ((rc = check_decode_error(s, st))) return rc;   // synchronises the stream
    } else {
      PB_TRY_CUDA(cudaStreamSynchronize(st));
    }
    *h_out_id = s->h_ctl->token;
  }
  return PB_OK;
}

extern "C" int pb_decode_greedy(pb_model* m, pb_state* s, int token, int pos0, int n, int* d_ids,
                                void* stream) {
  if (!m || !s || token < 0 || token >= m->V || pos0 < 0 || n <= 0 || pos0 + n > s->max_ctx)
    return pb_set_error(PB_EINVAL, "pb_decode_greedy: bad argument");
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
  if (s->persistent) {
    if ((rc = build_phases(s))) return rc;
    if ((rc = set_ctl(s, token, pos0, d_ids, st))) return rc;
    return launch_decode(s, n, st);
  }
  if ((rc = build_graph(s))) return rc;
  if ((rc = set_ctl(s, token, pos0, d_ids, st))) return rc;
  for (int i = 0; i < n; i++) {
    PB_TRY_CUDA(cudaGraphLaunch(s->exec, st));
    pb_count_launch(s->graph_launches);
  }
  return PB_OK;
}

extern "C" int pb_nccl_unique_id(void* out, size_t bytes) {
  if (!out || bytes < sizeof(ncclUniqueId))
    return pb_set_error(PB_EINVAL, "pb_nccl_unique_id: buffer under %zu bytes", sizeof(ncclUniqueId));
  NcclApi& api = nccl();
  if (!api.ok) return pb_set_error(PB_ENOTSUP, "pb_nccl_unique_id: libnccl.so.2 not found");
  ncclUniqueId id;
  const ncclResult_t r = api.get_unique_id(&id);
  if (r != ncclSuccess) return pb_set_error(PB_ECUDA, "ncclGetUniqueId: %s", api.error_string(r));
  memcpy(out, &id, sizeof id);
  return PB_OK;
}

extern "C" int pb_state_shard(pb_state* s, int rank, int world, const void* id) {
  if (!s || !id || world < 1 || rank < 0 || rank >= world) return pb_set_error(PB_EINVAL, "pb_state_shard: bad argument");
  if (s->comm) return pb_set_error(PB_EINVAL, "pb_state_shard: state already sharded");
  const pb_model* m = s->m;
  if (!m->decode_ok) return pb_set_error(PB_ENOTSUP, "pb_state_shard: decode needs the streaming layout");
  auto fits = [&](const pb_q8& w, int mult) { return w.N % (world * mult) == 0; };
  for (int L = 0; L < m->L; L++) {
    const Layer& Ly = m->layers[L];
    if (!fits(Ly.first, 1) || !fits(Ly.mix, 1) || !fits(Ly.w13, 2) || !fits(Ly.w2, 1))
      return pb_set_error(PB_ENOTSUP, "pb_state_shard: layer %d rows do not split over %d ranks", L, world);
  }
  if (!fits(m->head, 1)) return pb_set_error(PB_ENOTSUP, "pb_state_shard: head rows do not split over %d ranks", world);
  if (world == 1) return PB_OK;
  NcclApi& api = nccl();
  if (!api.ok) return pb_set_error(PB_ENOTSUP, "pb_state_shard: libnccl.so.2 not found");
  PB_TRY_CUDA(cudaSetDevice(m->device));
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof uid);
  ncclComm_t comm = nullptr;
  const ncclResult_t r = api.comm_init_rank(&comm, world, uid, rank);   // collective over the ranks
  if (r != ncclSuccess) return pb_set_error(PB_ECUDA, "ncclCommInitRank: %s", api.error_string(r));
  s->comm = comm;
  s->tp_rank = rank;
  s->tp_world = world;
  s->persistent = false;   // the per-kernel graph carries the all-gathers
  if (s->exec) { cudaGraphExecDestroy(s->exec); s->exec = nullptr; }
  if (s->graph) { cudaGraphDestroy(s->graph); s->graph = nullptr; }
  return PB_OK;
}

extern "C" int pb_state_status(pb_state* s, void* stream) {
  if (!s) return pb_set_error(PB_EINVAL, "pb_state_status: null state");
  cudaStream_t st = (cudaStream_t)stream;
  PB_TRY_CUDA(cudaStreamSynchronize(st));
  return check_decode_error(s, st);
}

// test/inspection helpers (not in the public header): device pointers of a
// state's buffers so that tests can compare intermediate state
extern "C" int pb_state_debug(pb_state* s, int which, void** ptr, size_t* bytes) {
  if (!s || !ptr) return PB_EINVAL;
  const pb_model* m = s->m;
  switch (which) {
    case 0: *ptr = s->kv; if (bytes) *bytes = (size_t)m->n_attn * 2 * s->max_ctx * m->NKV * m->HD * 2; return PB_OK;
    case 1: *ptr = s->ring; if (bytes) *bytes = (size_t)(m->L - m->n_attn) * m->W * m->H * 2; return PB_OK;
    case 2: *ptr = s->res[s->graph_res]; if (bytes) *bytes = (size_t)m->H * 2; return PB_OK;
    case 3: *ptr = s->logits; if (bytes) *bytes = (size_t)m->V * 4; return PB_OK;
    case 4: *ptr = &s->ctl->pos; if (bytes) *bytes = 4; return PB_OK;
    case 5: *ptr = s->d_trace; if (bytes) *bytes = s->d_trace ? (size_t)pb_num_sms() * s->nphase * 8 * 8 : 0; return PB_OK;
  }
  return PB_EINVAL;
}

extern "C" int pb_decode_prompt(pb_model* m, pb_state* s, const int* d_tokens, int n, int pos0,
                                int* d_ids, void* stream) {
  if (!m || !s || !d_tokens || n <= 0 || pos0 < 0 || pos0 + n > s->max_ctx)
    return pb_set_error(PB_EINVAL, "pb_decode_prompt: bad argument");
  cudaStream_t st = (cudaStream_t)stream;
  int rc = s->persistent ? build_phases(s) : build_graph(s);
  if (rc) return rc;
  int first = 0;
  PB_TRY_CUDA(cudaMemcpy(&first, d_tokens, sizeof(int), cudaMemcpyDeviceToHost));
  if (first < 0 || first >= m->V) return pb_set_error(PB_EINVAL, "pb_decode_prompt: token %d", first);
  if ((rc = set_ctl(s, first, pos0, d_ids, st, d_tokens, n))) return rc;
  if (s->persistent) return launch_decode(s, n, st);
  for (int i = 0; i < n; i++) {
    PB_TRY_CUDA(cudaGraphLaunch(s->exec, st));
    pb_count_launch(s->graph_launches);
  }
  return PB_OK;
}

extern "C" int pb_decode_kernels_per_token(pb_state* s) {
  if (!s) return pb_set_error(PB_EINVAL, "null state");
  if (s->persistent) return 1;     // one cooperative launch decodes any number of tokens
  int rc = build_graph(s);
  return rc ? rc : (int)s->graph_launches;
}

// Times one of the decode step's fused GEMV kernels alone: `which` 0 = the
// layer's first GEMV (q|k|v|gate or in_proj), 1 = o_proj/out_proj, 2 = w1|w3,
// 3 = w2, 4 = the head. Launches cycle over every layer that has the tensor
// (distinct weights, more bytes than L2), `iters` launches between two events
// on `stream`; returns the mean ms per launch and the algorithmic bytes of one
// launch (codes + scales of its matrix).
extern "C" int pb_time_step_kernel(pb_model* m, pb_state* s, int which, int iters, float* ms,
                                   double* bytes, void* stream) {
  if (!m || !s || !ms || iters <= 0 || which < 0 || which > 4) return pb_set_error(PB_EINVAL, "pb_time_step_kernel");
  cudaStream_t st = (cudaStream_t)stream;
  std::vector<const pb_q8*> ws;
  std::vector<int> layer;
  for (int L = 0; L < m->L; L++) {
    const Layer& Ly = m->layers[L];
    if (which == 0) { ws.push_back(&Ly.first); layer.push_back(L); }
    if (which == 1) { ws.push_back(&Ly.mix); layer.push_back(L); }
    if (which == 2) { ws.push_back(&Ly.w13); layer.push_back(L); }
    if (which == 3) { ws.push_back(&Ly.w2); layer.push_back(L); }
  }
  if (which == 4) { ws.push_back(&m->head); layer.push_back(m->L - 1); }
  // uniform shape subset: the most common shape among the candidates
  const pb_q8* ref = ws[0];
  std::vector<const pb_q8*> sel;
  std::vector<int> sl;
  for (size_t i = 0; i < ws.size(); i++)
    if (ws[i]->N == ref->N && ws[i]->K == ref->K) { sel.push_back(ws[i]); sl.push_back(layer[i]); }
  cudaEvent_t e0, e1;
  PB_TRY_CUDA(cudaEventCreate(&e0));
  PB_TRY_CUDA(cudaEventCreate(&e1));
  auto one = [&](int i) -> int {
    const pb_q8* w = sel[i % sel.size()];
    const Layer& Ly = m->layers[sl[i % sl.size()]];
    StepArgs a = base_args(m, s);
    int epi = EPI_BF16;
    if (which == 2) {
      a.pro = PRO_ADDNORM; a.xin = s->res[0]; a.hin = s->h_mix; a.wpost = Ly.post_op_norm;
      a.wnorm = Ly.ffn_norm; a.y = s->h_u; epi = EPI_SILU;
    } else if (which == 4) {
      a.pro = PRO_ADDNORM; a.xin = s->res[0]; a.hin = s->h_w2; a.wpost = Ly.post_ffn_norm;
      a.wnorm = m->final_norm; a.y = s->logits; epi = EPI_ARGMAX;
    } else if (which == 3) {
      a.pro = PRO_PLAIN; a.xin = s->h_u; a.y = s->h_w2;
    } else if (which == 1) {
      a.pro = PRO_PLAIN; a.xin = s->h_attn; a.y = s->h_mix;     // same stream cost either mixer
    } else {
      a.pro = PRO_ADDNORM; a.xin = s->res[0]; a.hin = s->h_w2; a.wpost = Ly.post_ffn_norm;
      a.wnorm = Ly.op_norm; a.y = s->h_first;
    }
    return launch_step(*w, epi, a, st, true);
  };
  int rc = PB_OK;
  for (int i = 0; i < 3 && rc == PB_OK; i++) rc = one(i);         // warm-up
  if (rc == PB_OK) rc = cudaEventRecord(e0, st) == cudaSuccess ? PB_OK : PB_ECUDA;
  for (int i = 0; i < iters && rc == PB_OK; i++) rc = one(i);
  if (rc == PB_OK && cudaEventRecord(e1, st) != cudaSuccess) rc = PB_ECUDA;
  if (rc == PB_OK && cudaEventSynchronize(e1) != cudaSuccess) rc = pb_set_error(PB_ECUDA, "timing sync");
  float t = 0;
  if (rc == PB_OK) cudaEventElapsedTime(&t, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (rc) return rc;
  *ms = t / iters;
  if (bytes) *bytes = (double)ref->N * ref->K + (double)ref->N * (ref->K / 32) * (ref->sdt == PB_DT_F32 ? 4 : 2);
  return PB_OK;
}

namespace {
__global__ void k_test_expf(const float* x, float* y, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = pb_expf(x[i]);
}
}  // namespace
// test hook: the device e^x over n values (not part of the public ABI)
extern "C" int pb_test_expf(const float* d_x, float* d_y, int n, void* stream) {
  k_test_expf<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(d_x, d_y, n);
  PB_LAUNCHED("k_test_expf");
  return PB_OK;
}

namespace {
// the persistent kernel's grid wait on a counter that nothing advances: it
// must give up after `limit` polls and report it, as the kernel does with
// its error word (status 1 = gave up, 2 = passed)
__global__ void k_test_grid_wait(const unsigned* bar, unsigned target, unsigned limit, int* status) {
  if (threadIdx.x == 0) *status = grid_wait(bar, target, limit) ? 2 : 1;
}
}  // namespace
// test hook (not part of the public ABI): one bounded grid wait; d_bar and
// d_status are device ints, limit the number of polls
extern "C" int pb_test_grid_wait(const unsigned* d_bar, unsigned target, unsigned limit, int* d_status,
                                 void* stream) {
  if (!d_bar || !d_status) return pb_set_error(PB_EINVAL, "pb_test_grid_wait: null argument");
  k_test_grid_wait<<<1, 32, 0, (cudaStream_t)stream>>>(d_bar, target, limit, d_status);
  PB_LAUNCHED("k_test_grid_wait");
  return PB_OK;
}

// ============================================ layer step without allocation
// Some callers cannot call cudaMalloc at all: a host runtime that owns every
// allocation through its own pool or arena, code running where allocation is
// forbidden after start-up, or a caller that must not grow device memory in a
// latency-critical loop. pb_layer_step_noalloc gives them the layer step with
// its intermediate activations (the q|k|v|gate or in_proj output, the
// attention output, the mixer output, SiLU(w1)*w3, the w2 output, a residual
// and the control block) in one file-scope device array instead of buffers
// that pb_state_create allocated. The model (weights) and the state (KV cache,
// conv rings, RoPE table) are still the caller's existing objects.
namespace {
constexpr size_t PB_NOALLOC_SCRATCH_BYTES = 512 * 1024;   // the stated maximum
__device__ __align__(256) unsigned char g_noalloc_scratch[PB_NOALLOC_SCRATCH_BYTES];

constexpr int PB_MAX_DEVICES = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[PB_MAX_DEVICES] = {};

__global__ void k_noalloc_set_ctl(Ctl* ctl, int pos) {
  ctl->token = 0;
  ctl->pos = pos;
  ctl->step = 0;
  ctl->counter = 0;
  ctl->ids = nullptr;
  ctl->prompt = nullptr;
  ctl->n_prompt = 0;
}

struct NoAllocBufs {
  bf16_t *res1, *h_first, *h_attn, *h_mix, *h_u, *h_w2;
  Ctl* ctl;
};

size_t noalloc_bytes(const pb_model* m) {
  const size_t firstn = std::max((size_t)3 * m->H, (size_t)m->NH * m->HD + 2 * (size_t)m->NKV * m->HD + m->NH);
  return align256((size_t)m->H * 2) + align256(firstn * 2) + align256((size_t)m->NH * m->HD * 2) +
         align256((size_t)m->H * 2) + align256((size_t)m->F * 2) + align256((size_t)m->H * 2) +
         align256(sizeof(Ctl));
}
}  // namespace

extern "C" int pb_layer_step_noalloc(pb_model* m, pb_state* s, int layer, int pos, uint16_t* d_x,
                                     void* stream) {
  if (!m || !s || !d_x || layer < 0 || layer >= m->L || pos < 0 || pos >= s->max_ctx)
    return pb_set_error(PB_EINVAL, "pb_layer_step_noalloc: bad argument");
  // a row-sharded state's layer step needs the all-gathers of the state's
  // graph path; this step has none, so it serves unsharded states only
  if (s->tp_world > 1)
    return pb_set_error(PB_ENOTSUP, "pb_layer_step_noalloc: the state is row-sharded over %d ranks", s->tp_world);
  const size_t need = noalloc_bytes(m);
  if (need > PB_NOALLOC_SCRATCH_BYTES)
    return pb_set_error(PB_EINVAL, "pb_layer_step_noalloc: this model needs %zu bytes of scratch, "
                        "more than the static %zu", need, PB_NOALLOC_SCRATCH_BYTES);
  int dev = 0;
  PB_TRY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= PB_MAX_DEVICES) return pb_set_error(PB_EINVAL, "pb_layer_step_noalloc: device %d", dev);
  void* base = nullptr;
  {
    // set-up, once per device with that device current: the array's device
    // address (its name in host code is only a stand-in, not an address). The
    // cached address is valid for the life of the device's primary context;
    // after a cudaDeviceReset the process must not call this entry point again.
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      void* p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || !p)
        return pb_set_error(PB_ECUDA, "pb_layer_step_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      g_noalloc_ptr[dev] = p;
    }
    base = g_noalloc_ptr[dev];
  }
  char* p = reinterpret_cast<char*>(base);
  NoAllocBufs b;
  const size_t firstn = std::max((size_t)3 * m->H, (size_t)m->NH * m->HD + 2 * (size_t)m->NKV * m->HD + m->NH);
  b.res1 = reinterpret_cast<bf16_t*>(p); p += align256((size_t)m->H * 2);
  b.h_first = reinterpret_cast<bf16_t*>(p); p += align256(firstn * 2);
  b.h_attn = reinterpret_cast<bf16_t*>(p); p += align256((size_t)m->NH * m->HD * 2);
  b.h_mix = reinterpret_cast<bf16_t*>(p); p += align256((size_t)m->H * 2);
  b.h_u = reinterpret_cast<bf16_t*>(p); p += align256((size_t)m->F * 2);
  b.h_w2 = reinterpret_cast<bf16_t*>(p); p += align256((size_t)m->H * 2);
  b.ctl = reinterpret_cast<Ctl*>(p);
  cudaStream_t st = (cudaStream_t)stream;
  // the previous call's control block is stale: every field it reads is set here
  k_noalloc_set_ctl<<<1, 1, 0, st>>>(b.ctl, pos);
  PB_LAUNCHED("k_noalloc_set_ctl");
  const Layer& Ly = m->layers[layer];
  int rc;
  auto args = [&]() { StepArgs a = {}; a.H = m->H; a.eps = m->eps; a.ctl = b.ctl; a.convw = m->W; return a; };
  StepArgs a = args();
  a.pro = PRO_ADDNORM; a.xin = d_x; a.wnorm = Ly.op_norm; a.y = b.h_first;
  if ((rc = launch_step(Ly.first, EPI_BF16, a, st, false))) return rc;
  if (Ly.attn) {
    AttnArgs t;
    t.qkvg = b.h_first; t.qnorm = Ly.q_norm; t.knorm = Ly.k_norm;
    t.rope_cos = layer_cos(s, layer); t.rope_sin = layer_sin(s, layer);
    const size_t per = (size_t)s->max_ctx * m->NKV * m->HD;
    t.kc = s->kv + (size_t)Ly.attn_idx * 2 * per; t.vc = t.kc + per;
    t.out = b.h_attn; t.ctl = b.ctl;
    t.nh = m->NH; t.nkv = m->NKV; t.half = layer_half(m, layer); t.win = layer_win(m, layer); t.max_ctx = s->max_ctx;
    t.scaling = 1.0f / sqrtf((float)m->HD); t.eps = m->eps;
    const size_t sm = (size_t)s->max_ctx * sizeof(float);
    switch (m->HD) {
      case 32: cudaFuncSetAttribute(k_attn<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
               k_attn<1><<<m->NH, 256, sm, st>>>(t); break;
      case 64: cudaFuncSetAttribute(k_attn<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
               k_attn<2><<<m->NH, 256, sm, st>>>(t); break;
      case 128: cudaFuncSetAttribute(k_attn<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
                k_attn<4><<<m->NH, 256, sm, st>>>(t); break;
      default: return pb_set_error(PB_ENOTSUP, "attention head_dim %d", m->HD);
    }
    PB_LAUNCHED("k_attn");
    StepArgs o = args();
    o.pro = PRO_PLAIN; o.xin = b.h_attn; o.y = b.h_mix;
    if ((rc = launch_step(Ly.mix, EPI_BF16, o, st, false))) return rc;
  } else {
    StepArgs o = args();
    o.pro = PRO_CONV; o.xin = b.h_first; o.ring = s->ring + (size_t)Ly.conv_idx * m->W * m->H;
    o.taps = Ly.taps; o.y = b.h_mix;
    if ((rc = launch_step(Ly.mix, EPI_BF16, o, st, false))) return rc;
  }
  StepArgs c = args();
  c.pro = PRO_ADDNORM; c.xin = d_x; c.hin = b.h_mix; c.wpost = Ly.post_op_norm; c.wnorm = Ly.ffn_norm;
  c.rout = b.res1; c.y = b.h_u;
  if ((rc = launch_step(Ly.w13, EPI_SILU, c, st, false))) return rc;
  StepArgs d = args();
  d.pro = PRO_PLAIN; d.xin = b.h_u; d.y = b.h_w2;
  if ((rc = launch_step(Ly.w2, EPI_BF16, d, st, false))) return rc;
  StepArgs e = args();
  e.pro = PRO_ADDNORM; e.xin = b.res1; e.hin = b.h_w2; e.wpost = Ly.post_ffn_norm; e.wnorm = nullptr;
  e.rout = d_x; e.K = m->H;
  k_tail<<<1, 256, step_smem(m->H, m->H), st>>>(e);
  PB_LAUNCHED("k_tail");
  return PB_OK;
}

// ------------------------------------------------------------ chunked prefill
namespace {

int launch_b16_head_T(const pb_model* m, const bf16_t* x, float* lg, int T, cudaStream_t st) {
  const size_t smem = (size_t)32 * m->H * 2;
  int grid = pb_num_sms();
  if (grid > (m->V + 7) / 8) grid = (m->V + 7) / 8;
  const uint16_t* w = m->head16;
  switch (m->H) {
    case 256:
      PB_TRY_CUDA(cudaFuncSetAttribute(k_b16_head_T<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      k_b16_head_T<1><<<grid, 256, smem, st>>>(w, x, lg, m->V, T);
      break;
    case 512:
      PB_TRY_CUDA(cudaFuncSetAttribute(k_b16_head_T<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      k_b16_head_T<2><<<grid, 256, smem, st>>>(w, x, lg, m->V, T);
      break;
    case 1024:
      PB_TRY_CUDA(cudaFuncSetAttribute(k_b16_head_T<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      k_b16_head_T<4><<<grid, 256, smem, st>>>(w, x, lg, m->V, T);
      break;
    case 2048:
      PB_TRY_CUDA(cudaFuncSetAttribute(k_b16_head_T<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      k_b16_head_T<8><<<grid, 256, smem, st>>>(w, x, lg, m->V, T);
      break;
    default: return pb_set_error(PB_ENOTSUP, "bf16 head with hidden %d", m->H);
  }
  PB_LAUNCHED("k_b16_head_T");
  return PB_OK;
}

int prefill_prepare(pb_model* m, pb_state* s, int T, cudaStream_t st) {
  if (!m->tc_arena) {
    std::vector<const pb_q8*> src;
    for (auto& Ly : m->layers) { src.push_back(&Ly.first); src.push_back(&Ly.mix); src.push_back(&Ly.w13); src.push_back(&Ly.w2); }
    if (m->head.layout != PB_Q8_B16) src.push_back(&m->head);   // (a bf16 table is read as it is)
    size_t tot = 0;
    for (auto* w : src) tot += align256(pb_q80tc_bytes(w->N, w->K));
    if (cudaMalloc(&m->tc_arena, tot) != cudaSuccess) {
      cudaGetLastError();
      m->tc_arena = nullptr;
      return pb_set_error(PB_ENOMEM, "prefill: tensor-core weight copies (%zu bytes)", tot);
    }
    m->tc.assign(src.size(), pb_q8());
    size_t off = 0;
    for (size_t i = 0; i < src.size(); i++) {
      int rc = pb_q80tc_from_stream(src[i], m->tc_arena + off, &m->tc[i], st);
      if (rc) return rc;
      off += align256(pb_q80tc_bytes(src[i]->N, src[i]->K));
    }
  }
  if (s->pf_cap < T) {
    cudaFree(s->pf_mem);
    s->pf_mem = nullptr;
    s->pf_cap = 0;
    const int H = m->H, F = m->F;
    const int nq = m->NH * m->HD + 2 * m->NKV * m->HD + m->NH;
    const int kmax = std::max(H, std::max(F, m->NH * m->HD));
    int nmax = std::max(std::max(3 * H, nq), std::max(2 * F, H));
    const size_t sizes[] = {(size_t)T * H * 2, (size_t)T * kmax, (size_t)T * (kmax / 32) * 2, (size_t)T * nmax * 4,
                            (size_t)T * nq * 2, (size_t)T * m->NH * m->HD * 2, (size_t)T * m->V * 4, (size_t)T * 4,
                            (size_t)T * H * 2};
    size_t tot = 0;
    for (size_t x : sizes) tot += align256(x);
    if (cudaMalloc(&s->pf_mem, tot) != cudaSuccess) {
      cudaGetLastError();
      s->pf_mem = nullptr;
      return pb_set_error(PB_ENOMEM, "prefill: buffers");
    }
    void** slots[] = {(void**)&s->pf_R, (void**)&s->pf_qx, (void**)&s->pf_dx, (void**)&s->pf_y, (void**)&s->pf_qkvg,
                      (void**)&s->pf_att, (void**)&s->pf_logits, (void**)&s->pf_tok, (void**)&s->pf_R2};
    char* p = s->pf_mem;
    for (size_t i = 0; i < sizeof(sizes) / sizeof(sizes[0]); i++) { *slots[i] = p; p += align256(sizes[i]); }
    s->pf_cap = T;
  }
  return PB_OK;
}

int pf_norm(const pb_model* m, pb_state* s, int T, const int* tokens, const float* hin, const float* wpost,
            const float* wnorm, cudaStream_t st, bf16_t* xout = nullptr) {
  PfNormArgs a = {};
  a.xout = xout;
  a.tokens = tokens;
  a.emb_codes = reinterpret_cast<const uint4*>(m->head.codes);
  a.emb_scales = m->head.scales;
  a.emb_nch = m->head.nch;
  a.emb_f32 = m->head.sdt == PB_DT_F32;
  a.emb16 = m->head.layout == PB_Q8_B16 ? m->head16 : nullptr;
  a.rin = s->pf_R;
  a.hin = hin;
  a.wpost = wpost;
  a.wnorm = wnorm;
  a.rout = s->pf_R;
  a.qx = s->pf_qx;
  a.dx = s->pf_dx;
  a.H = m->H;
  a.eps = m->eps;
  k_pf_norm_quant<8><<<T, 256, 0, st>>>(a);
  PB_LAUNCHED("k_pf_norm_quant");
  return PB_OK;
}

}  // namespace

// The chunked prefill on the integer path (see pb_prefill.cuh): T prompt
// tokens (device int32, T a multiple of 16, at most 256) at positions
// pos0 .. pos0+T-1 through every layer, the KV caches and conv rings updated
// as T decode steps would update them. d_ids (optional, int32 [T]) receives
// each position's greedy id, d_logits (optional, fp32 [T][vocab]) the logits.
// Compiled for the LFM3 2B shape (hidden 2048, head_dim 64, conv width 3).
extern "C" int pb_prefill_chunk(pb_model* m, pb_state* s, const int* d_tokens, int T, int pos0, int* d_ids,
                                float* d_logits, void* stream) {
  if (!m || !s || !d_tokens || T <= 0) return pb_set_error(PB_EINVAL, "pb_prefill_chunk: bad argument");
  if (T % 16 || T > 256) return pb_set_error(PB_ENOTSUP, "pb_prefill_chunk: T=%d (a multiple of 16, at most 256)", T);
  if (pos0 < 0 || pos0 + T > s->max_ctx) return pb_set_error(PB_EINVAL, "pb_prefill_chunk: positions beyond max_ctx");
  if (!chunk_shape(m)) return pb_set_error(PB_ENOTSUP, "pb_prefill_chunk: shape not compiled");
  if (!m->decode_ok) return pb_set_error(PB_ENOTSUP, "pb_prefill_chunk: needs every matrix in the streaming layout");
  PB_TRY_CUDA(cudaSetDevice(m->device));
  cudaStream_t st = (cudaStream_t)stream;
  int rc = prefill_prepare(m, s, T, st);
  if (rc) return rc;
  const int H = m->H, F = m->F;
  const int nq = m->NH * m->HD + 2 * m->NKV * m->HD + m->NH;
  const size_t per = (size_t)s->max_ctx * m->NKV * m->HD;
  for (int L = 0; L < m->L; L++) {
    const Layer& Ly = m->layers[L];
    const pb_q8* tc = &m->tc[(size_t)L * 4];
    if (L == 0) rc = pf_norm(m, s, T, d_tokens, nullptr, nullptr, Ly.op_norm, st);
    else rc = pf_norm(m, s, T, nullptr, s->pf_y, m->layers[L - 1].post_ffn_norm, Ly.op_norm, st);
    if (rc) return rc;
    if ((rc = pb_q80_gemm(&tc[0], T, s->pf_qx, s->pf_dx, s->pf_y, nullptr, st))) return rc;
    if (Ly.attn) {
      PfQkvArgs q = {};
      q.y = s->pf_y;
      q.qkvg = s->pf_qkvg;
      q.knorm = Ly.k_norm;
      q.rope_cos = layer_cos(s, L);
      q.rope_sin = layer_sin(s, L);
      q.kc = s->kv + (size_t)Ly.attn_idx * 2 * per;
      q.vc = q.kc + per;
      q.nq = nq; q.nh = m->NH; q.nkv = m->NKV; q.half = layer_half(m, L); q.pos0 = pos0; q.eps = m->eps;
      if (m->HD == 128) k_pf_qkv<4><<<T, 256, 0, st>>>(q);
      else k_pf_qkv<2><<<T, 256, 0, st>>>(q);
      PB_LAUNCHED("k_pf_qkv");
      AttnArgs a = attn_args(m, s, L);
      a.qkvg = s->pf_qkvg;
      a.out = s->pf_att;
      const size_t asm_b = (size_t)s->max_ctx * sizeof(float);
      if (m->HD == 128) {
        PB_TRY_CUDA(cudaFuncSetAttribute(k_pf_attn<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
        k_pf_attn<4><<<dim3(m->NH, T), 256, asm_b, st>>>(a, pos0, nq, m->NH * m->HD);
      } else {
        PB_TRY_CUDA(cudaFuncSetAttribute(k_pf_attn<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
        k_pf_attn<2><<<dim3(m->NH, T), 256, asm_b, st>>>(a, pos0, nq, m->NH * m->HD);
      }
      PB_LAUNCHED("k_pf_attn");
      k_pf_quant<8><<<T, 256, 0, st>>>(s->pf_att, m->NH * m->HD, s->pf_qx, s->pf_dx);
      PB_LAUNCHED("k_pf_quant");
    } else {
      PfConvArgs c = {};
      c.y = s->pf_y;
      c.ring = s->ring + (size_t)Ly.conv_idx * m->W * H;
      c.taps = Ly.taps;
      c.qx = s->pf_qx;
      c.dx = s->pf_dx;
      c.H = H;
      c.pos0 = pos0;
      if (m->W == 7) k_pf_conv_quant<8, 7><<<T, 256, 0, st>>>(c);
      else k_pf_conv_quant<8, 3><<<T, 256, 0, st>>>(c);
      PB_LAUNCHED("k_pf_conv_quant");
      k_pf_ring<<<dim3((H + 255) / 256, m->W), 256, 0, st>>>(s->pf_y, s->ring + (size_t)Ly.conv_idx * m->W * H,
                                                             H, m->W, T, pos0);
      PB_LAUNCHED("k_pf_ring");
    }
    if ((rc = pb_q80_gemm(&tc[1], T, s->pf_qx, s->pf_dx, s->pf_y, nullptr, st))) return rc;
    if ((rc = pf_norm(m, s, T, nullptr, s->pf_y, Ly.post_op_norm, Ly.ffn_norm, st))) return rc;
    if ((rc = pb_q80_gemm(&tc[2], T, s->pf_qx, s->pf_dx, s->pf_y, nullptr, st))) return rc;
    switch (F / 256) {
      case 8: k_pf_silu_quant<8><<<T, 256, 0, st>>>(s->pf_y, F, s->pf_qx, s->pf_dx); break;
      case 16: k_pf_silu_quant<16><<<T, 256, 0, st>>>(s->pf_y, F, s->pf_qx, s->pf_dx); break;
      default: k_pf_silu_quant<32><<<T, 256, 0, st>>>(s->pf_y, F, s->pf_qx, s->pf_dx); break;
    }
    PB_LAUNCHED("k_pf_silu_quant");
    if ((rc = pb_q80_gemm(&tc[3], T, s->pf_qx, s->pf_dx, s->pf_y, nullptr, st))) return rc;
  }
  float* lg = d_logits ? d_logits : s->pf_logits;
  if (m->head.layout == PB_Q8_B16) {
    // the bf16 head on each position's x (the float path's head: there is no
    // integer form of k_gemv_bf16)
    if ((rc = pf_norm(m, s, T, nullptr, s->pf_y, m->layers[m->L - 1].post_ffn_norm, m->final_norm, st, s->pf_R2))) return rc;
    if ((rc = launch_b16_head_T(m, s->pf_R2, lg, T, st))) return rc;
  } else {
    if ((rc = pf_norm(m, s, T, nullptr, s->pf_y, m->layers[m->L - 1].post_ffn_norm, m->final_norm, st))) return rc;
    if ((rc = pb_q80_gemm(&m->tc.back(), T, s->pf_qx, s->pf_dx, lg, nullptr, st))) return rc;
  }
  if (d_ids) {
    k_pf_argmax<<<T, PF_AM_T, 0, st>>>(lg, m->V, d_ids);
    PB_LAUNCHED("k_pf_argmax");
  }
  return PB_OK;
}


// ------------------------------------------------------------ batched decode
namespace {
struct BatchTable {
  std::mutex mu;
  std::vector<pb_state*> key;
  SeqPtrs* d = nullptr;
  size_t cap = 0;
};
BatchTable g_bt;
}  // namespace

// One decode step of B independent sequences (B a multiple of 16, at most
// 256), each at its own position, every projection (and the head) one
// integer-path GEMM on the tensor cores over the B sequences: the per
// sequence values equal the decode step's with the integer path (the
// oracle's integer mode). states: B states of model m (host array); d_tokens,
// d_pos: device int32 [B]; d_ids (device int32 [B]) receives the greedy ids,
// d_logits (optional, fp32 [B][vocab]) the logits. The states' caches and
// rings advance by one position each. Compiled for the LFM3 2B shape.
extern "C" int pb_decode_batch(pb_model* m, pb_state* const* states, int B, const int* d_tokens, const int* d_pos,
                               int* d_ids, float* d_logits, void* stream) {
  if (!m || !states || !d_tokens || !d_pos || !d_ids || B <= 0) return pb_set_error(PB_EINVAL, "pb_decode_batch: bad argument");
  if (B % 16 || B > 256) return pb_set_error(PB_ENOTSUP, "pb_decode_batch: B=%d (a multiple of 16, at most 256)", B);
  if (!chunk_shape(m)) return pb_set_error(PB_ENOTSUP, "pb_decode_batch: shape not compiled");
  if (!m->decode_ok) return pb_set_error(PB_ENOTSUP, "pb_decode_batch: needs every matrix in the streaming layout");
  int max_ctx = 0;
  for (int b = 0; b < B; b++) {
    if (!states[b] || states[b]->m != m) return pb_set_error(PB_EINVAL, "pb_decode_batch: state %d is not of this model", b);
    max_ctx = std::max(max_ctx, states[b]->max_ctx);
  }
  PB_TRY_CUDA(cudaSetDevice(m->device));
  cudaStream_t st = (cudaStream_t)stream;
  pb_state* ws = states[0];        // its prefill buffers are the step's workspace
  int rc = prefill_prepare(m, ws, B, st);
  if (rc) return rc;
  const SeqPtrs* seq = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_bt.mu);
    std::vector<pb_state*> key(states, states + B);
    if (key != g_bt.key) {
      std::vector<SeqPtrs> h(B);
      for (int b = 0; b < B; b++) {
        const pb_state* s = states[b];
        h[b].kv = s->kv; h[b].ring = s->ring; h[b].rope_cos = s->rope_cos; h[b].rope_sin = s->rope_sin;
        h[b].rope_cos_s = s->rope_cos_s; h[b].rope_sin_s = s->rope_sin_s;
        h[b].max_ctx = s->max_ctx; h[b]._pad = 0;
      }
      if (g_bt.cap < (size_t)B) {
        PB_TRY_CUDA(cudaDeviceSynchronize());   // the table may still be read by a step in flight
        cudaFree(g_bt.d);
        g_bt.d = nullptr;
        g_bt.cap = 0;
        if (cudaMalloc(&g_bt.d, 256 * sizeof(SeqPtrs)) != cudaSuccess) {
          cudaGetLastError();
          return pb_set_error(PB_ENOMEM, "pb_decode_batch: sequence table");
        }
        g_bt.cap = 256;
      } else {
        PB_TRY_CUDA(cudaStreamSynchronize(st));
      }
      PB_TRY_CUDA(cudaMemcpy(g_bt.d, h.data(), B * sizeof(SeqPtrs), cudaMemcpyHostToDevice));
      g_bt.key = key;
    }
    seq = g_bt.d;
  }
  const int H = m->H, F = m->F;
  const int nq = m->NH * m->HD + 2 * m->NKV * m->HD + m->NH;
  for (int L = 0; L < m->L; L++) {
    const Layer& Ly = m->layers[L];
    const pb_q8* tc = &m->tc[(size_t)L * 4];
    if (L == 0) rc = pf_norm(m, ws, B, d_tokens, nullptr, nullptr, Ly.op_norm, st);
    else rc = pf_norm(m, ws, B, nullptr, ws->pf_y, m->layers[L - 1].post_ffn_norm, Ly.op_norm, st);
    if (rc) return rc;
    if ((rc = pb_q80_gemm(&tc[0], B, ws->pf_qx, ws->pf_dx, ws->pf_y, nullptr, st))) return rc;
    if (Ly.attn) {
      BdArgs a = {};
      a.seq = seq;
      a.pos = d_pos;
      a.y = ws->pf_y;
      a.qkvg = ws->pf_qkvg;
      a.qnorm = Ly.q_norm;
      a.knorm = Ly.k_norm;
      a.att = ws->pf_att;
      a.attn_idx = Ly.attn_idx;
      a.nq = nq; a.nh = m->NH; a.nkv = m->NKV; a.half = layer_half(m, L); a.win = layer_win(m, L);
      a.slide = Ly.slide ? 1 : 0;
      a.eps = m->eps;
      a.scaling = 1.0f / sqrtf((float)m->HD);
      if (m->HD == 128) k_bd_qkv<4><<<B, 256, 0, st>>>(a);
      else k_bd_qkv<2><<<B, 256, 0, st>>>(a);
      PB_LAUNCHED("k_bd_qkv");
      if (m->HD == 128) {
        PB_TRY_CUDA(cudaFuncSetAttribute(k_bd_attn<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
        k_bd_attn<4><<<dim3(m->NH, B), 256, (size_t)max_ctx * sizeof(float), st>>>(a);
      } else {
        PB_TRY_CUDA(cudaFuncSetAttribute(k_bd_attn<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
        k_bd_attn<2><<<dim3(m->NH, B), 256, (size_t)max_ctx * sizeof(float), st>>>(a);
      }
      PB_LAUNCHED("k_bd_attn");
      k_pf_quant<8><<<B, 256, 0, st>>>(ws->pf_att, m->NH * m->HD, ws->pf_qx, ws->pf_dx);
      PB_LAUNCHED("k_pf_quant");
    } else {
      BdConvArgs c = {};
      c.seq = seq;
      c.pos = d_pos;
      c.y = ws->pf_y;
      c.taps = Ly.taps;
      c.conv_idx = Ly.conv_idx;
      c.H = H;
      c.qx = ws->pf_qx;
      c.dx = ws->pf_dx;
      if (m->W == 7) k_bd_conv_quant<8, 7><<<B, 256, 0, st>>>(c);
      else k_bd_conv_quant<8, 3><<<B, 256, 0, st>>>(c);
      PB_LAUNCHED("k_bd_conv_quant");
    }
    if ((rc = pb_q80_gemm(&tc[1], B, ws->pf_qx, ws->pf_dx, ws->pf_y, nullptr, st))) return rc;
    if ((rc = pf_norm(m, ws, B, nullptr, ws->pf_y, Ly.post_op_norm, Ly.ffn_norm, st))) return rc;
    if ((rc = pb_q80_gemm(&tc[2], B, ws->pf_qx, ws->pf_dx, ws->pf_y, nullptr, st))) return rc;
    switch (F / 256) {
      case 8: k_pf_silu_quant<8><<<B, 256, 0, st>>>(ws->pf_y, F, ws->pf_qx, ws->pf_dx); break;
      case 16: k_pf_silu_quant<16><<<B, 256, 0, st>>>(ws->pf_y, F, ws->pf_qx, ws->pf_dx); break;
      default: k_pf_silu_quant<32><<<B, 256, 0, st>>>(ws->pf_y, F, ws->pf_qx, ws->pf_dx); break;
    }
    PB_LAUNCHED("k_pf_silu_quant");
    if ((rc = pb_q80_gemm(&tc[3], B, ws->pf_qx, ws->pf_dx, ws->pf_y, nullptr, st))) return rc;
  }
  if (m->head.layout == PB_Q8_B16) {
    if ((rc = pf_norm(m, ws, B, nullptr, ws->pf_y, m->layers[m->L - 1].post_ffn_norm, m->final_norm, st, ws->pf_R2))) return rc;
  } else if ((rc = pf_norm(m, ws, B, nullptr, ws->pf_y, m->layers[m->L - 1].post_ffn_norm, m->final_norm, st))) {
    return rc;
  }
  float* lg = d_logits ? d_logits : ws->pf_logits;
  if (m->head.layout == PB_Q8_B16) {
    if ((rc = launch_b16_head_T(m, ws->pf_R2, lg, B, st))) return rc;
  } else if ((rc = pb_q80_gemm(&m->tc.back(), B, ws->pf_qx, ws->pf_dx, lg, nullptr, st))) {
    return rc;
  }
  k_pf_argmax<<<B, PF_AM_T, 0, st>>>(lg, m->V, d_ids);
  PB_LAUNCHED("k_pf_argmax");
  return PB_OK;
}
