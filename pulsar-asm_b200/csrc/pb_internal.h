// pb_internal.h -- host-side declarations shared by the library's translation
// units (not part of the public ABI; include/pulsar_b200.h is).
#pragma once
#include <cstdint>
#include <cstddef>
#include <cuda_runtime.h>
#include "../../include/pulsar_b200.h"

// thread-local last error (pb_last_error) and a process-wide launch counter
int pb_set_error(int code, const char* fmt, ...);
void pb_count_launch(uint64_t n = 1);
// while set on this thread, pb_count_launch ignores launches (graph capture)
void pb_set_capturing(bool on);

#define PB_TRY_CUDA(expr)                                                        \
  do {                                                                           \
    cudaError_t e__ = (expr);                                                    \
    if (e__ != cudaSuccess)                                                      \
      return pb_set_error(PB_ECUDA, "%s: %s (%s:%d)", #expr, cudaGetErrorString(e__), \
                          __FILE__, __LINE__);                                   \
  } while (0)

// after a <<<>>> launch: count it and surface launch-configuration errors
#define PB_LAUNCHED(name)                                                        \
  do {                                                                           \
    cudaError_t e__ = cudaGetLastError();                                        \
    if (e__ != cudaSuccess)                                                      \
      return pb_set_error(PB_ECUDA, "launch %s: %s", name, cudaGetErrorString(e__)); \
    pb_count_launch();                                                           \
  } while (0)

// Q8 tensor layouts
// PB_Q8_UMMA: 128-row tiles in the tensor cores' K-major 128-byte-swizzle order,
// fp32 scales [tile][block][128] (pb_q80tc_pack; only pb_q80_gemm reads it)
// PB_Q8_B16: the bf16 tied table (blob dtype 3) in the head layout
// (b16_index); codes points at it, no scales, nch = K / 1024 (2048-byte
// segments per row)
enum { PB_Q8_ROWMAJOR = 0, PB_Q8_STREAM = 1, PB_Q8_UMMA = 2, PB_Q8_B16 = 3 };

struct pb_q8 {
  int N = 0, K = 0;
  int sdt = PB_DT_F16;       // scale dtype: PB_DT_F16 or PB_DT_F32
  int layout = PB_Q8_ROWMAJOR;
  int nch = 1;               // 2048-code chunks per row (stream layout)
  int one = 0;               // stream layout of a K that is not a multiple of
                             // 2048: one chunk per row (the lane chains run on
                             // over the row's segments, one tree), codes and
                             // scales zero past K up to nch * 2048
  int8_t* codes = nullptr;   // device
  void* scales = nullptr;    // device
  bool owner = true;         // false: views into a model arena
};

struct pb_q1 {
  int rows = 0, K = 0;
  uint32_t* bits = nullptr;      // device, stream layout (see pb_q1.cu)
  uint16_t* scales = nullptr;    // device
  bool owner = true;
};

// streaming layout: 2048-code segments, chunks | 8. A K that is a multiple of
// 2048 reduces per 2048-code chunk; any other K (a multiple of 32) reduces as
// ONE chunk (pick(), lfm3_nanode.cu:1763-1768: KCHUNK = K unless 2048 divides
// K) and is padded with zero blocks to whole segments. 0: row-major layout.
inline int pb_q8_stream_chunks(int K, int* one) {
  if (K <= 0 || K % 32) return 0;
  const int n = (K + 2047) / 2048;
  if (!(n == 1 || n == 2 || n == 4 || n == 8)) return 0;
  if (one) *one = K % 2048 != 0;
  return n;
}
inline bool pb_q8_stream_ok(int K) { return pb_q8_stream_chunks(K, nullptr) > 0; }
// device bytes of a tensor's codes / scales in its layout
inline size_t pb_q8_code_bytes(int N, int K) {
  const int n = pb_q8_stream_chunks(K, nullptr);
  return n ? (size_t)N * n * 2048 : (size_t)N * K;
}
inline size_t pb_q8_layout_scale_bytes(int N, int K, int sdt) {
  const int n = pb_q8_stream_chunks(K, nullptr);
  return (size_t)N * (n ? n * 64 : K / 32) * (sdt == PB_DT_F32 ? 4 : 2);
}
inline size_t pb_q8_scale_bytes(int N, int K, int sdt) {
  return (size_t)N * (K / 32) * (sdt == PB_DT_F32 ? 4 : 2);
}

// pack src_rows row-major rows into caller-provided storage at destination
// rows r*rmul + radd (the model arena merges and interleaves tensors this way)
int pb_q8_pack_into(pb_q8* w, const int8_t* d_codes, const void* d_scales, cudaStream_t st,
                    int src_rows, int rmul, int radd);

// Bonsai state access for the host hooks (pb_pq1hooks.cpp)
int pb_bonsai_state_set_rope_row(pb_bonsai_state* s, int pos, const float* h_cos, const float* h_sin,
                                 cudaStream_t st);
const float* pb_bonsai_state_logits(const pb_bonsai_state* s);
// a state over a K/V cache the caller owns ([layer][2][n_kv][max_ctx][128]
// f16, not freed with the state)
int pb_bonsai_state_create_kv(pb_bonsai* m, int max_ctx, uint16_t* d_kv, pb_bonsai_state** out);
// a TurboQuant cache the caller owns: all layers' code words and scales
// ([layer][n_kv][max_ctx][CW], [layer][n_kv][max_ctx]); per layer, the same
// four pointers advanced to that layer
struct PbTqCache {
  uint32_t *kc = nullptr, *vc = nullptr;
  float *ks = nullptr, *vs = nullptr;
};
int pb_bonsai_state_create_tq_ext(pb_bonsai* m, int max_ctx, int kv_bits, const PbTqCache* cache,
                                  pb_bonsai_state** out);

// TurboQuant K/V cache (pb_tq.cu): bits 3, 4 or 43 (4-bit K, 3-bit V); the
// store takes the position from d_npos when it is non-null (graph replays)
size_t pb_tq_scratch_floats(int nkv, int ctx);
int pb_tq_store_launch(int bits, const uint16_t* d_rows, const int* d_npos, int npos, uint32_t* kc, float* ks,
                       uint32_t* vc, float* vs, int nkv, int ctx, cudaStream_t st, bool pdl);
// T positions, or (d_npos non-null) *d_npos + 1 read on the device
int pb_tq_attention_launch(int bits, const float* d_q, const uint32_t* kc, const float* ks, const uint32_t* vc,
                           const float* vs, int nkv, int ctx, int T, const int* d_npos, float* d_atto, float* d_scratch,
                           cudaStream_t st, bool pdl);
// per-layer TurboQuant cache sizes: code words per row and bytes per layer
inline int pb_tq_cw(int b) { return b == 3 ? 12 : 16; }
inline int pb_tq_bk(int bits) { return bits == 43 ? 4 : bits; }
inline int pb_tq_bv(int bits) { return bits == 43 ? 3 : bits; }

// one layer's attention block / FFN tail from the caller's host Q8_K
// activation, for fwd8.c's per-layer hooks (pb_bonsai.cu); blocking
struct pb_bs_blocks;
int pb_bs_blocks_create(int device, pb_bs_blocks** out);
void pb_bs_blocks_destroy(pb_bs_blocks* b);
int pb_bs_attn_block(pb_bs_blocks* b, const pb_q1* wq, const pb_q1* wk, const pb_q1* wv, const pb_q1* wo,
                     const float* d_qn, const float* d_kn, uint16_t* kc, uint16_t* vc, int max_ctx, int npos,
                     float attn_scale, const float* h_cos, const float* h_sin, const uint8_t* h_xq, float* h_ao,
                     cudaStream_t st);
int pb_bs_attn_block_tq(pb_bs_blocks* b, int bits, const pb_q1* wq, const pb_q1* wk, const pb_q1* wv, const pb_q1* wo,
                        const float* d_qn, const float* d_kn, const PbTqCache* layer, int max_ctx, int npos,
                        const float* h_cos, const float* h_sin, const uint8_t* h_xq, float* h_ao, cudaStream_t st);
int pb_bs_ffn_block(pb_bs_blocks* b, const pb_q1* wg, const pb_q1* wu, const pb_q1* wd, const uint8_t* h_xq,
                    float* h_fo, cudaStream_t st);
// the last attention block's post-rope q and attention output (fp32 [nh][128]);
// the last FFN tail's down activation (Q8_K blocks, at most n bytes)
int pb_bs_blocks_attn_debug(pb_bs_blocks* b, float* h_q, float* h_atto, int nh);
int pb_bs_blocks_ffn_xq(pb_bs_blocks* b, uint8_t* h_dst, size_t n);

// the bf16 tied table (blob dtype 3) re-laid for the head GEMV (pb_q8.cu)
int pb_b16_pack(const uint16_t* d_src, uint16_t* d_dst, int N, int K, cudaStream_t st);

// launch helpers used by the model's step (pdl: programmatic dependent launch)
int pb_q8_gemv_launch(const pb_q8* w, const uint16_t* d_x, void* d_y, int y_dtype,
                      cudaStream_t st);
int pb_num_sms();

// tensor-core (kind::i8) copies of streaming-layout tensors, for the
// chunked prefill: bytes of the copy, and the conversion into caller storage
size_t pb_q80tc_bytes(int N, int K);
int pb_q80tc_from_stream(const pb_q8* src, char* storage, pb_q8* out, cudaStream_t st);

// Q1_0 GEMV launch (pdl: programmatic dependent launch) and packing of device
// Q1_0 blocks into rows [row0, row0 + rows) of an allocated tensor
int pb_q1_gemv_launch(const pb_q1* w, const uint8_t* d_xq, float* d_y, int32_t* d_isum,
                      cudaStream_t st, bool pdl);
int pb_q1_pack_into(pb_q1* w, const uint8_t* d_blocks, int rows, int row0, cudaStream_t st);
