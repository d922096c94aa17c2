/* pulsar_b200.h -- C ABI of the B200 (sm_100a) quantized weight-streaming path.
 *
 * Drop-in boundary for PULSAR-ASM's decode hot path. Reference interfaces each
 * entry point replaces are cited as file:line relative to the PULSAR-ASM root.
 *
 * Conventions
 *  - Every function returns int: 0 (PB_OK) or a negative PB_E* code. No exits,
 *    no printing; pb_last_error() returns the message of the calling thread's
 *    last failure.
 *  - Pointers named d_* are device pointers (cudaMalloc'd or equivalent) on the
 *    current device; h_* are host pointers. `stream` is a cudaStream_t passed as
 *    void* so that this header needs no CUDA include (NULL = legacy stream).
 *  - bf16 activations are passed as uint16_t bit patterns, fp16 as uint16_t.
 *  - The caller owns activations, outputs and streams; the library owns packed
 *    weights (pb_q8 / pb_q1 tensors), models and states.
 *  - Calls on one object are not thread-safe; distinct objects may be used
 *    from different host threads and streams.
 */
#ifndef PULSAR_B200_H
#define PULSAR_B200_H
#include <stddef.h>
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

#define PB_OK 0
#define PB_EINVAL (-1)    /* bad argument or shape */
#define PB_ENOMEM (-2)    /* device or host allocation failed */
#define PB_ECUDA (-3)     /* a CUDA call or launch failed */
#define PB_EIO (-4)       /* open/read failure or short read */
#define PB_ECRC (-5)      /* per-tensor CRC mismatch */
#define PB_EFORMAT (-6)   /* bad magic, malformed header or record */
#define PB_ENOTSUP (-8)   /* shape/dtype this build does not implement */

#define PB_DT_BF16 0
#define PB_DT_F32 1
#define PB_DT_F16 2

int pb_version(void);
int pb_last_error(char* buf, size_t n);
/* number of this library's kernel launches issued so far by the calling process */
uint64_t pb_launch_count(void);

/* ------------------------------------------------------------------ Q8 ---- *
 * Q8 tensor: int8 codes [N][K] row-major plus one scale per 32-code block,
 * fp16 (Q8_0, PB_DT_F16) or fp32 (.lfm3q8 dtype 1, PB_DT_F32). pb_q8_pack
 * copies it into the library's streaming layout (16-byte granules ordered so
 * that each warp load instruction is one contiguous 512-byte segment).
 * Replaces the loader's tiler, lfm3_nanode.cu:1359-1375 / :4510-4521.        */
typedef struct pb_q8 pb_q8;
int pb_q8_pack(const int8_t* codes, const void* scales, int scale_dtype, int N, int K,
               int src_on_device, void* stream, pb_q8** out);
int pb_q8_free(pb_q8* w);
int pb_q8_shape(const pb_q8* w, int* N, int* K);
/* y = W x, REF_FLOAT numerics: bf16 x, fp32 FMA chains in the reference's
 * 32-leaf tree order, K-chunks of 2048 summed ascending (a K that 2048 does
 * not divide is one chunk, pick() :1763-1768), output rounded to
 * bf16 (y_dtype PB_DT_BF16, the Linear) or kept fp32 (PB_DT_F32, the head).
 * Replaces gemv() lfm3_nanode.cu:1916-1966 (q8_partial + k_combine_bf) and
 * gemv_f() :3634-3664 (q8_partial + k_combine_f).                            */
int pb_q8_gemv(const pb_q8* w, const uint16_t* d_x, void* d_y, int y_dtype, void* stream);
/* T positions, x [T][K] position-major, y [T][N]: the values of the chunked
 * prefill pf_gemv_T (lfm3_nanode.cu:4840-4968), bit-identical per position.  */
int pb_q8_gemm(const pb_q8* w, int T, const uint16_t* d_x, void* d_y, int y_dtype,
               void* stream);

/* The certified arm's head over the bf16 tied table (blob dtype 3): logits[n]
 * = the 32 lane chains s = s + bf16(W[n][k]) * x[k] (k = l, l+32, ...;
 * product and sum rounded apart) combined by the shuffle-down tree, fp32 as
 * is. Replaces k_gemv_bf16 / lm_head_bf16, lfm3_nanode.cu:3517-3560. The table
 * is first re-laid (d_src [N][K] row-major bf16 -> d_dst, 16-byte aligned,
 * N*K*2 bytes; K a multiple of 256); pb_bf16_gemv takes the re-laid table,
 * K = 256, 512, 1024, 2048 or 4096. A .lfm3q8 model with a dtype-3 embedding uses the
 * same head inside every decode path.                                        */
int pb_bf16_relayout(const uint16_t* d_src, uint16_t* d_dst, int N, int K, void* stream);
int pb_bf16_gemv(const uint16_t* d_w, int N, int K, const uint16_t* d_x, float* d_y, void* stream);

/* Q8_0 x Q8_0 integer path. x (fp32) is quantised per 32-block to int8 codes
 * and fp16 scales (fwd35_ref.c:332-343); y[n] = sum_b (dw*dx)*(float)isum_b in
 * block order where isum_b is the exact int32 block dot (pq1_host.c:112-116
 * pattern). d_isum ([N][K/32] int32) is optional.                            */
int pb_q80_quantize(const float* d_x, int K, int8_t* d_qx, uint16_t* d_dx, void* stream);
int pb_q80_gemv(const pb_q8* w, const int8_t* d_qx, const uint16_t* d_dx, float* d_y,
                int32_t* d_isum, void* stream);

/* The integer path for T positions on the tensor cores (tcgen05.mma
 * kind::i8, int32 block dots in TMEM): the chunked prefill (T = 32,
 * pf_gemv_T's role, lfm3_nanode.cu:4840-4968) and batched decode (T = 64)
 * forms of pb_q80_gemv. pb_q80tc_pack lays a Q8 tensor (fp16 or fp32 block
 * scales, K % 256 == 0) out for it; pb_q80_gemm takes T (a multiple of 16,
 * at most 256) positions of quantised activations (qx [T][K] int8, dx [T][K/32] fp16, as
 * pb_q80_quantize writes them for a [T][K] array), writes y [T][N] fp32 and
 * optionally the exact block dots isum [T][N][K/32]. Per position the values
 * equal pb_q80_gemv's bit for bit. pb_q80_gemm_status synchronises `stream`
 * and reports a bounded wait inside the kernel that gave up.               */
int pb_q80tc_pack(const int8_t* codes, const void* scales, int scale_dtype, int N, int K,
                  int src_on_device, void* stream, pb_q8** out);
int pb_q80_gemm(const pb_q8* w, int T, const int8_t* d_qx, const uint16_t* d_dx, float* d_y,
                int32_t* d_isum, void* stream);
int pb_q80_gemm_status(void* stream);

/* ------------------------------------------------------------------ Q1 ---- *
 * Q1_0: 18-byte blocks per 128 weights along K, fp16 scale then 16 bytes of
 * LSB-first sign bits, bit 1 => +1 (pq1_wrap.h:24-35).                        */
typedef struct pb_q1 pb_q1;
/* replaces pq1_split_repack + arena upload (pq1_host.c:78-97,
 * pq1_fwd8_glue.c:562-620) */
int pb_q1_pack(const uint8_t* blocks, int rows, int K, int src_on_device, void* stream,
               pb_q1** out);
int pb_q1_free(pb_q1* w);
/* Q8_K activation quantiser, 292 bytes per 256 values (fwd8.c:67-139) */
int pb_q8k_quantize(const float* d_x, int K, uint8_t* d_xq, void* stream);
/* y = W xq: per 128-group exact int32 sum, acc += (ws*db)*(float)isum in group
 * order (pq1_gemv_cpu, pq1_host.c:99-120; device form pq1_gemv_hs,
 * pq1_swar_sm53.cu:924-1175). d_isum ([rows][K/128]) is optional.           */
int pb_q1_gemv(const pb_q1* w, const uint8_t* d_xq, float* d_y, int32_t* d_isum, void* stream);

/* The Bonsai engine's host ABI, same signatures and conventions
 * (pq1_fwd8_shim.h:12-23): host Q1_0 weights w (also the cache key, packed
 * and uploaded on first use), host Q8_K activation xq, host fp32 output y;
 * x is unused. The batch form returns 0 when it ran, nonzero when the caller
 * must fall back to the per-tensor call.                                     */
void pq1_pq1_compat_gemv(int rows, int cols, const unsigned char* w, const float* x, float* y,
                         const unsigned char* xq);
int pq1_pq1_compat_gemv_batch(const unsigned char* const* w, const int* rows, int n, int cols,
                              float* const* ys, const unsigned char* xq);

/* --------------------------------------------------------------- model ---- *
 * An LFM3-style backbone loaded from an .lfm3q8 blob (magic "LFM3Q8\1\0",
 * u32 header length, JSON header with cfg and tensor table, payloads; per
 * tensor CRC32). Tensor dtypes: 1 = Q8 codes + fp32 scales, 2 = fp32,
 * 3 = bf16 (rejected by this build: PB_ENOTSUP), 8 = Q8_0 codes + fp16
 * scales. Replaces load_blob
 * (lfm3_nanode.cu:1404-1733).                                                */
typedef struct pb_model pb_model;
typedef struct pb_state pb_state;
typedef struct {
  int hidden, inter, n_layers, n_heads, n_kv, head_dim, vocab, conv_w;
  int n_attn, sliding_window;
  float rope_theta, rope_partial, norm_eps;
  uint64_t weight_bytes;       /* bytes of weights streamed per decode token */
} pb_model_info;
/* device < 0: validate only (header, shapes, every payload CRC) without touching
 * a GPU; returns the status and leaves *out NULL. */
int pb_open(const char* blob_path, int device, pb_model** out);
int pb_close(pb_model* m);
int pb_model_get_info(const pb_model* m, pb_model_info* info);
/* index of a tensor by its blob name, or PB_EINVAL */
int pb_tensor_id(const pb_model* m, const char* name);
/* gemv(model, name, x, y) for a model holding Q4 / Q5 records (blob dtypes 6
 * / 7, lfm3_nanode.cu:1494-1501): pb_open then loads every 2-D Q8 / Q4 / Q5
 * matrix by itself (no fused decode arena; pb_state_create returns
 * PB_ENOTSUP), and this dispatches one by dtype as the reference's gemv()
 * does (lfm3_nanode.cu:1916-1922): y (bf16 [N]) = W x (x bf16 [K], 16-byte
 * aligned). PB_ENOTSUP for an all-Q8 model (its projections are fused for
 * the decode entry points). */
int pb_model_gemv(pb_model* m, int tensor_id, const uint16_t* d_x, uint16_t* d_y, void* stream);
/* KV cache (fp16, [layer][max_ctx][n_kv][head_dim]) and conv rings, zeroed */
int pb_state_create(pb_model* m, int max_ctx, pb_state** out);
int pb_state_destroy(pb_state* s);
int pb_state_reset(pb_state* s, void* stream);
/* one T=1 layer on the device residual x (bf16 [hidden], updated in place):
 * layer_body, lfm3_nanode.cu:3739-3856 */
int pb_layer_step(pb_model* m, pb_state* s, int layer, int pos, uint16_t* d_x, void* stream);
/* one token: embedding row, every layer, final norm, tied head, greedy id.
 * h_out_id (host, optional) receives the id after the call synchronises
 * `stream`; d_logits (fp32 [vocab], optional) receives the logits. */
int pb_decode_token(pb_model* m, pb_state* s, int token, int pos, int* h_out_id,
                    float* d_logits, void* stream);
/* n greedy steps on the device: step i feeds the previous id (the first feeds
 * `token`), at positions pos0..pos0+n-1, no host round trip (one persistent
 * kernel launch for all n tokens; one CUDA graph launch per token with
 * PB_DECODE_MODE=graph); d_ids (int32 [n]) receives the generated ids. */
int pb_decode_greedy(pb_model* m, pb_state* s, int token, int pos0, int n, int* d_ids,
                     void* stream);
/* teacher-forced prompt: step i feeds d_tokens[i] (device int32 [n]) at
 * position pos0+i, launched like pb_decode_greedy, no host round trip; d_ids
 * (optional, int32 [n]) receives the greedy prediction after each token.
 * The prompt feed of the reference's step loop (lfm3_nanode.cu:5828-6030). */
int pb_decode_prompt(pb_model* m, pb_state* s, const int* d_tokens, int n, int pos0, int* d_ids,
                     void* stream);
/* pb_layer_step for callers that cannot allocate device memory (a runtime
 * that owns every allocation through its own pool, or code that must not
 * allocate after start-up). This entry point has no counterpart in the
 * reference. It calls no cudaMalloc/cudaFree and no allocating routine: the
 * layer's intermediate activations live in one static device array of at most
 * 512 KB per GPU (held by every GPU that loads the library until exit); models
 * needing more scratch get PB_EINVAL. The first call on a device looks up that
 * array's device address, and the first use of the library's kernels may load
 * its module, which commits the array: make that first call (or any earlier
 * call into the library) in the caller's start-up phase, before any stream
 * capture. The looked-up address lasts for the life of the device's primary
 * context. All calls share the array, so calls that overlap on the GPU race:
 * serialise them on one stream. Row-sharded states (pb_state_shard) get
 * PB_ENOTSUP. Results are identical to pb_layer_step's. */
int pb_layer_step_noalloc(pb_model* m, pb_state* s, int layer, int pos, uint16_t* d_x,
                          void* stream);
/* chunked prefill on the integer path (the tensor-core GEMMs of pb_q80_gemm
 * for every projection): T prompt tokens (device int32, T a multiple of 16,
 * at most 256) at positions pos0 .. pos0+T-1 through every layer, updating
 * the KV caches and conv rings as T decode steps would. Each position's
 * values are those of the decode step with every projection (and the head)
 * on the Q8_0 integer path: activations quantised per 32-block, exact int32
 * block dots, in-order fp32 fold, bf16 outputs. d_ids (optional, int32 [T])
 * receives each position's greedy id, d_logits (optional, fp32 [T][vocab])
 * the logits. The first call builds tensor-core copies of the weights.
 * Replaces layer_chunk_T / prefill_e2e (lfm3_nanode.cu:4997-5162,
 * :5248-5313) in its integer form. */
int pb_prefill_chunk(pb_model* m, pb_state* s, const int* d_tokens, int T, int pos0, int* d_ids,
                     float* d_logits, void* stream);
/* one decode step of B independent sequences (B a multiple of 16, at most
 * 256; batched decode, the multi-stream form of the reference's step loop):
 * sequence b is states[b] (a host array of states of model m) at position
 * d_pos[b] fed d_tokens[b] (device int32 [B]). Every projection and the head
 * is one integer-path GEMM over the B sequences on the tensor cores; each
 * sequence's values are those of its own decode step on the integer path.
 * d_ids (device int32 [B]) receives the greedy ids, d_logits (optional,
 * fp32 [B][vocab]) the logits; each state's caches and rings advance by one
 * position. The step's scratch is states[0]'s prefill workspace. */
int pb_decode_batch(pb_model* m, pb_state* const* states, int B, const int* d_tokens, const int* d_pos,
                    int* d_ids, float* d_logits, void* stream);
/* synchronise `stream` and report a decode failure recorded on the device
 * (a bounded wait inside the decode kernel that gave up): PB_OK or PB_ECUDA */
int pb_state_status(pb_state* s, void* stream);
/* Row sharding of one sequence's decode over `world` GPUs (one process per
 * GPU, every rank holding the same model and calling the same decode entry
 * points in the same order): each GEMV computes the rank's rows [rank*N/world,
 * (rank+1)*N/world) and an in-place NCCL all-gather over NVLink completes the
 * output vector before the next kernel; the head's logits are gathered and a
 * global greedy argmax publishes the id. Results equal the unsharded decode
 * bit for bit (every row is computed whole on one rank). `id` is the
 * ncclUniqueId from pb_nccl_unique_id on rank 0, shared by the caller;
 * pb_state_shard is collective. NCCL is resolved at run time (libnccl.so.2).
 * The survey's row-sharded layout with per-layer all-gather (no reference
 * counterpart: the reference engine runs on one device). */
int pb_nccl_unique_id(void* out, size_t bytes);
int pb_state_shard(pb_state* s, int rank, int world, const void* id);
/* kernel launches per decode token: 1 on the persistent path (one launch
 * decodes any number of tokens), the CUDA graph's node count otherwise */
int pb_decode_kernels_per_token(pb_state* s);
/* measurement hook: mean ms of one of the decode step's fused GEMV kernels
 * launched alone (which: 0 first GEMV, 1 o/out_proj, 2 w1|w3, 3 w2, 4 head),
 * cycling over the layers' distinct weights, and its algorithmic bytes */
int pb_time_step_kernel(pb_model* m, pb_state* s, int which, int iters, float* ms, double* bytes,
                        void* stream);

/* ------------------------------------------------------- Bonsai decoder ---- *
 * The Q1_0 token step of pulsar_arm/bonsai2/fwd8.c (Qwen3-style dense GQA
 * layers, head_dim 128, f16 K/V cache): per layer rms -> q|k|v -> head norms +
 * YaRN rope -> f16 flash-attention decode in the fork's order (pq1_host.c:
 * 404-434) -> o -> rms -> gate|up -> silu(g)*u -> down; output norm, head,
 * greedy argmax. Replaces the device side of pq1_token_fused
 * (pq1_fwd8_shim.h:44-51, pq1_fwd8_glue.c:1530) with device-pointer calls.
 * Shapes: hidden and inter multiples of 256 (hidden <= 8192), n_heads even
 * and <= 128, n_heads/n_kv <= 8.                                              */
typedef struct pb_bonsai pb_bonsai;
typedef struct pb_bonsai_state pb_bonsai_state;
typedef struct {
  int hidden, inter, n_layers, n_heads, n_kv, vocab;
  float rope_factor;   /* YaRN factor (fwd8.c:51: 4) */
  int rope_orig_ctx;   /* YaRN original context (fwd8.c:56: 16384 for the 8B) */
  float rope_base;     /* fwd8.c:57: 1e6 for the 8B */
  float attn_scale;    /* fwd8.c:566: 0.0883883476 */
} pb_bonsai_cfg;
/* tensor slots: the 7 per-layer tensors in pq1_token_fused's wt order, then
 * the layer -1 tensors (token_embd; output.weight, absent = tied) */
enum { PB_BS_Q = 0, PB_BS_K, PB_BS_V, PB_BS_O, PB_BS_GATE, PB_BS_UP, PB_BS_DOWN,
       PB_BS_EMBED = 16, PB_BS_HEAD = 17 };
/* norm slots in pq1_token_fused's nw order, then output_norm (layer -1) */
enum { PB_BS_ATTN_NORM = 0, PB_BS_FFN_NORM, PB_BS_Q_NORM, PB_BS_K_NORM, PB_BS_OUT_NORM = 16 };
int pb_bonsai_create(const pb_bonsai_cfg* cfg, int device, pb_bonsai** out);
int pb_bonsai_destroy(pb_bonsai* m);
/* Q1_0 18-byte blocks [rows][K/128] (GGUF layout, pq1_wrap.h:24-26) of one
 * tensor; q|k|v and gate|up are merged into one matrix each on the device */
int pb_bonsai_set_q1(pb_bonsai* m, int layer, int slot, const uint8_t* blocks, int src_on_device,
                     void* stream);
/* fp32 norm weights: hidden values (attn, ffn, output) or 128 (q, k) */
int pb_bonsai_set_norm(pb_bonsai* m, int layer, int slot, const float* w, int src_on_device,
                       void* stream);
/* per sequence: K/V cache [layer][K|V][n_kv][max_ctx][128] f16 and the rope
 * table of every position (max_ctx a multiple of 32, <= 8192) */
int pb_bonsai_state_create(pb_bonsai* m, int max_ctx, pb_bonsai_state** out);
/* a state whose K/V cache is TurboQuant-coded (kv_bits 3, 4 or 43; 0 is the
 * f16 cache of pb_bonsai_state_create): every position's post-rope K/V rows
 * are coded as they are stored and the attention runs over the codes
 * (pb_tq_store / pb_tq_attention inside the token's graph). The reference's
 * glue does this by default (PQ1_KVTQ=4, pq1_fwd8_glue.c:211-232). Needs
 * n_heads = 4 n_kv (PB_ENOTSUP otherwise). */
int pb_bonsai_state_create_tq(pb_bonsai* m, int max_ctx, int kv_bits, pb_bonsai_state** out);
int pb_bonsai_state_destroy(pb_bonsai_state* s);
/* device address of one layer's K (which 0) or V (which 1) cache [n_kv][max_ctx][128] */
int pb_bonsai_state_kv(pb_bonsai_state* s, int layer, int which, void** d_ptr);
/* copy the residual stream after the last step (fp32 [hidden]) */
int pb_bonsai_state_residual(pb_bonsai_state* s, float* d_x, void* stream);
/* RMS norms that fell back to the serial double chain since creation */
int pb_bonsai_state_fallbacks(pb_bonsai_state* s, int* out);
/* synchronise `stream` and report a failure recorded on the device (a bounded
 * wait that gave up): PB_OK or PB_ECUDA */
int pb_bonsai_state_status(pb_bonsai_state* s, void* stream);
/* one token at position pos: the embedding row of `token`, or d_x (fp32
 * [hidden], the caller's row, as pq1_token_fused receives it) when non-null.
 * d_logits (fp32 [vocab]) and out_id (host, synchronises) are optional. */
int pb_bonsai_decode(pb_bonsai* m, pb_bonsai_state* s, int token, int pos, const float* d_x,
                     float* d_logits, int* out_id, void* stream);
/* n greedy tokens from (token, pos), each step's id fed back on the device;
 * d_ids (int [n]) receives them; synchronises */
int pb_bonsai_decode_greedy(pb_bonsai* m, pb_bonsai_state* s, int token, int pos, int n, int* d_ids,
                            void* stream);

/* ---- low-bit backbone GEMV: Q4 / Q5 (blob dtypes 6 / 7) ------------------
 * pulsar_arm/asm/lfm3_qlow.cuh:1-113 (k_qlow + k_qlow_combine, dispatched by
 * qlow_gemv, lfm3_nanode.cu:1894-1915). codes / scales are the exporter's
 * tiled payload as the blob stores it (32-row tiles; per tile and 32-weight
 * group 32 x 16 bytes of nibbles, for Q5 then 32 x 4 bytes of high-bit
 * planes; scales 32 x half2 (128 d, mn) per tile and group): N*K/32*16 (Q4)
 * or *20 (Q5) code bytes and N*K/32*4 scale bytes; N % 32 == 0, K % 256 ==
 * 0. pb_qlow_gemv: y (bf16 [N]) = W x (x bf16 [K]) with the reference's
 * arithmetic bit for bit (K slices of 2, 4 from K = 4096, added in order).
 * pb_qlow_gemm: T positions (x [T][K], y [T][N]), each position's values
 * those of pb_qlow_gemv (the prefill's per-position loop, :4847). x must be
 * 16-byte aligned, and x and y must not overlap. */
typedef struct pb_qlow pb_qlow;
int pb_qlow_pack(const void* codes, const void* scales, int bits, int N, int K, int src_on_device, void* stream,
                 pb_qlow** out);
int pb_qlow_free(pb_qlow* w);
int pb_qlow_gemv(const pb_qlow* w, const uint16_t* d_x, uint16_t* d_y, void* stream);
int pb_qlow_gemm(const pb_qlow* w, int T, const uint16_t* d_x, uint16_t* d_y, void* stream);
/* synchronise `stream` and report a failure recorded on the device (a
 * bounded wait for the streamed weights that gave up): PB_OK or PB_ECUDA */
int pb_qlow_status(const pb_qlow* w, void* stream);

/* ---- TurboQuant K/V cache (pulsar_arm/bonsai2/pq1_swar_sm53.cu:3264-3990;
 * PQ1_KVTQ, pq1_fwd8_glue.c:211-232, 4 bits by default there) ---------------
 * bits: 3 or 4 for K and V alike, 43 for 4-bit K with 3-bit V. A 128-value
 * f16 row becomes 12 (3-bit) or 16 (4-bit) uint32 code words and one fp32
 * scale (random-sign Hadamard rotation, Lloyd-Max levels of the d = 128
 * sphere marginal, s = |x| / |c|). Layout per layer: K codes
 * [n_kv][ctx][CW], K scales [n_kv][ctx], V alike; ctx is the position stride.
 * pb_tq_store: rows [2 n_kv][128] f16 (the n_kv K rows, then the V rows, post
 * rope) encoded at position npos (pq1_tq_store). pb_tq_attention: the query
 * heads q [4 n_kv][128] fp32 (post rope, 4 per KV head as in the reference)
 * over positions 0..T-1 -> atto [4 n_kv][128] fp32 (pq1_tq_qk2, pq1_tq_sm,
 * pq1_tq_pv2, pq1_tq_out: the same reductions, in the same orders; rsqrtf and
 * expf replaced by 1/sqrt and this library's expf); scratch of
 * pb_tq_scratch_bytes(n_kv, ctx) bytes, 16-byte aligned. Asynchronous. */
long long pb_tq_scratch_bytes(int nkv, int ctx);
int pb_tq_store(int bits, const uint16_t* d_rows, int npos, uint32_t* d_kcode, float* d_kscale, uint32_t* d_vcode,
                float* d_vscale, int nkv, int ctx, void* stream);
int pb_tq_attention(int bits, const float* d_q, const uint32_t* d_kcode, const float* d_kscale,
                    const uint32_t* d_vcode, const float* d_vscale, int nkv, int ctx, int T, float* d_atto,
                    void* d_scratch, void* stream);

/* ---- sampler: sample_topkpp + frand01 (pulsar_arm/bonsai2/fwd8.c:465-521) ----
 * for each of B rows of fp32 logits (row b at d_logits + b*ld, n values):
 * top-k (topk <= 0 or > 1024 means 1024; ties in the reference's order,
 * value descending then index ascending), min-p and top-p on the raw logits,
 * temperature last, softmax draw with the row's 64-bit LCG state d_rng[b]
 * (advanced once per draw). temp <= 0 is greedy (the first maximum, the state
 * untouched; d_rng may be null). d_ids[b] receives the id, or -1 for a row
 * holding a NaN. One launch for all rows; asynchronous on `stream`. The
 * exponentials are this library's expf (within about 1 ulp of the C
 * library's, which the reference uses); logf(minp) is the host's. */
int pb_sample_topkpp(const float* d_logits, int B, int n, long long ld, float temp, float topp, int topk,
                     float minp, unsigned long long* d_rng, int* d_ids, void* stream);

/* ---- the Bonsai host hooks of pulsar_arm/bonsai2/pq1_fwd8_shim.h:24-60 ----
 * (the reference implements them in pq1_fwd8_glue.c:235-246, :1483-1760):
 * fwd8.c built with that shim and linked against this library runs each
 * token on the device in one call. Weights and norms are fwd8's host arrays
 * (wt: q k v o gate up down per layer, then output.weight; nw: attn ffn q k
 * norms per layer, then output_norm), uploaded on first use and keyed by
 * their pointers; x is the token's fp32 embedding row, rcc/rcs the 64 cos /
 * sin values of position npos; head (fp32 [vocab]) receives the logits unless
 * pq1_head_need(0). pq1_token_fused returns 0 when the step ran and -1 when it
 * declines (the caller then runs its own path): no pq1_kv_shape, a shape the
 * decoder does not take, or npos not the next position of the session's
 * cache. pq1_head_top: the last step's greedy id and its logit, or -1.
 * pq1_sess_init(n) (before the first step, 1 <= n <= 64) gives n sessions
 * with their own caches and positions; pq1_sess_select picks the current one.
 * pq1_attn_kv_put: the K / V rows ([nkv][128] f16, post-rope) of layer il at
 * position npos that fwd8 computed on the host (it runs a sequence's first
 * token there), mirrored into the current session's cache; 0, or -1 when npos
 * is not that layer's next position.
 * pq1_attn_fused (layer il's attention block: q|k|v, head norms, rope, the
 * K/V rows stored at npos in the current session's cache, f16 attention over
 * positions 0..npos, attn_output; xq is fwd8's host Q8_K of attn_norm(x), ao
 * the host fp32 output) and pq1_ffn_fused (the FFN tail: gate|up, silu(g)*u,
 * its Q8_K, down; fo the host output): 0 when the block ran, -1 when it
 * declines (for attention: no pq1_kv_shape, or npos not the layer's next
 * position). Tensors are fwd8's host arrays, uploaded on first use and keyed
 * by pointer (pq1_fwd8_glue.c:1156-1235, :1376-1470). pq1_attn_dbg and
 * pq1_ffn_dbg_xq return the device's K/V rows, post-rope q and attention
 * output of the last attention block, and the Q8_K down activation of the
 * last FFN tail (fwd8's PQ1_ATT_CHECK / PQ1_FFN_CHECK). pb_pq1_hooks_reset
 * (no reference counterpart) frees every device object the hooks hold and
 * returns them to their initial state (no shape, one session). */
void pq1_kv_shape(int nl, int nkv, int ctx);
int pq1_token_fused(int nl, const unsigned char* const* wt, const float* const* nw, int nh, int nkv, int hid,
                    int inter, int vocab, int ctx, int npos, const float* rcc, const float* rcs, const float* x,
                    float* head);
void pq1_head_need(int need);
int pq1_head_top(float* val);
int pq1_sess_init(int n);
void pq1_sess_select(int s);
int pq1_attn_kv_put(int il, int nl, int nkv, int ctx, int npos, const uint16_t* k16, const uint16_t* v16);
int pq1_attn_fused(int il, const unsigned char* wq, const unsigned char* wk, const unsigned char* wv,
                   const unsigned char* wo, const float* qnw, const float* knw, int nh, int nkv, int hid, int ctx,
                   int npos, const float* rcc, const float* rcs, const unsigned char* xq, float* ao);
int pq1_ffn_fused(const unsigned char* wg, const unsigned char* wu, const unsigned char* wd, int inter, int hid,
                  const unsigned char* xq, float* fo);
void pq1_attn_dbg(int il, int npos, uint16_t* k16, uint16_t* v16, float* q, float* atto, int nh);
void pq1_ffn_dbg_xq(unsigned char* dst, unsigned long n);
int pb_pq1_hooks_reset(void);
/* the shim's host helpers (pq1_fwd8_shim.h:21-22, :64): silu(g)*u in place
 * on the host, lu[i] = (g * (1/(1+expf(-g)))) * lu[i] with the C library's
 * expf, every operation rounded (pq1_host.c:196-227); and the GPU memory
 * report fwd8 prints under PQ1_STATS=1 */
void pq1_silu_mul(float* lu, const float* lg, int n);
const char* pq1_gpu_stats_mb(char* buf, int n);

#ifdef __cplusplus
}
#endif
#endif
