// pb_q1.cu -- Q1_0 x Q8_K weight streaming on sm_100a, the Q8_K activation
// quantiser, and the Bonsai engine's host compat entry points.
//
// Arithmetic (pq1_host.c:99-120): per 128-weight group g of a row,
//   isum_g = sum_i (bit_i ? +q_i : -q_i)          exact int32
//   acc    = acc + (ws_g * db) * (float)isum_g      group order, no contraction
// with ws_g the group's fp16 scale (widened; -0 widens to +0 as pq1_h2f does)
// and db the Q8_K block scale of the 256 activations holding the group.
//
// Device form: isum_g = 2 P_g - A_g with A_g = sum_i q_i (from the activations
// alone) and P_g = sum_{bit_i = 1} q_i. P_g is computed with dp4a on 0/1 byte
// masks: for a 32-bit word w of weight bits, (w >> k) & 0x01010101 selects the
// weights at bit positions k, k+8, k+16, k+24, so the 32 activations of that
// word are staged in shared memory pre-permuted as words
// (q_k, q_{k+8}, q_{k+16}, q_{k+24}), k = 0..7.
#include "pb_common.cuh"
#include "pb_internal.h"
#include "pb_q8k.cuh"
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

// --------------------------------------------------------------- packing
// 18-byte blocks (fp16 scale, 16 sign bytes) -> bits [rows][K/32] u32 and
// scales [rows][K/128] fp16 (pq1_split_repack, pq1_host.c:78-97).
__global__ void k_q1_pack(const uint8_t* __restrict__ src, uint32_t* __restrict__ bits,
                          uint16_t* __restrict__ scales, int rows, int K) {
  const int nb = K / 128;
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;   // one block
  if (i >= (size_t)rows * nb) return;
  const uint8_t* b = src + i * 18;
  scales[i] = (uint16_t)(b[0] | (b[1] << 8));
#pragma unroll
  for (int w = 0; w < 4; w++)
    bits[i * 4 + w] = (uint32_t)b[2 + 4 * w] | ((uint32_t)b[3 + 4 * w] << 8) |
                      ((uint32_t)b[4 + 4 * w] << 16) | ((uint32_t)b[5 + 4 * w] << 24);
}

// ------------------------------------------------------- Q8_K quantiser
// One CTA (256 threads) per 256-value block (pb_q8k.cuh).
__global__ void __launch_bounds__(256) k_q8k_quantize(const float* __restrict__ x,
                                                      uint8_t* __restrict__ xq) {
  __shared__ Q8kScratch sc;
  const int b = blockIdx.x;
  pb_q8k_block256(x[(size_t)b * 256 + threadIdx.x], xq + (size_t)b * 292, sc);
}

// ------------------------------------------------------------ Q1 GEMV
// One warp per batch of Q1_R rows, lane l owns groups l, l+32, ... (GPL per
// lane); products (ws*db)*(float)isum go to a per-warp row buffer and lane r
// folds row r in group order. Every weight word of a batch is requested
// before any is used, and the next batch's words while this one computes.
// Activations staged once per CTA, permuted as described above, 528 bytes per
// group (512 + 16 of padding so that lanes on consecutive groups hit distinct
// banks).
#define PB_Q1_GSTRIDE 528
constexpr int Q1_R = 4;   // rows per warp batch
template <int GPL>
PB_DEV void q1_load(uint4 (&wv)[GPL][Q1_R], unsigned short (&hs)[GPL][Q1_R], const uint4* __restrict__ bits,
                    const uint16_t* __restrict__ wsc, int row0, int rows, int ng, int lane) {
#pragma unroll
  for (int j = 0; j < GPL; j++) {
    const int g = lane + 32 * j;
    if (g < ng) {
#pragma unroll
      for (int r = 0; r < Q1_R; r++) {
        const int row = min(row0 + r, rows - 1);
        wv[j][r] = pb_ldg_stream(bits + (size_t)row * ng + g);
        hs[j][r] = wsc[(size_t)row * ng + g];
      }
    }
  }
}
template <int GPL>
__global__ void __launch_bounds__(256, GPL <= 2 ? 2 : 1)
k_q1_gemv(const uint4* __restrict__ bits, const uint16_t* __restrict__ wsc,
          const uint8_t* __restrict__ xq, float* __restrict__ y, int32_t* __restrict__ isum,
          int rows, int K) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int ng = K / 128, nbk = K / 256, ps = ng + 1;
  unsigned char* act = smem;                                         // ng * 528
  int* asum = reinterpret_cast<int*>(smem + (size_t)ng * PB_Q1_GSTRIDE);   // ng
  float* dbs = reinterpret_cast<float*>(asum + ng);                 // ng (db per group)
  float* prod = dbs + ng;                                           // 8 warps x Q1_R x (ng + 1)
  unsigned char* raw = reinterpret_cast<unsigned char*>(prod + (size_t)8 * Q1_R * ps);   // nbk * 292
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row_first = (blockIdx.x * 8 + warp) * Q1_R;
  const int stride = gridDim.x * 8 * Q1_R;
  uint4 wv[GPL][Q1_R];
  unsigned short hs[GPL][Q1_R];
  // the first weight words do not depend on the previous kernel: request them
  // before waiting on it (programmatic dependent launch; no-op otherwise)
  if (row_first < rows) q1_load<GPL>(wv, hs, bits, wsc, row_first, rows, ng, lane);
  pb_grid_wait();
  pb_grid_launch_dependents();
  // the Q8_K activation into shared memory once (coalesced words), then
  // permuted from there
  for (int i = threadIdx.x; i < nbk * 73; i += blockDim.x)
    reinterpret_cast<uint32_t*>(raw)[i] = reinterpret_cast<const uint32_t*>(xq)[i];
  __syncthreads();
  // thread per (group, word-of-32, k): words (q_k, q_k+8, q_k+16, q_k+24)
  for (int i = threadIdx.x; i < ng * 32; i += blockDim.x) {
    const int g = i >> 5, j = (i >> 3) & 3, k = i & 7;
    const unsigned char* qs = raw + (size_t)(g >> 1) * 292 + 4 + (g & 1) * 128 + j * 32;
    const uint32_t w = (uint32_t)qs[k] | ((uint32_t)qs[k + 8] << 8) | ((uint32_t)qs[k + 16] << 16) |
                       ((uint32_t)qs[k + 24] << 24);
    reinterpret_cast<uint32_t*>(act + (size_t)g * PB_Q1_GSTRIDE)[j * 8 + k] = w;
  }
  // A_g: the group's activation sum, 8 lanes per group (dp4a over 16 bytes each)
  // (the loop bound is a multiple of 32: whole warps take part in the shuffles)
  for (int i = threadIdx.x; i < ((ng * 8 + 31) & ~31); i += blockDim.x) {
    const int g = i >> 3, part = i & 7;
    const bool valid = g < ng;
    const unsigned char* qs = raw + (size_t)(valid ? g >> 1 : 0) * 292 + 4 + (g & 1) * 128 + part * 16;
    int sum = 0;
#pragma unroll
    for (int k = 0; valid && k < 4; k++) {
      const uint32_t w = (uint32_t)qs[4 * k] | ((uint32_t)qs[4 * k + 1] << 8) | ((uint32_t)qs[4 * k + 2] << 16) |
                         ((uint32_t)qs[4 * k + 3] << 24);
      sum = __dp4a((int)w, 0x01010101, sum);
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    if (valid && part == 0) {
      asum[g] = sum;
      float db;
      memcpy(&db, raw + (size_t)(g >> 1) * 292, 4);
      dbs[g] = db;
    }
  }
  __syncthreads();
  float* pw = prod + (size_t)warp * Q1_R * ps;
  for (int row0 = row_first; row0 < rows; row0 += stride) {
    uint4 cw[GPL][Q1_R];
    unsigned short ch[GPL][Q1_R];
#pragma unroll
    for (int j = 0; j < GPL; j++)
#pragma unroll
      for (int r = 0; r < Q1_R; r++) { cw[j][r] = wv[j][r]; ch[j][r] = hs[j][r]; }
    if (row0 + stride < rows) q1_load<GPL>(wv, hs, bits, wsc, row0 + stride, rows, ng, lane);
#pragma unroll
    for (int j = 0; j < GPL; j++) {
      const int g = lane + 32 * j;
      if (g >= ng) break;
      const uint4* av = reinterpret_cast<const uint4*>(act + (size_t)g * PB_Q1_GSTRIDE);
      int P[Q1_R];
#pragma unroll
      for (int r = 0; r < Q1_R; r++) P[r] = 0;
#pragma unroll
      for (int jj = 0; jj < 4; jj++) {
        const uint4 a0 = av[2 * jj], a1 = av[2 * jj + 1];
        const unsigned aw[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
        for (int r = 0; r < Q1_R; r++) {
          const unsigned ws = jj == 0 ? cw[j][r].x : jj == 1 ? cw[j][r].y : jj == 2 ? cw[j][r].z : cw[j][r].w;
#pragma unroll
          for (int k = 0; k < 8; k++) P[r] = __dp4a((int)((ws >> k) & 0x01010101u), (int)aw[k], P[r]);
        }
      }
      const int ag = asum[g];
      const float dbg = dbs[g];
#pragma unroll
      for (int r = 0; r < Q1_R; r++) {
        const int sm = 2 * P[r] - ag;
        if (isum && row0 + r < rows) isum[(size_t)(row0 + r) * ng + g] = sm;
        const float wsf = ch[j][r] == 0x8000u ? 0.0f : pb_h2f(ch[j][r]);
        pw[r * ps + g] = __fmul_rn(__fmul_rn(wsf, dbg), __int2float_rn(sm));
      }
    }
    __syncwarp();
    if (lane < Q1_R && row0 + lane < rows) {
      const float* pr = pw + lane * ps;
      float acc = 0.0f;
      for (int g = 0; g < ng; g++) acc = __fadd_rn(acc, pr[g]);
      y[row0 + lane] = acc;
    }
    __syncwarp();
  }
}

static size_t q1_smem(int K) {
  const int ng = K / 128;
  return (size_t)ng * PB_Q1_GSTRIDE + (size_t)ng * 4 * 2 + (size_t)8 * Q1_R * (ng + 1) * 4 +
         (size_t)(K / 256) * 292;
}

int pb_q1_gemv_launch(const pb_q1* w, const uint8_t* d_xq, float* d_y, int32_t* d_isum,
                      cudaStream_t st, bool pdl) {
  const size_t smem = q1_smem(w->K);
  if (smem > 220 * 1024) return pb_set_error(PB_ENOTSUP, "pb_q1_gemv: K=%d too large", w->K);
  const int gpl = (w->K / 128 + 31) / 32;
  if (gpl > 4) return pb_set_error(PB_ENOTSUP, "pb_q1_gemv: K=%d above 16384", w->K);
  void (*kern)(const uint4*, const uint16_t*, const uint8_t*, float*, int32_t*, int, int) =
      gpl == 1 ? k_q1_gemv<1> : gpl == 2 ? k_q1_gemv<2> : gpl == 3 ? k_q1_gemv<3> : k_q1_gemv<4>;
  static bool smem_set[64][4] = {};   // the attribute is per device and instance
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !smem_set[dev][gpl - 1]) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
    if (dev >= 0 && dev < 64) smem_set[dev][gpl - 1] = true;
  }
  // one resident wave: every CTA walks its row batches with the next batch's
  // words in flight
  static int occ[64][4] = {};
  if (dev >= 0 && dev < 64 && !occ[dev][gpl - 1]) {
    int n = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, 256, smem);
    occ[dev][gpl - 1] = n > 0 ? n : 1;
  }
  int grid = (dev >= 0 && dev < 64 ? occ[dev][gpl - 1] : 1) * pb_num_sms();
  if (grid * 8 * Q1_R > w->rows) grid = (w->rows + 8 * Q1_R - 1) / (8 * Q1_R);
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
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, reinterpret_cast<const uint4*>(w->bits),
                                     (const uint16_t*)w->scales, d_xq, d_y, d_isum, w->rows, w->K);
  if (e != cudaSuccess) return pb_set_error(PB_ECUDA, "launch k_q1_gemv: %s", cudaGetErrorString(e));
  pb_count_launch();
  return PB_OK;
}
static int q1_gemv_launch(const pb_q1* w, const uint8_t* d_xq, float* d_y, int32_t* d_isum,
                          cudaStream_t st) {
  return pb_q1_gemv_launch(w, d_xq, d_y, d_isum, st, false);
}

// ---------------------------------------------------------------- C ABI
extern "C" int pb_q1_pack(const uint8_t* blocks, int rows, int K, int src_on_device, void* stream,
                          pb_q1** out) {
  if (!out || !blocks) return pb_set_error(PB_EINVAL, "pb_q1_pack: null argument");
  *out = nullptr;
  if (rows <= 0 || K <= 0 || K % 256) return pb_set_error(PB_EINVAL, "pb_q1_pack: bad shape %dx%d", rows, K);
  cudaStream_t st = (cudaStream_t)stream;
  const size_t nblk = (size_t)rows * (K / 128), src_bytes = nblk * 18;
  pb_q1* w = new pb_q1();
  w->rows = rows; w->K = K;
  if (cudaMalloc(&w->bits, nblk * 16) != cudaSuccess || cudaMalloc(&w->scales, nblk * 2) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(w->bits); cudaFree(w->scales); delete w;
    return pb_set_error(PB_ENOMEM, "pb_q1_pack: cannot allocate");
  }
  const uint8_t* src = blocks;
  uint8_t* tmp = nullptr;
  int rc = PB_OK;
  if (!src_on_device) {
    if (cudaMalloc(&tmp, src_bytes) != cudaSuccess) { cudaGetLastError(); rc = pb_set_error(PB_ENOMEM, "pb_q1_pack: staging"); }
    else if (cudaMemcpyAsync(tmp, blocks, src_bytes, cudaMemcpyHostToDevice, st) != cudaSuccess)
      rc = pb_set_error(PB_ECUDA, "pb_q1_pack: upload");
    src = tmp;
  }
  if (rc == PB_OK) {
    k_q1_pack<<<(unsigned)((nblk + 255) / 256), 256, 0, st>>>(src, w->bits, w->scales, rows, K);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) rc = pb_set_error(PB_ECUDA, "launch k_q1_pack: %s", cudaGetErrorString(e));
    else pb_count_launch();
  }
  if (rc == PB_OK && cudaStreamSynchronize(st) != cudaSuccess)
    rc = pb_set_error(PB_ECUDA, "pb_q1_pack: %s", cudaGetErrorString(cudaGetLastError()));
  cudaFree(tmp);
  if (rc != PB_OK) { cudaFree(w->bits); cudaFree(w->scales); delete w; return rc; }
  *out = w;
  return PB_OK;
}

// device Q1_0 blocks of `rows` rows into w's storage from row row0 on (the
// merged tensors of the Bonsai decoder are filled this way)
int pb_q1_pack_into(pb_q1* w, const uint8_t* d_blocks, int rows, int row0, cudaStream_t st) {
  if (row0 < 0 || row0 + rows > w->rows) return pb_set_error(PB_EINVAL, "pb_q1_pack_into: rows out of range");
  const size_t nblk = (size_t)rows * (w->K / 128);
  k_q1_pack<<<(unsigned)((nblk + 255) / 256), 256, 0, st>>>(d_blocks, w->bits + (size_t)row0 * (w->K / 32),
                                                           w->scales + (size_t)row0 * (w->K / 128), rows, w->K);
  PB_LAUNCHED("k_q1_pack");
  return PB_OK;
}

extern "C" int pb_q1_free(pb_q1* w) {
  if (!w) return PB_OK;
  if (w->owner) { cudaFree(w->bits); cudaFree(w->scales); }
  delete w;
  return PB_OK;
}

extern "C" int pb_q8k_quantize(const float* d_x, int K, uint8_t* d_xq, void* stream) {
  if (!d_x || !d_xq || K <= 0 || K % 256) return pb_set_error(PB_EINVAL, "pb_q8k_quantize: bad argument");
  k_q8k_quantize<<<K / 256, 256, 0, (cudaStream_t)stream>>>(d_x, d_xq);
  PB_LAUNCHED("k_q8k_quantize");
  return PB_OK;
}

extern "C" int pb_q1_gemv(const pb_q1* w, const uint8_t* d_xq, float* d_y, int32_t* d_isum, void* stream) {
  if (!w || !d_xq || !d_y) return pb_set_error(PB_EINVAL, "pb_q1_gemv: null argument");
  return q1_gemv_launch(w, d_xq, d_y, d_isum, (cudaStream_t)stream);
}

// ------------------------------------------------ host compat (Bonsai ABI)
// pq1_fwd8_shim.h:12-23 / pq1_fwd8_glue.c:549-620: the host weight pointer
// (with its shape) is the cache key; the first call packs and uploads it.
namespace {
struct Compat {
  std::mutex mu;
  std::map<std::tuple<const void*, int, int>, pb_q1*> cache;
  cudaStream_t st = nullptr;
  uint8_t* d_xq = nullptr; size_t xq_cap = 0;
  float* d_y = nullptr; size_t y_cap = 0;
  float* h_y = nullptr;
};
Compat& compat() { static Compat c; return c; }

int compat_ensure(Compat& c, size_t xq_bytes, size_t y_elems) {
  if (!c.st && cudaStreamCreateWithFlags(&c.st, cudaStreamNonBlocking) != cudaSuccess)
    return pb_set_error(PB_ECUDA, "compat: stream");
  if (xq_bytes > c.xq_cap) {
    cudaFree(c.d_xq); c.d_xq = nullptr; c.xq_cap = 0;
    if (cudaMalloc(&c.d_xq, xq_bytes) != cudaSuccess) return pb_set_error(PB_ENOMEM, "compat: xq");
    c.xq_cap = xq_bytes;
  }
  if (y_elems > c.y_cap) {
    cudaFree(c.d_y); cudaFreeHost(c.h_y); c.d_y = nullptr; c.h_y = nullptr; c.y_cap = 0;
    if (cudaMalloc(&c.d_y, y_elems * 4) != cudaSuccess || cudaMallocHost(&c.h_y, y_elems * 4) != cudaSuccess)
      return pb_set_error(PB_ENOMEM, "compat: y");
    c.y_cap = y_elems;
  }
  return PB_OK;
}
pb_q1* compat_tensor(Compat& c, const unsigned char* w, int rows, int cols) {
  auto key = std::make_tuple((const void*)w, rows, cols);
  auto it = c.cache.find(key);
  if (it != c.cache.end()) return it->second;
  pb_q1* t = nullptr;
  if (pb_q1_pack(w, rows, cols, 0, c.st, &t) != PB_OK) return nullptr;
  c.cache[key] = t;
  return t;
}
}  // namespace

extern "C" int pq1_pq1_compat_gemv_batch(const unsigned char* const* w, const int* rows, int n, int cols,
                                         float* const* ys, const unsigned char* xq) {
  if (!w || !rows || !ys || !xq || n <= 0 || cols <= 0 || cols % 256) return PB_EINVAL;
  Compat& c = compat();
  std::lock_guard<std::mutex> lk(c.mu);
  size_t tot = 0;
  for (int i = 0; i < n; i++) tot += (size_t)rows[i];
  const size_t xqb = (size_t)(cols / 256) * 292;
  if (compat_ensure(c, xqb, tot) != PB_OK) return PB_ECUDA;
  std::vector<pb_q1*> ts((size_t)n);
  for (int i = 0; i < n; i++) {
    ts[i] = compat_tensor(c, w[i], rows[i], cols);
    if (!ts[i]) return PB_ENOMEM;
  }
  if (cudaMemcpyAsync(c.d_xq, xq, xqb, cudaMemcpyHostToDevice, c.st) != cudaSuccess) return PB_ECUDA;
  size_t off = 0;
  for (int i = 0; i < n; i++) {
    if (q1_gemv_launch(ts[i], c.d_xq, c.d_y + off, nullptr, c.st) != PB_OK) return PB_ECUDA;
    off += (size_t)rows[i];
  }
  if (cudaMemcpyAsync(c.h_y, c.d_y, tot * 4, cudaMemcpyDeviceToHost, c.st) != cudaSuccess) return PB_ECUDA;
  if (cudaStreamSynchronize(c.st) != cudaSuccess) return PB_ECUDA;
  off = 0;
  for (int i = 0; i < n; i++) { memcpy(ys[i], c.h_y + off, (size_t)rows[i] * 4); off += (size_t)rows[i]; }
  return PB_OK;
}

extern "C" void pq1_pq1_compat_gemv(int rows, int cols, const unsigned char* w, const float* x, float* y,
                                    const unsigned char* xq) {
  (void)x;
  const unsigned char* const ws[1] = {w};
  const int rs[1] = {rows};
  float* const yv[1] = {y};
  if (pq1_pq1_compat_gemv_batch(ws, rs, 1, cols, yv, xq) != PB_OK) {
    // The reference's compat entry has no status; a failure leaves y as NaN
    // so that a caller comparing results cannot mistake it for an answer.
    for (int i = 0; i < rows; i++) y[i] = __builtin_nanf("");
  }
}
