// pb_qlow.cu -- the low-bit backbone GEMV: Q4 / Q5 weights (blob dtypes 6 / 7,
// pulsar_arm/asm/lfm3_qlow.cuh:1-113, records lfm3_nanode.cu:1494-1501,
// dispatch qlow_gemv :1894-1915) at one position, and the same for T positions
// with each 32-row tile's codes read once per P positions (the reference's
// prefill calls the one-position kernel per position, :4847).
//
// Format (the exporter's tiling, kept as the device layout): 32-row tiles;
// per tile and 32-weight group g, 32 uint4 (lane = row: byte b of word i
// holds weight 8i+b in its low nibble and 8i+4+b in its high nibble), for Q5
// then 32 uint32 high-bit planes (bit 8b+p = bit 4 of weight 4p+b); scales
// per tile and group 32 half2 (d' = 128 d, mn): w = d q + mn.
//
// Arithmetic, per row (identical to the reference's k_qlow + k_qlow_combine):
//   K splits into KS slices (2; 4 from K = 4096), each slice's groups chained
//   in order: per group the code q becomes the float 1 + q/128 (exact), four
//   fma chains a_b over weights b, b+4, ..., b+28 against x, acc = (a0 + a1) +
//   (a2 + a3), sx = the group's x summed in order from 0, and
//   y = fma(d', acc - sx, fma(mn, sx, y)); the slices' partials are added in
//   slice order to 0 and rounded to bf16.
// B200 layout of the work: one warp per (tile, slice), lane = row, the row's
// four chains run as two packed fma.rn.f32x2 chains (each half an fmaf); a
// CTA holds TW tiles x KS slices and combines the slices in shared memory in
// slice order (no second kernel, no scratch). x (and its group sums) for P
// positions is staged as fp32 in shared memory. A warp's codes and scales are
// one contiguous range, streamed by its lane 0 with 1-D TMA bulk copies (no
// multicast) through a ring of 4 stages of CG groups issued before x is
// staged; waits are time-bounded, the warp agrees on their outcome, and a
// give-up is reported through an error word (pb_qlow_status). (A layout with
// a row's four chains on four lanes gave 4x the warps but ran slower: the
// per-group gather, shuffles and fold cost more than the extra warps hid.)
#include "pb_internal.h"
#include "pb_common.cuh"

#include <cuda_fp16.h>

struct pb_qlow {
  int bits = 0, N = 0, K = 0;
  uint4* codes = nullptr;      // device, the exporter's tiled payload
  __half2* scales = nullptr;   // device
  int* err = nullptr;          // device: a bounded wait in the kernel gave up
};

namespace {

__host__ __device__ constexpr int ql_slices(int K) { return K >= 4096 ? 4 : 2; }

struct QlArgs {
  const uint4* q;
  const __half2* s;
  const uint16_t* x;   // [T][K] bf16
  uint16_t* y;         // [T][N] bf16
  int N, K, T;
  int* err;            // set when a bounded wait gave up
};

PB_DEV uint32_t ql_smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
PB_DEV unsigned long long ql_time() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
PB_DEV bool ql_try(uint64_t* b, unsigned parity) {
  uint32_t ok;
  asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
               : "=r"(ok) : "r"(ql_smem_u32(b)), "r"(parity) : "memory");
  return ok != 0;
}
// waits at most about a second for the stage's bytes: try_wait suspends in
// hardware for a while per attempt; the clock is read every 64 attempts
PB_DEV bool ql_wait(uint64_t* b, unsigned parity) {
  if (ql_try(b, parity)) return true;
  const unsigned long long t0 = ql_time();
  for (unsigned i = 1;; i++) {
    if (ql_try(b, parity)) return true;
    if ((i & 63u) == 0u && ql_time() - t0 > 1000000000ull) return false;
  }
}
PB_DEV void ql_issue(void* dst_c, const void* src_c, unsigned bc, void* dst_s, const void* src_s, unsigned bs,
                     uint64_t* bar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(ql_smem_u32(bar)), "r"(bc + bs)
               : "memory");
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(ql_smem_u32(dst_c)), "l"(src_c), "r"(bc), "r"(ql_smem_u32(bar)) : "memory");
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(ql_smem_u32(dst_s)), "l"(src_s), "r"(bs), "r"(ql_smem_u32(bar)) : "memory");
}

template <int B, int CG, int NS>
struct QlGeo {
  static constexpr int GW = B == 4 ? 32 : 40;   // uint4 slots per (tile, group)
  static constexpr int REC = GW * 16;           // code bytes per (tile, group)
  static constexpr int SC = CG * REC;           // code bytes per stage
  static constexpr int SS = CG * 128;           // scale bytes per stage
  static constexpr int S = NS;                  // stages per warp
  static constexpr int WARP = S * (SC + SS) + 64;   // ring + barriers, per warp
};

typedef unsigned long long ql_f2;   // two floats in one 64-bit register pair
PB_DEV ql_f2 ql_pk(float a, float b) {
  ql_f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
PB_DEV void ql_upk(ql_f2 v, float& a, float& b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
// two independent fma.rn (one per half): the same bits as two fmaf
PB_DEV ql_f2 ql_fma2(ql_f2 a, ql_f2 b, ql_f2 c) {
  ql_f2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// the weights 8i+4hf+b (b = 0..3) of one group as the floats 1 + q/128,
// packed (b 0, 1) and (b 2, 3)
template <int B>
PB_DEV void ql_decode4(uint32_t word, uint32_t plane, int i, int hf, ql_f2& f01, ql_f2& f23) {
  uint32_t m = ((hf ? (word >> 4) : word) & 0x0F0F0F0Fu) | 0x80808080u;
  if (B == 5) {
    const int p = 2 * i + hf;   // bit 8b+p of the plane -> bit 4 of byte b
    const uint32_t hs = p <= 4 ? (plane << (4 - p)) : (plane >> (p - 4));
    m |= hs & 0x10101010u;
  }
  // byte b of m (0x80 | q) becomes byte 2 of 0x3F000000: 0x3F800000 | q << 16
  f01 = ql_pk(__uint_as_float(__byte_perm(m, 0x3F00u, 0x5044)), __uint_as_float(__byte_perm(m, 0x3F00u, 0x5144)));
  f23 = ql_pk(__uint_as_float(__byte_perm(m, 0x3F00u, 0x5244)), __uint_as_float(__byte_perm(m, 0x3F00u, 0x5344)));
}

// grid (ceil(N / (32 TW)), ceil(T / P)), block 32 * TW * KS threads: warp =
// (tile, slice), lane = row; its codes and scales are one contiguous range,
// streamed by lane 0 through S stages of CG groups
template <int B, int KS, int TW, int P, int CG, int NS>
__global__ void __launch_bounds__(32 * TW * KS) k_qlow_tile(QlArgs a) {
  using Geo = QlGeo<B, CG, NS>;
  extern __shared__ __align__(128) unsigned char ql_smem[];
  const int K = a.K, G = K / 32, GL = G / KS, N = a.N;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  unsigned char* ring = ql_smem + (size_t)w * Geo::WARP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + Geo::S * (Geo::SC + Geo::SS));
  float* xs = reinterpret_cast<float*>(ql_smem + (size_t)TW * KS * Geo::WARP);   // [P][K]
  float* sx = xs + (size_t)P * K;                                                   // [P][G]
  float* part = sx + (size_t)P * G;                                                 // [KS][TW][P][32]
  const int slice = w % KS, tl = w / KS;
  const int tile = blockIdx.x * TW + tl, row = tile * 32 + lane;
  const bool active = tile * 32 < N;
  const int g0 = slice * GL, nchunk = (GL + CG - 1) / CG;
  const unsigned char* csrc = reinterpret_cast<const unsigned char*>(a.q) + ((size_t)tile * G + g0) * Geo::REC;
  const unsigned char* ssrc = reinterpret_cast<const unsigned char*>(a.s) + ((size_t)tile * G + g0) * 128;
  auto issue = [&](int c) {
    const int ng = min(CG, GL - c * CG), sl = c % Geo::S;
    ql_issue(ring + (size_t)sl * Geo::SC, csrc + (size_t)c * Geo::SC, (unsigned)(ng * Geo::REC),
             ring + (size_t)Geo::S * Geo::SC + (size_t)sl * Geo::SS, ssrc + (size_t)c * Geo::SS,
             (unsigned)(ng * 128), &bars[sl]);
  };
  if (active && lane == 0) {
    for (int k = 0; k < Geo::S; k++)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(ql_smem_u32(&bars[k])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    for (int c = 0; c < Geo::S && c < nchunk; c++) issue(c);
  }
  // x (and its group sums) for the CTA's positions, while the weights stream in:
  // 8 bf16 per 16-byte load, a thread's loads issued before its stores
  const int p0 = blockIdx.y * P;
  {
    const int K8 = K / 8, n8 = P * K8;
    constexpr int U = 4;
    for (int j0 = tid; j0 < n8; j0 += U * blockDim.x) {
      uint4 v[U];
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int j = j0 + u * blockDim.x, p = j / K8;
        v[u] = (j < n8 && p0 + p < a.T)
                   ? *reinterpret_cast<const uint4*>(a.x + (size_t)(p0 + p) * K + (size_t)(j - p * K8) * 8)
                   : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < U; u++) {
        const int j = j0 + u * blockDim.x;
        if (j < n8) {
          const uint32_t wv[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
          float4* d = reinterpret_cast<float4*>(xs + (size_t)j * 8);
          d[0] = make_float4(__uint_as_float(wv[0] << 16), __uint_as_float(wv[0] & 0xFFFF0000u),
                             __uint_as_float(wv[1] << 16), __uint_as_float(wv[1] & 0xFFFF0000u));
          d[1] = make_float4(__uint_as_float(wv[2] << 16), __uint_as_float(wv[2] & 0xFFFF0000u),
                             __uint_as_float(wv[3] << 16), __uint_as_float(wv[3] & 0xFFFF0000u));
        }
      }
    }
  }
  __syncthreads();
  for (int i = tid; i < P * G; i += blockDim.x) {   // group sums in order from 0
    const float* xg = xs + (size_t)i * 32;
    float t = 0.0f;
#pragma unroll
    for (int k = 0; k < 32; k++) t = __fadd_rn(t, xg[k]);
    sx[i] = t;
  }
  __syncthreads();
  float yv[P];
#pragma unroll
  for (int p = 0; p < P; p++) yv[p] = 0.0f;
  if (active) {
    int failed = -1;
    for (int c = 0; c < nchunk; c++) {
      const int sl = c % Geo::S, ng = min(CG, GL - c * CG);
      // every lane waits (bounded) itself; the warp then agrees, so that its
      // lanes go on, or give up, together
      const bool ok = ql_wait(&bars[sl], (unsigned)(c / Geo::S) & 1u);
      if (!__all_sync(0xffffffffu, ok)) { failed = c; break; }
      const unsigned char* cbase = ring + (size_t)sl * Geo::SC;
      const unsigned char* sbase = ring + (size_t)Geo::S * Geo::SC + (size_t)sl * Geo::SS;
      // GB groups' sums are independent: compute them together, then fold y
      // through them in group order (the chain the reference runs)
      constexpr int GB = P == 1 ? 8 : 2;
      for (int gb = 0; gb < ng; gb += GB) {
        float accs[GB][P];
        float2 fds[GB];
#pragma unroll
        for (int u = 0; u < GB; u++) {
          const int gi = gb + u < ng ? gb + u : ng - 1;   // a short batch repeats its last group, unused
          const uint4 cw = *reinterpret_cast<const uint4*>(cbase + ((size_t)gi * Geo::GW + lane) * 16);
          const uint32_t ch = B == 5 ? *reinterpret_cast<const uint32_t*>(cbase + ((size_t)gi * Geo::GW + 32) * 16 + lane * 4) : 0u;
          fds[u] = __half22float2(*reinterpret_cast<const __half2*>(sbase + (size_t)gi * 128 + lane * 4));
          const uint32_t wd[4] = {cw.x, cw.y, cw.z, cw.w};
          ql_f2 a01[P], a23[P];
#pragma unroll
          for (int p = 0; p < P; p++) a01[p] = a23[p] = 0ull;
          const int gg = g0 + c * CG + gi;
#pragma unroll
          for (int i = 0; i < 4; i++) {
#pragma unroll
            for (int hf = 0; hf < 2; hf++) {
              ql_f2 f01, f23;
              ql_decode4<B>(wd[i], ch, i, hf, f01, f23);
#pragma unroll
              for (int p = 0; p < P; p++) {
                const ulonglong2 xv = *reinterpret_cast<const ulonglong2*>(xs + (size_t)p * K + gg * 32 + 8 * i + 4 * hf);
                a01[p] = ql_fma2(f01, xv.x, a01[p]);
                a23[p] = ql_fma2(f23, xv.y, a23[p]);
              }
            }
          }
#pragma unroll
          for (int p = 0; p < P; p++) {
            float a0, a1, a2, a3;
            ql_upk(a01[p], a0, a1);
            ql_upk(a23[p], a2, a3);
            accs[u][p] = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
          }
        }
#pragma unroll
        for (int u = 0; u < GB; u++) {
          if (gb + u < ng) {
            const int gg = g0 + c * CG + gb + u;
#pragma unroll
            for (int p = 0; p < P; p++) {
              const float sg = sx[(size_t)p * G + gg];
              yv[p] = __fmaf_rn(fds[u].x, __fsub_rn(accs[u][p], sg), __fmaf_rn(fds[u].y, sg, yv[p]));
            }
          }
        }
      }
      __syncwarp();   // every lane has read the slot: refill it
      if (lane == 0 && c + Geo::S < nchunk) issue(c + Geo::S);
    }
    if (failed >= 0 && lane == 0) {   // report, then let the copies in flight land (bounded) before leaving
      atomicExch(a.err, 1);
      for (int c = failed; c < min(nchunk, failed + Geo::S); c++) ql_wait(&bars[c % Geo::S], (unsigned)(c / Geo::S) & 1u);
    }
    __syncwarp();
  }
#pragma unroll
  for (int p = 0; p < P; p++) part[(((size_t)slice * TW + tl) * P + p) * 32 + lane] = yv[p];
  __syncthreads();
  if (slice == 0 && row < N) {
#pragma unroll
    for (int p = 0; p < P; p++) {
      if (p0 + p >= a.T) break;
      float v = 0.0f;
#pragma unroll
      for (int sl = 0; sl < KS; sl++) v = __fadd_rn(v, part[(((size_t)sl * TW + tl) * P + p) * 32 + lane]);
      // round to nearest even with no inf / NaN case, as the reference's combine rounds
      const uint32_t u = __float_as_uint(v);
      a.y[(size_t)(p0 + p) * N + row] = (uint16_t)((u + 0x7fffu + ((u >> 16) & 1u)) >> 16);
    }
  }
}

// Work shape: one tile per CTA (KS warps), the most CTAs for the fixed
// number of (tile, slice) chains the format allows, except for T positions
// with 2 slices (two tiles share the staged x). The ring: 4 stages of 8
// groups per warp (16 to 20 KB in flight) while the grid has few warps, 2
// stages of 4 groups once it has 8 or more per SM (occupancy then hides the
// latency; measured: 36.9 against 30.9 us for the reference's kernel at
// 65536 x 2048 with the deep ring).
template <int B, int KS, int P, int CG, int NS, int TW>
int launch_ql_geo(const pb_qlow* w, const uint16_t* x, uint16_t* y, int T, cudaStream_t st) {
  using Geo = QlGeo<B, CG, NS>;
  const int K = w->K, G = K / 32;
  const size_t smem = (size_t)TW * KS * Geo::WARP + ((size_t)P * K + (size_t)P * G + (size_t)KS * TW * P * 32) * 4;
  auto k = k_qlow_tile<B, KS, TW, P, CG, NS>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return pb_set_error(PB_ECUDA, "k_qlow_tile: shared memory %zu: %s", smem, cudaGetErrorString(e));
  QlArgs a{w->codes, w->scales, x, y, w->N, K, T, w->err};
  dim3 grid((unsigned)((w->N + 32 * TW - 1) / (32 * TW)), (unsigned)((T + P - 1) / P));
  k<<<grid, 32 * TW * KS, smem, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return pb_set_error(PB_ECUDA, "k_qlow_tile: %s", cudaGetErrorString(e));
  pb_count_launch();
  return PB_OK;
}

template <int B, int KS, int P>
int launch_ql(const pb_qlow* w, const uint16_t* x, uint16_t* y, int T, cudaStream_t st) {
  constexpr int TW = (P > 1 && KS == 2) ? 2 : 1;
  const bool wide = (long long)(w->N / 32) * KS >= 8LL * pb_num_sms();
  if (P == 1 && !wide) return launch_ql_geo<B, KS, P, 8, 4, TW>(w, x, y, T, st);
  return launch_ql_geo<B, KS, P, 4, 2, TW>(w, x, y, T, st);
}

template <int B, int P>
int launch_ql_ks(const pb_qlow* w, const uint16_t* x, uint16_t* y, int T, cudaStream_t st) {
  return ql_slices(w->K) == 4 ? launch_ql<B, 4, P>(w, x, y, T, st) : launch_ql<B, 2, P>(w, x, y, T, st);
}

template <int P>
int launch_ql_b(const pb_qlow* w, const uint16_t* x, uint16_t* y, int T, cudaStream_t st) {
  return w->bits == 5 ? launch_ql_ks<5, P>(w, x, y, T, st) : launch_ql_ks<4, P>(w, x, y, T, st);
}

bool overlaps(const void* a, size_t na, const void* b, size_t nb) {
  const char* pa = static_cast<const char*>(a);
  const char* pb = static_cast<const char*>(b);
  return pa < pb + nb && pb < pa + na;
}

}  // namespace

size_t pb_qlow_code_bytes(int bits, int N, int K) { return (size_t)N * K / 32 * (bits == 5 ? 20 : 16); }
size_t pb_qlow_scale_bytes(int N, int K) { return (size_t)N * K / 32 * 4; }

extern "C" int pb_qlow_pack(const void* codes, const void* scales, int bits, int N, int K, int src_on_device,
                            void* stream, pb_qlow** out) {
  if (!codes || !scales || !out) return pb_set_error(PB_EINVAL, "pb_qlow_pack: null argument");
  *out = nullptr;
  if ((bits != 4 && bits != 5) || N <= 0 || K <= 0 || N % 32 || K % 256)
    return pb_set_error(PB_EINVAL, "pb_qlow_pack: bits %d (4 or 5), N %d (multiple of 32), K %d (multiple of 256)",
                        bits, N, K);
  const size_t cb = pb_qlow_code_bytes(bits, N, K), sb = pb_qlow_scale_bytes(N, K);
  pb_qlow* w = new pb_qlow();
  w->bits = bits; w->N = N; w->K = K;
  if (cudaMalloc(&w->codes, cb) != cudaSuccess || cudaMalloc(&w->scales, sb) != cudaSuccess ||
      cudaMalloc(&w->err, sizeof(int)) != cudaSuccess || cudaMemset(w->err, 0, sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(w->codes);
    cudaFree(w->scales);
    cudaFree(w->err);
    delete w;
    return pb_set_error(PB_ENOMEM, "pb_qlow_pack: %zu bytes", cb + sb);
  }
  cudaStream_t st = (cudaStream_t)stream;
  const cudaMemcpyKind kind = src_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  if (cudaMemcpyAsync(w->codes, codes, cb, kind, st) != cudaSuccess ||
      cudaMemcpyAsync(w->scales, scales, sb, kind, st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(w->codes);
    cudaFree(w->scales);
    cudaFree(w->err);
    delete w;
    return pb_set_error(PB_ECUDA, "pb_qlow_pack: upload");
  }
  *out = w;
  return PB_OK;
}

extern "C" int pb_qlow_status(const pb_qlow* w, void* stream) {
  if (!w) return pb_set_error(PB_EINVAL, "pb_qlow_status: null argument");
  PB_TRY_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  int err = 0;
  PB_TRY_CUDA(cudaMemcpy(&err, w->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (err) return pb_set_error(PB_ECUDA, "k_qlow_tile: a bounded wait for streamed weights gave up");
  return PB_OK;
}

extern "C" int pb_qlow_free(pb_qlow* w) {
  if (!w) return PB_OK;
  cudaFree(w->codes);
  cudaFree(w->scales);
  cudaFree(w->err);
  delete w;
  return PB_OK;
}

extern "C" int pb_qlow_gemm(const pb_qlow* w, int T, const uint16_t* d_x, uint16_t* d_y, void* stream) {
  if (!w || !d_x || !d_y || T <= 0) return pb_set_error(PB_EINVAL, "pb_qlow_gemm: bad argument");
  if (overlaps(d_x, (size_t)T * w->K * 2, d_y, (size_t)T * w->N * 2))
    return pb_set_error(PB_EINVAL, "pb_qlow_gemm: x and y overlap");
  if (reinterpret_cast<uintptr_t>(d_x) & 15u)
    return pb_set_error(PB_EINVAL, "pb_qlow_gemm: x must be 16-byte aligned (it is read 8 values at a time)");
  cudaStream_t st = (cudaStream_t)stream;
  if (T == 1) return launch_ql_b<1>(w, d_x, d_y, 1, st);
  // positions per CTA: 4 while x for them fits next to the partials
  if ((size_t)4 * (w->K + w->K / 32) * 4 <= 160 * 1024) return launch_ql_b<4>(w, d_x, d_y, T, st);
  return launch_ql_b<2>(w, d_x, d_y, T, st);
}

extern "C" int pb_qlow_gemv(const pb_qlow* w, const uint16_t* d_x, uint16_t* d_y, void* stream) {
  return pb_qlow_gemm(w, 1, d_x, d_y, stream);
}
