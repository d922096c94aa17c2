// pb_q80tc.cu -- the Q8_0 x Q8_0 integer path for T positions on the 5th
// generation tensor cores: tcgen05.mma kind::i8 with TMEM accumulators.
//
// y[t][n] = sum_b (dw[n][b] * dx[t][b]) * (float)isum[t][n][b], the sum in
// block order with no contraction, isum the exact int32 dot of one 32-code
// block (the I2 pattern of pq1_host.c:112-116, per position; the activation
// quantiser is fwd35_ref.c:332-343). One MMA of K = 32 bytes computes exactly
// one block's isum for a 128-row x T tile, so each block gets its own TMEM
// accumulator (no accumulation across blocks in the tensor core) and the
// epilogue warps fold the blocks in order in fp32.
//
// CTA = 6 warps, one 128-row tile of W and 16 of the T positions (grid
// tiles x T/16; the CTAs of one tile run side by side and share its weights
// in L2), two CTAs per SM:
//   warp 0  lane 0: TMA producer, 1-D bulk copies of each stage (8 blocks of
//                   weights, activations and their scales) into a ring of NS
//                   shared-memory stages (full/empty mbarriers);
//   warp 1  lane 0: MMA issuer, one tcgen05.mma (M 128, N 16, K 32) per block
//                   into one of NB TMEM buffers of 16 columns, tcgen05.commit
//                   to the buffer's mbarrier; warp 1 also allocates and frees
//                   the TMEM;
//   warps 2-5:      epilogue, TMEM lane quarter warp % 4: tcgen05.ld of BK
//                   blocks' int32 tiles at a time, release of the buffers,
//                   fp32 fold in block order (int32 -> fp32 by the exact
//                   2^23 + 2^22 exponent trick: |isum| < 2^22).
// Operands sit in shared memory in the canonical K-major no-swizzle layout:
// 8-row x 16-byte core matrices, the two 16-byte halves of a block 128 bytes
// apart (leading byte offset), 8-row groups 256 bytes apart (stride byte
// offset). The weights are stored that way in HBM at pack time and the
// activations are re-laid once per call, so every stage is four contiguous
// bulk copies. All waits are bounded; a wait that gives up records an error,
// every role leaves its loop, the issuer waits (bounded) for its MMAs and the
// producer for its copies, and the TMEM is freed before the CTA exits.
#include "pb_common.cuh"
#include "pb_internal.h"
#include <algorithm>
#include <mutex>

namespace {

constexpr int TC_M = 128;            // rows per tile (MMA M)
constexpr int TC_CB = 8;             // 32-code blocks per stage
constexpr unsigned TC_WAIT = 1u << 24;

struct TcArgs {
  const int8_t* a;     // weights [tile][block][16 groups][2 halves][8 rows][16 bytes]
  const float* dw;     // weight scales [tile][block][128]
  const int8_t* b;     // activations [block][T/8 groups][2 halves][8 rows][16 bytes]
  const float* dx;     // activation scales [block][T]
  float* y;            // [T][N]
  int32_t* isum;       // optional [T][N][K/32]
  int N, K, ns;
  int* err;
};

PB_DEV uint32_t s32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
PB_DEV void mb_init(uint64_t* b, unsigned c) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(s32(b)), "r"(c) : "memory");
}
PB_DEV void mb_expect(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s32(b)), "r"(bytes) : "memory");
}
PB_DEV void mb_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(s32(b)) : "memory");
}
PB_DEV bool mb_try(uint64_t* b, unsigned par) {
  uint32_t ok;
  asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
               : "=r"(ok) : "r"(s32(b)), "r"(par) : "memory");
  return ok != 0;
}
// bounded wait; false when it gave up or another role aborted
// (try_wait itself suspends the thread until the phase completes or a short
// hardware time limit passes, so the loop needs no sleep)
PB_DEV bool mb_wait(uint64_t* b, unsigned par, volatile int* abort_f) {
  for (unsigned i = 0; i < TC_WAIT; i++) {
    if (mb_try(b, par)) return true;
    if ((i & 255) == 255 && *abort_f) return false;
  }
  return false;
}
PB_DEV void bulk(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(s32(dst)), "l"(src), "r"(bytes), "r"(s32(bar)) : "memory");
}
// K-major, no swizzle: LBO 128 B between the block's two 16-byte halves,
// SBO 256 B between 8-row groups, descriptor version 1 (sm_100)
PB_DEV uint64_t umma_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) |
         (1ull << 46);
}
PB_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
PB_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
PB_DEV void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(s32(bar)) : "memory");
}
// D (int32, TMEM) = A (128 x 32 int8, smem) . B (T x 32 int8, smem)^T, no accumulation
PB_DEV void tc_mma_i8(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc) {
  const uint32_t z = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
      ::"r"(dtmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(z), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}
// 8 consecutive int32 columns of this thread's TMEM lane
PB_DEV void tc_ld8(uint32_t taddr, int32_t* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr));
}
PB_DEV void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

constexpr int TC_TS = 16;            // positions per CTA (MMA N)
constexpr int TC_NB = 16;            // TMEM buffers of 16 columns
constexpr int TC_BK = 4;             // blocks per epilogue step
constexpr int TC_SA = TC_M * 32 * TC_CB;       // weights of a stage
constexpr int TC_SB = TC_TS * 32 * TC_CB;      // activations
constexpr int TC_SW = TC_CB * TC_M * 4;        // weight scales
constexpr int TC_SX = TC_CB * TC_TS * 4;       // activation scales
constexpr int TC_STAGE = TC_SA + TC_SB + TC_SW + TC_SX;
constexpr int TC_NS = 2;

PB_DEV float i2f_exact(int32_t v) { return __fsub_rn(__int_as_float(v + 0x4B400000), 12582912.0f); }

__global__ void __launch_bounds__(192, 2) k_q80tc(TcArgs p) {
  extern __shared__ __align__(1024) unsigned char tsm[];
  __shared__ uint64_t full[TC_NS], empty[TC_NS], tfull[TC_NB], tempty[TC_NB], done;
  __shared__ uint32_t tbase;
  __shared__ int abort_f;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nblk = p.K / 32, nst = nblk / TC_CB, tile = blockIdx.x, ts = blockIdx.y;
  if (threadIdx.x == 0) {
    for (int i = 0; i < TC_NS; i++) { mb_init(&full[i], 1); mb_init(&empty[i], 1 + 4); }
    for (int i = 0; i < TC_NB; i++) { mb_init(&tfull[i], 1); mb_init(&tempty[i], 4); }
    mb_init(&done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    abort_f = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;" ::"r"(s32(&tbase)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tbase;
  const int8_t* bsrc = p.b + (size_t)ts * nblk * (TC_TS * 32);
  const float* xsrc = p.dx + (size_t)ts * nblk * TC_TS;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int s = 0; s < nst; s++) {
        const int slot = s % TC_NS;
        if (s >= TC_NS && !mb_wait(&empty[slot], (unsigned)((s / TC_NS) - 1) & 1u, &abort_f)) {
          abort_f = 1;
          atomicCAS(p.err, 0, 1);
          break;
        }
        unsigned char* st = tsm + (size_t)slot * TC_STAGE;
        mb_expect(&full[slot], TC_STAGE);
        bulk(st, p.a + ((size_t)tile * nblk + (size_t)s * TC_CB) * 4096, TC_SA, &full[slot]);
        bulk(st + TC_SA, bsrc + (size_t)s * TC_SB, TC_SB, &full[slot]);
        bulk(st + TC_SA + TC_SB, p.dw + ((size_t)tile * nblk + (size_t)s * TC_CB) * TC_M, TC_SW, &full[slot]);
        bulk(st + TC_SA + TC_SB + TC_SW, xsrc + (size_t)s * TC_CB * TC_TS, TC_SX, &full[slot]);
        issued = s + 1;
      }
      // no copy may land after the CTA exits: each slot's last issued stage (bounded)
      for (int s = issued > TC_NS ? issued - TC_NS : 0; s < issued; s++) {
        unsigned n = 0;
        while (!mb_try(&full[s % TC_NS], (unsigned)(s / TC_NS) & 1u) && n < TC_WAIT) { n++; if (n > 64) __nanosleep(32); }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // kind::i8: D s32 (bits 4-5 = 2), A and B signed (bits 7-9, 10-12 = 1),
      // both K-major, N = 16 (bits 17-22 = 16/8), M = 128 (bits 24-28 = 128/16)
      const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TC_TS >> 3) << 17) |
                             ((uint32_t)(TC_M >> 4) << 24);
      int b = 0;
      for (; b < nblk; b++) {
        const int s = b / TC_CB, j = b % TC_CB, slot = s % TC_NS, nb = b % TC_NB;
        if (j == 0 && !mb_wait(&full[slot], (unsigned)(s / TC_NS) & 1u, &abort_f)) break;
        if (b >= TC_NB && !mb_wait(&tempty[nb], (unsigned)((b / TC_NB) - 1) & 1u, &abort_f)) break;
        tc_fence_after();
        const uint32_t sa = s32(tsm + (size_t)slot * TC_STAGE) + j * (TC_M * 32);
        const uint32_t sb = s32(tsm + (size_t)slot * TC_STAGE + TC_SA) + j * (TC_TS * 32);
        tc_mma_i8(tmem + (uint32_t)(nb * TC_TS), umma_desc(sa), umma_desc(sb), idesc);
        tc_commit(&tfull[nb]);
        if (j == TC_CB - 1) tc_commit(&empty[slot]);
      }
      if (b < nblk) { abort_f = 1; atomicCAS(p.err, 0, 2); }
      // every MMA issued so far has completed before the TMEM is freed (bounded)
      tc_commit(&done);
      unsigned n = 0;
      while (!mb_try(&done, 0) && n < TC_WAIT) { n++; if (n > 64) __nanosleep(32); }
    }
  } else {
    const int q = warp & 3;                     // TMEM lane quarter of this warp
    const int rloc = q * 32 + lane;
    const int n = tile * TC_M + rloc;
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    float acc[TC_TS];
#pragma unroll
    for (int t = 0; t < TC_TS; t++) acc[t] = 0.0f;
    int b0 = 0;
    bool ok = true;
    for (; b0 < nblk && ok; b0 += TC_BK) {
      // TC_BK blocks per step: one wait for all their TMEM loads
#pragma unroll
      for (int k = 0; k < TC_BK; k++) {
        const int b = b0 + k, s = b / TC_CB, j = b % TC_CB, slot = s % TC_NS;
        // the stage's scales are visible once its copies completed
        if (j == 0 && !mb_wait(&full[slot], (unsigned)(s / TC_NS) & 1u, &abort_f)) { ok = false; break; }
        if (!mb_wait(&tfull[b % TC_NB], (unsigned)(b / TC_NB) & 1u, &abort_f)) { ok = false; break; }
      }
      if (!ok) break;
      tc_fence_after();
      int32_t v[TC_BK][TC_TS];
#pragma unroll
      for (int k = 0; k < TC_BK; k++) {
        const int nb = (b0 + k) % TC_NB;
        tc_ld8(tq + (uint32_t)(nb * TC_TS), &v[k][0]);
        tc_ld8(tq + (uint32_t)(nb * TC_TS + 8), &v[k][8]);
      }
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0)
        for (int k = 0; k < TC_BK; k++) mb_arrive(&tempty[(b0 + k) % TC_NB]);
#pragma unroll
      for (int k = 0; k < TC_BK; k++) {
        const int b = b0 + k, s = b / TC_CB, j = b % TC_CB, slot = s % TC_NS;
        const unsigned char* st = tsm + (size_t)slot * TC_STAGE;
        const float dwv = reinterpret_cast<const float*>(st + TC_SA + TC_SB)[j * TC_M + rloc];
        const float4* dx4 = reinterpret_cast<const float4*>(st + TC_SA + TC_SB + TC_SW) + j * (TC_TS / 4);
#pragma unroll
        for (int t4 = 0; t4 < TC_TS / 4; t4++) {
          const float4 d = dx4[t4];
          const float dd[4] = {d.x, d.y, d.z, d.w};
#pragma unroll
          for (int u = 0; u < 4; u++) {
            const int t = 4 * t4 + u;
            acc[t] = __fadd_rn(acc[t], __fmul_rn(__fmul_rn(dwv, dd[u]), i2f_exact(v[k][t])));
          }
        }
        if (p.isum && n < p.N) {
#pragma unroll
          for (int t = 0; t < TC_TS; t++) p.isum[((size_t)(ts * TC_TS + t) * p.N + n) * nblk + b] = v[k][t];
        }
        if (j == TC_CB - 1) {
          __syncwarp();
          if (lane == 0) mb_arrive(&empty[slot]);
        }
      }
    }
    if (b0 < nblk) { abort_f = 1; atomicCAS(p.err, 0, 3); }
    if (n < p.N) {
#pragma unroll
      for (int t = 0; t < TC_TS; t++) p.y[(size_t)(ts * TC_TS + t) * p.N + n] = acc[t];
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;" ::"r"(tmem));
}

// row-major codes/scales -> tiles of 128 rows in the K-major core-matrix
// order (rows >= N are zero); one thread per 16-byte (row, block, half)
template <typename S>
__global__ void k_q80tc_pack(const int8_t* __restrict__ codes, const S* __restrict__ scales, int N, int K,
                             int ntile, int8_t* __restrict__ a, float* __restrict__ dw) {
  const int nblk = K / 32;
  const size_t total = (size_t)ntile * TC_M * nblk * 2;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int kh = (int)(i & 1);
    const size_t rb = i >> 1;                 // (row, block), row fastest within a tile's block
    const int row = (int)(rb % TC_M);
    const size_t tb = rb / TC_M;              // tile * nblk + block
    const int b = (int)(tb % nblk);
    const int tile = (int)(tb / nblk);
    const int n = tile * TC_M + row;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (n < N) v = *reinterpret_cast<const uint4*>(codes + (size_t)n * K + b * 32 + kh * 16);
    int8_t* dst = a + tb * 4096 + (row >> 3) * 256 + kh * 128 + (row & 7) * 16;
    *reinterpret_cast<uint4*>(dst) = v;
    if (kh == 0) {
      float s = 0.0f;
      if (n < N) {
        if (sizeof(S) == 2) s = pb_h2f((unsigned short)scales[(size_t)n * nblk + b]);
        else s = (float)scales[(size_t)n * nblk + b];
      }
      dw[tb * TC_M + row] = s;
    }
  }
}

// the same tiles from a tensor in the streaming layout (pb_q8.cu): granule
// h*32 + l of segment (row, chunk) holds codes [16(h&1), +16) of block
// l + 32(h>>1) of the chunk; scales are pairs (s_l, s_{l+32}) per segment
template <typename S>
__global__ void k_q80tc_from_stream(const uint4* __restrict__ codes, const S* __restrict__ scales, int N, int K,
                                    int ntile, int8_t* __restrict__ a, float* __restrict__ dw) {
  const int nblk = K / 32, nch = K / 2048;
  const size_t total = (size_t)ntile * TC_M * nblk * 2;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int kh = (int)(i & 1);
    const size_t rb = i >> 1;
    const int row = (int)(rb % TC_M);
    const size_t tb = rb / TC_M;
    const int b = (int)(tb % nblk);
    const int tile = (int)(tb / nblk);
    const int n = tile * TC_M + row;
    const int c = b / 64, bl = b % 64, l = bl % 32, hb = bl / 32;
    uint4 v = make_uint4(0, 0, 0, 0);
    float sc = 0.0f;
    if (n < N) {
      const size_t seg = (size_t)n * nch + c;
      v = codes[seg * 128 + (hb * 2 + kh) * 32 + l];
      if (sizeof(S) == 2) sc = pb_h2f((unsigned short)scales[(seg * 32 + l) * 2 + hb]);
      else sc = (float)scales[(seg * 32 + l) * 2 + hb];
    }
    *reinterpret_cast<uint4*>(a + tb * 4096 + (row >> 3) * 256 + kh * 128 + (row & 7) * 16) = v;
    if (kh == 0) dw[tb * TC_M + row] = sc;
  }
}

// activations [T][K] int8 + fp16 scales [T][K/32] -> the kernel's layout:
// per 16 positions, per block, 2 groups of 8 positions x 2 halves x 16 bytes
__global__ void k_q80tc_act(const int8_t* __restrict__ qx, const uint16_t* __restrict__ dxh, int T, int K,
                            int8_t* __restrict__ bq, float* __restrict__ dx) {
  const int nblk = K / 32;
  const int total = nblk * T * 2;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int kh = i & 1, t = (i >> 1) % T, b = (i >> 1) / T;
    const int ts = t / TC_TS, tl = t % TC_TS;
    const size_t blk = (size_t)ts * nblk + b;
    const uint4 v = *reinterpret_cast<const uint4*>(qx + (size_t)t * K + b * 32 + kh * 16);
    *reinterpret_cast<uint4*>(bq + blk * (TC_TS * 32) + (tl >> 3) * 256 + kh * 128 + (tl & 7) * 16) = v;
    if (kh == 0) dx[blk * TC_TS + tl] = pb_h2f(dxh[(size_t)t * nblk + b]);
  }
}

int launch_tc(const pb_q8* w, int T, const int8_t* bq, const float* dx, float* y, int32_t* isum, int* err,
              cudaStream_t st) {
  const size_t smem = (size_t)TC_NS * TC_STAGE;
  PB_TRY_CUDA(cudaFuncSetAttribute(k_q80tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  TcArgs a;
  a.a = w->codes;
  a.dw = reinterpret_cast<const float*>(w->scales);
  a.b = bq;
  a.dx = dx;
  a.y = y;
  a.isum = isum;
  a.N = w->N;
  a.K = w->K;
  a.ns = TC_NS;
  a.err = err;
  const int ntile = (w->N + TC_M - 1) / TC_M;
  k_q80tc<<<dim3(ntile, T / TC_TS), 192, smem, st>>>(a);
  PB_LAUNCHED("k_q80tc");
  return PB_OK;
}

// per-device scratch of the activation re-layout and the error word, grown on demand
struct TcScratch {
  std::mutex mu;
  char* p[64] = {};
  size_t cap[64] = {};
};
TcScratch g_tc;

}  // namespace

extern "C" int pb_q80tc_pack(const int8_t* codes, const void* scales, int scale_dtype, int N, int K,
                             int src_on_device, void* stream, pb_q8** out) {
  if (!out || !codes || !scales) return pb_set_error(PB_EINVAL, "pb_q80tc_pack: null argument");
  *out = nullptr;
  if (N <= 0 || K <= 0 || K % (32 * TC_CB)) return pb_set_error(PB_EINVAL, "pb_q80tc_pack: bad shape %dx%d (K %% 256)", N, K);
  if (scale_dtype != PB_DT_F16 && scale_dtype != PB_DT_F32)
    return pb_set_error(PB_EINVAL, "pb_q80tc_pack: scale dtype %d", scale_dtype);
  cudaStream_t st = (cudaStream_t)stream;
  const int ntile = (N + TC_M - 1) / TC_M, nblk = K / 32;
  const size_t ab = (size_t)ntile * TC_M * K, wb = (size_t)ntile * TC_M * nblk * 4;
  const size_t cb = (size_t)N * K, sb = pb_q8_scale_bytes(N, K, scale_dtype);
  pb_q8* w = new pb_q8();
  w->N = N; w->K = K; w->sdt = scale_dtype; w->layout = PB_Q8_UMMA; w->nch = 1;
  if (cudaMalloc(&w->codes, ab) != cudaSuccess || cudaMalloc(&w->scales, wb) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(w->codes); cudaFree(w->scales); delete w;
    return pb_set_error(PB_ENOMEM, "pb_q80tc_pack: cannot allocate %zu bytes", ab + wb);
  }
  const int8_t* dc = codes;
  const void* ds = scales;
  int8_t* tc = nullptr; void* ts = nullptr;
  int rc = PB_OK;
  if (!src_on_device) {
    if (cudaMalloc(&tc, cb) != cudaSuccess || cudaMalloc(&ts, sb) != cudaSuccess) {
      cudaGetLastError();
      rc = pb_set_error(PB_ENOMEM, "pb_q80tc_pack: staging");
    } else if (cudaMemcpyAsync(tc, codes, cb, cudaMemcpyHostToDevice, st) != cudaSuccess ||
               cudaMemcpyAsync(ts, scales, sb, cudaMemcpyHostToDevice, st) != cudaSuccess) {
      rc = pb_set_error(PB_ECUDA, "pb_q80tc_pack: upload failed");
    }
    dc = tc; ds = ts;
  }
  if (rc == PB_OK) {
    const size_t units = (size_t)ntile * TC_M * nblk * 2;
    const int grid = (int)std::min<size_t>((units + 255) / 256, (size_t)pb_num_sms() * 16);
    if (scale_dtype == PB_DT_F16)
      k_q80tc_pack<unsigned short><<<grid, 256, 0, st>>>(dc, (const unsigned short*)ds, N, K, ntile, w->codes,
                                                         (float*)w->scales);
    else
      k_q80tc_pack<float><<<grid, 256, 0, st>>>(dc, (const float*)ds, N, K, ntile, w->codes, (float*)w->scales);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) rc = pb_set_error(PB_ECUDA, "launch k_q80tc_pack: %s", cudaGetErrorString(e));
    else pb_count_launch();
  }
  if (rc == PB_OK && cudaStreamSynchronize(st) != cudaSuccess)
    rc = pb_set_error(PB_ECUDA, "pb_q80tc_pack: %s", cudaGetErrorString(cudaGetLastError()));
  cudaFree(tc); cudaFree(ts);
  if (rc != PB_OK) { cudaFree(w->codes); cudaFree(w->scales); delete w; return rc; }
  *out = w;
  return PB_OK;
}

// a tensor-core copy of a tensor held in the streaming layout (the model's
// weights), into caller-provided storage of pb_q80tc_bytes() bytes
size_t pb_q80tc_bytes(int N, int K) {
  const size_t ntile = (size_t)(N + TC_M - 1) / TC_M;
  return ntile * TC_M * K + ntile * TC_M * (K / 32) * 4;
}
int pb_q80tc_from_stream(const pb_q8* src, char* storage, pb_q8* out, cudaStream_t st) {
  if (src->layout != PB_Q8_STREAM || src->K % (32 * TC_CB))
    return pb_set_error(PB_ENOTSUP, "tensor-core copy: needs the streaming layout");
  const int N = src->N, K = src->K, ntile = (N + TC_M - 1) / TC_M;
  out->N = N; out->K = K; out->sdt = src->sdt; out->layout = PB_Q8_UMMA; out->nch = 1; out->owner = false;
  out->codes = reinterpret_cast<int8_t*>(storage);
  out->scales = storage + (size_t)ntile * TC_M * K;
  const size_t units = (size_t)ntile * TC_M * (K / 32) * 2;
  const int grid = (int)std::min<size_t>((units + 255) / 256, (size_t)pb_num_sms() * 16);
  if (src->sdt == PB_DT_F32)
    k_q80tc_from_stream<float><<<grid, 256, 0, st>>>(reinterpret_cast<const uint4*>(src->codes),
                                                     (const float*)src->scales, N, K, ntile, out->codes,
                                                     (float*)out->scales);
  else
    k_q80tc_from_stream<unsigned short><<<grid, 256, 0, st>>>(reinterpret_cast<const uint4*>(src->codes),
                                                              (const unsigned short*)src->scales, N, K, ntile,
                                                              out->codes, (float*)out->scales);
  PB_LAUNCHED("k_q80tc_from_stream");
  return PB_OK;
}

extern "C" int pb_q80_gemm(const pb_q8* w, int T, const int8_t* d_qx, const uint16_t* d_dx, float* d_y,
                           int32_t* d_isum, void* stream) {
  if (!w || !d_qx || !d_dx || !d_y) return pb_set_error(PB_EINVAL, "pb_q80_gemm: null argument");
  if (w->layout != PB_Q8_UMMA) return pb_set_error(PB_EINVAL, "pb_q80_gemm: tensor not packed by pb_q80tc_pack");
  if (T <= 0 || T % TC_TS || T > 256)
    return pb_set_error(PB_ENOTSUP, "pb_q80_gemm: T=%d (a multiple of 16 up to 256)", T);
  if (((uintptr_t)d_qx & 15) != 0) return pb_set_error(PB_EINVAL, "pb_q80_gemm: qx must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  int dev = 0;
  PB_TRY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return pb_set_error(PB_ENOTSUP, "pb_q80_gemm: device %d", dev);
  const int nblk = w->K / 32;
  const size_t bqb = (size_t)T * w->K, dxb = (size_t)nblk * T * 4, need = 256 + bqb + dxb;
  std::lock_guard<std::mutex> lk(g_tc.mu);
  if (g_tc.cap[dev] < need) {
    // the scratch may still be read by work queued earlier on another stream
    PB_TRY_CUDA(cudaDeviceSynchronize());
    cudaFree(g_tc.p[dev]);
    g_tc.p[dev] = nullptr;
    g_tc.cap[dev] = 0;
    if (cudaMalloc(&g_tc.p[dev], need) != cudaSuccess) {
      cudaGetLastError();
      return pb_set_error(PB_ENOMEM, "pb_q80_gemm: scratch");
    }
    g_tc.cap[dev] = need;
    PB_TRY_CUDA(cudaMemset(g_tc.p[dev], 0, 256));
  }
  int* err = reinterpret_cast<int*>(g_tc.p[dev]);
  int8_t* bq = reinterpret_cast<int8_t*>(g_tc.p[dev] + 256);
  float* dx = reinterpret_cast<float*>(g_tc.p[dev] + 256 + bqb);
  const int units = nblk * T * 2;
  k_q80tc_act<<<(units + 255) / 256, 256, 0, st>>>(d_qx, d_dx, T, w->K, bq, dx);
  PB_LAUNCHED("k_q80tc_act");
  int rc = launch_tc(w, T, bq, dx, d_y, d_isum, err, st);
  return rc;
}

extern "C" int pb_q80_gemm_status(void* stream) {
  int dev = 0;
  PB_TRY_CUDA(cudaGetDevice(&dev));
  PB_TRY_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  int e = 0;
  {
    std::lock_guard<std::mutex> lk(g_tc.mu);
    if (dev < 0 || dev >= 64 || !g_tc.p[dev]) return PB_OK;
    PB_TRY_CUDA(cudaMemcpy(&e, g_tc.p[dev], sizeof(int), cudaMemcpyDeviceToHost));
    if (e) PB_TRY_CUDA(cudaMemset(g_tc.p[dev], 0, sizeof(int)));
  }
  return e ? pb_set_error(PB_ECUDA, "k_q80tc: a bounded wait gave up (role %d)", e) : PB_OK;
}
