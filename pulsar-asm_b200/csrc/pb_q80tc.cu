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
// CTA = 10 warps, one 128-row tile of W and TS (16, 32 or 64) of the T
// positions: a TMA producer warp, an MMA warp and eight epilogue warps (two
// per TMEM lane quarter, each folding half of the positions); see k_q80tc.
// The weight scales keep the tensor's own dtype (fp16 for Q8_0, fp32 for the
// .lfm3q8 dtype-1 format).
// Operands sit in shared memory in the K-major 128-byte-swizzle layout: a
// stage's 8 blocks (256 bytes of K per row) are two 128-byte-wide column
// slabs of 128-byte rows, 8-row groups 1024 bytes apart, the 16-byte chunk c
// of row r stored at chunk c ^ (r & 7); the MMA of block j starts at slab
// j / 4, byte (j % 4) * 32. (The no-swizzle core-matrix layout feeds the
// tensor cores about 16 bytes a cycle: an M128 N32 K32 MMA then takes some 500
// cycles.) The weights are stored that way in HBM at pack time and the
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
constexpr unsigned long long TC_WAIT_NS = 1000000000ull;   // a wait gives up after about a second

struct TcArgs {
  const int8_t* a;     // weights [tile][stage][128 rows x 256 bytes, 128-byte swizzle]
  const void* dw;      // weight scales [tile][stage][128 rows][8 blocks] (fp16 or fp32, the tensor's dtype)
  const int8_t* b;     // activations [T/TS][stage][TS rows x 256 bytes, 128-byte swizzle]
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
PB_DEV unsigned long long tc_now() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
PB_DEV bool mb_wait(uint64_t* b, unsigned par, volatile int* abort_f) {
  if (mb_try(b, par)) return true;
  const unsigned long long t0 = tc_now();
  for (unsigned i = 0; i < TC_WAIT; i++) {
    if (mb_try(b, par)) return true;
    if ((i & 63) == 63 && (*abort_f || tc_now() - t0 > TC_WAIT_NS)) return false;
  }
  return false;
}
// wait for a phase whatever the other roles did (in-flight copies and MMAs
// before exit), bounded by time
PB_DEV void mb_drain(uint64_t* b, unsigned par) {
  const unsigned long long t0 = tc_now();
  for (unsigned i = 0; !mb_try(b, par); i++)
    if ((i & 63) == 63 && tc_now() - t0 > TC_WAIT_NS) return;
}
// the same, by a whole warp, with one answer for every lane
PB_DEV bool mb_wait_warp(uint64_t* b, unsigned par, volatile int* abort_f) {
  return __all_sync(0xffffffffu, mb_wait(b, par, abort_f));
}
PB_DEV void bulk(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(s32(dst)), "l"(src), "r"(bytes), "r"(s32(bar)) : "memory");
}
// K-major, 128-byte swizzle (layout type 2, bits 61-63): LBO 16 B (unused by
// swizzled K-major layouts), SBO 1024 B between 8-row groups, descriptor
// version 1 (sm_100, bits 46-47), base offset 0 (slabs are 1024-byte aligned)
PB_DEV uint64_t umma_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}
// byte offset of (row r, K byte c of the stage, c < 256) in a stage region of
// R rows (R a multiple of 8) in the 128-byte-swizzle layout
PB_DEV size_t tc_sw(int r, int c, int R) {
  return (size_t)(c >> 7) * (R * 128) + (size_t)(r >> 3) * 1024 + (r & 7) * 128 + ((((c >> 4) & 7) ^ (r & 7)) << 4) +
         (c & 15);
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

// 8 consecutive / 16 / 32 int32 columns of this thread's TMEM lane
PB_DEV void tc_ld16(uint32_t taddr, int32_t* v) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
               "%14, %15}, [%16];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                 "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
               : "r"(taddr));
}
template <int NC>
PB_DEV void tc_ld_cols(uint32_t taddr, int32_t* v) {
#pragma unroll
  for (int c = 0; c < NC; c += 16) {
    if (NC - c >= 16) tc_ld16(taddr + (uint32_t)c, v + c);
    else tc_ld8(taddr + (uint32_t)c, v + c);
  }
}

constexpr int TC_NS = 4;             // shared-memory stages
#ifndef PB_TC_EW
#define PB_TC_EW 8
#endif
constexpr int TC_EW = PB_TC_EW;      // epilogue warps: TC_EW / 4 per TMEM lane quarter
constexpr int TC_EP = TC_EW / 4;     // position parts per lane quarter
// registers of an epilogue thread for one group of TMEM columns
constexpr int TC_VREGS = TC_EW >= 16 ? 32 : 128;

// shared-memory geometry of one stage for TS positions per CTA and weight
// scales of SB bytes
template <int TS, int SB>
struct TcGeo {
  static constexpr int SA = TC_M * 32 * TC_CB;       // weights
  static constexpr int SBX = TS * 32 * TC_CB;        // activations
  static constexpr int SW = TC_CB * TC_M * SB;       // weight scales [row][8 blocks]
  static constexpr int SX = TC_CB * TS * 4;          // activation scales (fp32)
  static constexpr int BYTES = SA + SBX + SW + SX;                // copied per stage
  static constexpr int STAGE = (BYTES + 1023) / 1024 * 1024;     // stride: slabs stay 1024-aligned
  static constexpr int NB = (512 / TS) < 16 ? (512 / TS) : 16;   // TMEM buffers of TS columns
  static constexpr int HT = TS / TC_EP;                           // positions per epilogue thread
  // blocks per TMEM group (one handshake per group): an epilogue thread
  // holds one group's columns, GB HT registers
  static constexpr int GBR = TC_VREGS / HT;
  static constexpr int GB = GBR >= TC_CB ? TC_CB : (GBR >= 4 ? 4 : (GBR >= 2 ? 2 : 1));
  static constexpr int NG = NB / GB;                 // buffer groups
  static constexpr int SMEM = TC_NS * STAGE + 1024;  // + room to align the base
};

// packed fp32 pairs; every operation rounds on its own (explicit .rn: no
// contraction into an fma)
typedef unsigned long long tc_f2;
PB_DEV tc_f2 tc_pk(float a, float b) {
  tc_f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
PB_DEV void tc_upk(tc_f2 v, float& a, float& b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
PB_DEV tc_f2 tc_mul2(tc_f2 a, tc_f2 b) {
  tc_f2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
PB_DEV tc_f2 tc_add2(tc_f2 a, tc_f2 b) {
  tc_f2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// two int32 block dots -> fp32, exactly (|isum| < 2^22): the integer is added
// to the mantissa of 1.5 * 2^23 and the bias subtracted
PB_DEV tc_f2 tc_i2f2(int32_t a, int32_t b) {
  tc_f2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(a + 0x4B400000), "r"(b + 0x4B400000));
  return tc_add2(r, tc_pk(-12582912.0f, -12582912.0f));
}

// the weight scales of GB consecutive blocks of one row (GB * sizeof(ST)
// bytes, aligned to that size) in one vector load, as fp32
template <int GB, typename ST>
PB_DEV void tc_scales(const ST* p, float (&o)[GB]) {
  if constexpr (sizeof(ST) == 4) {
    if constexpr (GB >= 4) {
#pragma unroll
      for (int i = 0; i < GB; i += 4) {
        const float4 v = reinterpret_cast<const float4*>(p)[i / 4];
        o[i] = v.x; o[i + 1] = v.y; o[i + 2] = v.z; o[i + 3] = v.w;
      }
    } else if constexpr (GB == 2) {
      const float2 v = *reinterpret_cast<const float2*>(p);
      o[0] = v.x; o[1] = v.y;
    } else {
      o[0] = p[0];
    }
  } else {
    unsigned w[(GB + 1) / 2];
    if constexpr (GB == 8) {
      const uint4 v = *reinterpret_cast<const uint4*>(p);
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    } else if constexpr (GB == 4) {
      const uint2 v = *reinterpret_cast<const uint2*>(p);
      w[0] = v.x; w[1] = v.y;
    } else if constexpr (GB == 2) {
      w[0] = *reinterpret_cast<const unsigned*>(p);
    } else {
      w[0] = p[0];
    }
#pragma unroll
    for (int i = 0; i < GB; i++) o[i] = pb_h2f((unsigned short)(w[i / 2] >> (16 * (i & 1))));
  }
}

// CTA = 2 + TC_EW warps, one 128-row tile of W and TS of the T positions (grid
// tiles x T/TS; for T <= 64 every weight byte is read once):
//   warp 0:     TMA producer (lane 0 issues), 1-D bulk copies of each stage
//               (8 blocks of weights, activations and their scales) into a
//               ring of TC_NS shared-memory stages (full/empty mbarriers);
//   warp 1:     MMA issuer (lane 0 issues), one tcgen05.mma (M 128, N TS,
//               K 32) per block into one of NB TMEM buffers of TS columns, one
//               tcgen05.commit per group of GB blocks; warp 1 allocates and
//               frees the TMEM (all 512 columns: one CTA per SM);
//   warps 2-:   epilogue; warp w reads TMEM lane quarter w % 4 and part
//               (w - 2) / 4 of the positions: per group one wait,
//               tcgen05.ld of its columns of the group's blocks, release of
//               the group's buffers,
//               fp32 fold in block order (products two positions per packed
//               multiply, the accumulation scalar).
// The issuing loops run one stage per iteration with every block of the
// stage unrolled: a single issuing thread runs its instructions back to back,
// so each index or descriptor computed at run time costs tens of cycles per
// MMA (a loop computing them per block issued one M128 N32 MMA per 470
// cycles; precomputed descriptors plus constants reach about 50).
template <int TS, typename ST, bool ISUM>
__global__ void __launch_bounds__(32 * (2 + TC_EW), 1) k_q80tc(TcArgs p) {
  typedef TcGeo<TS, (int)sizeof(ST)> Gm;
  constexpr int NB = Gm::NB, NG = Gm::NG, HT = Gm::HT, GB = Gm::GB, GPS = TC_CB / GB;
  static_assert((NB & (NB - 1)) == 0 && NB % TC_CB == 0, "TMEM buffers: whole stages, a power of two");
  static_assert(TC_CB % GB == 0 && HT % 2 == 0, "group shape");
  extern __shared__ __align__(1024) unsigned char tsm_raw[];
  __shared__ uint64_t full[TC_NS], empty[TC_NS], tfull[NG], tempty[NG], done;
  __shared__ uint32_t tbase;
  __shared__ int abort_f;
  unsigned char* tsm = tsm_raw + ((1024u - (s32(tsm_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nblk = p.K / 32, nst = nblk / TC_CB, ngrp = nblk / GB, tile = blockIdx.x, ts = blockIdx.y;
  if (threadIdx.x == 0) {
    for (int i = 0; i < TC_NS; i++) { mb_init(&full[i], 1); mb_init(&empty[i], 1 + TC_EW); }
    for (int i = 0; i < NG; i++) { mb_init(&tfull[i], 1); mb_init(&tempty[i], TC_EW); }   // every epilogue warp reads every group
    mb_init(&done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    abort_f = 0;
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(s32(&tbase)));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tbase;

  if (warp == 0) {
    // the whole warp runs the loop; lane 0 issues the copies
    const int8_t* pa = p.a + (size_t)tile * nblk * 4096;
    const int8_t* pbx = p.b + (size_t)ts * nblk * (TS * 32);
    const unsigned char* pw = reinterpret_cast<const unsigned char*>(p.dw) + (size_t)tile * nblk * TC_M * sizeof(ST);
    const float* px = p.dx + (size_t)ts * nblk * TS;
    int slot = 0, issued = 0;
    unsigned epar = 1;   // parity of the empty phase a refill of this slot waits for (flips per ring pass)
    for (int s = 0; s < nst; s++) {
      if (s >= TC_NS && !mb_wait_warp(&empty[slot], epar, &abort_f)) {
        if (lane == 0) { abort_f = 1; atomicCAS(p.err, 0, 1); }
        break;
      }
      if (lane == 0) {
        unsigned char* st = tsm + (size_t)slot * Gm::STAGE;
        mb_expect(&full[slot], Gm::BYTES);
        bulk(st, pa, Gm::SA, &full[slot]);
        bulk(st + Gm::SA, pbx, Gm::SBX, &full[slot]);
        bulk(st + Gm::SA + Gm::SBX, pw, Gm::SW, &full[slot]);
        bulk(st + Gm::SA + Gm::SBX + Gm::SW, px, Gm::SX, &full[slot]);
      }
      __syncwarp();
      pa += Gm::SA;
      pbx += Gm::SBX;
      pw += Gm::SW;
      px += Gm::SX / 4;
      issued = s + 1;
      if (++slot == TC_NS) { slot = 0; epar ^= 1; }
    }
    // no copy may land after the CTA exits: each slot's last issued stage (bounded)
    for (int s = issued > TC_NS ? issued - TC_NS : 0; s < issued; s++) mb_drain(&full[s % TC_NS], (unsigned)(s / TC_NS) & 1u);
  } else if (warp == 1) {
    // kind::i8: D s32 (bits 4-5 = 2), A and B signed (bits 7-9, 10-12 = 1),
    // both K-major, N = TS (bits 17-22 = TS/8), M = 128 (bits 24-28 = 128/16)
    constexpr uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(TS >> 3) << 17) |
                               ((uint32_t)(TC_M >> 4) << 24);
    // descriptors of slot 0, block 0; others add constant offsets (in 16-byte
    // units) to the start-address field, which never carries
    const uint64_t da0 = umma_desc(s32(tsm)), db0 = umma_desc(s32(tsm + Gm::SA));
    int slot = 0, gs = 0, nb0 = 0;
    unsigned fpar = 0;   // parity of full[slot]
    unsigned tpass = 0;  // passes over the TMEM group slots completed
    bool ok = true;
    for (int s = 0; s < nst && ok; s++) {
      if (!mb_wait_warp(&full[slot], fpar, &abort_f)) { ok = false; break; }
      tc_fence_after();
      const uint64_t so = (uint64_t)((slot * Gm::STAGE) >> 4);
      const uint64_t da = da0 + so, db = db0 + so;
#pragma unroll
      for (int q = 0; q < GPS; q++) {
        if (tpass > 0 && !mb_wait_warp(&tempty[gs], (tpass - 1) & 1u, &abort_f)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
#pragma unroll
          for (int k = 0; k < GB; k++) {
            const int j = q * GB + k;
            tc_mma_i8(tmem + (uint32_t)((nb0 + j) * TS),
                      da + (uint64_t)(((j >> 2) * (TC_M * 128) + (j & 3) * 32) >> 4),
                      db + (uint64_t)(((j >> 2) * (TS * 128) + (j & 3) * 32) >> 4), idesc);
          }
          tc_commit(&tfull[gs]);
          if (q == GPS - 1) tc_commit(&empty[slot]);
        }
        __syncwarp();
        if (++gs == NG) { gs = 0; tpass++; }
      }
      nb0 = (nb0 + TC_CB) & (NB - 1);
      if (++slot == TC_NS) { slot = 0; fpar ^= 1; }
    }
    if (!ok && lane == 0) { abort_f = 1; atomicCAS(p.err, 0, 2); }
    // every MMA issued so far has completed before the TMEM is freed (bounded)
    if (lane == 0) tc_commit(&done);
    __syncwarp();
    mb_drain(&done, 0);
  } else {
    const int q = warp & 3;                     // TMEM lane quarter of this warp
    const int part = (warp - 2) >> 2;           // which part of the positions
    const int rloc = q * 32 + lane;
    const int n = tile * TC_M + rloc;
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(part * HT);
    float acc[HT];
#pragma unroll
    for (int t = 0; t < HT; t++) acc[t] = 0.0f;
    int32_t va[GB][HT];
    bool ok = true;
    // wait until group g is in TMEM (its stage's scales are then in shared
    // memory too: the MMAs read the same stage), then load it into v
    auto fetch = [&](int g, int32_t (&v)[GB][HT]) -> bool {
      if (!mb_wait(&tfull[g % NG], (unsigned)(g / NG) & 1u, &abort_f)) return false;
      tc_fence_after();
#pragma unroll
      for (int k = 0; k < GB; k++) tc_ld_cols<HT>(tq + (uint32_t)(((g * GB + k) % NB) * TS), v[k]);
      return true;
    };
    // the loads of group g have landed: hand its buffers back to the MMA warp
    auto landed = [&](int g) {
      tc_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mb_arrive(&tempty[g % NG]);
    };
    auto fold = [&](int g, const int32_t (&v)[GB][HT]) {
      const int s = (g * GB) / TC_CB, slot = s % TC_NS, j0 = (g * GB) % TC_CB;
      const unsigned char* st = tsm + (size_t)slot * Gm::STAGE;
      float dws[GB];
      tc_scales<GB, ST>(reinterpret_cast<const ST*>(st + Gm::SA + Gm::SBX) + rloc * TC_CB + j0, dws);
#pragma unroll
      for (int k = 0; k < GB; k++) {
        const int j = j0 + k, b = g * GB + k;
        const tc_f2 dw2 = tc_pk(dws[k], dws[k]);
        const float4* dx4 = reinterpret_cast<const float4*>(st + Gm::SA + Gm::SBX + Gm::SW) + j * (TS / 4) + part * (HT / 4);
#pragma unroll
        for (int t4 = 0; t4 < HT / 4; t4++) {
          const float4 d = dx4[t4];
          // acc += (dw * dx) * (float)isum, per position, in block order; the
          // products as packed pairs, the accumulation scalar (a packed add
          // after a packed multiply is not kept apart: its results differ)
          float p0, p1, p2, p3;
          tc_upk(tc_mul2(tc_mul2(dw2, tc_pk(d.x, d.y)), tc_i2f2(v[k][4 * t4], v[k][4 * t4 + 1])), p0, p1);
          tc_upk(tc_mul2(tc_mul2(dw2, tc_pk(d.z, d.w)), tc_i2f2(v[k][4 * t4 + 2], v[k][4 * t4 + 3])), p2, p3);
          acc[4 * t4] = __fadd_rn(acc[4 * t4], p0);
          acc[4 * t4 + 1] = __fadd_rn(acc[4 * t4 + 1], p1);
          acc[4 * t4 + 2] = __fadd_rn(acc[4 * t4 + 2], p2);
          acc[4 * t4 + 3] = __fadd_rn(acc[4 * t4 + 3], p3);
        }
        if (ISUM && n < p.N) {
#pragma unroll
          for (int t = 0; t < HT; t++) p.isum[((size_t)(ts * TS + part * HT + t) * p.N + n) * nblk + b] = v[k][t];
        }
        if (j == TC_CB - 1) {
          __syncwarp();
          if (lane == 0) mb_arrive(&empty[slot]);
        }
      }
    };
    // one register set: the fold keeps the registers for its own parallelism
    // (a second set, loaded a group ahead, left too few and was slower)
    int b = 0;
    for (int g = 0; g < ngrp; g++) {
      if (!(ok = fetch(g, va))) break;
      landed(g);
      fold(g, va);
      b = (g + 1) * GB;
    }
    if (b < nblk) { abort_f = 1; atomicCAS(p.err, 0, 3); }
    if (n < p.N) {
#pragma unroll
      for (int t = 0; t < HT; t++) p.y[(size_t)(ts * TS + part * HT + t) * p.N + n] = acc[t];
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem));
}

// row-major codes/scales -> tiles of 128 rows, per stage of 8 blocks in the
// 128-byte-swizzle order (rows >= N are zero); one thread per 16-byte
// (row, block, half)
template <typename S>
__global__ void k_q80tc_pack(const int8_t* __restrict__ codes, const S* __restrict__ scales, int N, int K,
                             int ntile, int8_t* __restrict__ a, S* __restrict__ dw) {
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
    int8_t* dst = a + ((size_t)tile * nblk + (b & ~(TC_CB - 1))) * 4096 + tc_sw(row, (b % TC_CB) * 32 + kh * 16, TC_M);
    *reinterpret_cast<uint4*>(dst) = v;
    if (kh == 0) dw[((tb >> 3) * TC_M + row) * TC_CB + (b % TC_CB)] = n < N ? scales[(size_t)n * nblk + b] : (S)0;
  }
}

// the same tiles from a tensor in the streaming layout (pb_q8.cu): granule
// h*32 + l of segment (row, chunk) holds codes [16(h&1), +16) of block
// l + 32(h>>1) of the chunk; scales are pairs (s_l, s_{l+32}) per segment;
// only the K / 32 real blocks are copied (the integer fold is block-serial,
// whatever the float path's chunking)
template <typename S>
__global__ void k_q80tc_from_stream(const uint4* __restrict__ codes, const S* __restrict__ scales, int N, int K,
                                    int ntile, int8_t* __restrict__ a, S* __restrict__ dw) {
  const int nblk = K / 32, nch = (K + 2047) / 2048;   // segments per row (a one-chunk row is padded)
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
    S sc = (S)0;
    if (n < N) {
      const size_t seg = (size_t)n * nch + c;
      v = codes[seg * 128 + (hb * 2 + kh) * 32 + l];
      sc = scales[(seg * 32 + l) * 2 + hb];
    }
    *reinterpret_cast<uint4*>(a + ((size_t)tile * nblk + (b & ~(TC_CB - 1))) * 4096 +
                              tc_sw(row, (b % TC_CB) * 32 + kh * 16, TC_M)) = v;
    if (kh == 0) dw[((tb >> 3) * TC_M + row) * TC_CB + (b % TC_CB)] = sc;
  }
}

// positions per CTA for T positions (T a multiple of 16)
int tc_ts(int T) { return T % 64 == 0 ? 64 : (T % 32 == 0 ? 32 : 16); }

// activations [T][K] int8 + fp16 scales [T][K/32] -> the kernel's layout:
// per TS positions, per stage of 8 blocks, TS rows in the 128-byte-swizzle
// order; scales fp32 [TS group][block][TS]
__global__ void k_q80tc_act(const int8_t* __restrict__ qx, const uint16_t* __restrict__ dxh, int T, int K, int TS,
                            int8_t* __restrict__ bq, float* __restrict__ dx) {
  const int nblk = K / 32;
  const int total = nblk * T * 2;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int kh = i & 1, t = (i >> 1) % T, b = (i >> 1) / T;
    const int ts = t / TS, tl = t % TS;
    const size_t blk = (size_t)ts * nblk + b;
    const uint4 v = *reinterpret_cast<const uint4*>(qx + (size_t)t * K + b * 32 + kh * 16);
    *reinterpret_cast<uint4*>(bq + ((size_t)ts * nblk + (b & ~(TC_CB - 1))) * (TS * 32) +
                              tc_sw(tl, (b % TC_CB) * 32 + kh * 16, TS)) = v;
    if (kh == 0) dx[blk * TS + tl] = pb_h2f(dxh[(size_t)t * nblk + b]);
  }
}

template <int TS, typename ST, bool ISUM>
int launch_tc_t2(const pb_q8* w, int T, const int8_t* bq, const float* dx, float* y, int32_t* isum, int* err,
                cudaStream_t st) {
  typedef TcGeo<TS, (int)sizeof(ST)> Gm;
  static bool attr[64] = {};
  int dev = 0;
  PB_TRY_CUDA(cudaGetDevice(&dev));
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    PB_TRY_CUDA(cudaFuncSetAttribute(k_q80tc<TS, ST, ISUM>, cudaFuncAttributeMaxDynamicSharedMemorySize, Gm::SMEM));
    attr[dev] = true;
  }
  TcArgs a;
  a.a = w->codes;
  a.dw = w->scales;
  a.b = bq;
  a.dx = dx;
  a.y = y;
  a.isum = isum;
  a.N = w->N;
  a.K = w->K;
  a.ns = TC_NS;
  a.err = err;
  const int ntile = (w->N + TC_M - 1) / TC_M;
  k_q80tc<TS, ST, ISUM><<<dim3(ntile, T / TS), 32 * (2 + TC_EW), Gm::SMEM, st>>>(a);
  PB_LAUNCHED("k_q80tc");
  return PB_OK;
}
// the block dots are written out only when asked for (tests)
template <int TS, typename ST>
int launch_tc_t(const pb_q8* w, int T, const int8_t* bq, const float* dx, float* y, int32_t* isum, int* err,
                cudaStream_t st) {
  return isum ? launch_tc_t2<TS, ST, true>(w, T, bq, dx, y, isum, err, st)
              : launch_tc_t2<TS, ST, false>(w, T, bq, dx, y, isum, err, st);
}

int launch_tc(const pb_q8* w, int T, const int8_t* bq, const float* dx, float* y, int32_t* isum, int* err,
              cudaStream_t st) {
  const bool f32 = w->sdt == PB_DT_F32;
  switch (tc_ts(T)) {
    case 64: return f32 ? launch_tc_t<64, float>(w, T, bq, dx, y, isum, err, st)
                        : launch_tc_t<64, unsigned short>(w, T, bq, dx, y, isum, err, st);
    case 32: return f32 ? launch_tc_t<32, float>(w, T, bq, dx, y, isum, err, st)
                        : launch_tc_t<32, unsigned short>(w, T, bq, dx, y, isum, err, st);
    default: return f32 ? launch_tc_t<16, float>(w, T, bq, dx, y, isum, err, st)
                        : launch_tc_t<16, unsigned short>(w, T, bq, dx, y, isum, err, st);
  }
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
  const size_t ab = (size_t)ntile * TC_M * K, wb = (size_t)ntile * TC_M * nblk * (scale_dtype == PB_DT_F32 ? 4 : 2);
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
                                                         (unsigned short*)w->scales);
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
  return ntile * TC_M * K + ntile * TC_M * (K / 32) * 4;   // room for fp32 scales
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
                                                              out->codes, (unsigned short*)out->scales);
  PB_LAUNCHED("k_q80tc_from_stream");
  return PB_OK;
}

extern "C" int pb_q80_gemm(const pb_q8* w, int T, const int8_t* d_qx, const uint16_t* d_dx, float* d_y,
                           int32_t* d_isum, void* stream) {
  if (!w || !d_qx || !d_dx || !d_y) return pb_set_error(PB_EINVAL, "pb_q80_gemm: null argument");
  if (w->layout != PB_Q8_UMMA) return pb_set_error(PB_EINVAL, "pb_q80_gemm: tensor not packed by pb_q80tc_pack");
  if (T <= 0 || T % 16 || T > 256)
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
  k_q80tc_act<<<(units + 255) / 256, 256, 0, st>>>(d_qx, d_dx, T, w->K, tc_ts(T), bq, dx);
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
