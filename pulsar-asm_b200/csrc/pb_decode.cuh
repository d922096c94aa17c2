// pb_decode.cuh -- the persistent decode kernel: every phase of a token (each
// fused GEMV, each attention layer, the greedy argmax), for any number of
// tokens, in ONE cooperative launch with one CTA (8 warps) per SM.
//
// Weight stream: the CTA's row slice of every GEMV of every token is a fixed
// sequence of stages (16 segments of 2048 codes + their scales), known before
// the launch (host-built schedule: per CTA and GEMV its rows and first stage,
// and a stage -> GEMV map). Stages flow through a ring of DS shared-memory
// slots filled by 1-D TMA bulk copies (cp.async.bulk ... complete_tx on the
// slot's mbarrier). There is no producer warp: the warp that is the last of
// the eight to finish reading a slot (a shared counter) issues the copy of the
// stage DS places ahead into it. Weights never depend on activations, so the
// stream runs ahead across phases: while the warps sit in a grid barrier,
// compute a prologue or run attention, the next GEMV's first DS stages land.
//
// Phases: wait until every CTA finished the previous phase (a global arrival
// counter), compute the fused prologue (pb_step.cuh), then consume stages:
// two 2048-code segments per warp per stage, in the reference's reduction
// order, with the FMA chains of a lane's two blocks (l and l+32) packed into
// one fma.rn.f32x2 (each half is an IEEE fma, so the values are unchanged).
// All spin waits are bounded: on a timeout the kernel records an error code,
// every warp leaves at the next phase boundary, and thread 0 waits (bounded)
// for the copies still in flight before the CTA exits; the host reports the
// error.
#pragma once
#include "pb_step.cuh"

namespace {

constexpr int PH_GEMV = 0, PH_ARGMAX = 2, PH_SCORE = 3, PH_SOFTMAX = 4, PH_PV = 5;
constexpr int PV_DIMS = 16;                    // head dims per P.V task
constexpr int DSEGS = 16;                      // 2048-byte segments per stage
constexpr int STAGE_CODES = DSEGS * 2048;      // 32 KB

struct Phase {
  int kind, nch, epi;
  int rowoff;     // GEMV: float offset in the activation region of the row values
  int gidx;       // GEMV: index in the per-CTA GEMV schedule
  int _pad;
  StepArgs a;     // GEMV: weights, prologue, epilogue
  AttnArgs at;    // ATTN
};

// one CTA's share of one GEMV: rows [r0, r1), stages base .. base + ceil((r1-r0)/RB) - 1
struct GemvSched {
  const char* codes;
  const char* scales;
  int r0, r1, base, nch;
};

// one stage of a CTA's weight stream: codes and scales as 16-byte offsets
// into the model's weight arena, and their byte counts
struct StageDesc {
  unsigned codes16, scales16, bc, bs;
};

// the weight stream's bookkeeping, at the start of dynamic shared memory
struct IssueCtx {
  uint64_t pol;           // L2 evict-first policy of the stream
  const char* arena;      // the model's weight arena
  unsigned spt;           // stages per token of this CTA
  unsigned total;         // stages of the launch (spt * tokens)
  unsigned ds;            // ring slots
  unsigned ngemv;
  unsigned cnt[8];        // per slot: warps done reading the current stage
  unsigned issued[8];     // per slot: last stage issued into it (+1; 0 = none)
  uint32_t sched_s;       // shared address of GemvSched[ngemv]
  uint32_t desc_s;        // shared address of StageDesc[spt]
};
constexpr int ISSUE_BYTES = 128;
constexpr int MAX_DS = 8;

struct DecodeArgs {
  const Phase* phases;
  int nphase;
  int ntok;
  Ctl* ctl;
  unsigned* bar;       // phase arrival counter (zeroed before the launch)
  int* err;            // 0, or the code of the wait that gave up
  int xregion;         // floats of the activation region in shared memory
  int nh;              // attention heads = CTAs that run an attention phase
  int ds;              // ring stages
  int pv_per_warp;     // floats of shared memory per warp in a P.V phase
  unsigned long long* trace;   // optional: per (CTA, phase) globaltimer marks of token 0
  const GemvSched* sched;      // [CTA][ngemv]
  const StageDesc* sdesc;      // [CTA][spt_max]: the stages of a token
  const int* spt;              // [CTA]: stages per token
  const char* arena;           // the model's weight arena
  int ngemv, spt_max;
  int sched_off, desc_off;     // byte offsets of the tables in dynamic shared memory
};

PB_DEV unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// trace marks: 0 phase entered, 1 grid barrier passed, 2 prologue done, 3 work done, 4 arrived;
// in a build with PB_TRACE_STAGE_LOOP defined, GEMV phases add warp 0's
// stage-loop totals: 5 slot releases with their refill issues, 6 waits for
// stage data, 7 chain and tree arithmetic (these timers cost about 4.5 % of
// decode throughput even with tracing off, so default builds leave them out)
PB_DEV void tmark(const DecodeArgs& d, int tok, int p, int k) {
  if (d.trace && tok == 0 && threadIdx.x == 0) d.trace[((size_t)blockIdx.x * d.nphase + p) * 8 + k] = gtime();
}

template <bool F32S>
struct DGeo {
  static constexpr int SB = F32S ? 8 : 4;                  // bytes per scale pair
  static constexpr int STAGE_SCALES = DSEGS * 32 * SB;
  static constexpr int STAGE = STAGE_CODES + STAGE_SCALES;
};

PB_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
PB_DEV void mbar_init(uint64_t* b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
PB_DEV void mbar_expect_tx(uint64_t* b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
PB_DEV void mbar_arrive(uint64_t* b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}
PB_DEV bool mbar_try(uint64_t* b, unsigned parity) {
  uint32_t ok;
  asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
               : "=r"(ok) : "r"(smem_u32(b)), "r"(parity) : "memory");
  return ok != 0;
}
PB_DEV bool mbar_wait(uint64_t* b, unsigned parity, volatile int* abort_flag) {
  for (unsigned i = 0; i < PB_WAIT_LIMIT; i++) {
    if (mbar_try(b, parity)) return true;
    if ((i & 255) == 255 && *abort_flag) return false;
    if (i > 64) __nanosleep(32);
  }
  return false;
}
// the weight stream is read once per token: an evict-first L2 policy keeps it
// from pushing the small reused state (activations, KV cache, conv rings,
// norm weights) out of L2
PB_DEV uint64_t l2_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
PB_DEV void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar, uint64_t pol) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol) : "memory");
}
PB_DEV void grid_arrive(unsigned* bar) {
  asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
}

// packed fp32 pairs
typedef unsigned long long f2x;
PB_DEV f2x pk(float a, float b) {
  f2x r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
PB_DEV f2x pku(unsigned a, unsigned b) {
  f2x r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(a), "r"(b));
  return r;
}
PB_DEV void upk(f2x v, float& a, float& b) { asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v)); }
PB_DEV f2x fma2(f2x a, f2x b, f2x c) {
  f2x d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
PB_DEV f2x add2(f2x a, f2x b) {
  f2x d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// the two chains of lane l (block l in the low half, block l+32 in the high
// half) over one pair of 16-code granules, continuing d
PB_DEV f2x dot16x2(uint4 ga, uint4 gb, const f2x* xr, f2x d) {
  const unsigned wa[4] = {ga.x, ga.y, ga.z, ga.w}, wb[4] = {gb.x, gb.y, gb.z, gb.w};
  const f2x bias = pk(-8388736.0f, -8388736.0f);
#pragma unroll
  for (int k = 0; k < 4; k++) {
    const unsigned ua = wa[k] ^ 0x80808080u, ub = wb[k] ^ 0x80808080u;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const f2x c = add2(pku(__byte_perm(ua, 0x4B000000u, 0x7440u + j), __byte_perm(ub, 0x4B000000u, 0x7440u + j)), bias);
      d = fma2(c, xr[4 * k + j], d);
    }
  }
  return d;
}
PB_DEV float leaf2(const uint4 (&q)[4], float slo, float shi, const f2x (&xr)[32]) {
  f2x d = pk(0.0f, 0.0f);
  d = dot16x2(q[0], q[2], xr, d);
  d = dot16x2(q[1], q[3], xr + 16, d);
  float d0, d1;
  upk(d, d0, d1);
  return __fmaf_rn(shi, d1, __fmaf_rn(slo, d0, 0.0f));
}


extern __shared__ __align__(128) unsigned char dsm[];
PB_DEV IssueCtx* issue_ctx() { return reinterpret_cast<IssueCtx*>(dsm); }

// Copy the stage at position k of a token into ring slot `slot`. Called by
// thread 0 for the first DS stages and afterwards by lane 0 of the warp that
// releases the slot's previous stage (stage S + DS follows stage S in the same
// slot), so every copy follows the slot's last read.
template <bool F32S>
PB_DEV void issue_stage(unsigned k, unsigned slot, unsigned S, unsigned char* ring, uint64_t* full) {
  typedef DGeo<F32S> Gm;
  IssueCtx* ic = issue_ctx();
  uint4 dsc;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(dsc.x), "=r"(dsc.y), "=r"(dsc.z), "=r"(dsc.w) : "r"(ic->desc_s + 16 * k));
  const char* arena = ic->arena;
  const uint64_t pol = ic->pol;
  mbar_expect_tx(&full[slot], dsc.z + dsc.w);
  bulk_g2s(ring + (size_t)slot * Gm::STAGE, arena + (size_t)dsc.x * 16, dsc.z, &full[slot], pol);
  bulk_g2s(ring + (size_t)slot * Gm::STAGE + STAGE_CODES, arena + (size_t)dsc.y * 16, dsc.w, &full[slot], pol);
  ic->issued[slot] = S + 1;
}
// arrival of a warp that finished reading a slot; true for the last of the 8
PB_DEV bool slot_release(unsigned slot) {
  unsigned old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
               : "=r"(old) : "r"(smem_u32(&issue_ctx()->cnt[slot])) : "memory");
  return old == 7u;
}

// One GEMV phase on the consumer warps. Warp (g, c) owns rows 2g, 2g+1 of
// every stage in chunk c. The stage loop only waits, computes each row's
// chunk value (the lane chains and the shuffle-down tree) and parks it in
// shared memory (rowv, [local row][chunk]); after one consumer barrier the
// 256 threads combine the chunks in order and run the epilogue for all of
// the CTA's rows at once, so no per-row latency sits in the stage loop. A
// wait that gives up breaks out of the loop and the phase still ends with
// the same barriers as on the other warps.
template <bool F32S, int EPI, int EH, int W>
__device__ __forceinline__ unsigned gemv_phase(const DecodeArgs& d, const Phase& ph, unsigned char* ring,
                           float* xreg, uint64_t* full, unsigned it, float* red,
                           float* bestv, int* besti,
                           volatile int* abort_flag, unsigned long long* tmark2, const GridWait* gw, int pos) {
  typedef DGeo<F32S> Gm;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sx = xreg;
  step_prologue_fixed<1, EH, W>(ph.a, sx, red, gw, pos);   // grid barrier inside; ends with a consumer barrier
  if (tmark2 && threadIdx.x == 0) *tmark2 = gtime();
  // the few fields the stage loop needs, read once into registers (the loop's
  // global stores would otherwise force the compiler to re-read them)
  void* const yout = ph.a.y;
  Ctl* const ctl = ph.a.ctl;
  const int nch = ph.nch, RB = DSEGS / nch;
  float* const rowv = xreg + ph.rowoff;
  const int c = warp % nch, g = warp / nch;
  const unsigned ds = (unsigned)d.ds;
  f2x xr[32];
  {
    const float* x0 = sx + (c * 64 + lane) * 33;
    const float* x1 = sx + (c * 64 + 32 + lane) * 33;
#pragma unroll
    for (int j = 0; j < 32; j++) xr[j] = pk(x0[j], x1[j]);
  }
  int r0, r1;
  {
    const GemvSched* gs = reinterpret_cast<const GemvSched*>(dsm + (issue_ctx()->sched_s - smem_u32(dsm)));
    r0 = gs[ph.gidx].r0;
    r1 = gs[ph.gidx].r1;
  }
  unsigned slot = it % ds, par = (it / ds) & 1;
  // position within the token of the stage that refills the current slot
  const unsigned spt = issue_ctx()->spt, total = issue_ctx()->total;
  unsigned kn = it % spt + ds;
  while (kn >= spt) kn -= spt;
  for (int r = r0; r < r1; r += RB) {
#ifdef PB_TRACE_STAGE_LOOP
    const unsigned long long tw = (tmark2 && threadIdx.x == 0) ? gtime() : 0;
#endif
    if (!mbar_wait(&full[slot], par, abort_flag)) {
      *abort_flag = 1;
      atomicCAS(d.err, 0, 2);
      break;
    }
#ifdef PB_TRACE_STAGE_LOOP
    if (tmark2 && threadIdx.x == 0) tmark2[4] += gtime() - tw;   // slot 6 of the phase: data waits
#endif
    const unsigned char* st = ring + (size_t)slot * Gm::STAGE;
    uint4 q[2][4];
    float slo[2], shi[2];
#pragma unroll
    for (int u = 0; u < 2; u++) {
      const int rel = g * 2 + u;
      const int seg = rel * nch + c;
      if (r + rel < r1) {
        const uint4* gp = reinterpret_cast<const uint4*>(st + (size_t)seg * 2048) + lane;
#pragma unroll
        for (int h = 0; h < 4; h++) q[u][h] = gp[32 * h];
        if (F32S) {
          const float2 s2 = reinterpret_cast<const float2*>(st + STAGE_CODES)[seg * 32 + lane];
          slo[u] = s2.x; shi[u] = s2.y;
        } else {
          const unsigned w = reinterpret_cast<const unsigned*>(st + STAGE_CODES)[seg * 32 + lane];
          slo[u] = pb_h2f((unsigned short)(w & 0xffffu));
          shi[u] = pb_h2f((unsigned short)(w >> 16));
        }
      } else {
#pragma unroll
        for (int h = 0; h < 4; h++) q[u][h] = make_uint4(0, 0, 0, 0);
        slo[u] = shi[u] = 0.0f;
      }
    }
    // release the slot as soon as its data sit in registers (the empty asm
    // makes every load complete first), so the refill of the stage DS ahead
    // overlaps this stage's arithmetic; the last warp to release issues it
    asm volatile("" ::"r"(q[0][0].x), "r"(q[0][0].y), "r"(q[0][0].z), "r"(q[0][0].w), "r"(q[0][1].x),
                 "r"(q[0][1].y), "r"(q[0][1].z), "r"(q[0][1].w), "r"(q[0][2].x), "r"(q[0][2].y),
                 "r"(q[0][2].z), "r"(q[0][2].w), "r"(q[0][3].x), "r"(q[0][3].y), "r"(q[0][3].z),
                 "r"(q[0][3].w), "f"(slo[0]), "f"(shi[0]));
    asm volatile("" ::"r"(q[1][0].x), "r"(q[1][0].y), "r"(q[1][0].z), "r"(q[1][0].w), "r"(q[1][1].x),
                 "r"(q[1][1].y), "r"(q[1][1].z), "r"(q[1][1].w), "r"(q[1][2].x), "r"(q[1][2].y),
                 "r"(q[1][2].z), "r"(q[1][2].w), "r"(q[1][3].x), "r"(q[1][3].y), "r"(q[1][3].z),
                 "r"(q[1][3].w), "f"(slo[1]), "f"(shi[1]));
    __syncwarp();
#ifdef PB_TRACE_STAGE_LOOP
    const unsigned long long tr0 = (tmark2 && threadIdx.x == 0) ? gtime() : 0;
#endif
    if (lane == 0 && slot_release(slot)) {
      issue_ctx()->cnt[slot] = 0;
      if (it + ds < total) issue_stage<F32S>(kn, slot, it + ds, ring, full);
    }
#ifdef PB_TRACE_STAGE_LOOP
    const unsigned long long tr1 = (tmark2 && threadIdx.x == 0) ? gtime() : 0;
#endif
    float v[2];
#pragma unroll
    for (int u = 0; u < 2; u++) v[u] = pb_warp_tree(leaf2(q[u], slo[u], shi[u], xr));
#ifdef PB_TRACE_STAGE_LOOP
    if (tmark2 && threadIdx.x == 0) {
      asm volatile("" ::"f"(v[0]), "f"(v[1]));
      tmark2[3] += tr1 - tr0;            // slot 5: release (+ refill issue) of warp 0
      tmark2[5] += gtime() - tr1;        // slot 7: chains and trees of warp 0
    }
#endif
    if (lane == 0) {
      const int lr = r - r0 + g * 2;
      rowv[lr * nch + c] = v[0];
      if (r + g * 2 + 1 < r1) rowv[(lr + 1) * nch + c] = v[1];
    }
    it++;
    if (++slot == ds) { slot = 0; par ^= 1; }
    if (++kn == spt) kn = 0;
  }
  csync<1>();
  // epilogue over the CTA's rows: chunk values added in chunk order from 0
  const int nr = r1 - r0;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  if (EPI == EPI_SILU) {
    // rows 2i (w1) and 2i+1 (w3): k_silu_mul_bf, lfm3_nanode.cu:821-829
    for (int i = 2 * threadIdx.x; i + 1 < nr; i += 512) {
      float o0 = 0.0f, o1 = 0.0f;
      for (int cc = 0; cc < nch; cc++) {
        o0 = __fadd_rn(o0, rowv[i * nch + cc]);
        o1 = __fadd_rn(o1, rowv[(i + 1) * nch + cc]);
      }
      const float av = pb_bf2f(pb_f2bf(o0)), bw = pb_bf2f(pb_f2bf(o1));
      reinterpret_cast<bf16_t*>(yout)[(r0 + i) >> 1] = pb_f2bf(__fmul_rn(__fmul_rn(av, pb_sigmoid(av)), bw));
    }
  } else {
    for (int i = threadIdx.x; i < nr; i += 256) {
      float o = 0.0f;
      for (int cc = 0; cc < nch; cc++) o = __fadd_rn(o, rowv[i * nch + cc]);
      if (EPI == EPI_ARGMAX) {
        reinterpret_cast<float*>(yout)[r0 + i] = o;
        if (o > bv || (o == bv && r0 + i < bi)) { bv = o; bi = r0 + i; }
      } else {
        reinterpret_cast<bf16_t*>(yout)[r0 + i] = pb_f2bf(o);
      }
    }
  }
  if (EPI == EPI_ARGMAX) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_down_sync(0xffffffffu, bv, o);
      const int oi = __shfl_down_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { bestv[warp] = bv; besti[warp] = bi; }
    csync<1>();
    if (threadIdx.x == 0) {
      float b = bestv[0];
      int ix = besti[0];
      for (int w = 1; w < 8; w++)
        if (bestv[w] > b || (bestv[w] == b && besti[w] < ix)) { b = bestv[w]; ix = besti[w]; }
      ctl->slot_val[blockIdx.x] = b;
      ctl->slot_idx[blockIdx.x] = ix;
    }
  }
  return it;
}

// ------------------------------------------------------- split attention
// k_attn_head (lfm3_nanode.cu:503-602) as three grid-wide phases with the
// reference's exact arithmetic. Each phase issues all of a task's global
// loads before it consumes any of them (one L2 round trip per task), and the
// loops stay rolled so that the code of these rarely run phases stays small.
//  SCORE   task = (head, 32 positions), one warp: lane p forms the score of
//          position p alone: its 32 per-lane chains (((0 + q0k0) + q1k1) ...)
//          and then the shuffle-down tree's additions, replayed in registers;
//          * scaling. The task holding position pos for a group's first head
//          appends the new fp16 k/v row to the cache.
//  SOFTMAX task = head, one CTA: the 256 consumer threads are the reference's
//          256 strided chains i = t, t+256, ...; max over the window;
//          e = expf(s - m) kept in place; chains summed ascending, eight
//          shuffle-down trees and the 8-lane tree; inv = 1/sum.
//  PV      task = (head, segment, 16 dims), one warp: the segment's chain over
//          p = seg, seg+8, ... of (e_p * inv) * v_p, staged through shared
//          memory; the 8 segment partials meet in the o_proj prologue.
// Window spans above 2048 positions take the per-kernel path (host check).

PB_DEV void cp_async16(void* sdst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(sdst)), "l"(gsrc) : "memory");
}
PB_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// head RMSNorm (k_headnorm, lfm3_nanode.cu:460-479) + NeoX RoPE (k_rope,
// :483-498) of one warp from values already in registers: lane holds
// elements lane*E + j; c/s are the rope factors of those elements (i < half)
template <int E>
PB_DEV void norm_rope_regs(const float (&v)[E], const float (&w)[E], const float (&c)[E],
                           const float (&sv)[E], int half, float eps, float* o) {
  constexpr int HD = 32 * E;
  const int lane = threadIdx.x & 31;
  float ss[E];
#pragma unroll
  for (int j = 0; j < E; j++) ss[j] = __fmul_rn(v[j], v[j]);
#pragma unroll
  for (int width = E; width > 1; width >>= 1)
#pragma unroll
    for (int i = 0; i < width / 2; i++) ss[i] = __fadd_rn(ss[2 * i], ss[2 * i + 1]);
  float s = pb_warp_tree(__fadd_rn(ss[0], 0.0f));
  s = __shfl_sync(0xffffffffu, s, 0);
  const float rs = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(s, __fdiv_rn(1.0f, (float)HD)), eps)));
  float n[E], part[E];
#pragma unroll
  for (int j = 0; j < E; j++) n[j] = pb_bf2f(pb_f2bf(__fmul_rn(w[j], pb_bf2f(pb_f2bf(__fmul_rn(v[j], rs))))));
  // element i + HD/2 sits in lane + 16 at the same j
#pragma unroll
  for (int j = 0; j < E; j++) part[j] = __shfl_xor_sync(0xffffffffu, n[j], 16);
#pragma unroll
  for (int j = 0; j < E; j++) {
    const int i = lane * E + j;
    float r = n[j];
    if (lane < 16 && i < half) {          // lo = n, hi = part
      r = pb_bf2f(pb_f2bf(__fadd_rn(__fmul_rn(n[j], c[j]), __fmul_rn(-part[j], sv[j]))));
    } else if (lane >= 16 && i - HD / 2 < half) {   // hi = n, lo = part; factors of i - HD/2
      r = pb_bf2f(pb_f2bf(__fadd_rn(__fmul_rn(n[j], c[j]), __fmul_rn(part[j], sv[j]))));
    }
    o[i] = r;
  }
}

template <int E>
__device__ __noinline__ void attn_score_phase(const AttnArgs& a, int pos, float* wsm) {
  constexpr int HD = 32 * E;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * 8 + warp, GW = gridDim.x * 8;
  const int grp = a.nh / a.nkv, nkv = a.nkv, half = a.half;
  const int npos = pos + 1;
  const int lo = (a.win > 0 && npos > a.win) ? npos - a.win : 0;
  const int np = npos - lo, nblk = (np + 31) / 32, ntask = a.nh * nblk;
  const float scaling = a.scaling, eps = a.eps;
  float* qs = wsm + warp * 2 * HD;
  float* ks = qs + HD;
  const bf16_t* qkvg = a.qkvg;
  unsigned short* kc = a.kc;
  unsigned short* vc = a.vc;
  float* scores = a.scores;
  const float* qnorm = a.qnorm;
  const float* knorm = a.knorm;
  const size_t max_ctx = (size_t)a.max_ctx;
  // rope factors of this lane's elements: lanes >= 16 use those of i - HD/2
  const int ri = (lane & 15) * E;
  const float* cs = a.rope_cos + (size_t)pos * half;
  const float* sn = a.rope_sin + (size_t)pos * half;
  const size_t koff = (size_t)a.nh * HD, voff = koff + (size_t)nkv * HD;
  int cur = -1;
  for (int task = gw; task < ntask; task += GW) {
    const int h = task / nblk, pb = task - h * nblk, kvh = h / grp;
    const int p = lo + pb * 32 + lane;
    const bool writer = (h % grp == 0) && pos >= lo + pb * 32 && pos < lo + pb * 32 + 32;
    // all loads first: this lane's cached key row, the new v row (writer),
    // and when the head changes its q/k rows, norm weights and rope factors
    uint4 kg[HD / 8];
    if (p < pos) {
      const uint4* kr = reinterpret_cast<const uint4*>(kc + ((size_t)p * nkv + kvh) * HD);
#pragma unroll
      for (int g = 0; g < HD / 8; g++) kg[g] = __ldcg(kr + g);
    }
    unsigned short vraw[E];
    if (writer) {
#pragma unroll
      for (int j = 0; j < E; j++) vraw[j] = __ldcg(qkvg + voff + (size_t)kvh * HD + lane * E + j);
    }
    if (h != cur) {
      float qx[E], kx[E], qw[E], kw[E], c[E], sv[E];
#pragma unroll
      for (int j = 0; j < E; j++) {
        const int i = lane * E + j;
        qx[j] = pb_bf2f(__ldcg(qkvg + (size_t)h * HD + i));
        kx[j] = pb_bf2f(__ldcg(qkvg + koff + (size_t)kvh * HD + i));
        qw[j] = __ldg(qnorm + i);
        kw[j] = __ldg(knorm + i);
        c[j] = ri + j < half ? __ldg(cs + ri + j) : 0.0f;
        sv[j] = ri + j < half ? __ldg(sn + ri + j) : 0.0f;
      }
      __syncwarp();                       // previous task's reads of qs/ks are done
      norm_rope_regs<E>(qx, qw, c, sv, half, eps, qs);
      norm_rope_regs<E>(kx, kw, c, sv, half, eps, ks);
#pragma unroll
      for (int j = 0; j < E; j++) ks[lane * E + j] = pb_h2f(pb_f2h(ks[lane * E + j]));
      __syncwarp();
      cur = h;
    }
    if (writer) {
      unsigned short* kd = kc + ((size_t)pos * nkv + kvh) * HD;
      unsigned short* vd = vc + ((size_t)pos * nkv + kvh) * HD;
#pragma unroll
      for (int j = 0; j < E; j++) {
        kd[lane * E + j] = pb_f2h(ks[lane * E + j]);
        vd[lane * E + j] = pb_f2h(pb_bf2f(vraw[j]));
      }
    }
    if (p < npos) {
      float v[32];
#pragma unroll
      for (int l = 0; l < 32; l++) {
        float sl = 0.0f;
#pragma unroll
        for (int j = 0; j < E; j++) {
          const int dd = l * E + j;
          float kf;
          if (p < pos) {
            const unsigned w = reinterpret_cast<const unsigned*>(&kg[dd >> 3])[(dd & 7) >> 1];
            kf = pb_h2f((unsigned short)((dd & 1) ? (w >> 16) : (w & 0xffffu)));
          } else {
            kf = ks[dd];
          }
          sl = __fadd_rn(sl, __fmul_rn(qs[dd], kf));
        }
        v[l] = sl;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int l = 0; l < o; l++) v[l] = __fadd_rn(v[l], v[l + o]);
      scores[(size_t)h * max_ctx + (p - lo)] = __fmul_rn(v[0], scaling);
    }
  }
}

__device__ __noinline__ void attn_softmax_phase(const AttnArgs& a, int pos, float* red) {
  constexpr int PER = 8;     // scores per thread: window spans up to 2048
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int npos = pos + 1;
  const int lo = (a.win > 0 && npos > a.win) ? npos - a.win : 0;
  const int np = npos - lo;
  for (int h = blockIdx.x; h < a.nh; h += gridDim.x) {
    float* sc = a.scores + (size_t)h * a.max_ctx;
    float sv[PER];
#pragma unroll
    for (int k = 0; k < PER; k++) sv[k] = (t + 256 * k < np) ? __ldcg(sc + t + 256 * k) : -1e30f;
    float m = sv[0];
#pragma unroll
    for (int k = 1; k < PER; k++) m = fmaxf(m, sv[k]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red[warp] = m;
    csync<1>();
    m = red[0];
#pragma unroll
    for (int w = 1; w < 8; w++) m = fmaxf(m, red[w]);
    m = fmaxf(-1e30f, m);
    float sum = 0.0f;            // chain t: i = t, t + 256, ... ascending
#pragma unroll
    for (int k = 0; k < PER; k++) {
      const int i = t + 256 * k;
      if (i < np) {
        const float e = pb_expf(__fadd_rn(sv[k], -m));
        sc[i] = e;
        sum = __fadd_rn(sum, e);
      }
    }
    sum = pb_warp_tree(sum);
    if (lane == 0) red[8 + warp] = sum;
    csync<1>();
    if (t == 0) {
      const float* W = red + 8;
      const float tot = __fadd_rn(__fadd_rn(__fadd_rn(W[0], W[4]), __fadd_rn(W[2], W[6])),
                                  __fadd_rn(__fadd_rn(W[1], W[5]), __fadd_rn(W[3], W[7])));
      a.inv[h] = __fdiv_rn(1.0f, tot);
    }
    csync<1>();                  // red is reused by the next head
  }
}

template <int E>
__device__ __noinline__ void attn_pv_phase(const AttnArgs& a, int pos, float* wsm, int per_warp) {
  constexpr int HD = 32 * E, NDQ = HD / PV_DIMS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * 8 + warp, GW = gridDim.x * 8;
  const int grp = a.nh / a.nkv, nkv = a.nkv;
  const int npos = pos + 1;
  const int lo = (a.win > 0 && npos > a.win) ? npos - a.win : 0;
  const int np = npos - lo, ntask = a.nh * 8 * NDQ;
  const size_t max_ctx = (size_t)a.max_ctx;
  const float* scores = a.scores;
  const float* invp = a.inv;
  const unsigned short* vc = a.vc;
  float* segp = a.segp;
  // per warp: e values [cnt] then v rows [cnt][16 halves] (16-byte aligned)
  float* we = wsm + (size_t)warp * per_warp;
  unsigned short* wv = reinterpret_cast<unsigned short*>(we + (per_warp / 9));
  for (int task = gw; task < ntask; task += GW) {
    const int h = task / (8 * NDQ), rem = task - h * 8 * NDQ, seg = rem / NDQ, dq = rem - seg * NDQ;
    const int kvh = h / grp;
    const int cnt = seg < np ? (np - seg + 7) / 8 : 0;     // <= 256
    const float* sc = scores + (size_t)h * max_ctx;
    __syncwarp();                 // previous task's reads of we/wv are done
    // v rows by asynchronous copies, e values and inv by plain loads: all in flight together
    for (int it = lane; it < 2 * cnt; it += 32) {
      const int j = it >> 1, hf = it & 1;
      cp_async16(wv + it * 8, vc + ((size_t)(lo + seg + 8 * j) * nkv + kvh) * HD + dq * PV_DIMS + hf * 8);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    float ev[8];
#pragma unroll
    for (int r = 0; r < 8; r++) {
      const int j = lane + 32 * r;
      ev[r] = j < cnt ? __ldcg(sc + seg + 8 * j) : 0.0f;
    }
    const float inv = __ldcg(invp + h);
#pragma unroll
    for (int r = 0; r < 8; r++)
      if (lane + 32 * r < cnt) we[lane + 32 * r] = ev[r];
    cp_async_wait_all();
    __syncwarp();
    if (lane < PV_DIMS) {
      float acc = 0.0f;
      for (int j = 0; j < cnt; j++)
        acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(we[j], inv), pb_h2f(wv[j * PV_DIMS + lane])));
      segp[((size_t)h * 8 + seg) * HD + dq * PV_DIMS + lane] = acc;
    }
  }
}

// greedy id from the per-CTA maxima (ties to the lowest index); the next
// input is the prompt's next token while a prompt is being fed
__device__ void argmax_phase(const DecodeArgs& d) {
  // warp 0 of CTA 0: lanes reduce strided slots, then a shuffle tree; ties
  // resolve to the lowest index (the per-CTA maxima carry their row index)
  Ctl* ctl = d.ctl;
  const int lane = threadIdx.x & 31;
  float b = -INFINITY;
  int ix = 0x7fffffff;
  for (int k = lane; k < (int)gridDim.x; k += 32) {
    const float ov = __ldcg(&ctl->slot_val[k]);
    const int oi = __ldcg(&ctl->slot_idx[k]);
    if (ov > b || (ov == b && oi < ix)) { b = ov; ix = oi; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_down_sync(0xffffffffu, b, o);
    const int oi = __shfl_down_sync(0xffffffffu, ix, o);
    if (ov > b || (ov == b && oi < ix)) { b = ov; ix = oi; }
  }
  if (lane == 0) {
    const int step = __ldcg(&ctl->step);
    const int np = __ldcg(&ctl->n_prompt);
    ctl->token = (step + 1 < np) ? __ldcg(ctl->prompt + step + 1) : ix;
    if (ctl->ids) ctl->ids[step] = ix;
    ctl->step = step + 1;
    ctl->pos = __ldcg(&ctl->pos) + 1;
  }
}

template <bool F32S, int E, int EH, int W>
__global__ void __launch_bounds__(256, 1) k_decode(DecodeArgs d) {
  typedef DGeo<F32S> Gm;
  IssueCtx* ic = issue_ctx();
  unsigned char* ring = dsm + ISSUE_BYTES;
  float* xreg = reinterpret_cast<float*>(ring + (size_t)d.ds * Gm::STAGE);
  uint64_t* full = reinterpret_cast<uint64_t*>(xreg + ((d.xregion + 1) & ~1));
  __shared__ float red[16];
  __shared__ float bestv[8];
  __shared__ int besti[8];
  __shared__ int abort_flag;
  // this CTA's weight-stream schedule into shared memory
  {
    const uint4* src = reinterpret_cast<const uint4*>(d.sched + (size_t)blockIdx.x * d.ngemv);
    uint4* dst = reinterpret_cast<uint4*>(dsm + d.sched_off);
    for (int i = threadIdx.x; i < d.ngemv * (int)(sizeof(GemvSched) / 16); i += blockDim.x) dst[i] = __ldg(src + i);
    const int spt = __ldg(d.spt + blockIdx.x);
    const uint4* ms = reinterpret_cast<const uint4*>(d.sdesc + (size_t)blockIdx.x * d.spt_max);
    uint4* md = reinterpret_cast<uint4*>(dsm + d.desc_off);
    for (int i = threadIdx.x; i < spt; i += blockDim.x) md[i] = __ldg(ms + i);
    if (threadIdx.x == 0) {
      ic->pol = l2_evict_first();
      ic->arena = d.arena;
      ic->spt = (unsigned)spt;
      ic->total = (unsigned)spt * (unsigned)d.ntok;
      ic->ds = (unsigned)d.ds;
      ic->ngemv = (unsigned)d.ngemv;
      for (int i = 0; i < MAX_DS; i++) { ic->cnt[i] = 0; ic->issued[i] = 0; }
      ic->sched_s = smem_u32(dsm + d.sched_off);
      ic->desc_s = smem_u32(dsm + d.desc_off);
      for (int i = 0; i < d.ds; i++) mbar_init(&full[i], 1);
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      abort_flag = 0;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && ic->spt > 0)
    for (unsigned i = 0; i < (unsigned)d.ds && i < ic->total; i++) issue_stage<F32S>(i % ic->spt, i, i, ring, full);
  const unsigned G = gridDim.x;
  // the position advances by one per token (argmax phase), so it is read once
  const int pos0 = __ldcg(&d.ctl->pos);
  unsigned it = 0;
  bool stop = false;
  for (int tok = 0; tok < d.ntok && !stop; tok++) {
    for (int p = 0; p < d.nphase; p++) {
      const unsigned q = (unsigned)(tok * d.nphase + p);
      tmark(d, tok, p, 0);
      const Phase& ph = d.phases[p];
      const int kind = ph.kind;
      // a GEMV phase takes the grid barrier inside its prologue, once the
      // loads that do not depend on the previous phase are in flight (the
      // trace's mark 1 then precedes the barrier)
      if (kind != PH_GEMV) {
        if (q > 0) {
          if (threadIdx.x == 0 && !abort_flag && !grid_wait(d.bar, G * q)) { abort_flag = 1; atomicCAS(d.err, 0, 3); }
          csync<1>();
        }
        if (abort_flag) { stop = true; break; }   // every thread leaves here together
      }
      tmark(d, tok, p, 1);
      unsigned long long* tm2 = (d.trace && tok == 0) ? d.trace + ((size_t)blockIdx.x * d.nphase + p) * 8 + 2 : nullptr;
      if (kind == PH_GEMV) {
        const GridWait gw = {d.bar, G * q, &abort_flag, d.err};
        const GridWait* gwp = q > 0 ? &gw : nullptr;
        const int epi = ph.epi, pos = pos0 + tok;
        if (epi == EPI_SILU)
          it = gemv_phase<F32S, EPI_SILU, EH, W>(d, ph, ring, xreg, full, it, red, bestv, besti, &abort_flag, tm2, gwp, pos);
        else if (epi == EPI_ARGMAX)
          it = gemv_phase<F32S, EPI_ARGMAX, EH, W>(d, ph, ring, xreg, full, it, red, bestv, besti, &abort_flag, tm2, gwp, pos);
        else
          it = gemv_phase<F32S, EPI_BF16, EH, W>(d, ph, ring, xreg, full, it, red, bestv, besti, &abort_flag, tm2, gwp, pos);
      } else if (kind == PH_SCORE) {
        attn_score_phase<E>(ph.at, pos0 + tok, xreg);
      } else if (kind == PH_SOFTMAX) {
        attn_softmax_phase(ph.at, pos0 + tok, red);
      } else if (kind == PH_PV) {
        attn_pv_phase<E>(ph.at, pos0 + tok, xreg, d.pv_per_warp);
      } else {
        if (blockIdx.x == 0 && threadIdx.x < 32) argmax_phase(d);
      }
      tmark(d, tok, p, 3);
      // every thread's writes of this phase are issued: publish them. The
      // CTA barrier orders them before thread 0's arrival, and the arrival is
      // a release add at GPU scope, which makes them visible to every CTA
      // that acquires the counter (no separate full fence: it cost about
      // 0.5 us per phase)
      csync<1>();
      if (threadIdx.x == 0) grid_arrive(d.bar);
      if (abort_flag) { stop = true; break; }     // read after the barrier: the same value on every thread
      tmark(d, tok, p, 4);
    }
  }
  // never leave with copies in flight: each slot's last issued stage must
  // have landed (bounded); every issue happened before the barrier above
  if (threadIdx.x == 0) {
    for (int i = 0; i < d.ds; i++) {
      const unsigned s1 = ic->issued[i];
      if (!s1) continue;
      const unsigned par = ((s1 - 1) / (unsigned)d.ds) & 1;
      unsigned n = 0;
      while (!mbar_try(&full[i], par) && n < PB_WAIT_LIMIT) { n++; if (n > 64) __nanosleep(32); }
    }
  }
}

}  // namespace
