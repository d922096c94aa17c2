// pb_decode.cuh -- the persistent decode kernel: every phase of a token (each
// fused GEMV, each attention layer, the greedy argmax), for any number of
// tokens, in ONE cooperative launch with one CTA of 16 warps per SM.
//
// Weight stream: the CTA's row slice of every GEMV of every token is a fixed
// sequence of stages (16 segments of 2048 codes + their scales), known before
// the launch (host-built schedule: per CTA and GEMV its rows and first stage,
// and one descriptor per stage). Stages flow through a ring of DS shared-memory
// slots filled by 1-D TMA bulk copies (cp.async.bulk ... complete_tx on the
// slot's mbarrier). There is no producer warp: the warp that is the last of
// the sixteen to finish reading a slot (a shared counter) issues the copy of
// the stage DS places ahead into it. Weights never depend on activations, so
// the stream runs ahead across phases: while the warps wait for a phase's
// input, compute a prologue or run attention, the next GEMV's stages land.
//
// Stage loop: warp (g, c) consumes rows 2g and 2g+1 of chunk c of every
// stage (two 2048-code segments), in the reference's reduction order, with the
// FMA chains of a lane's two blocks (l and l+32) packed into one fma.rn.f32x2
// (each half is an IEEE fma, so the values are unchanged).
//
// Phase hand-off without an arrival counter: every activation vector that one
// phase produces and the next consumes is stored as TAGGED words (the bf16
// value in the low half, the low 16 bits of the producing phase's sequence
// number in the high half; attention scores as fp32 bits with the full
// sequence number in a 64-bit word), each a single-copy-atomic store at GPU
// scope. A consumer polls exactly the words it needs until every tag is the
// producer's, so readiness and data arrive in one L2 round trip. The residual
// stream never leaves the CTA: every CTA computes it in its prologues anyway
// and keeps its own copy in shared memory. The only grid-wide barrier is the
// one per token after the head (a release add and acquire polls on one
// counter): it publishes the per-CTA argmax slots, the KV rows and the conv
// ring slot that later tokens read, and every CTA then reduces the argmax
// slots itself.
//
// Attention (k_attn_head's arithmetic, lfm3_nanode.cu:503-602) runs as two
// phases: SCORE over the whole grid, one warp per (head, 32 positions), the
// lane of a position replaying the reference's 32 lane chains and shuffle tree
// in registers; then P.V on NH * 4 CTAs, one (head, quarter of the head dims)
// each: the V slice is prefetched into shared memory by asynchronous copies
// while the head's scores arrive, the softmax runs on 256 threads exactly as
// the reference's block does, and the (segment, dim) chains, the segment
// combine and the sigmoid gate follow.
//
// All spin waits are bounded: on a timeout the kernel records an error code,
// every warp leaves at the next phase boundary, and thread 0 waits (bounded)
// for the copies still in flight before the CTA exits; the host reports the
// error.
#pragma once
#include "pb_step.cuh"
#include <type_traits>

namespace {

constexpr int PH_GEMV = 0, PH_SCORE = 1, PH_PV = 2;
constexpr int DTHREADS = 256, DWARPS = 8;
constexpr int DSEGS = 16;                      // 2048-byte segments per stage (two per warp)
constexpr int STAGE_CODES = DSEGS * 2048;      // 32 KB
constexpr unsigned PB_POLL_LIMIT = 1u << 22;   // tagged-word polls before a wait gives up

// One phase of the token. GEMV: a fused prologue producing the GEMV input x
// (fp32 values of bf16 numbers) in shared memory, the weight stream, and a
// fused epilogue. SCORE / PV: the two attention phases.
struct DPhase {
  int kind;            // PH_GEMV or PH_ATTN
  int pro, epi;        // GEMV prologue (PRO_*) and epilogue (EPI_*)
  int N, K, nch;       // GEMV rows, input length, 2048-code segments per row
  int one;             // one-chunk rows (K not a multiple of 2048): lane chains
                       // run on over the segments; the row values region then
                       // holds (dot_lo, dot_hi, s_lo, s_hi) per segment and lane
  int gidx;            // index in the per-CTA GEMV schedule
  int rowoff;          // float offset of the row values in the activation region
  int H;
  float eps;
  const uint32_t* tin; // tagged input: the previous phase's output
  uint32_t* tout;      // tagged output (EPI_BF16, EPI_SILU, PV)
  unsigned long long* tsc;   // SCORE output / PV input: [NH][max_ctx] tagged scores
  float* fout;         // fp32 logits (EPI_ARGMAX)
  const float* wpost;  // ADDNORM: post-norm weight of the input vector
  const float* wnorm;  // norm that gives x from the residual
  bf16_t* rout;        // the residual, written by CTA 0 (null: not written)
  bf16_t* ring;        // CONV: [W][H], slot = position mod W
  const float* taps;   // CONV: [H][W]
  const uint4* emb_codes;   // EMBED: tied table, streaming layout
  const void* emb_scales;
  int emb_nch, emb_f32;
  const uint16_t* emb16;    // EMBED: the bf16 table (head layout) instead
  int b16;             // GEMV over the bf16 table (the dtype-3 head): 8 rows per stage
  AttnArgs at;         // SCORE, PV
};

// one CTA's share of one GEMV: rows [r0, r1)
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
  const DPhase* phases;
  int nphase;
  int ntok;
  unsigned qbase;      // sequence number of the launch's first phase (tags continue across launches)
  Ctl* ctl;
  unsigned* bar;       // per-token arrival counter (zeroed before the launch)
  int* err;            // 0, or the code of the wait that gave up
  int xregion;         // floats of the activation region in shared memory
  int nh;              // attention heads
  int ds;              // ring stages
  unsigned long long* trace;   // optional: per (CTA, phase) globaltimer marks of token 0
  const GemvSched* sched;      // [CTA][ngemv]
  const StageDesc* sdesc;      // [CTA][spt_max]: the stages of a token
  const int* spt;              // [CTA]: stages per token
  const char* arena;           // the model's weight arena
  int ngemv, spt_max;
  int sched_off, desc_off;     // byte offsets of the tables in dynamic shared memory
  int res_off;                 // byte offset of the CTA's residual copy (bf16 [H])
};

PB_DEV unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// trace marks: 0 phase entered, 1 prologue done (input arrived and x built),
// 2 thread 0's input poll ended (GEMV), 3 work done, 4 phase left; in a build with PB_TRACE_STAGE_LOOP defined, GEMV
// phases add warp 0's stage-loop totals: 5 slot releases with their refill
// issues, 6 waits for stage data, 7 chain and tree arithmetic
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
PB_DEV void dsync() { asm volatile("bar.sync 0;" ::: "memory"); }   // all warps of the CTA

// ---------------------------------------------------------- tagged words
PB_DEV void st_tag(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
PB_DEV uint4 ld_tag4(const uint32_t* p) {
  uint4 r;
  asm volatile("ld.relaxed.gpu.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p) : "memory");
  return r;
}
PB_DEV uint2 ld_tag2(const uint32_t* p) {
  uint2 r;
  asm volatile("ld.relaxed.gpu.global.v2.u32 {%0, %1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p) : "memory");
  return r;
}
PB_DEV uint32_t ld_tag1(const uint32_t* p) {
  uint32_t r;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(r) : "l"(p) : "memory");
  return r;
}
PB_DEV int ld_relaxed_int(const int* p) {
  int r;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(r) : "l"(p) : "memory");
  return r;
}

struct PollCtx {
  volatile int* abort;  // the CTA's abort flag (shared memory)
  int* err;             // the launch's error word
};
// N words from p (N a multiple of 4 and p 16-byte aligned, or N = 1, 2),
// polled until every word carries tag tw (in its high half). false: the wait
// gave up (poll limit, or a failure reported elsewhere); the caller raises
// the abort flag and still meets every barrier of the phase.
template <int N>
PB_DEV bool poll_words(const uint32_t* p, uint32_t tw, uint32_t (&w)[N], const PollCtx& pc) {
  for (unsigned i = 0;; i++) {
    if (N == 1) {
      w[0] = ld_tag1(p);
    } else if (N == 2) {
      const uint2 v = ld_tag2(p);
      w[0] = v.x; w[1 % N] = v.y;
    } else {
#pragma unroll
      for (int v = 0; v < N / 4; v++) {
        const uint4 q = ld_tag4(p + 4 * v);
        w[4 * v] = q.x; w[(4 * v + 1) % N] = q.y; w[(4 * v + 2) % N] = q.z; w[(4 * v + 3) % N] = q.w;
      }
    }
    uint32_t bad = 0;
#pragma unroll
    for (int j = 0; j < N; j++) bad |= w[j] ^ tw;
    if (bad < 0x10000u) return true;
    if (i >= PB_POLL_LIMIT) return false;
    if ((i & 255) == 255 && (*pc.abort || ld_relaxed_int(pc.err))) return false;
  }
}
PB_DEV void poll_fail(const PollCtx& pc, int code) {
  *pc.abort = 1;
  atomicCAS(pc.err, 0, code);
}
PB_DEV uint32_t tagged(uint32_t tw, float v) { return tw | (uint32_t)pb_f2bf(v); }

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
// the two block dots of lane l (blocks l and l+32 of the segment)
PB_DEV void dots2(const uint4 (&q)[4], const f2x (&xr)[32], float& d0, float& d1) {
  f2x d = pk(0.0f, 0.0f);
  d = dot16x2(q[0], q[2], xr, d);
  d = dot16x2(q[1], q[3], xr + 16, d);
  upk(d, d0, d1);
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
  if (dsc.w) bulk_g2s(ring + (size_t)slot * Gm::STAGE + STAGE_CODES, arena + (size_t)dsc.y * 16, dsc.w, &full[slot], pol);
  ic->issued[slot] = S + 1;
}
// arrival of a warp that finished reading a slot; true for the last of the 8
PB_DEV bool slot_release(unsigned slot) {
  unsigned old;
  asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
               : "=r"(old) : "r"(smem_u32(&issue_ctx()->cnt[slot])) : "memory");
  return old == (unsigned)(DWARPS - 1);
}

// ---------------------------------------------------------------- prologues
// All prologues run on the 256 threads and write the GEMV input x (fp32
// values of bf16 numbers) into sx, padded (element i at padx(i)), ending
// before the caller's CTA barrier. The RMS norms keep the reference's
// 256-thread reduction tree (rmsnorm_body, lfm3_nanode.cu:383-440), with
// E = H/256 elements per thread.

// residual (embedding row, or the CTA's residual copy + the post-normalised
// input vector) -> the CTA's residual copy (and the global one when rout) ->
// norm -> x.
// trace mark 2 of a GEMV phase: thread 0's input poll ended
PB_DEV void mark_input(unsigned long long* tm2) {
  if (tm2 && threadIdx.x == 0) tm2[0] = gtime();
}

template <int E>
PB_DEV void dpro_residual(const DPhase& ph, float* sx, bf16_t* res_s, float* red, uint32_t tw, int tok_id,
                          const PollCtx& pc, unsigned long long* tm2) {
  const int t = threadIdx.x;
  const int H = ph.H;
  const float eps = ph.eps;
  const bool embed = ph.pro == PRO_EMBED;
  float wp[E], wn[E], R[E];
  if (!embed) ld_f32<E>(ph.wpost + (size_t)t * E, wp);
  ld_f32<E>(ph.wnorm + (size_t)t * E, wn);
  if (embed) {
    // the token's row of the tied table
#pragma unroll
    for (int j = 0; j < E; j++)
      R[j] = emb_value(ph.emb_codes, ph.emb_scales, ph.emb_nch, ph.emb_f32, ph.emb16, H, tok_id, t * E + j);
  } else {
    uint32_t w[E];
    if (!poll_words<E>(ph.tin + (size_t)t * E, tw, w, pc)) poll_fail(pc, 4);
    mark_input(tm2);
    float Hv[E], hn[E];
#pragma unroll
    for (int j = 0; j < E; j++) Hv[j] = pb_lo2f(w[j]);
    rms_reg<E, 1>(Hv, wp, hn, H, eps, red);
#pragma unroll
    for (int j = 0; j < E; j++) R[j] = pb_bf2f(pb_f2bf(__fadd_rn(pb_bf2f(res_s[t * E + j]), hn[j])));
  }
#pragma unroll
  for (int j = 0; j < E; j++) res_s[t * E + j] = pb_f2bf(R[j]);
  if (ph.rout && blockIdx.x == 0) st_bf<E>(ph.rout + (size_t)t * E, R);
  float X[E];
  rms_reg<E, 1>(R, wn, X, H, eps, red + 8);
#pragma unroll
  for (int j = 0; j < E; j++) sx[padx(t * E + j)] = X[j];
}

// gated short conv (lfm3_nanode.cu:3790-3818): bx = bf16(B*x) enters the ring
// as the newest slot; y = sum_k taps[i][k] * ring_k (oldest first), one fp32
// chain; out = bf16(C * bf16(y)). The W-1 older slots hold positions of
// earlier tokens (published by the per-token barrier); the slot of position
// pos held pos - W, which no CTA reads any more, and CTA 0 writes the new value
// there. E = H/256 channels per thread.
template <int E, int W>
PB_DEV void dpro_conv(const DPhase& ph, float* sx, uint32_t tw, int pos, const PollCtx& pc,
                      unsigned long long* tm2) {
  const int t = threadIdx.x, H = ph.H;
  bf16_t* ring = ph.ring;
  float tp[E * W];
  ld_f32<E * W>(ph.taps + (size_t)t * E * W, tp);
  float rg[W - 1][E];
#pragma unroll
  for (int k = 0; k < W - 1; k++) {
    const int p = pos - (W - 1) + k;
    ld_bf<E, 1>(ring + (size_t)(((p % W) + W) % W) * H + (size_t)t * E, rg[k]);
  }
  uint32_t wB[E], wC[E], wX[E];
  bool ok = poll_words<E>(ph.tin + (size_t)t * E, tw, wB, pc);
  ok = ok && poll_words<E>(ph.tin + H + (size_t)t * E, tw, wC, pc);
  ok = ok && poll_words<E>(ph.tin + 2 * H + (size_t)t * E, tw, wX, pc);
  if (!ok) poll_fail(pc, 4);
  mark_input(tm2);
  float bx[E];
#pragma unroll
  for (int j = 0; j < E; j++) {
    bx[j] = pb_bf2f(pb_f2bf(__fmul_rn(pb_lo2f(wB[j]), pb_lo2f(wX[j]))));
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < W; k++) acc = __fadd_rn(acc, __fmul_rn(tp[j * W + k], k == W - 1 ? bx[j] : rg[k][j]));
    sx[padx(t * E + j)] = pb_bf2f(pb_f2bf(__fmul_rn(pb_lo2f(wC[j]), pb_bf2f(pb_f2bf(acc)))));
  }
  if (blockIdx.x == 0) st_bf<E>(ring + (size_t)(pos % W) * H + (size_t)t * E, bx);
}

// plain input: 256 EK values staged, EK per thread: the K tagged values,
// then zeros (a one-chunk tensor's padding; K is a multiple of 32, so a
// thread's EK values are all inside or all past it)
template <int EK>
PB_DEV void dpro_plain(const DPhase& ph, float* sx, uint32_t tw, const PollCtx& pc, unsigned long long* tm2) {
  const int t = threadIdx.x;
  uint32_t w[EK];
  if (t * EK < ph.K) {
    if (!poll_words<EK>(ph.tin + (size_t)t * EK, tw, w, pc)) poll_fail(pc, 4);
  } else {
#pragma unroll
    for (int j = 0; j < EK; j++) w[j] = 0u;   // bf16 +0
  }
  mark_input(tm2);
#pragma unroll
  for (int j = 0; j < EK; j++) sx[padx(t * EK + j)] = pb_lo2f(w[j]);
}

// ------------------------------------------------------------- GEMV phase
// The stage loop only waits, computes each row's chunk value (the lane chains
// and the shuffle-down tree) and parks it in shared memory (rowv, [local row]
// [chunk]); after one CTA barrier the 256 threads combine the chunks in order
// and run the epilogue for all of the CTA's rows at once. A wait that gives up
// breaks out of the loop and the phase still ends with the same barriers as
// on the other warps.
// EXT: the build that also takes one-chunk rows and the bf16 head (a model
// without them runs the build that compiles them out)
template <bool F32S, int EH, int W, bool EXT>
__device__ __forceinline__ unsigned gemv_phase(const DecodeArgs& d, const DPhase& ph, unsigned char* ring,
                                               float* xreg, bf16_t* res_s, uint64_t* full, unsigned it,
                                               float* red, float* bestv, int* besti, volatile int* abort_flag,
                                               unsigned long long* tm2, uint32_t tw_in, uint32_t tw_out, int pos,
                                               int tok_id) {
  typedef DGeo<F32S> Gm;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* sx = xreg;
  {
    const PollCtx pc = {abort_flag, d.err};
    const int pro = ph.pro;
    if (pro == PRO_EMBED || pro == PRO_ADDNORM) {
      dpro_residual<EH>(ph, sx, res_s, red, tw_in, tok_id, pc, tm2);
    } else if (pro == PRO_CONV) {
      dpro_conv<EH, W>(ph, sx, tw_in, pos, pc, tm2);
    } else {
      switch (pb_kpad(ph.K) >> 8) {
        case 8: dpro_plain<8>(ph, sx, tw_in, pc, tm2); break;
        case 16: dpro_plain<16>(ph, sx, tw_in, pc, tm2); break;
        case 32: dpro_plain<32>(ph, sx, tw_in, pc, tm2); break;
        default: break;   // other K: the host keeps this kernel off
      }
    }
  }
  dsync();
  if (tm2 && threadIdx.x == 0) tm2[-1] = gtime();    // mark 1: prologue done
  // the few fields the stage loop needs, read once into registers
  const int nch = ph.nch, RB = DSEGS / nch;
  float* const rowv = xreg + ph.rowoff;
  const int c = warp % nch, g = warp / nch;
  const unsigned ds = (unsigned)d.ds;
  f2x xr[32];
  if (EXT && ph.b16) {
    // the bf16 head's lane chain: x[l + 32 m], m = 0..63, in pairs
#pragma unroll
    for (int j = 0; j < 32; j++) xr[j] = pk(sx[lane + 33 * (2 * j)], sx[lane + 33 * (2 * j + 1)]);
  } else {
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
  // the stage loop, compiled once per row kind so that the common one carries
  // no per-stage test: 0 chunked rows, 1 one-chunk rows, 2 the bf16 head
  auto stage_loop = [&](auto mode) {
    constexpr int MODE = decltype(mode)::value;
    for (int r = r0; r < r1; r += RB) {
#ifdef PB_TRACE_STAGE_LOOP
      const unsigned long long tw0 = (tm2 && threadIdx.x == 0) ? gtime() : 0;
#endif
      if (!mbar_wait(&full[slot], par, abort_flag)) {
        *abort_flag = 1;
        atomicCAS(d.err, 0, 2);
        break;
      }
#ifdef PB_TRACE_STAGE_LOOP
      if (tm2 && threadIdx.x == 0) tm2[4] += gtime() - tw0;
#endif
      const unsigned char* st = ring + (size_t)slot * Gm::STAGE;
      if constexpr (MODE == 2) {
        // bf16 head (k_gemv_bf16, lfm3_nanode.cu:3517-3534): warp w takes row
        // r + w of the stage's 8 (4 KB each, head layout); lane l's chain over
        // k = l + 32 m is s = s + bf16(W[k]) * x[k], products and sums rounded
        // apart; the shuffle-down tree gives the logit as is
        const bool live = r + warp < r1;
        const uint4* gp = reinterpret_cast<const uint4*>(st + (size_t)warp * 4096) + lane;
        uint4 qb[8];
#pragma unroll
        for (int h = 0; h < 8; h++) qb[h] = live ? gp[32 * h] : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int h = 0; h < 8; h++) asm volatile("" ::"r"(qb[h].x), "r"(qb[h].y), "r"(qb[h].z), "r"(qb[h].w));
        __syncwarp();
        if (lane == 0 && slot_release(slot)) {
          issue_ctx()->cnt[slot] = 0;
          if (it + ds < total) issue_stage<F32S>(kn, slot, it + ds, ring, full);
        }
        float acc = 0.0f;
#pragma unroll
        for (int h = 0; h < 8; h++) {
          const unsigned ws[4] = {qb[h].x, qb[h].y, qb[h].z, qb[h].w};
#pragma unroll
          for (int i = 0; i < 4; i++) {
            float xa, xb;
            upk(xr[4 * h + i], xa, xb);
            acc = __fadd_rn(acc, __fmul_rn(pb_lo2f(ws[i]), xa));
            acc = __fadd_rn(acc, __fmul_rn(pb_hi2f(ws[i]), xb));
          }
        }
        const float v = pb_warp_tree(acc);
        if (lane == 0 && live) rowv[(r - r0 + warp) * nch] = v;
        it++;
        if (++slot == ds) { slot = 0; par ^= 1; }
        if (++kn == spt) kn = 0;
        continue;
      }
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
      const unsigned long long tr0 = (tm2 && threadIdx.x == 0) ? gtime() : 0;
#endif
      if (lane == 0 && slot_release(slot)) {
        issue_ctx()->cnt[slot] = 0;
        if (it + ds < total) issue_stage<F32S>(kn, slot, it + ds, ring, full);
      }
#ifdef PB_TRACE_STAGE_LOOP
      const unsigned long long tr1 = (tm2 && threadIdx.x == 0) ? gtime() : 0;
#endif
      if constexpr (MODE == 1) {
        // park this lane's two block dots and scales per (row, segment)
        float4* rq = reinterpret_cast<float4*>(rowv);
#pragma unroll
        for (int u = 0; u < 2; u++) {
          float d0, d1;
          dots2(q[u], xr, d0, d1);
          const int lr = r - r0 + g * 2 + u;
          if (r + g * 2 + u < r1) rq[(lr * nch + c) * 32 + lane] = make_float4(d0, d1, slo[u], shi[u]);
        }
        it++;
        if (++slot == ds) { slot = 0; par ^= 1; }
        if (++kn == spt) kn = 0;
        continue;
      }
      float v[2];
#pragma unroll
      for (int u = 0; u < 2; u++) v[u] = pb_warp_tree(leaf2(q[u], slo[u], shi[u], xr));
#ifdef PB_TRACE_STAGE_LOOP
      if (tm2 && threadIdx.x == 0) {
        asm volatile("" ::"f"(v[0]), "f"(v[1]));
        tm2[3] += tr1 - tr0;            // slot 5: release (+ refill issue) of warp 0
        tm2[5] += gtime() - tr1;        // slot 7: chains and trees of warp 0
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
  };
  if constexpr (EXT) {
    if (ph.b16) stage_loop(std::integral_constant<int, 2>{});
    else if (ph.one) stage_loop(std::integral_constant<int, 1>{});
    else stage_loop(std::integral_constant<int, 0>{});
  } else {
    stage_loop(std::integral_constant<int, 0>{});
  }
  dsync();
  // epilogue over the CTA's rows: chunk values added in chunk order from 0
  const int nr = r1 - r0;
  if (EXT && ph.one) {
    // one-chunk rows (bf16 output only): a warp per row chains every lane's
    // blocks l, l+32, l+64, ... in order, then the tree; the chunk sum is 0 + v
    const float4* rq = reinterpret_cast<const float4*>(rowv);
    for (int i = warp; i < nr; i += DWARPS) {
      float acc = 0.0f;
      for (int cc = 0; cc < nch; cc++) {
        const float4 pv = rq[(i * nch + cc) * 32 + lane];
        acc = __fmaf_rn(pv.z, pv.x, acc);
        acc = __fmaf_rn(pv.w, pv.y, acc);
      }
      const float v = pb_warp_tree(acc);
      if (lane == 0) st_tag(ph.tout + r0 + i, tagged(tw_out, __fadd_rn(0.0f, v)));
    }
  } else if (ph.epi == EPI_SILU) {
    // rows 2i (w1) and 2i+1 (w3): k_silu_mul_bf, lfm3_nanode.cu:821-829
    uint32_t* out = ph.tout;
    for (int i = 2 * threadIdx.x; i + 1 < nr; i += 2 * DTHREADS) {
      float o0 = 0.0f, o1 = 0.0f;
      for (int cc = 0; cc < nch; cc++) {
        o0 = __fadd_rn(o0, rowv[i * nch + cc]);
        o1 = __fadd_rn(o1, rowv[(i + 1) * nch + cc]);
      }
      const float av = pb_bf2f(pb_f2bf(o0)), bw = pb_bf2f(pb_f2bf(o1));
      st_tag(out + ((r0 + i) >> 1), tagged(tw_out, __fmul_rn(__fmul_rn(av, pb_sigmoid(av)), bw)));
    }
  } else if (ph.epi == EPI_BF16) {
    uint32_t* out = ph.tout;
    for (int i = threadIdx.x; i < nr; i += DTHREADS) {
      float o = 0.0f;
      for (int cc = 0; cc < nch; cc++) o = __fadd_rn(o, rowv[i * nch + cc]);
      st_tag(out + r0 + i, tagged(tw_out, o));
    }
  } else {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    float* out = ph.fout;
    for (int i = threadIdx.x; i < nr; i += DTHREADS) {
      float o = 0.0f;
      if (EXT && ph.b16) o = rowv[i * nch];    // the bf16 head's logit is the tree's value
      else
        for (int cc = 0; cc < nch; cc++) o = __fadd_rn(o, rowv[i * nch + cc]);
      out[r0 + i] = o;
      if (o > bv || (o == bv && r0 + i < bi)) { bv = o; bi = r0 + i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_down_sync(0xffffffffu, bv, o);
      const int oi = __shfl_down_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { bestv[warp] = bv; besti[warp] = bi; }
    dsync();
    if (threadIdx.x == 0) {
      float b = bestv[0];
      int ix = besti[0];
      for (int w = 1; w < DWARPS; w++)
        if (bestv[w] > b || (bestv[w] == b && besti[w] < ix)) { b = bestv[w]; ix = besti[w]; }
      Ctl* ctl = ph.at.ctl;
      ctl->slot_val[blockIdx.x] = b;
      ctl->slot_idx[blockIdx.x] = ix;
    }
  }
  return it;
}

// ------------------------------------------------------------- attention
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

PB_DEV void cp_async16(void* sdst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(sdst)), "l"(gsrc) : "memory");
}
PB_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
PB_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
PB_DEV void st_score(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
PB_DEV unsigned long long ld_score(const unsigned long long* p) {
  unsigned long long r;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(r) : "l"(p) : "memory");
  return r;
}

// SCORE: task = (head, 32 positions), one warp; lane p forms the score of
// position p alone: its 32 per-lane chains (((0 + q0k0) + q1k1) ...) over E
// dims and then the shuffle-down tree's additions, replayed in registers;
// * scaling. The head's q and k (tagged words of the first GEMV) get the head
// norm and RoPE in the warp (per task); the current position's k is used from
// there, and the task holding position pos for a group's first head appends
// the new fp16 k/v row to the cache. Scores go out as (sequence number << 32 |
// fp32 bits). wsm: 2 HD floats per warp.
template <int E>
__device__ __noinline__ void score_phase(const DPhase& ph, int pos, float* wsm, uint32_t tw_in,
                                         unsigned long long tq, volatile int* abort_flag, int* err) {
  constexpr int HD = 32 * E;
  const AttnArgs& a = ph.at;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * DWARPS + warp, GW = gridDim.x * DWARPS;
  const int nh = a.nh, nkv = a.nkv, grp = nh / nkv, half = a.half;
  const int npos = pos + 1;
  const int lo = (a.win > 0 && npos > a.win) ? npos - a.win : 0;
  const int np = npos - lo, nblk = (np + 31) / 32, ntask = nh * nblk;
  const float scaling = a.scaling;
  float* qs = wsm + warp * 2 * HD;
  float* ks = qs + HD;
  const PollCtx pc = {abort_flag, err};
  const uint32_t* in = ph.tin;
  const size_t koff = (size_t)nh * HD, voff = koff + (size_t)nkv * HD;
  const size_t max_ctx = (size_t)a.max_ctx;
  // rope factors of this lane's elements: lanes >= 16 use those of i - HD/2
  const int ri = (lane & 15) * E;
  const float* cs = a.rope_cos + (size_t)pos * half;
  const float* sn = a.rope_sin + (size_t)pos * half;
  int cur = -1;
  for (int task = gw; task < ntask; task += GW) {
    const int h = task / nblk, pb = task - h * nblk, kvh = h / grp;
    const int p = lo + pb * 32 + lane;
    const bool writer = (h % grp == 0) && pos >= lo + pb * 32 && pos < lo + pb * 32 + 32;
    // the cached key row of this lane's position (an earlier token's) first
    uint4 kg[HD / 8];
    if (p < pos) {
      const uint4* kr = reinterpret_cast<const uint4*>(a.kc + ((size_t)p * nkv + kvh) * HD);
#pragma unroll
      for (int g = 0; g < HD / 8; g++) kg[g] = __ldcg(kr + g);
    }
    if (h != cur) {
      float qw[E], kw[E], c[E], sv[E];
#pragma unroll
      for (int j = 0; j < E; j++) {
        const int i = lane * E + j;
        qw[j] = __ldg(a.qnorm + i);
        kw[j] = __ldg(a.knorm + i);
        c[j] = ri + j < half ? __ldg(cs + ri + j) : 0.0f;
        sv[j] = ri + j < half ? __ldg(sn + ri + j) : 0.0f;
      }
      uint32_t wq[E], wk[E];
      bool ok = poll_words<E>(in + (size_t)h * HD + lane * E, tw_in, wq, pc);
      ok = ok && poll_words<E>(in + koff + (size_t)kvh * HD + lane * E, tw_in, wk, pc);
      if (!ok) poll_fail(pc, 5);
      float qx[E], kx[E];
#pragma unroll
      for (int j = 0; j < E; j++) { qx[j] = pb_lo2f(wq[j]); kx[j] = pb_lo2f(wk[j]); }
      __syncwarp();                       // previous task's reads of qs/ks are done
      norm_rope_regs<E>(qx, qw, c, sv, half, a.eps, qs);
      norm_rope_regs<E>(kx, kw, c, sv, half, a.eps, ks);
#pragma unroll
      for (int j = 0; j < E; j++) ks[lane * E + j] = pb_h2f(pb_f2h(ks[lane * E + j]));
      __syncwarp();
      cur = h;
    }
    if (writer) {
      uint32_t wv[E];
      if (!poll_words<E>(in + voff + (size_t)kvh * HD + lane * E, tw_in, wv, pc)) poll_fail(pc, 5);
      unsigned short* kd = a.kc + ((size_t)pos * nkv + kvh) * HD;
      unsigned short* vd = a.vc + ((size_t)pos * nkv + kvh) * HD;
#pragma unroll
      for (int j = 0; j < E; j++) {
        kd[lane * E + j] = pb_f2h(ks[lane * E + j]);
        vd[lane * E + j] = pb_f2h(pb_lo2f(wv[j]));
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
      st_score(ph.tsc + (size_t)h * max_ctx + (p - lo), tq | __float_as_uint(__fmul_rn(v[0], scaling)));
    }
  }
}

// dims of a P.V task: a quarter of the head
template <int E>
struct PvGeo {
  static constexpr int HD = 32 * E;
  static constexpr int DQ = HD / 4;        // dims per task
  static constexpr int CH = 32768 / (DQ * 2);   // positions per V chunk in shared memory (32 KB)
};

// P.V: CTA b < 4 NH takes head b/4 and dims [DQ (b%4), +DQ). The V slice of
// the window (earlier tokens' rows) is brought into shared memory by
// asynchronous copies, a chunk of CH positions at a time, the first while the
// head's scores arrive; the current position's v row comes from the first
// GEMV's tagged output. Softmax on the 256 threads as k_attn_head's block:
// max over the window, e = expf(s - m) in place, chain t over i = t, t+256, ...
// ascending, the warp shuffle-down trees and the 8-lane tree, inv = 1/sum. Then
// the chains of (segment, dim) over p = seg, seg+8, ... of (e_p * inv) * v_p,
// the segment combine ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7)), bf16, and the
// sigmoid gate (k_sigmoid_gate, :852-864): bf16(out * 1/(1+e^-g)).
template <int E>
__device__ __noinline__ void pv_phase(const DPhase& ph, int pos, float* xs, float* red, uint32_t tw_in,
                                      unsigned long long tq_sc, uint32_t tw_out, volatile int* abort_flag,
                                      int* err) {
  typedef PvGeo<E> P;
  constexpr int HD = P::HD, DQ = P::DQ, CH = P::CH;
  const AttnArgs& a = ph.at;
  const int b = blockIdx.x;
  if (b >= 4 * a.nh) return;
  const int h = b >> 2, dq = b & 3;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int nkv = a.nkv, grp = a.nh / nkv, kvh = h / grp;
  const int npos = pos + 1;
  const int lo = (a.win > 0 && npos > a.win) ? npos - a.win : 0;
  const int np = npos - lo;
  const size_t max_ctx = (size_t)a.max_ctx;
  unsigned short* vsm = reinterpret_cast<unsigned short*>(xs);    // [CH][DQ] fp16
  float* sc = xs + CH * DQ / 2;                                    // [np]
  float* segp = sc + ((np + 3) & ~3);                              // [8][DQ]
  float* vcur = segp + 8 * DQ;                                     // [DQ]
  float* gsig = vcur + DQ;                                         // [1]
  const PollCtx pc = {abort_flag, err};
  const size_t rowst = (size_t)nkv * HD;
  const unsigned short* vsrc = a.vc + (size_t)kvh * HD + dq * DQ;
  constexpr int G16 = DQ / 8;          // 16-byte pieces per V row slice
  // chunk 0 of the V slice: rows lo .. min(pos, lo + CH) - 1
  const int n0 = min(np - 1, CH);
  for (int k = t; k < n0 * G16; k += DTHREADS) {
    const int j = k / G16, gq = k - j * G16;
    cp_async16(vsm + j * DQ + gq * 8, vsrc + (size_t)(lo + j) * rowst + gq * 8);
  }
  cp_async_commit();
  const uint32_t* in = ph.tin;
  const size_t voff = (size_t)a.nh * HD + (size_t)nkv * HD, goff = voff + (size_t)nkv * HD;
  if (t < DQ) {
    uint32_t w[1];
    if (!poll_words<1>(in + voff + (size_t)kvh * HD + dq * DQ + t, tw_in, w, pc)) poll_fail(pc, 6);
    vcur[t] = pb_h2f(pb_f2h(pb_lo2f(w[0])));
  } else if (t == DQ) {
    uint32_t w[1];
    if (!poll_words<1>(in + goff + h, tw_in, w, pc)) poll_fail(pc, 6);
    gsig[0] = pb_sigmoid(pb_lo2f(w[0]));
  }
  // the head's scores
  const unsigned long long* scs = ph.tsc + (size_t)h * max_ctx;
  for (int i = t; i < np; i += DTHREADS) {
    unsigned long long v = 0;
    for (unsigned n = 0;; n++) {
      v = ld_score(scs + i);
      if ((v & 0xffffffff00000000ull) == tq_sc) break;
      if (n >= PB_POLL_LIMIT || ((n & 255) == 255 && (*abort_flag || ld_relaxed_int(err)))) {
        poll_fail(pc, 6);
        break;
      }
    }
    sc[i] = __uint_as_float((unsigned)v);
  }
  dsync();
  float m = -1e30f;
  for (int i = t; i < np; i += DTHREADS) m = fmaxf(m, sc[i]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane == 0) red[warp] = m;
  dsync();
  m = red[0];
#pragma unroll
  for (int w = 1; w < 8; w++) m = fmaxf(m, red[w]);
  m = fmaxf(-1e30f, m);
  float sum = 0.0f;
  for (int i = t; i < np; i += DTHREADS) {
    const float e = pb_expf(__fadd_rn(sc[i], -m));
    sc[i] = e;
    sum = __fadd_rn(sum, e);
  }
  sum = pb_warp_tree(sum);
  if (lane == 0) red[8 + warp] = sum;
  dsync();
  const float* Wp = red + 8;
  const float inv = __fdiv_rn(1.0f, __fadd_rn(__fadd_rn(__fadd_rn(Wp[0], Wp[4]), __fadd_rn(Wp[2], Wp[6])),
                                              __fadd_rn(__fadd_rn(Wp[1], Wp[5]), __fadd_rn(Wp[3], Wp[7]))));
  // (segment, dim) chains: 8 x DQ of them, thread t < 8 DQ
  constexpr int NCHAIN = 8 * DQ;
  const int seg = t / DQ, dd = t - seg * DQ;
  float acc = 0.0f;
  for (int c0 = 0; c0 < np - 1 || c0 == 0; c0 += CH) {
    const int cn = min(np - 1 - c0, CH);      // cached rows in this chunk
    if (c0 > 0) {
      dsync();                                 // the previous chunk's reads are done
      for (int k = t; k < cn * G16; k += DTHREADS) {
        const int j = k / G16, gq = k - j * G16;
        cp_async16(vsm + j * DQ + gq * 8, vsrc + (size_t)(lo + c0 + j) * rowst + gq * 8);
      }
      cp_async_commit();
    }
    cp_async_wait_all();
    dsync();
    if (t < NCHAIN) {
      // positions i = c0 + j with i = seg (mod 8), ascending
      int j0 = (seg - c0 % 8 + 8) % 8;
      for (int j = j0; j < cn; j += 8)
        acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(sc[c0 + j], inv), pb_h2f(vsm[j * DQ + dd])));
    }
    if (c0 + CH >= np - 1) break;
  }
  // the current position (i = np - 1) closes the chain of its segment
  if (t < NCHAIN && ((np - 1) & 7) == seg)
    acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(sc[np - 1], inv), vcur[dd]));
  if (t < NCHAIN) segp[seg * DQ + dd] = acc;
  dsync();
  if (t < DQ) {
    const float* r = segp + t;
    const float o = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[DQ]), __fadd_rn(r[2 * DQ], r[3 * DQ])),
                              __fadd_rn(__fadd_rn(r[4 * DQ], r[5 * DQ]), __fadd_rn(r[6 * DQ], r[7 * DQ])));
    st_tag(ph.tout + (size_t)h * HD + dq * DQ + t, tagged(tw_out, __fmul_rn(pb_bf2f(pb_f2bf(o)), gsig[0])));
  }
}

// greedy id from the per-CTA maxima (ties to the lowest index), by warp 0
PB_DEV int argmax_slots(const Ctl* ctl) {
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
  return __shfl_sync(0xffffffffu, ix, 0);
}

template <bool F32S, int E, int EH, int W, bool EXT>
__global__ void __launch_bounds__(DTHREADS, 1) k_decode(DecodeArgs d) {
  typedef DGeo<F32S> Gm;
  IssueCtx* ic = issue_ctx();
  unsigned char* ring = dsm + ISSUE_BYTES;
  float* xreg = reinterpret_cast<float*>(ring + (size_t)d.ds * Gm::STAGE);
  uint64_t* full = reinterpret_cast<uint64_t*>(xreg + ((d.xregion + 1) & ~1));
  bf16_t* res_s = reinterpret_cast<bf16_t*>(dsm + d.res_off);
  __shared__ float red[16];
  __shared__ float bestv[DWARPS];
  __shared__ int besti[DWARPS];
  __shared__ int abort_flag;
  __shared__ int s_tok;
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
      s_tok = __ldcg(&d.ctl->token);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && ic->spt > 0)
    for (unsigned i = 0; i < (unsigned)d.ds && i < ic->total; i++) issue_stage<F32S>(i % ic->spt, i, i, ring, full);
  const unsigned G = gridDim.x;
  Ctl* ctl = d.ctl;
  // the position advances by one per token, so it is read once; so are the
  // prompt (teacher-forced inputs) and the id output
  const int pos0 = __ldcg(&ctl->pos), step0 = __ldcg(&ctl->step), n_prompt = __ldcg(&ctl->n_prompt);
  const int* prompt = ctl->prompt;
  int* ids = ctl->ids;
  unsigned it = 0;
  bool stop = false;
  for (int tok = 0; tok < d.ntok && !stop; tok++) {
    const int pos = pos0 + tok;
    const int tok_id = s_tok;
    for (int p = 0; p < d.nphase; p++) {
      const unsigned q = d.qbase + (unsigned)(tok * d.nphase + p);
      const uint32_t tw_in = ((q - 1u) & 0xffffu) << 16, tw_out = (q & 0xffffu) << 16;
      tmark(d, tok, p, 0);
      const DPhase& ph = d.phases[p];
      unsigned long long* tm2 = (d.trace && tok == 0) ? d.trace + ((size_t)blockIdx.x * d.nphase + p) * 8 + 2 : nullptr;
      if (ph.kind == PH_GEMV) {
        it = gemv_phase<F32S, EH, W, EXT>(d, ph, ring, xreg, res_s, full, it, red, bestv, besti, &abort_flag, tm2,
                                     tw_in, tw_out, pos, tok_id);
      } else if (ph.kind == PH_SCORE) {
        score_phase<E>(ph, pos, xreg, tw_in, (unsigned long long)q << 32, &abort_flag, d.err);
      } else {
        pv_phase<E>(ph, pos, xreg, red, ((q - 2u) & 0xffffu) << 16, (unsigned long long)(q - 1u) << 32, tw_out,
                    &abort_flag, d.err);
      }
      tmark(d, tok, p, 3);
      dsync();      // the phase's shared-memory use ends; the abort flag is final
      if (abort_flag) { stop = true; break; }
      tmark(d, tok, p, 4);
    }
    if (stop) break;
    // token end: publish this token's writes (argmax slots, KV rows, ring
    // slot) and wait for every CTA; then every CTA reduces the argmax slots
    if (threadIdx.x == 0) {
      grid_arrive(d.bar);
      if (!grid_wait(d.bar, G * (unsigned)(tok + 1))) { abort_flag = 1; atomicCAS(d.err, 0, 3); }
    }
    dsync();
    if (abort_flag) break;
    if (threadIdx.x < 32) {
      const int ix = argmax_slots(ctl);
      const int step = step0 + tok;
      const int next = (step + 1 < n_prompt) ? __ldg(prompt + step + 1) : ix;
      if (threadIdx.x == 0) {
        s_tok = next;
        if (blockIdx.x == 0) {
          if (ids) ids[step] = ix;
          ctl->token = next;
          ctl->step = step + 1;
          ctl->pos = pos + 1;
        }
      }
    }
    dsync();
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
