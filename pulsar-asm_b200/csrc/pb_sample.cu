// pb_sample.cu -- the Bonsai decoder's sampler on the device: top-k -> min-p
// -> top-p on the raw logits, temperature last, then a softmax draw from a
// 64-bit LCG (sample_topkpp and frand01, pulsar_arm/bonsai2/fwd8.c:471-521),
// for B rows at once, each row with its own generator state (fwd8.c:736: every
// session draws from its own copy of the seeded stream). temp <= 0 is greedy:
// the first maximum (argmax, fwd8.c:465-469), and the state is not advanced.
//
// One CTA of 1024 threads per row:
//  1. a radix select (4 passes of 8 bits over an order-preserving uint32 key,
//     -0 keyed as +0 because the reference compares with <=) finds the k-th
//     largest key T;
//  2. every key above T, and the first keys equal to T in index order, are
//     compacted into shared memory;
//  3. a bitonic sort orders them by value descending, then index ascending:
//     the order the reference's insertion list builds (a later equal value
//     goes after the earlier ones, and a full list drops it);
//  4. the exponentials are evaluated in parallel; the double-precision running
//     sums, the top-p cut and the draw run on one thread in the reference's
//     order and rounding (float exp terms promoted to double).
// expf is pb_expf, as everywhere in this library (within about 1 ulp of the
// correctly rounded value; the reference calls the C library's expf on the
// host), logf(minp) is taken on the host with the C library. Rows holding a
// NaN get id -1 (the reference's insertion walk has no defined order for
// them) and keep their generator state.
#include "pb_internal.h"
#include "pb_common.cuh"

#include <cmath>

namespace {

constexpr int ST = 1024;     // threads per row
constexpr int KMAX = 1024;   // the reference's list length (fwd8.c:480-483)

__device__ __forceinline__ uint32_t skey(float v) {
  uint32_t u = __float_as_uint(v);
  if ((u << 1) == 0u) u = 0u;   // -0 keys as +0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

struct SampleArgs {
  const float* lg;
  long long ld;
  int n, topk, use_minp;
  float temp, topp, lminp;
  unsigned long long* rng;
  int* ids;
};

// block-wide exclusive scan of two counts (1024 threads)
__device__ __forceinline__ void scan2(int a, int b, int& xa, int& xb, int (*ws)[32]) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int ia = a, ib = b;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int ta = __shfl_up_sync(0xffffffffu, ia, o), tb = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) { ia += ta; ib += tb; }
  }
  if (lane == 31) { ws[0][w] = ia; ws[1][w] = ib; }
  __syncthreads();
  if (w == 0) {
    int va = ws[0][lane], vb = ws[1][lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int ta = __shfl_up_sync(0xffffffffu, va, o), tb = __shfl_up_sync(0xffffffffu, vb, o);
      if (lane >= o) { va += ta; vb += tb; }
    }
    ws[0][lane] = va;
    ws[1][lane] = vb;
  }
  __syncthreads();
  const int pa = w ? ws[0][w - 1] : 0, pb = w ? ws[1][w - 1] : 0;
  xa = pa + ia - a;
  xb = pb + ib - b;
}

__global__ void __launch_bounds__(ST) k_sample(SampleArgs a) {
  __shared__ unsigned long long cand[KMAX];   // (key << 32) | ~index
  __shared__ float e1[KMAX], e2[KMAX], sv[KMAX];
  __shared__ int si[KMAX];
  __shared__ unsigned hist[256];
  __shared__ int ws[2][32];
  __shared__ float wv[32];
  __shared__ int wi[32];
  __shared__ uint32_t s_prefix;
  __shared__ int s_rem;
  const int b = blockIdx.x, t = threadIdx.x, n = a.n, lane = t & 31, w = t >> 5;
  const float* lg = a.lg + (size_t)b * (size_t)a.ld;
  int nan = 0;
  if (a.temp <= 0.0f) {   // greedy: the first maximum
    float bv = -INFINITY;
    int bi = -1;
    for (int i0 = t; i0 < n; i0 += 8 * ST) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) v[u] = i0 + u * ST < n ? lg[i0 + u * ST] : 0.0f;
#pragma unroll
      for (int u = 0; u < 8; u++) {   // increasing index: the first maximum stays
        if (i0 + u * ST >= n) break;
        if (v[u] != v[u]) nan = 1;
        if (bi < 0 || v[u] > bv) { bv = v[u]; bi = i0 + u * ST; }
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_down_sync(0xffffffffu, bv, o);
      const int oi = __shfl_down_sync(0xffffffffu, bi, o);
      if (oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
    }
    if (lane == 0) { wv[w] = bv; wi[w] = bi; }
    nan = __syncthreads_or(nan);
    if (t == 0) {
      float v = wv[0];
      int id = wi[0];
      for (int k = 1; k < 32; k++)
        if (wi[k] >= 0 && (id < 0 || wv[k] > v || (wv[k] == v && wi[k] < id))) { v = wv[k]; id = wi[k]; }
      a.ids[b] = nan ? -1 : id;
    }
    return;
  }
  int k = (a.topk <= 0 || a.topk > KMAX) ? KMAX : a.topk;
  if (k > n) k = n;
  // 1. radix select of the k-th largest key
  uint32_t prefix = 0u, mask = 0u;
  int rem = k;
  for (int pass = 0; pass < 4; pass++) {
    const int shift = 24 - 8 * pass;
    if (t < 256) hist[t] = 0u;
    __syncthreads();
    // 8 loads issued before any is used: the row is read from L2 in flight
    for (int i0 = t; i0 < n; i0 += 8 * ST) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) v[u] = i0 + u * ST < n ? lg[i0 + u * ST] : 0.0f;
#pragma unroll
      for (int u = 0; u < 8; u++) {
        if (i0 + u * ST >= n) break;
        if (pass == 0 && v[u] != v[u]) nan = 1;
        const uint32_t key = skey(v[u]);
        if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
      }
    }
    if (pass == 0) {
      nan = __syncthreads_or(nan);
      if (nan) {
        if (t == 0) a.ids[b] = -1;
        return;
      }
    } else {
      __syncthreads();
    }
    // the highest bin d whose count, with every bin above it, reaches rem
    // (bin 0 when none does): warp 0, lane l holding bins 255-8l down to
    // 248-8l, scans the lanes' sums, and the first lane to reach rem walks
    // its own eight bins
    if (w == 0) {
      int c8[8], sum = 0;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        c8[j] = (int)hist[255 - 8 * lane - j];
        sum += c8[j];
      }
      int inc = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int up = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += up;
      }
      const unsigned hit = __ballot_sync(0xffffffffu, inc >= rem);
      if (lane == (hit ? __ffs(hit) - 1 : 31)) {
        int cum = inc - sum, d = 255 - 8 * lane;
#pragma unroll
        for (int j = 0; j < 8; j++) {
          if (d == 0 || cum + c8[j] >= rem) break;
          cum += c8[j];
          d--;
        }
        s_prefix = prefix | ((uint32_t)d << shift);
        s_rem = rem - cum;
      }
    }
    __syncthreads();
    prefix = s_prefix;
    rem = s_rem;
    mask |= 0xFFu << shift;
  }
  // 2. compaction: keys above T anywhere, the first `rem` keys equal to T in
  // index order. Warp w walks the contiguous segment [w S, (w + 1) S) in
  // coalesced 32-key steps; ballots give each key its place among the warp's
  // keys, a block scan of the warps' counts places the segments
  const uint32_t T = prefix;
  const int S = (n + 32 * 32 - 1) / (32 * 32) * 32;
  const int s0 = w * S, s1 = min(n, s0 + S);
  const unsigned lt = (1u << lane) - 1u;
  int ngt = 0, neq = 0;
  for (int j0 = s0; j0 < s1; j0 += 8 * 32) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int i = j0 + u * 32 + lane;
      v[u] = i < s1 ? lg[i] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const bool in = j0 + u * 32 + lane < s1;
      const uint32_t key = skey(v[u]);
      ngt += __popc(__ballot_sync(0xffffffffu, in && key > T));
      neq += __popc(__ballot_sync(0xffffffffu, in && key == T));
    }
  }
  int pgt, peq;
  scan2(lane ? 0 : ngt, lane ? 0 : neq, pgt, peq, ws);
  pgt = __shfl_sync(0xffffffffu, pgt, 0);
  peq = __shfl_sync(0xffffffffu, peq, 0);
  const int base_eq = k - rem;   // the number of keys above T
  for (int j0 = s0; j0 < s1; j0 += 8 * 32) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int i = j0 + u * 32 + lane;
      v[u] = i < s1 ? lg[i] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 8; u++) {
      const int i = j0 + u * 32 + lane;
      const uint32_t key = skey(v[u]);
      const bool gt = i < s1 && key > T, eq = i < s1 && key == T;
      const unsigned bg = __ballot_sync(0xffffffffu, gt), be = __ballot_sync(0xffffffffu, eq);
      const unsigned long long e = ((unsigned long long)key << 32) | (uint32_t)~(uint32_t)i;
      // the counts keep every place of a key above T below k - rem, and
      // rem equal keys are taken; the guards keep the writes inside the list
      // whatever the input
      if (gt) {
        const int p = pgt + __popc(bg & lt);
        if (p < base_eq) cand[p] = e;
      }
      if (eq) {
        const int p = peq + __popc(be & lt);
        if (p < rem && base_eq + p < KMAX) cand[base_eq + p] = e;
      }
      pgt += __popc(bg);
      peq += __popc(be);
    }
  }
  if (t >= k) cand[t] = 0ull;   // below every real entry (no key is 0 once NaN is excluded)
  // 3. bitonic sort, descending, of the first kp2 >= k entries (a power of two)
  int kp2 = 2;
  while (kp2 < k) kp2 <<= 1;
  for (int size = 2; size <= kp2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      const int j = t ^ stride;
      if (t < kp2 && j > t) {
        const unsigned long long x = cand[t], y = cand[j];
        const bool desc = (t & size) == 0;
        if (desc ? (x < y) : (x > y)) { cand[t] = y; cand[j] = x; }
      }
    }
  }
  __syncthreads();
  if (t < k) {
    int idx = (int)~(uint32_t)cand[t];
    if ((unsigned)idx >= (unsigned)n) idx = 0;   // cannot happen with exact counts; keeps the read in the row
    si[t] = idx;
    sv[t] = lg[idx];
  }
  __syncthreads();
  // 4. min-p on the raw logits: the list is sorted, so the survivors are the
  // prefix with sc >= mx + log(minp) (at least one)
  const float mx = sv[0];
  int m = k;
  if (a.use_minp) {
    const float thr = __fadd_rn(mx, a.lminp);
    m = __syncthreads_count(t < k && !(sv[t] < thr));
    if (m < 1) m = 1;
  }
  if (t < m) {
    const float d = __fsub_rn(sv[t], mx);
    e1[t] = pb_expf(d);
    e2[t] = pb_expf(__fdiv_rn(d, a.temp));
  }
  __syncthreads();
  if (t == 0) {
    double es = 0.0;
    for (int j = 0; j < m; j++) es = __dadd_rn(es, (double)e1[j]);
    double acc = 0.0;
    int keep = m;
    for (int j = 0; j < m; j++) {
      acc = __dadd_rn(acc, __ddiv_rn((double)e1[j], es));
      if (acc >= (double)a.topp) { keep = j + 1; break; }
    }
    double es2 = 0.0;
    for (int j = 0; j < keep; j++) es2 = __dadd_rn(es2, (double)e2[j]);
    unsigned long long rs = a.rng[b];
    rs = rs * 6364136223846793005ull + 1442695040888963407ull;
    const float r01 = __double2float_rn(__dmul_rn(__ull2double_rn(rs >> 11), 1.0 / 9007199254740992.0));
    const double r = __dmul_rn((double)r01, es2);
    double a2 = 0.0;
    int id = si[keep - 1];
    for (int j = 0; j < keep; j++) {
      a2 = __dadd_rn(a2, (double)e2[j]);
      if (r < a2 || j == keep - 1) { id = si[j]; break; }
    }
    a.ids[b] = id;
    a.rng[b] = rs;
  }
}

}  // namespace

extern "C" int pb_sample_topkpp(const float* d_logits, int B, int n, long long ld, float temp, float topp, int topk,
                                float minp, unsigned long long* d_rng, int* d_ids, void* stream) {
  if (!d_logits || !d_ids || B <= 0 || n <= 0 || ld < n) return pb_set_error(PB_EINVAL, "pb_sample_topkpp: bad argument");
  if (temp > 0.0f && !d_rng) return pb_set_error(PB_EINVAL, "pb_sample_topkpp: sampling needs the generator states");
  if (B > 65535) return pb_set_error(PB_EINVAL, "pb_sample_topkpp: B %d > 65535", B);
  SampleArgs a{};
  a.lg = d_logits;
  a.ld = ld;
  a.n = n;
  a.topk = topk;
  a.temp = temp;
  a.topp = topp;
  a.use_minp = minp > 0.0f;
  a.lminp = minp > 0.0f ? logf(minp) : 0.0f;
  a.rng = d_rng;
  a.ids = d_ids;
  k_sample<<<B, ST, 0, (cudaStream_t)stream>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return pb_set_error(PB_ECUDA, "k_sample: %s", cudaGetErrorString(e));
  pb_count_launch();
  return PB_OK;
}
