// pb_pq1hooks.cpp -- the Bonsai host hooks fwd8.c calls through
// pulsar_arm/bonsai2/pq1_fwd8_shim.h:24-60 (implemented by the reference in
// pq1_fwd8_glue.c:1156-1470, :1483-1760), here over this library's Bonsai
// decoder (pb_bonsai_*). A fwd8.c built with that shim and linked against this
// library runs every token on the B200 in one call, or a layer's attention
// block and FFN tail in one call each:
//   pq1_kv_shape(nl, nkv, ctx)   the K/V cache shape, before the first call;
//   pq1_sess_init(n) / pq1_sess_select(s)   n time-sliced sessions, each with
//                                its own K/V cache and position, one model;
//   pq1_token_fused(...)         one whole token: host Q1_0 weights (uploaded
//                                on first use; the pointer set is the cache
//                                key), the caller's fp32 embedding row and
//                                this position's rope row; logits written to
//                                the host unless pq1_head_need(0);
//   pq1_head_top(&val)           the device argmax of the last token, or -1;
//   pq1_attn_fused(il, ...)      layer il's attention block from the host Q8_K
//                                of attn_norm(x): q|k|v, head norms, rope, the
//                                K/V rows stored at npos in the session's
//                                cache, attention, attn_output -> ao (host);
//   pq1_ffn_fused(...)           the FFN tail from the host Q8_K of
//                                ffn_norm(x): gate|up, silu(g)*u, its Q8_K,
//                                down -> fo (host);
//   pq1_attn_kv_put(il, ...)     a layer's K/V rows of a position fwd8 ran on
//                                the host (it always runs a sequence's first
//                                token there, fwd8.c:780-787), mirrored into
//                                the session's cache;
//   pq1_attn_dbg / pq1_ffn_dbg_xq   the device's values of the last block for
//                                fwd8's PQ1_ATT_CHECK / PQ1_FFN_CHECK;
//   pq1_silu_mul, pq1_gpu_stats_mb   the shim's two host helpers.
// The cache is f16, or TurboQuant-coded when PQ1_KVTQ is 3, 4 or 43 (unset:
// 4, the reference glue's default; 0: the exact f16 cache), read when a
// session's cache is made. Per-layer tensors are keyed by their host
// pointers, as the reference's glue keys them; the whole-token path keeps its own copy of the weight set. A
// session's K/V cache belongs to the session, so the per-layer hooks, the
// mirrored rows and the whole-token path all continue one cache.
// As in the reference, a hook declines (returns -1, the caller runs its own
// path) when it cannot run the step exactly: a shape it does not support, no
// cache shape announced, or a position that is not the next one the layer's
// cache holds (the caller ran earlier positions itself without mirroring
// their K/V rows). Errors print nothing; pb_last_error keeps the reason.
#include "pb_internal.h"

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

namespace {

// fwd8.c:566: the attention scale 1/sqrt(128)
constexpr float kAttnScale = 0.0883883476f;

struct HookSession {
  pb_bonsai_state* st = nullptr;   // the whole-token path's state, over the session's cache
  uint16_t* kv = nullptr;          // f16 cache: [nl][2][nkv][mc][128]
  int nl = 0, nkv = 0, mc = 0;     // the cache's shape
  int tq = 0;                      // TurboQuant bits (3, 4, 43), 0 for the f16 cache
  char* tq_mem = nullptr;          // TurboQuant cache: codes and scales of every layer, then 2 nkv staged rows
  PbTqCache tqc;                   // its layer-0 pointers ([layer][nkv][mc][CW], [layer][nkv][mc])
  uint16_t* stage = nullptr;       // [2 nkv][128] f16 rows put by the host
  std::vector<int> next;           // per layer: the position its cache takes next
};

struct Q1Entry {
  pb_q1* t = nullptr;
  int rows = 0, K = 0;
};

struct Hooks {
  std::mutex mu;
  int nl = 0, nkv = 0, ctx = 0;          // pq1_kv_shape
  int nsess = 1, cur = 0;
  bool sess_fixed = false;               // pq1_sess_init after the first device call is refused
  bool head_need = true;
  int top_valid = 0, top_id = -1;
  float top_val = 0.0f;
  pb_bonsai* m = nullptr;
  int hid = 0, inter = 0, nh = 0, vocab = 0;
  std::vector<const void*> key;          // the weight and norm pointers the model was built from
  std::vector<HookSession> sess;
  float* d_x = nullptr;                  // the caller's row on the device
  cudaStream_t stream = nullptr;
  // per-layer hooks: device copies of host tensors and head-norm weights
  std::map<const void*, Q1Entry> q1;
  std::map<const void*, float*> hnorm;
  pb_bs_blocks* blk = nullptr;
};
Hooks g_h;

int cache_len(int ctx) { return (ctx + 31) / 32 * 32; }

// PQ1_KVTQ as the reference's glue reads it (pq1_fwd8_glue.c:219-229): 3, 4
// or 43 codes the cache with TurboQuant, anything else is the f16 cache; unset
// is 4, the reference's default. Read when a session's cache is made.
int kv_mode() {
  const char* e = getenv("PQ1_KVTQ");
  const int v = e ? atoi(e) : 4;
  return (v == 3 || v == 4 || v == 43) ? v : 0;
}

// layer il's TurboQuant code and scale arrays
PbTqCache tq_layer(const HookSession& S, int il) {
  const size_t rows = (size_t)S.nkv * S.mc;
  PbTqCache c;
  c.kc = S.tqc.kc + (size_t)il * rows * pb_tq_cw(pb_tq_bk(S.tq));
  c.vc = S.tqc.vc + (size_t)il * rows * pb_tq_cw(pb_tq_bv(S.tq));
  c.ks = S.tqc.ks + (size_t)il * rows;
  c.vs = S.tqc.vs + (size_t)il * rows;
  return c;
}

bool ensure_stream() {
  if (g_h.stream) return true;
  if (cudaStreamCreateWithFlags(&g_h.stream, cudaStreamNonBlocking) != cudaSuccess) {
    cudaGetLastError();
    g_h.stream = nullptr;
    pb_set_error(PB_ECUDA, "pq1 hooks: stream");
    return false;
  }
  return true;
}

// a new weight set: the whole-token states built for the old one go and every
// cache starts again from position 0. Rows mirrored or computed before the
// first model existed stay: they belong to it.
void drop_model() {
  if (!g_h.m) return;
  for (auto& s : g_h.sess) {
    pb_bonsai_state_destroy(s.st);
    s.st = nullptr;
    s.next.assign(s.next.size(), 0);
  }
  pb_bonsai_destroy(g_h.m);
  g_h.m = nullptr;
  g_h.key.clear();
}

// build (or keep) the device model for this weight set; false: decline
bool ensure_model(int nl, const unsigned char* const* wt, const float* const* nw, int nh, int nkv, int hid,
                  int inter, int vocab) {
  std::vector<const void*> key;
  key.reserve((size_t)7 * nl + 1 + 4 * nl + 1);
  for (int i = 0; i < 7 * nl + 1; i++) key.push_back(wt[i]);
  for (int i = 0; i < 4 * nl + 1; i++) key.push_back(nw[i]);
  if (g_h.m && key == g_h.key && hid == g_h.hid && inter == g_h.inter && nh == g_h.nh && vocab == g_h.vocab)
    return true;
  drop_model();
  if (!ensure_stream()) return false;
  // fwd8.c's Bonsai-8B constants: YaRN factor 4 over 16384 positions, base
  // 1e6 (fwd8.c:51-57; the table itself comes from the caller per call), and
  // the attention scale
  pb_bonsai_cfg c = {hid, inter, nl, nh, nkv, vocab, 4.0f, 16384, 1e6f, kAttnScale};
  int dev = 0;
  cudaGetDevice(&dev);
  if (pb_bonsai_create(&c, dev, &g_h.m) != PB_OK) { g_h.m = nullptr; return false; }
  int rc = PB_OK;
  for (int il = 0; il < nl && rc == PB_OK; il++) {
    for (int k = 0; k < 7 && rc == PB_OK; k++) rc = pb_bonsai_set_q1(g_h.m, il, k, wt[7 * il + k], 0, g_h.stream);
    for (int k = 0; k < 4 && rc == PB_OK; k++) rc = pb_bonsai_set_norm(g_h.m, il, k, nw[4 * il + k], 0, g_h.stream);
  }
  // output.weight [vocab][hid]: the head; loaded as the (tied) table slot,
  // which the decoder reads as the head when no separate one is set (the
  // embedding itself is the caller's: every call brings its row)
  if (rc == PB_OK) rc = pb_bonsai_set_q1(g_h.m, -1, PB_BS_EMBED, wt[7 * nl], 0, g_h.stream);
  if (rc == PB_OK) rc = pb_bonsai_set_norm(g_h.m, -1, PB_BS_OUT_NORM, nw[4 * nl], 0, g_h.stream);
  if (rc == PB_OK && cudaStreamSynchronize(g_h.stream) != cudaSuccess) {
    cudaGetLastError();
    rc = pb_set_error(PB_ECUDA, "pq1 hooks: weight upload");
  }
  if (rc != PB_OK) { drop_model(); return false; }
  g_h.key = key;
  g_h.hid = hid; g_h.inter = inter; g_h.nh = nh; g_h.vocab = vocab;
  return true;
}

HookSession& session() {
  if ((int)g_h.sess.size() != g_h.nsess) g_h.sess.resize(g_h.nsess);
  HookSession& S = g_h.sess[g_h.cur];
  if ((int)S.next.size() != g_h.nl) S.next.assign(g_h.nl, 0);
  return S;
}

// the session's K/V cache for the announced shape; false: decline (the
// shape changed after the cache was made, or is too long for the attention
// kernel)
bool ensure_kv(HookSession& S) {
  const int mc = cache_len(g_h.ctx);
  if (S.kv) {
    if (S.nl == g_h.nl && S.nkv == g_h.nkv && S.mc == mc) return true;
    pb_set_error(PB_EINVAL, "pq1 hooks: the cache shape changed after the cache was made");
    return false;
  }
  if (S.tq_mem) {
    if (S.nl == g_h.nl && S.nkv == g_h.nkv && S.mc == mc) return true;
    pb_set_error(PB_EINVAL, "pq1 hooks: the cache shape changed after the cache was made");
    return false;
  }
  if (g_h.nl <= 0 || g_h.nkv <= 0 || mc <= 0 || mc > 8192) {
    pb_set_error(PB_EINVAL, "pq1 hooks: cache shape %d x %d x %d", g_h.nl, g_h.nkv, g_h.ctx);
    return false;
  }
  const int tq = g_h.nkv <= 16 ? kv_mode() : 0;
  if (tq) {   // codes and scales of every layer, then the staged rows
    const size_t rows = (size_t)g_h.nl * g_h.nkv * mc;
    const size_t kcb = rows * pb_tq_cw(pb_tq_bk(tq)) * 4, vcb = rows * pb_tq_cw(pb_tq_bv(tq)) * 4;
    const size_t bytes = kcb + vcb + 2 * rows * 4 + (size_t)2 * g_h.nkv * 128 * 2;
    if (cudaMalloc(&S.tq_mem, bytes) != cudaSuccess || cudaMemset(S.tq_mem, 0, bytes) != cudaSuccess) {
      cudaGetLastError();
      if (S.tq_mem) cudaFree(S.tq_mem);
      S.tq_mem = nullptr;
      pb_set_error(PB_ENOMEM, "pq1 hooks: TurboQuant cache of %zu bytes", bytes);
      return false;
    }
    char* p = S.tq_mem;
    S.tqc.kc = reinterpret_cast<uint32_t*>(p); p += kcb;
    S.tqc.vc = reinterpret_cast<uint32_t*>(p); p += vcb;
    S.tqc.ks = reinterpret_cast<float*>(p); p += rows * 4;
    S.tqc.vs = reinterpret_cast<float*>(p); p += rows * 4;
    S.stage = reinterpret_cast<uint16_t*>(p);
    S.tq = tq;
  } else {
    const size_t bytes = (size_t)g_h.nl * 2 * g_h.nkv * mc * 128 * 2;
    if (cudaMalloc(&S.kv, bytes) != cudaSuccess || cudaMemset(S.kv, 0, bytes) != cudaSuccess) {
      cudaGetLastError();
      if (S.kv) cudaFree(S.kv);
      S.kv = nullptr;
      pb_set_error(PB_ENOMEM, "pq1 hooks: K/V cache of %zu bytes", bytes);
      return false;
    }
  }
  S.nl = g_h.nl; S.nkv = g_h.nkv; S.mc = mc;
  return true;
}

uint16_t* kv_layer(HookSession& S, int il, int which) {
  return S.kv + ((size_t)il * 2 + which) * S.nkv * S.mc * 128;
}

// one layer's K and V rows of position pos ([n_kv][128] f16 each) into the
// session's cache ([n_kv][mc][128] per layer, K and V)
bool put_rows(HookSession& S, int il, int pos, const uint16_t* k16, const uint16_t* v16, cudaStream_t st) {
  if (S.tq) {   // stage the rows, code them at pos (the glue's pq1_tq_store_launch)
    const PbTqCache c = tq_layer(S, il);
    if (cudaMemcpyAsync(S.stage, k16, (size_t)S.nkv * 256, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(S.stage + (size_t)S.nkv * 128, v16, (size_t)S.nkv * 256, cudaMemcpyHostToDevice, st) !=
            cudaSuccess) {
      cudaGetLastError();
      pb_set_error(PB_ECUDA, "pq1 hooks: K/V rows");
      return false;
    }
    return pb_tq_store_launch(S.tq, S.stage, nullptr, pos, c.kc, c.ks, c.vc, c.vs, S.nkv, S.mc, st, false) == PB_OK;
  }
  for (int which = 0; which < 2; which++) {
    uint16_t* dst = kv_layer(S, il, which) + (size_t)pos * 128;
    if (cudaMemcpy2DAsync(dst, (size_t)S.mc * 128 * 2, which ? v16 : k16, 256, 256, (size_t)S.nkv,
                          cudaMemcpyHostToDevice, st) != cudaSuccess) {
      cudaGetLastError();
      pb_set_error(PB_ECUDA, "pq1 hooks: K/V rows");
      return false;
    }
  }
  return true;
}

// the device copy of a host Q1_0 tensor [rows][K/128 blocks], made on first use
const pb_q1* q1_of(const void* w, int rows, int K) {
  auto it = g_h.q1.find(w);
  if (it != g_h.q1.end()) {
    if (it->second.rows == rows && it->second.K == K) return it->second.t;
    pb_q1_free(it->second.t);
    g_h.q1.erase(it);
  }
  Q1Entry e;
  if (pb_q1_pack(static_cast<const uint8_t*>(w), rows, K, 0, g_h.stream, &e.t) != PB_OK) return nullptr;
  if (cudaStreamSynchronize(g_h.stream) != cudaSuccess) {
    cudaGetLastError();
    pb_q1_free(e.t);
    pb_set_error(PB_ECUDA, "pq1 hooks: tensor upload");
    return nullptr;
  }
  e.rows = rows;
  e.K = K;
  g_h.q1[w] = e;
  return e.t;
}

// the device copy of a head-norm weight (128 floats)
const float* hnorm_of(const float* w) {
  auto it = g_h.hnorm.find(w);
  if (it != g_h.hnorm.end()) return it->second;
  float* d = nullptr;
  if (cudaMalloc(&d, 128 * 4) != cudaSuccess || cudaMemcpy(d, w, 128 * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaGetLastError();
    if (d) cudaFree(d);
    pb_set_error(PB_ECUDA, "pq1 hooks: head-norm weights");
    return nullptr;
  }
  g_h.hnorm[w] = d;
  return d;
}

bool ensure_blocks() {
  if (g_h.blk) return true;
  int dev = 0;
  cudaGetDevice(&dev);
  return pb_bs_blocks_create(dev, &g_h.blk) == PB_OK;
}

// shapes the device decoder takes (pb_bonsai_create's limits)
bool shape_ok(int nh, int nkv, int hid) {
  return hid > 0 && hid % 256 == 0 && hid <= 8192 && nh > 0 && nh <= 128 && nh % 2 == 0 && nkv > 0 &&
         nh % nkv == 0 && nh / nkv <= 8;
}

}  // namespace

extern "C" {

void pq1_kv_shape(int nl, int nkv, int ctx) {
  std::lock_guard<std::mutex> lk(g_h.mu);
  g_h.nl = nl; g_h.nkv = nkv; g_h.ctx = ctx;
}

int pq1_sess_init(int n) {
  std::lock_guard<std::mutex> lk(g_h.mu);
  if (n < 1 || n > 64 || g_h.sess_fixed) return -1;   // before the first device call, once
  g_h.nsess = n;
  g_h.cur = 0;
  g_h.sess_fixed = true;
  return 0;
}

void pq1_sess_select(int s) {
  std::lock_guard<std::mutex> lk(g_h.mu);
  if (s < 0 || s >= g_h.nsess) return;
  g_h.cur = s;
}

void pq1_head_need(int need) {
  std::lock_guard<std::mutex> lk(g_h.mu);
  g_h.head_need = need != 0;
}

int pq1_head_top(float* val) {
  std::lock_guard<std::mutex> lk(g_h.mu);
  if (!g_h.top_valid) return -1;
  g_h.top_valid = 0;
  if (val) *val = g_h.top_val;
  return g_h.top_id;
}

int pq1_token_fused(int nl, const unsigned char* const* wt, const float* const* nw, int nh, int nkv, int hid,
                    int inter, int vocab, int ctx, int npos, const float* rcc, const float* rcs, const float* x,
                    float* head) {
  std::lock_guard<std::mutex> lk(g_h.mu);
  g_h.top_valid = 0;
  if (!wt || !nw || !rcc || !rcs || !x) return -1;
  if (nl != g_h.nl || nkv != g_h.nkv || ctx != g_h.ctx || npos < 0 || npos >= ctx) return -1;
  if (!shape_ok(nh, nkv, hid) || (inter & 255) || inter <= 0 || vocab <= 0) return -1;
  g_h.sess_fixed = true;
  if (!ensure_model(nl, wt, nw, nh, nkv, hid, inter, vocab)) return -1;
  HookSession& S = session();
  for (int il = 0; il < nl; il++)
    if (S.next[il] != npos) return -1;         // a layer's cache lacks earlier positions
  if (!ensure_kv(S)) return -1;
  if (S.tq && nh != 4 * nkv) return -1;   // the TurboQuant attention takes 4 query heads per KV head
  if (!S.st) {
    const int rc = S.tq ? pb_bonsai_state_create_tq_ext(g_h.m, S.mc, S.tq, &S.tqc, &S.st)
                        : pb_bonsai_state_create_kv(g_h.m, S.mc, S.kv, &S.st);
    if (rc != PB_OK) { S.st = nullptr; return -1; }
  }
  if (!g_h.d_x && cudaMalloc(&g_h.d_x, (size_t)8192 * 4) != cudaSuccess) {
    cudaGetLastError();
    g_h.d_x = nullptr;
    return -1;
  }
  cudaStream_t st = g_h.stream;
  if (pb_bonsai_state_set_rope_row(S.st, npos, rcc, rcs, st) != PB_OK) return -1;
  if (cudaMemcpyAsync(g_h.d_x, x, (size_t)hid * 4, cudaMemcpyHostToDevice, st) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  int id = -1;
  if (pb_bonsai_decode(g_h.m, S.st, 0, npos, g_h.d_x, nullptr, &id, st) != PB_OK) return -1;
  // from here the step has run: every layer's cache holds npos
  for (int il = 0; il < nl; il++) S.next[il] = npos + 1;
  const float* lg = pb_bonsai_state_logits(S.st);
  float v = 0.0f;
  if (cudaMemcpyAsync(&v, lg + id, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      (g_h.head_need && head && cudaMemcpyAsync(head, lg, (size_t)vocab * 4, cudaMemcpyDeviceToHost, st) != cudaSuccess) ||
      cudaStreamSynchronize(st) != cudaSuccess) {
    cudaGetLastError();
    pb_set_error(PB_ECUDA, "pq1_token_fused: logits");
    return -1;
  }
  g_h.top_id = id;
  g_h.top_val = v;
  g_h.top_valid = 1;
  return 0;
}

int pq1_attn_kv_put(int il, int nl, int nkv, int ctx, int npos, const uint16_t* k16, const uint16_t* v16) {
  std::lock_guard<std::mutex> lk(g_h.mu);
  if (!k16 || !v16 || nl != g_h.nl || nkv != g_h.nkv || ctx != g_h.ctx || il < 0 || il >= nl || npos < 0 ||
      npos >= ctx)
    return -1;
  g_h.sess_fixed = true;
  HookSession& S = session();
  if (S.next[il] != npos) return -1;
  if (!ensure_stream() || !ensure_kv(S)) return -1;
  if (!put_rows(S, il, npos, k16, v16, g_h.stream) || cudaStreamSynchronize(g_h.stream) != cudaSuccess) {
    cudaGetLastError();
    return -1;
  }
  S.next[il] = npos + 1;
  return 0;
}

int pq1_attn_fused(int il, const unsigned char* wq, const unsigned char* wk, const unsigned char* wv,
                   const unsigned char* wo, const float* qnw, const float* knw, int nh, int nkv, int hid, int ctx,
                   int npos, const float* rcc, const float* rcs, const unsigned char* xq, float* ao) {
  std::lock_guard<std::mutex> lk(g_h.mu);
  if (!wq || !wk || !wv || !wo || !qnw || !knw || !rcc || !rcs || !xq || !ao) return -1;
  if (g_h.nl <= 0 || nkv != g_h.nkv || ctx != g_h.ctx || il < 0 || il >= g_h.nl || npos < 0 || npos >= ctx)
    return -1;
  if (!shape_ok(nh, nkv, hid)) return -1;
  g_h.sess_fixed = true;
  HookSession& S = session();
  if (S.next[il] != npos) return -1;
  if (!ensure_stream() || !ensure_kv(S) || !ensure_blocks()) return -1;
  const pb_q1* tq = q1_of(wq, nh * 128, hid);
  const pb_q1* tk = tq ? q1_of(wk, nkv * 128, hid) : nullptr;
  const pb_q1* tv = tk ? q1_of(wv, nkv * 128, hid) : nullptr;
  const pb_q1* to = tv ? q1_of(wo, hid, nh * 128) : nullptr;
  const float* dq = to ? hnorm_of(qnw) : nullptr;
  const float* dk = dq ? hnorm_of(knw) : nullptr;
  if (!dk) return -1;
  int rc;
  if (S.tq) {
    if (nh != 4 * nkv) return -1;
    const PbTqCache c = tq_layer(S, il);
    rc = pb_bs_attn_block_tq(g_h.blk, S.tq, tq, tk, tv, to, dq, dk, &c, S.mc, npos, rcc, rcs, xq, ao, g_h.stream);
  } else {
    rc = pb_bs_attn_block(g_h.blk, tq, tk, tv, to, dq, dk, kv_layer(S, il, 0), kv_layer(S, il, 1), S.mc, npos,
                          kAttnScale, rcc, rcs, xq, ao, g_h.stream);
  }
  if (rc != PB_OK) {
    cudaGetLastError();
    return -1;
  }
  S.next[il] = npos + 1;
  return 0;
}

int pq1_ffn_fused(const unsigned char* wg, const unsigned char* wu, const unsigned char* wd, int inter, int hid,
                  const unsigned char* xq, float* fo) {
  std::lock_guard<std::mutex> lk(g_h.mu);
  if (!wg || !wu || !wd || !xq || !fo) return -1;
  if (hid <= 0 || hid % 256 || hid > 8192 || inter <= 0 || inter % 256) return -1;
  if (!ensure_stream() || !ensure_blocks()) return -1;
  const pb_q1* tg = q1_of(wg, inter, hid);
  const pb_q1* tu = tg ? q1_of(wu, inter, hid) : nullptr;
  const pb_q1* td = tu ? q1_of(wd, hid, inter) : nullptr;
  if (!td) return -1;
  if (pb_bs_ffn_block(g_h.blk, tg, tu, td, xq, fo, g_h.stream) != PB_OK) {
    cudaGetLastError();
    return -1;
  }
  return 0;
}

void pq1_ffn_dbg_xq(unsigned char* dst, unsigned long n) {
  std::lock_guard<std::mutex> lk(g_h.mu);
  if (g_h.blk && dst) pb_bs_blocks_ffn_xq(g_h.blk, dst, (size_t)n);
}

void pq1_attn_dbg(int il, int npos, uint16_t* k16, uint16_t* v16, float* q, float* atto, int nh) {
  std::lock_guard<std::mutex> lk(g_h.mu);
  if (g_h.sess.empty() || g_h.cur >= (int)g_h.sess.size()) return;
  HookSession& S = g_h.sess[g_h.cur];
  // no f16 rows under TurboQuant (the glue returns nothing there either)
  if (!S.kv || S.tq || il < 0 || il >= S.nl || npos < 0 || npos >= S.mc) return;
  const size_t pitch = (size_t)S.mc * 128 * 2;
  if (k16) cudaMemcpy2D(k16, 256, kv_layer(S, il, 0) + (size_t)npos * 128, pitch, 256, S.nkv, cudaMemcpyDeviceToHost);
  if (v16) cudaMemcpy2D(v16, 256, kv_layer(S, il, 1) + (size_t)npos * 128, pitch, 256, S.nkv, cudaMemcpyDeviceToHost);
  if (g_h.blk && (q || atto)) pb_bs_blocks_attn_debug(g_h.blk, q, atto, nh);
  cudaGetLastError();
}

// pq1_host.c:196-227: lu[i] = (g * (1 / (1 + expf(-g)))) * lu[i], the host
// helper fwd8.c calls when its FFN tail runs on the host. expf is the host
// C library's (glibc's expf on the reference's targets); the operations are
// rounded one by one, as the reference's -ffp-contract=off build does.
__attribute__((optimize("fp-contract=off"))) void pq1_silu_mul(float* lu, const float* lg, int n) {
  for (int i = 0; i < n; i++) {
    const float g = lg[i];
    const float e = expf(-g);
    const float d = 1.0f + e;
    const float sg = 1.0f / d;
    const float gs = g * sg;
    lu[i] = gs * lu[i];
  }
}

// the GPU memory report fwd8.c prints at exit under PQ1_STATS=1
// (pq1_fwd8_shim.h:64-77): device memory in use and total, in MB
const char* pq1_gpu_stats_mb(char* buf, int n) {
  if (!buf || n <= 0) return buf;
  size_t fr = 0, tot = 0;
  if (cudaMemGetInfo(&fr, &tot) != cudaSuccess) {
    cudaGetLastError();
    snprintf(buf, (size_t)n, "pq1: GPU memory unavailable");
    return buf;
  }
  snprintf(buf, (size_t)n, "pq1: GPU memory %.1f MB used of %.1f MB", (double)(tot - fr) / 1048576.0,
           (double)tot / 1048576.0);
  return buf;
}

int pb_pq1_hooks_reset(void) {
  std::lock_guard<std::mutex> lk(g_h.mu);
  drop_model();
  for (auto& s : g_h.sess) {
    pb_bonsai_state_destroy(s.st);
    if (s.kv) cudaFree(s.kv);
    if (s.tq_mem) cudaFree(s.tq_mem);
  }
  g_h.sess.clear();
  for (auto& e : g_h.q1) pb_q1_free(e.second.t);
  g_h.q1.clear();
  for (auto& e : g_h.hnorm) cudaFree(e.second);
  g_h.hnorm.clear();
  pb_bs_blocks_destroy(g_h.blk);
  g_h.blk = nullptr;
  if (g_h.d_x) cudaFree(g_h.d_x);
  g_h.d_x = nullptr;
  if (g_h.stream) cudaStreamDestroy(g_h.stream);
  g_h.stream = nullptr;
  g_h.nl = g_h.nkv = g_h.ctx = 0;
  g_h.nsess = 1;
  g_h.cur = 0;
  g_h.sess_fixed = false;
  g_h.head_need = true;
  g_h.top_valid = 0;
  g_h.top_id = -1;
  return PB_OK;
}

}  // extern "C"
