// pb_pq1hooks.cpp -- the Bonsai host hooks fwd8.c calls through
// pulsar_arm/bonsai2/pq1_fwd8_shim.h:24-60 (implemented by the reference in
// pq1_fwd8_glue.c:235-246, :1483-1760), here over this library's Bonsai
// decoder (pb_bonsai_*). A fwd8.c built with that shim and linked against this
// library runs every token on the B200 in one call:
//   pq1_kv_shape(nl, nkv, ctx)   the K/V cache shape, before the first call;
//   pq1_sess_init(n) / pq1_sess_select(s)   n time-sliced sessions, each with
//                                its own K/V cache and position, one model;
//   pq1_token_fused(...)         one whole token: host Q1_0 weights (uploaded
//                                on first use; the pointer set is the cache
//                                key), the caller's fp32 embedding row and
//                                this position's rope row; logits written to
//                                the host unless pq1_head_need(0);
//   pq1_head_top(&val)           the device argmax of the last token, or -1;
//   pq1_attn_kv_put(il, ...)     a layer's K/V rows of a position fwd8 ran on
//                                the host (it always runs a sequence's first
//                                token there, fwd8.c:780-787), mirrored into
//                                the session's cache (held on the host until
//                                the cache exists).
// As in the reference, pq1_token_fused declines (returns -1, the caller runs
// its own path) when it cannot run the step exactly: a shape it does not
// support, no cache shape announced, or a position that is not the next one
// every layer's cache holds (the caller ran earlier positions itself without
// mirroring their K/V rows). Errors print nothing; pb_last_error keeps the
// reason.
#include "pb_internal.h"

#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

namespace {

struct PendingKV {
  int il, pos;
  std::vector<uint16_t> k, v;   // [nkv][128] f16 each
};
struct HookSession {
  pb_bonsai_state* st = nullptr;
  int mc = 0;                       // the cache's positions (ctx rounded up to 32)
  std::vector<int> next;            // per layer: the position its cache takes next
  std::vector<PendingKV> pending;   // rows put before the cache existed
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
};
Hooks g_h;

// a new weight set: the caches built for the old one go (rows mirrored
// before any model existed stay, they belong to the first one)
void drop_model() {
  if (!g_h.m) return;
  for (auto& s : g_h.sess) {
    pb_bonsai_state_destroy(s.st);
    s.st = nullptr;
    s.next.assign(s.next.size(), 0);
    s.pending.clear();
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
  if (!g_h.stream && cudaStreamCreateWithFlags(&g_h.stream, cudaStreamNonBlocking) != cudaSuccess) {
    cudaGetLastError();
    pb_set_error(PB_ECUDA, "pq1 hooks: stream");
    return false;
  }
  // fwd8.c's Bonsai-8B constants: YaRN factor 4 over 16384 positions, base
  // 1e6 (fwd8.c:51-57; the table itself comes from the caller per call), and
  // attention scale 1/sqrt(128) (fwd8.c:566)
  pb_bonsai_cfg c = {hid, inter, nl, nh, nkv, vocab, 4.0f, 16384, 1e6f, 0.0883883476f};
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

// one layer's K and V rows of position pos ([n_kv][128] f16 each) into the
// session's cache ([n_kv][max_ctx][128] per layer, K and V)
bool put_rows(HookSession& S, int il, int pos, const uint16_t* k16, const uint16_t* v16, cudaStream_t st) {
  for (int which = 0; which < 2; which++) {
    void* d = nullptr;
    if (pb_bonsai_state_kv(S.st, il, which, &d) != PB_OK) return false;
    uint16_t* dst = static_cast<uint16_t*>(d) + (size_t)pos * 128;
    if (cudaMemcpy2DAsync(dst, (size_t)S.mc * 128 * 2, which ? v16 : k16, 256, 256, (size_t)g_h.nkv,
                          cudaMemcpyHostToDevice, st) != cudaSuccess) {
      cudaGetLastError();
      pb_set_error(PB_ECUDA, "pq1 hooks: K/V rows");
      return false;
    }
  }
  return true;
}

HookSession& session() {
  if ((int)g_h.sess.size() != g_h.nsess) g_h.sess.resize(g_h.nsess);
  HookSession& S = g_h.sess[g_h.cur];
  if ((int)S.next.size() != g_h.nl) S.next.assign(g_h.nl, 0);
  return S;
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
  if ((hid & 255) || hid > 8192 || (inter & 255) || nh <= 0 || nh > 128 || (nh & 1) || nkv <= 0 || nh % nkv ||
      nh / nkv > 8 || vocab <= 0)
    return -1;
  g_h.sess_fixed = true;
  if (!ensure_model(nl, wt, nw, nh, nkv, hid, inter, vocab)) return -1;
  HookSession& S = session();
  for (int il = 0; il < nl; il++)
    if (S.next[il] != npos) return -1;         // a layer's cache lacks earlier positions
  if (!S.st) {
    const int mc = (ctx + 31) / 32 * 32;
    if (mc > 8192 || pb_bonsai_state_create(g_h.m, mc, &S.st) != PB_OK) { S.st = nullptr; return -1; }
    S.mc = mc;
    for (const auto& pk : S.pending)
      if (!put_rows(S, pk.il, pk.pos, pk.k.data(), pk.v.data(), g_h.stream)) return -1;
    if (cudaStreamSynchronize(g_h.stream) != cudaSuccess) { cudaGetLastError(); return -1; }
    S.pending.clear();
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
  if (S.st) {
    if (!put_rows(S, il, npos, k16, v16, g_h.stream) || cudaStreamSynchronize(g_h.stream) != cudaSuccess) {
      cudaGetLastError();
      return -1;
    }
  } else {
    PendingKV pk;
    pk.il = il;
    pk.pos = npos;
    pk.k.assign(k16, k16 + (size_t)nkv * 128);
    pk.v.assign(v16, v16 + (size_t)nkv * 128);
    S.pending.push_back(std::move(pk));
  }
  S.next[il] = npos + 1;
  return 0;
}

}  // extern "C"
