"""ctypes front end for the CPU oracle (oracle/_build/libpb_oracle.so) and for
the reference-compiled pins (oracle/_ref/libpb_refpins.so).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's CPU
baseline arm import this module as the checker. The product never does.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libpb_oracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libpb_refpins.so")

_lib = None
_ref = None


def build():
    """Compile the oracle (and, where the reference tree exists, its pins)."""
    subprocess.check_call(["make", "-s", "-C", HERE])
    subprocess.check_call(["bash", os.path.join(HERE, "build_ref.sh")])


def _p(a):
    return a.ctypes.data_as(C.c_void_p)


class _Cfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "inter", "n_layers", "n_heads", "n_kv",
                                       "head_dim", "vocab", "conv_w", "max_ctx",
                                       "sliding_window")] + \
               [(n, C.c_float) for n in ("rope_theta", "rope_partial", "norm_eps")] + \
               [("slide_window", C.c_int), ("slide_theta", C.c_float), ("slide_partial", C.c_float)]


class _BsCfg(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "inter", "n_layers", "n_heads", "n_kv", "vocab",
                                       "max_ctx")] + \
               [("rope_factor", C.c_float), ("rope_orig_ctx", C.c_int), ("rope_base", C.c_float),
                ("attn_scale", C.c_float)]


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            subprocess.check_call(["make", "-s", "-C", HERE])
        L = C.CDLL(LIB_PATH)
        vp, i, f = C.c_void_p, C.c_int, C.c_float
        L.pbo_f2bf.restype = C.c_uint16; L.pbo_f2bf.argtypes = [f]
        L.pbo_bf2f.restype = f; L.pbo_bf2f.argtypes = [C.c_uint16]
        L.pbo_f2h.restype = C.c_uint16; L.pbo_f2h.argtypes = [f]
        L.pbo_h2f.restype = f; L.pbo_h2f.argtypes = [C.c_uint16]
        L.pbo_expf.restype = f; L.pbo_expf.argtypes = [f]
        L.pbo_q8_kchunk.restype = i; L.pbo_q8_kchunk.argtypes = [i]
        L.pbo_q8f_gemv.argtypes = [vp, vp, i, i, vp, vp]
        L.pbo_q8f_gemm.argtypes = [vp, vp, i, i, i, vp, vp]
        L.pbo_q80_quant_act.argtypes = [vp, i, vp, vp]
        L.pbo_q80_gemv.argtypes = [vp, vp, i, i, vp, vp, vp, vp]
        L.pbo_q1_repack.argtypes = [vp, i, i, vp, vp]
        L.pbo_q8k_quant.argtypes = [vp, i, vp]
        L.pbo_q1_gemv.argtypes = [i, i, vp, vp, vp, vp, vp]
        L.pbo_q1_rms_q8k.argtypes = [vp, vp, vp, i, f, vp, vp]
        L.pbo_rmsnorm.argtypes = [vp, vp, vp, i, f]
        L.pbo_headnorm.argtypes = [vp, vp, i, i, f]
        L.pbo_rope_invf.argtypes = [vp, f, i, f]
        L.pbo_rope_cs.argtypes = [vp, i, i, vp, vp]
        L.pbo_rope.argtypes = [vp, i, i, i, vp, vp]
        L.pbo_attn_head.argtypes = [vp, vp, vp, i, i, i, i, i, f, C.c_uint16, i, vp]
        L.pbo_argmax.restype = i; L.pbo_argmax.argtypes = [vp, i]
        L.pbo_qlow_gemv.argtypes = [vp, vp, i, i, i, i, vp, vp]
        L.pbo_tq_row.argtypes = [vp, i, vp, vp]
        L.pbo_tq_attn.argtypes = [vp, i, i, vp, vp, vp, vp, i, vp]
        L.pbo_sample_topkpp.restype = i
        L.pbo_sample_topkpp.argtypes = [vp, i, f, f, i, f, C.POINTER(C.c_uint64), i]
        L.pbo_conv_step.argtypes = [vp, vp, vp, i, i, vp]
        L.pbo_silu_mul_bf.argtypes = [vp, vp, vp, i]
        L.pbo_sigmoid_gate.argtypes = [vp, vp, i, i]
        L.pbo_model_new.restype = vp; L.pbo_model_new.argtypes = [C.POINTER(_Cfg), vp]
        L.pbo_model_free.argtypes = [vp]
        L.pbo_model_set_q8.argtypes = [vp, i, i, vp, vp, i, i]
        L.pbo_model_set_f32.argtypes = [vp, i, i, vp]
        L.pbo_model_set_int.argtypes = [vp, i]
        L.pbo_model_set_emb_bf16.argtypes = [vp, vp]
        L.pbo_gemv_bf16.argtypes = [vp, i, i, vp, vp]
        L.pbo_state_new.restype = vp; L.pbo_state_new.argtypes = [vp]
        L.pbo_state_free.argtypes = [vp]
        L.pbo_decode.restype = i; L.pbo_decode.argtypes = [vp, vp, i, i, vp, vp]
        L.pbo_state_kv.restype = vp; L.pbo_state_kv.argtypes = [vp, i, i]
        L.pbo_state_ring.restype = vp; L.pbo_state_ring.argtypes = [vp, i]
        L.pbo_threads.restype = i
        L.pbo_bs_rms.argtypes = [vp, vp, i, vp]
        L.pbo_bs_rope_table.argtypes = [i, f, i, f, vp, vp]
        L.pbo_bs_rope.argtypes = [vp, i, vp, vp]
        L.pbo_bs_fa16_head.argtypes = [vp, vp, vp, i, f, vp]
        L.pbo_bs_silu_mul.argtypes = [vp, vp, i]
        L.pbo_bs_model_new.restype = vp; L.pbo_bs_model_new.argtypes = [C.POINTER(_BsCfg)]
        L.pbo_bs_model_free.argtypes = [vp]
        L.pbo_bs_model_set_q1.argtypes = [vp, i, i, vp, i, i]
        L.pbo_bs_model_set_f32.argtypes = [vp, i, i, vp]
        L.pbo_bs_state_new.restype = vp; L.pbo_bs_state_new.argtypes = [vp]
        L.pbo_bs_state_new_tq.restype = vp; L.pbo_bs_state_new_tq.argtypes = [vp, i]
        L.pbo_bs_state_tq_recode.argtypes = [vp, vp, i]
        L.pbo_bs_state_free.argtypes = [vp]
        L.pbo_bs_state_kv.restype = vp; L.pbo_bs_state_kv.argtypes = [vp, i, i]
        L.pbo_bs_decode.restype = i; L.pbo_bs_decode.argtypes = [vp, vp, i, i, vp, vp, vp]
        _lib = L
    return _lib


def ref():
    """The reference's own functions, or None when they were not built here."""
    global _ref
    if _ref is None and os.path.exists(REF_PATH):
        R = C.CDLL(REF_PATH)
        vp, i = C.c_void_p, C.c_int
        R.pbref_h2f.restype = C.c_float; R.pbref_h2f.argtypes = [C.c_uint16]
        R.pbref_ff16.restype = C.c_uint16; R.pbref_ff16.argtypes = [C.c_float]
        R.pbref_f16f.restype = C.c_float; R.pbref_f16f.argtypes = [C.c_uint16]
        R.pbref_q1_repack.argtypes = [vp, i, i, vp, vp]
        R.pbref_q1_gemv.argtypes = [i, i, vp, vp, vp, vp]
        R.pbref_q80_quant.argtypes = [vp, i, vp, vp]
        R.pbref_mk_q8k.argtypes = [vp, i, C.c_uint]
        R.pbref_rms_q8k.argtypes = [vp, vp, vp, i, vp]
        R.pbref_parity_q1_weights.argtypes = [vp, i, i]
        R.pbref_gemv_q8.argtypes = [vp, vp, vp, vp, i, i]
        R.pbref_quant_row.argtypes = [vp, i, vp, vp]
        R.pbref_cpuchk.restype = C.c_long
        R.pbref_cpuchk.argtypes = [vp, vp, vp, vp, i, i, i, i]
        R.pbref_bs_rms.argtypes = [vp, vp, i, vp]
        R.pbref_bs_rope_table.argtypes = [i, vp, vp]
        R.pbref_bs_rope.argtypes = [vp, i, i]
        R.pbref_fa16_head.argtypes = [vp, vp, vp, i, C.c_float, vp]
        R.pbref_silu_mul.argtypes = [vp, vp, i]
        _ref = R
    return _ref


# ---------------------------------------------------------------- helpers ---
def f2bf(a):
    """vectorised lfm3_nanode.cu:116-121 (numpy; matches pbo_f2bf bit for bit)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    special = ((u >> 23) & 0xFF) == 0xFF
    r = ((u + np.uint32(0x7FFF) + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(special, (u >> 16).astype(np.uint16), r)


def bf2f(h):
    return (np.asarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def q8f_gemv(codes, scales_f32, x_bf16):
    N, K = codes.shape
    T = 1 if x_bf16.ndim == 1 else x_bf16.shape[0]
    y = np.zeros((T, N), np.float32)
    lib().pbo_q8f_gemm(_p(codes), _p(scales_f32), N, K, T, _p(np.ascontiguousarray(x_bf16)), _p(y))
    return y[0] if x_bf16.ndim == 1 else y


def gemv_bf16(w_bf16, x_bf16):
    """k_gemv_bf16 (the bf16 head): w [N][K] bf16 bits, x [K] bf16 bits -> fp32 [N]"""
    N, K = w_bf16.shape
    y = np.zeros(N, np.float32)
    lib().pbo_gemv_bf16(_p(np.ascontiguousarray(w_bf16, np.uint16)), N, K,
                        _p(np.ascontiguousarray(x_bf16, np.uint16)), _p(y))
    return y


def q80_quant_act(x):
    K = x.shape[0]
    qx = np.zeros(K, np.int8); dx = np.zeros(K // 32, np.uint16)
    lib().pbo_q80_quant_act(_p(np.ascontiguousarray(x, np.float32)), K, _p(qx), _p(dx))
    return qx, dx


def q80_gemv(codes, dw_h, qx, dx_h):
    N, K = codes.shape
    isum = np.zeros((N, K // 32), np.int32); y = np.zeros(N, np.float32)
    lib().pbo_q80_gemv(_p(codes), _p(dw_h), N, K, _p(qx), _p(dx_h), _p(isum), _p(y))
    return isum, y


def q1_repack(q1, rows, K):
    wb = np.zeros((rows, K // 32), np.uint32); sc = np.zeros((rows, K // 128), np.uint16)
    lib().pbo_q1_repack(_p(q1), rows, K, _p(wb), _p(sc))
    return wb, sc


def q8k_quant(x):
    K = x.shape[0]
    xq = np.zeros((K // 256) * 292, np.uint8)
    lib().pbo_q8k_quant(_p(np.ascontiguousarray(x, np.float32)), K, _p(xq))
    return xq


def q1_rms_q8k(x, w, r=None, eps=1e-6):
    x = np.array(x, np.float32)
    n = x.shape[0]
    y = np.zeros(n, np.float32); xq = np.zeros((n // 256) * 292, np.uint8)
    lib().pbo_q1_rms_q8k(_p(x), _p(np.ascontiguousarray(r, np.float32)) if r is not None else None,
                         _p(np.ascontiguousarray(w, np.float32)), n, eps, _p(y), _p(xq))
    return x, y, xq


def q1_gemv(wb, sc, xq, K):
    rows = wb.shape[0]
    isum = np.zeros((rows, K // 128), np.int32); y = np.zeros(rows, np.float32)
    lib().pbo_q1_gemv(rows, K, _p(wb), _p(sc), _p(xq), _p(isum), _p(y))
    return isum, y


def h2f_all():
    return np.array([lib().pbo_h2f(h) for h in range(65536)], np.float32)


class Model:
    """Oracle decode over numpy weights held by `weights` (a dict shaped like
    pulsar_b200.synth.make_weights)."""

    SLOTS_Q8 = {"q": 0, "k": 1, "v": 2, "gate": 3, "o": 4, "in_proj": 5, "out_proj": 6,
                "w1": 7, "w3": 8, "w2": 9}
    SLOTS_F = {"op_norm": 0, "post_op_norm": 1, "ffn_norm": 2, "post_ffn_norm": 3,
               "q_norm": 4, "k_norm": 5, "taps": 6}

    def __init__(self, cfg, weights, int_path=False):
        """int_path: every projection on the Q8_0 integer path (the chunked
        prefill's tensor-core form) instead of the reference's float path."""
        L = lib()
        self.cfg = cfg
        self._keep = []
        c = _Cfg(cfg["hidden"], cfg["inter"], cfg["n_layers"], cfg["n_heads"], cfg["n_kv"],
                 cfg["head_dim"], cfg["vocab"], cfg["conv_w"], cfg["max_ctx"],
                 cfg.get("sliding_window", 0), cfg["rope_theta"], cfg["rope_partial"],
                 cfg["norm_eps"], cfg.get("slide_window", 256), cfg.get("slide_theta", 1e4),
                 cfg.get("slide_partial", 1.0))
        kinds = {"conv": 0, "sliding_attention": 2}
        isa = np.array([kinds.get(t, 1) for t in cfg["layer_types"]], np.int32)
        self._keep.append(isa)
        self.m = L.pbo_model_new(C.byref(c), _p(isa))
        for li, lw in enumerate(weights["layers"]):
            for name, slot in self.SLOTS_Q8.items():
                if name in lw:
                    codes, sc16 = lw[name]
                    s32 = np.ascontiguousarray(h2f_vec(sc16))
                    self._keep += [codes, s32]
                    L.pbo_model_set_q8(self.m, li, slot, _p(codes), _p(s32), codes.shape[0], codes.shape[1])
            for name, slot in self.SLOTS_F.items():
                if name in lw:
                    a = np.ascontiguousarray(lw[name], np.float32)
                    self._keep.append(a)
                    L.pbo_model_set_f32(self.m, li, slot, _p(a))
        if "embed_bf16" in weights:
            e16 = np.ascontiguousarray(weights["embed_bf16"], np.uint16)
            self._keep.append(e16)
            L.pbo_model_set_emb_bf16(self.m, _p(e16))
        else:
            codes, sc16 = weights["embed"]
            s32 = np.ascontiguousarray(h2f_vec(sc16))
            self._keep += [codes, s32]
            L.pbo_model_set_q8(self.m, -1, 0, _p(codes), _p(s32), codes.shape[0], codes.shape[1])
        fn = np.ascontiguousarray(weights["final_norm"], np.float32)
        self._keep.append(fn)
        L.pbo_model_set_f32(self.m, -1, 0, _p(fn))
        L.pbo_model_set_int(self.m, 1 if int_path else 0)
        self.s = L.pbo_state_new(self.m)

    def reset(self):
        lib().pbo_state_free(self.s)
        self.s = lib().pbo_state_new(self.m)

    def decode(self, token, pos, want_logits=False):
        lg = np.zeros(self.cfg["vocab"], np.float32) if want_logits else None
        x = np.zeros(self.cfg["hidden"], np.uint16)
        tid = lib().pbo_decode(self.m, self.s, int(token), int(pos), _p(lg) if lg is not None else None, _p(x))
        return tid, lg, x

    def kv(self, layer, which, n):
        c = self.cfg
        ptr = lib().pbo_state_kv(self.s, layer, which)
        return np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_uint16)), shape=(n * c["n_kv"] * c["head_dim"],)).copy()

    def ring(self, layer):
        """the conv layer's ring [W][H] (bf16 bits), oldest position first"""
        c = self.cfg
        ptr = lib().pbo_state_ring(self.s, layer)
        return np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_uint16)),
                                     shape=(c["conv_w"] * c["hidden"],)).copy().reshape(c["conv_w"], c["hidden"])

    def set_kv(self, layer, which, a):
        """overwrite the attention layer's K (0) or V (1) cache with f16 bits
        [max_ctx][n_kv][head_dim]"""
        c = self.cfg
        a = np.ascontiguousarray(a, np.uint16)
        assert a.size == c["max_ctx"] * c["n_kv"] * c["head_dim"]
        C.memmove(lib().pbo_state_kv(self.s, layer, which), a.ctypes.data, a.nbytes)

    def set_ring(self, layer, a):
        """overwrite the conv layer's ring with bf16 bits [W][H]: row k holds
        position pos - W + k before the step at pos"""
        c = self.cfg
        a = np.ascontiguousarray(a, np.uint16)
        assert a.size == c["conv_w"] * c["hidden"]
        C.memmove(lib().pbo_state_ring(self.s, layer), a.ctypes.data, a.nbytes)

    def __del__(self):
        try:
            lib().pbo_state_free(self.s)
            lib().pbo_model_free(self.m)
        except Exception:
            pass


def h2f_vec(h):
    """exact fp16 -> fp32 widening (numpy's float16 conversion is exact); accepts
    float16 arrays or their uint16 bit patterns."""
    h = np.asarray(h)
    if h.dtype == np.uint16:
        h = h.view(np.float16)
    return h.astype(np.float32)


# ------------------------------------------------------------------ Bonsai ----
def bs_rms(x, w):
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros_like(x)
    lib().pbo_bs_rms(_p(x), _p(np.ascontiguousarray(w, np.float32)), x.shape[0], _p(y))
    return y


def bs_rope_table(pos, factor=4.0, orig_ctx=16384, base=1e6):
    c = np.zeros(64, np.float32); s = np.zeros(64, np.float32)
    lib().pbo_bs_rope_table(int(pos), factor, int(orig_ctx), base, _p(c), _p(s))
    return c, s


def bs_rope(x, c, s):
    x = np.array(x, np.float32)
    lib().pbo_bs_rope(_p(x), x.shape[0] // 128, _p(np.ascontiguousarray(c)), _p(np.ascontiguousarray(s)))
    return x


def bs_fa16_head(q, K16, V16, scale=0.0883883476):
    """q fp32 [128]; K16, V16 f16 bits [T][128]"""
    out = np.zeros(128, np.float32)
    T = K16.shape[0]
    lib().pbo_bs_fa16_head(_p(np.ascontiguousarray(q, np.float32)), _p(np.ascontiguousarray(K16, np.uint16)),
                           _p(np.ascontiguousarray(V16, np.uint16)), T, scale, _p(out))
    return out


def bs_silu_mul(lg, lu):
    u = np.array(lu, np.float32)
    lib().pbo_bs_silu_mul(_p(u), _p(np.ascontiguousarray(lg, np.float32)), u.shape[0])
    return u


class BsModel:
    """Oracle Bonsai decode (fwd8.c) over weights shaped like
    pulsar_b200.synth.make_bonsai_weights."""

    SLOTS = {"q": 0, "k": 1, "v": 2, "o": 3, "gate": 4, "up": 5, "down": 6}
    NORMS = {"attn_norm": 0, "ffn_norm": 1, "q_norm": 2, "k_norm": 3}

    def __init__(self, cfg, weights, max_ctx, kv_bits=0):
        L = lib()
        self.cfg = dict(cfg)
        self.max_ctx = max_ctx
        self._keep = []
        c = _BsCfg(cfg["hidden"], cfg["inter"], cfg["n_layers"], cfg["n_heads"], cfg["n_kv"], cfg["vocab"],
                   max_ctx, cfg["rope_factor"], cfg["rope_orig_ctx"], cfg["rope_base"], cfg["attn_scale"])
        self.m = L.pbo_bs_model_new(C.byref(c))
        for li, lw in enumerate(weights["layers"]):
            for name, slot in self.SLOTS.items():
                b = np.ascontiguousarray(lw[name], np.uint8)
                L.pbo_bs_model_set_q1(self.m, li, slot, _p(b), b.shape[0], b.shape[1] * 128)
            for name, slot in self.NORMS.items():
                a = np.ascontiguousarray(lw[name], np.float32)
                self._keep.append(a)
                L.pbo_bs_model_set_f32(self.m, li, slot, _p(a))
        e = np.ascontiguousarray(weights["embed"], np.uint8)
        L.pbo_bs_model_set_q1(self.m, -1, 0, _p(e), e.shape[0], e.shape[1] * 128)
        if weights.get("head") is not None:
            hd = np.ascontiguousarray(weights["head"], np.uint8)
            L.pbo_bs_model_set_q1(self.m, -1, 1, _p(hd), hd.shape[0], hd.shape[1] * 128)
        on = np.ascontiguousarray(weights["out_norm"], np.float32)
        self._keep.append(on)
        L.pbo_bs_model_set_f32(self.m, -1, 0, _p(on))
        self.s = L.pbo_bs_state_new_tq(self.m, int(kv_bits)) if kv_bits else L.pbo_bs_state_new(self.m)

    def decode(self, token, pos, x_in=None, want_logits=False):
        """-> (greedy id, logits or None, final residual fp32 [hidden])"""
        lg = np.zeros(self.cfg["vocab"], np.float32) if want_logits else None
        x = np.zeros(self.cfg["hidden"], np.float32)
        xi = None if x_in is None else np.ascontiguousarray(x_in, np.float32)
        tid = lib().pbo_bs_decode(self.m, self.s, int(token), int(pos), _p(xi) if xi is not None else None,
                                  _p(lg) if lg is not None else None, _p(x))
        return tid, lg, x

    def kv(self, layer, which):
        """the layer's K (0) or V (1) cache, f16 bits [n_kv][max_ctx][128]"""
        c = self.cfg
        ptr = lib().pbo_bs_state_kv(self.s, layer, which)
        n = c["n_kv"] * self.max_ctx * 128
        return np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_uint16)), shape=(n,)).copy().reshape(
            c["n_kv"], self.max_ctx, 128)

    def set_kv(self, layer, which, a):
        """overwrite the layer's K (0) or V (1) cache with f16 bits [n_kv][max_ctx][128]"""
        c = self.cfg
        a = np.ascontiguousarray(a, np.uint16)
        assert a.size == c["n_kv"] * self.max_ctx * 128
        C.memmove(lib().pbo_bs_state_kv(self.s, layer, which), a.ctypes.data, a.nbytes)

    def tq_recode(self, n):
        """a TurboQuant state: code positions < n again from the f16 rows (after set_kv)"""
        lib().pbo_bs_state_tq_recode(self.s, self.m, int(n))

    def __del__(self):
        try:
            lib().pbo_bs_state_free(self.s)
            lib().pbo_bs_model_free(self.m)
        except Exception:
            pass


def sample_topkpp(logits, temp, topp, topk, minp, rs, libm_exp=False):
    """fwd8.c:465-521 on one row: -> (id, the advanced generator state)"""
    lg = np.ascontiguousarray(logits, np.float32)
    st = C.c_uint64(int(rs))
    tid = lib().pbo_sample_topkpp(_p(lg), lg.shape[0], float(temp), float(topp), int(topk), float(minp),
                                  C.byref(st), 1 if libm_exp else 0)
    return tid, int(st.value)


def qlow_gemv(codes, scales, bits, N, K, x):
    """lfm3_qlow.cuh's GEMV; x bf16 bits [T][K] (or [K]) -> y bf16 bits [T][N]"""
    x = np.ascontiguousarray(x, np.uint16)
    T = 1 if x.ndim == 1 else x.shape[0]
    y = np.zeros((T, N), np.uint16)
    lib().pbo_qlow_gemv(_p(np.ascontiguousarray(codes, np.uint8)), _p(np.ascontiguousarray(scales, np.uint16)),
                        int(bits), int(N), int(K), T, _p(x), _p(y))
    return y if x.ndim == 2 else y[0]


def tq_cw(bits):
    return 12 if bits == 3 else 16


def tq_rows(rows16, bits):
    """TurboQuant encode of f16 rows [n][128] (bits) -> (codes uint32 [n][CW], scales fp32 [n])"""
    rows16 = np.ascontiguousarray(rows16, np.uint16).reshape(-1, 128)
    n = rows16.shape[0]
    cw = np.zeros((n, tq_cw(bits)), np.uint32)
    sc = np.zeros(n, np.float32)
    L = lib()
    for r in range(n):
        L.pbo_tq_row(_p(rows16[r]), int(bits), _p(cw[r]), C.cast(C.c_void_p(sc.ctypes.data + 4 * r), C.c_void_p))
    return cw, sc


def tq_attn(q4, bk, bv, kcw, ksc, vcw, vsc, T):
    """the 4 query heads q4 [4][128] of one KV head over positions 0..T-1 of a
    TurboQuant cache (codes [>=T][CW], scales [>=T]) -> atto [4][128]"""
    out = np.zeros((4, 128), np.float32)
    lib().pbo_tq_attn(_p(np.ascontiguousarray(q4, np.float32)), int(bk), int(bv),
                      _p(np.ascontiguousarray(kcw, np.uint32)), _p(np.ascontiguousarray(ksc, np.float32)),
                      _p(np.ascontiguousarray(vcw, np.uint32)), _p(np.ascontiguousarray(vsc, np.float32)), int(T),
                      _p(out))
    return out
