"""Generates tests/golden/tq.npz: what the REFERENCE's own TurboQuant K/V
kernels (pulsar_arm/bonsai2/pq1_swar_sm53.cu: pq1_tq_store, the long chain
pq1_tq_qk2 / pq1_tq_sm / pq1_tq_pv2 / pq1_tq_out, and the short pair
pq1_tq_qks / pq1_tq_tail, compiled where they lie into
oracle/_ref/libpb_reftq.so by oracle/build_ref.sh) produce on seeded K/V rows
and queries: the code words (as digests) and scales of every row, and the
attention outputs at several lengths, for 3-bit, 4-bit and 4-bit-K/3-bit-V
caches. TEST INFRASTRUCTURE: tests/test_tq.py checks the oracle against
these. Runs on a GPU box; the inputs are regenerated from the seeds by
case_rows() / case_q().

    bash oracle/build_ref.sh && python tests/golden/make_golden_tq.py
"""
import ctypes as C
import hashlib
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "tq.npz")
NKV, CTX = 2, 600
BITS = [(3, 3), (4, 4), (4, 3)]
T_LONG = [1, 37, 256, 257, 600]
T_SHORT = [1, 37, 200, 256]


def case_rows():
    """K and V rows, f16 bits [CTX][2 NKV][128] (NKV K rows then NKV V rows per
    position): normal values with a few outlier channels, as post-rope keys have"""
    rng = np.random.default_rng(424242)
    x = rng.standard_normal((CTX, 2 * NKV, 128)).astype(np.float32)
    x[:, :NKV, [3, 64, 100]] *= 8.0
    x[5] = 0.0                    # an all-zero position (scale 0)
    return x.astype(np.float16).view(np.uint16)


def case_q(T):
    rng = np.random.default_rng(1000 + T)
    return (rng.standard_normal((4 * NKV, 128)) * 1.5).astype(np.float32)


def cw(b):
    return 12 if b == 3 else 16


def main():
    L = C.CDLL(os.path.join(ROOT, "oracle", "_ref", "libpb_reftq.so"))
    vp, i = C.c_void_p, C.c_int
    L.pbref_gpu_tq_store.argtypes = [vp, i, i, i, vp, vp, vp, vp]
    L.pbref_gpu_tq_attn.argtypes = [vp, i, i, vp, vp, vp, vp, i, i, i, vp]
    L.pbref_gpu_tq_short.argtypes = [vp, vp, i, i, vp, vp, vp, vp, i, i, i, vp]
    rows = case_rows()
    out = {}
    for bk, bv in BITS:
        tag = "b%d%d" % (bk, bv)
        kc = np.zeros((NKV, CTX, cw(bk)), np.uint32); ks = np.zeros((NKV, CTX), np.float32)
        vc = np.zeros((NKV, CTX, cw(bv)), np.uint32); vs = np.zeros((NKV, CTX), np.float32)
        for t in range(CTX):
            a = np.ascontiguousarray(rows[t])
            k1 = np.zeros((NKV, cw(bk)), np.uint32); s1 = np.zeros(NKV, np.float32)
            v1 = np.zeros((NKV, cw(bv)), np.uint32); u1 = np.zeros(NKV, np.float32)
            assert L.pbref_gpu_tq_store(a.ctypes.data, NKV, bk, bv, k1.ctypes.data, s1.ctypes.data, v1.ctypes.data,
                                        u1.ctypes.data) == 0
            kc[:, t], ks[:, t], vc[:, t], vs[:, t] = k1, s1, v1, u1
        out[tag + "_kcode_sha256"] = np.frombuffer(hashlib.sha256(kc.tobytes()).digest(), np.uint8)
        out[tag + "_vcode_sha256"] = np.frombuffer(hashlib.sha256(vc.tobytes()).digest(), np.uint8)
        out[tag + "_ksc"], out[tag + "_vsc"] = ks, vs
        for T in T_LONG:
            q = case_q(T)
            at = np.zeros((4 * NKV, 128), np.float32)
            assert L.pbref_gpu_tq_attn(q.ctypes.data, bk, bv, kc.ctypes.data, ks.ctypes.data, vc.ctypes.data,
                                       vs.ctypes.data, NKV, CTX, T, at.ctypes.data) == 0
            out["%s_long_T%d" % (tag, T)] = at
        for T in T_SHORT:
            q = case_q(T)
            k2, s2, v2, u2 = kc.copy(), ks.copy(), vc.copy(), vs.copy()
            k2[:, T - 1] = 0; s2[:, T - 1] = 0; v2[:, T - 1] = 0; u2[:, T - 1] = 0
            st = np.ascontiguousarray(rows[T - 1])
            at = np.zeros((4 * NKV, 128), np.float32)
            assert L.pbref_gpu_tq_short(q.ctypes.data, st.ctypes.data, bk, bv, k2.ctypes.data, s2.ctypes.data,
                                        v2.ctypes.data, u2.ctypes.data, NKV, CTX, T, at.ctypes.data) == 0
            out["%s_short_T%d" % (tag, T)] = at
            # the short pair's own encode of position T-1 equals the store's
            out["%s_short_T%d_row_same" % (tag, T)] = np.array(
                [np.array_equal(k2[:, T - 1], kc[:, T - 1]) and np.array_equal(v2[:, T - 1], vc[:, T - 1]) and
                 np.array_equal(s2[:, T - 1].view(np.uint32), ks[:, T - 1].view(np.uint32)) and
                 np.array_equal(u2[:, T - 1].view(np.uint32), vs[:, T - 1].view(np.uint32))])
    np.savez(OUT, **out)
    print("wrote", OUT, len(out), "arrays")


if __name__ == "__main__":
    main()
