"""The TurboQuant oracle (pulsar_arm/bonsai2/pq1_swar_sm53.cu:3264-3990)
pinned to the reference's own kernels, run on a B200 (tests/golden/tq.npz):
every code word of 600 positions x 2 KV heads of K and V rows is identical
(3-bit, 4-bit, 4-bit K with 3-bit V; outlier channels and an all-zero row);
the row scales, where the reference multiplies by the approximate rsqrtf
and the oracle by a rounded 1/sqrt (2 ulp of rsqrtf error, then the
product's rounding), agree within 3 ulp; and the attention
outputs of the long chain (1 to 600 positions, one and three 256-position
chunks) and of the short pair (which also encodes the last position's rows)
agree within 2e-6 of their magnitude when the oracle reads the reference's
own scales (the rest is the reference's expf against the oracle's)."""
import hashlib
import importlib.util
import os

import numpy as np

from conftest import ROOT

GOLDEN = os.path.join(ROOT, "tests", "golden")


def _gen():
    spec = importlib.util.spec_from_file_location("make_golden_tq", os.path.join(GOLDEN, "make_golden_tq.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def _ulps(a, b):
    ia = np.ascontiguousarray(a, np.float32).view(np.int32).astype(np.int64)
    ib = np.ascontiguousarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(ia - ib)


def test_oracle_tq_matches_reference_kernels(oracle):
    g = _gen()
    z = np.load(os.path.join(GOLDEN, "tq.npz"))
    rows = g.case_rows()
    NKV, CTX = g.NKV, g.CTX
    for bk, bv in g.BITS:
        tag = "b%d%d" % (bk, bv)
        kc, ks = oracle.tq_rows(rows[:, :NKV].reshape(-1, 128), bk)
        vc, vs = oracle.tq_rows(rows[:, NKV:].reshape(-1, 128), bv)
        kc = np.ascontiguousarray(kc.reshape(CTX, NKV, -1).transpose(1, 0, 2))
        vc = np.ascontiguousarray(vc.reshape(CTX, NKV, -1).transpose(1, 0, 2))
        ks, vs = np.ascontiguousarray(ks.reshape(CTX, NKV).T), np.ascontiguousarray(vs.reshape(CTX, NKV).T)
        assert hashlib.sha256(kc.tobytes()).digest() == z[tag + "_kcode_sha256"].tobytes(), tag + " K code words"
        assert hashlib.sha256(vc.tobytes()).digest() == z[tag + "_vcode_sha256"].tobytes(), tag + " V code words"
        rks, rvs = z[tag + "_ksc"], z[tag + "_vsc"]
        assert _ulps(ks, rks).max() <= 3 and _ulps(vs, rvs).max() <= 3, tag + " scales"
        assert float(rks[0, 5]) == 0.0 and float(ks[0, 5]) == 0.0      # the all-zero row
        for kind, Ts in (("long", g.T_LONG), ("short", g.T_SHORT)):
            for T in Ts:
                want = z["%s_%s_T%d" % (tag, kind, T)]
                q = g.case_q(T)
                got = np.concatenate([oracle.tq_attn(q[4 * kh:4 * kh + 4], bk, bv, kc[kh], rks[kh], vc[kh], rvs[kh], T)
                                      for kh in range(NKV)])
                err = np.abs(got - want).max() / np.abs(want).max()
                assert err <= 2e-6, (tag, kind, T, err)
                if kind == "short":
                    assert bool(z["%s_short_T%d_row_same" % (tag, T)][0]), (tag, T)
