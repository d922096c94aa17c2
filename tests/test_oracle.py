"""The CPU oracle against the reference: committed golden fixtures (produced by
the reference's own compiled functions, tests/golden/make_golden.py) and, where
the reference tree was available at build time, the reference functions
themselves (oracle/_ref)."""
import os

import numpy as np
import pytest

from conftest import GOLDEN


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def test_golden_q1_parity(oracle):
    g = _load("q1_parity.npz")
    rows, K = int(g["rows"]), int(g["K"])
    wb, sc = oracle.q1_repack(g["q1"], rows, K)
    isum, y = oracle.q1_gemv(wb, sc, g["xq"], K)
    assert np.array_equal(y.view(np.uint32), g["y"].view(np.uint32))


def test_golden_q8k_rms(oracle):
    g = _load("q8k_rms.npz")
    n = g["x"].shape[1]
    mask = np.ones((n // 256) * 292, bool)
    for b in range(n // 256):          # bsums are not compared (the fork leaves them stale)
        mask[b * 292 + 260:b * 292 + 292] = False
    for x, want in zip(g["x"], g["xq"]):
        _, _, xq = oracle.q1_rms_q8k(x, g["w"])
        assert np.array_equal(xq[mask], want[mask])


def test_golden_q80_quant(oracle):
    g = _load("q80_quant.npz")
    qx, dx = oracle.q80_quant_act(g["x"])
    assert np.array_equal(qx, g["q"])
    assert np.array_equal(oracle.h2f_vec(dx), g["d"])


def test_golden_q8f_tree(oracle):
    g = _load("q8f_tree.npz")
    for t in ("a", "b", "c"):
        codes, s16, x, y = g[t + "_codes"], g[t + "_s16"], g[t + "_x"], g[t + "_y"]
        yo = oracle.q8f_gemv(codes, s16.astype(np.float32), x)
        assert np.array_equal(oracle.f2bf(np.float32(0) + yo), y)


def test_golden_q8_gemv_cpu_tolerance(oracle):
    g = _load("q8_gemv_cpu.npz")
    y = oracle.q8f_gemv(g["codes"], g["s"], g["x"])
    xf = oracle.bf2f(g["x"])
    N, K = g["codes"].shape
    mag = (np.abs(g["codes"].reshape(N, K // 32, 32).astype(np.float64) * xf.reshape(1, K // 32, 32)).sum(-1)
           * g["s"]).sum(-1)
    assert np.max(np.abs(y.astype(np.float64) - g["y"]) / mag) < 1e-6


def test_h2f_exhaustive(oracle):
    h = np.arange(65536, dtype=np.uint16)
    want = h.view(np.float16).astype(np.float32)
    got = np.array([oracle.lib().pbo_h2f(int(v)) for v in h], np.float32)
    nan = np.isnan(want)
    assert np.array_equal(got[~nan].view(np.uint32), want[~nan].view(np.uint32))
    assert np.isnan(got[nan]).all()


def test_f2h_rne(oracle):
    rng = np.random.default_rng(5)
    v = (rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 6, 20000)).astype(np.float32)
    v = np.concatenate([v, np.float32([0, -0.0, 65504, 65519.99, 65520, 1e9, 6.1e-5, 5.96e-8, 2.98e-8, 2.99e-8])])
    got = np.array([oracle.lib().pbo_f2h(float(x)) for x in v], np.uint16)
    want = v.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)


def test_expf_error_bound(oracle):
    xs = np.concatenate([np.linspace(-103.9, 88.7, 200001), np.linspace(-1, 1, 20001)]).astype(np.float32)
    got = np.array([oracle.lib().pbo_expf(float(x)) for x in xs], np.float32)
    ref = np.exp(xs.astype(np.float64))
    ok = (ref > 1.2e-38) & (ref < 3.4e38)
    ulp = np.abs(got[ok].astype(np.float64) - ref[ok]) / np.spacing(ref[ok].astype(np.float32)).astype(np.float64)
    assert ulp.max() < 1.5
    assert oracle.lib().pbo_expf(100.0) == float("inf")
    assert oracle.lib().pbo_expf(-200.0) == 0.0


def test_attention_matches_float64_softmax(oracle):
    """the restated attention order is still an attention (tolerance vs fp64)."""
    rng = np.random.default_rng(3)
    hd, nkv, T = 64, 2, 300
    q = oracle.f2bf(rng.standard_normal(hd).astype(np.float32))
    kc = rng.standard_normal((T, nkv, hd)).astype(np.float16)
    vc = rng.standard_normal((T, nkv, hd)).astype(np.float16)
    out = np.zeros(hd, np.uint16)
    L = oracle.lib()
    L.pbo_attn_head(oracle._p(q), oracle._p(kc.view(np.uint16)), oracle._p(vc.view(np.uint16)), 1, nkv, hd, T,
                    0, np.float32(0.125), 0, 0, oracle._p(out))
    qf = oracle.bf2f(q).astype(np.float64)
    s = kc[:, 1, :].astype(np.float64) @ qf * 0.125
    p = np.exp(s - s.max()); p /= p.sum()
    ref = p @ vc[:, 1, :].astype(np.float64)
    assert np.max(np.abs(oracle.bf2f(out) - ref)) < 2e-2 * max(1.0, np.abs(ref).max())


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(GOLDEN), "..", "oracle", "_ref",
                                                    "libpb_refpins.so")), reason="reference pins not built")
def test_pins_random_shapes(oracle):
    """more seeds and shapes straight against the reference-compiled functions."""
    R = oracle.ref()
    p = oracle._p
    rng = np.random.default_rng(11)
    for (N, K, T) in [(96, 2048, 1), (64, 4096, 2), (32, 512, 3), (64, 7680, 1), (32, 2048, 8)]:
        codes = rng.integers(-127, 128, (N, K), dtype=np.int8)
        s32 = (np.abs(rng.standard_normal((N, K // 32))) * 0.01).astype(np.float16).astype(np.float32)
        xb = oracle.f2bf(rng.standard_normal((T, K)).astype(np.float32))
        y = oracle.q8f_gemv(codes, s32, xb).reshape(T, N)
        if K // oracle.lib().pbo_q8_kchunk(K) == 1:        # cpuchk covers single-chunk shapes
            yb = oracle.f2bf(np.float32(0) + y)
            assert R.pbref_cpuchk(p(codes), p(s32), p(xb), p(yb), N, K, T, N) == 0
    for rows, K in [(64, 4096), (32, 12288)]:
        q1 = rng.integers(0, 256, rows * (K // 128) * 18, dtype=np.uint8)
        for r in range(rows):
            for b in range(K // 128):
                h = np.uint16(0x2800 + rng.integers(0, 0x1000))
                q1[(r * (K // 128) + b) * 18:(r * (K // 128) + b) * 18 + 2] = np.frombuffer(h.tobytes(), np.uint8)
        xq = np.zeros((K // 256) * 292, np.uint8)
        R.pbref_mk_q8k(p(xq), K, 7)
        wb, sc = oracle.q1_repack(q1, rows, K)
        yr = np.zeros(rows, np.float32)
        R.pbref_q1_gemv(rows, K, p(wb), p(sc), p(xq), p(yr))
        _, y = oracle.q1_gemv(wb, sc, xq, K)
        assert np.array_equal(y.view(np.uint32), yr.view(np.uint32))


# ------------------------------------------------------------------ Bonsai ----
def test_golden_bonsai_rms_rope(oracle):
    """fwd8.c's rms (:312-317) and YaRN rope (:320-369) as the reference computes them"""
    g = _load("bonsai.npz")
    for n in (4096, 128):
        y = oracle.bs_rms(g["rms%d_x" % n], g["rms%d_w" % n])
        assert np.array_equal(y.view(np.uint32), g["rms%d_y" % n].view(np.uint32))
    for i, pos in enumerate(g["rope_pos"]):
        c, s = oracle.bs_rope_table(int(pos))
        assert np.array_equal(np.concatenate([c, s]).view(np.uint32), g["rope_cs"][i].view(np.uint32)), pos
    c, s = oracle.bs_rope_table(37)
    y = oracle.bs_rope(g["rope_x"], c, s)
    assert np.array_equal(y.view(np.uint32), g["rope_y"].view(np.uint32))


def test_golden_bonsai_fa16_silu(oracle):
    """pq1_host.c's f16 flash-attention decode (:373-434) and silu tail (:226),
    bit for bit (both sides on the oracle's expf)"""
    g = _load("bonsai.npz")
    for T in (1, 2, 31, 33, 97, 512):
        out = oracle.bs_fa16_head(g["fa%d_q" % T], g["fa%d_k" % T], g["fa%d_v" % T])
        assert np.array_equal(out.view(np.uint32), g["fa%d_out" % T].view(np.uint32)), T
    o = oracle.bs_silu_mul(g["silu_g"], g["silu_u"])
    assert np.array_equal(o.view(np.uint32), g["silu_out"].view(np.uint32))


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(GOLDEN), "..", "oracle", "_ref",
                                                    "libpb_refpins.so")), reason="reference pins not built")
def test_pins_bonsai_libm_expf(oracle):
    """the reference's own attention and silu on the host libm's expf against
    the oracle (pbo_expf): the departure stays at the f16 rounding level"""
    import ctypes as C
    R = oracle.ref()
    p = oracle._p
    rng = np.random.default_rng(5)
    C.c_void_p.in_dll(R, "pbref_expf_hook").value = None
    worst = 0.0
    for T in (17, 300, 2048):
        q = rng.standard_normal(128).astype(np.float32) * 3
        K = rng.standard_normal((T, 128)).astype(np.float16).view(np.uint16)
        V = rng.standard_normal((T, 128)).astype(np.float16).view(np.uint16)
        ref = np.zeros(128, np.float32)
        R.pbref_fa16_head(p(q), p(K), p(V), T, np.float32(0.0883883476), p(ref))
        out = oracle.bs_fa16_head(q, K, V)
        worst = max(worst, float(np.max(np.abs(out - ref)) / max(1e-3, np.abs(ref).max())))
    assert worst < 2e-3, worst
    g = (rng.standard_normal(4096) * 4).astype(np.float32)
    u = rng.standard_normal(4096).astype(np.float32)
    ref = u.copy()
    R.pbref_silu_mul(p(ref), p(g), 4096)
    out = oracle.bs_silu_mul(g, u)
    rel = np.abs(out - ref) / np.maximum(np.abs(ref), 1e-30)
    assert rel.max() < 1e-6, rel.max()


def test_bonsai_oracle_decode_runs(oracle):
    """the whole Bonsai step on a tiny model: deterministic, finite, and the
    step's K/V rows are the post-rope f16 values it stored"""
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(GOLDEN), "..", "..", "pulsar-asm_b200"))
    from pulsar_b200 import synth
    c = synth.BONSAI_TINY
    w = synth.make_bonsai_weights(c, seed=3)
    a, b = oracle.BsModel(c, w, 32), oracle.BsModel(c, w, 32)
    for pos, tok in enumerate([5, 99, 1000, 7]):
        ia, la, xa = a.decode(tok, pos, want_logits=True)
        ib, lb, xb = b.decode(tok, pos, want_logits=True)
        assert ia == ib and np.array_equal(la, lb) and np.all(np.isfinite(la))
        assert ia == int(np.argmax(la))
    k = a.kv(0, 0)
    assert np.any(k[:, 3] != 0) and not np.any(k[:, 4:] != 0)
