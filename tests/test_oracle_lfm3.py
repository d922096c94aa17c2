"""The LFM3 layer oracle pinned to the reference's OWN kernels
(lfm3_nanode.cu, compiled for sm_100a and run on a B200 by
tests/golden/make_golden_lfm3.py; fixtures in tests/golden/lfm3_layer.npz).

Two checks per kernel:
 * replay: the reference's output is reproduced bit for bit by replaying its
   arithmetic in numpy (lfm3_replay.py) with CUDA's own rsqrtf / expf / cosf /
   sinf values for the arguments it forms. This pins every reduction order,
   tree shape and rounding point that the oracle and the B200 kernels share.
 * oracle: the C restatement (oracle/pb_oracle.c) gives the same bits where no
   transcendental enters (conv, B*x, argmax); where one does, it replaces
   CUDA's rsqrtf by a correctly rounded 1/sqrt, expf by its own Cody-Waite
   exponential and cosf/sinf by the double-precision table. Those values agree
   with CUDA's within 2 ulp (1.2e-7 relative), and the kernels' bf16 outputs
   then agree within one bf16 unit in the last place; the fp32-level error
   stays below the 1e-5 relative bound of the reference's own gate.
"""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "lfm3_layer.npz")
sys.path.insert(0, os.path.join(HERE, "golden"))
import lfm3_replay as R  # noqa: E402

pytestmark = pytest.mark.skipif(not os.path.exists(GOLDEN), reason="no lfm3_layer.npz fixture")


@pytest.fixture(scope="module")
def g():
    return dict(np.load(GOLDEN))


def _p(a):
    import ctypes as C
    return a.ctypes.data_as(C.c_void_p)


def _ulp_f32(a, b):
    ia = np.ascontiguousarray(a, np.float32).view(np.int32).astype(np.int64)
    ib = np.ascontiguousarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(ia - ib)


def _within_one_bf16_ulp(a, b):
    """every pair of bf16 codes equal in value (+0 / -0 included) or adjacent"""
    ia = np.asarray(a, np.uint16).astype(np.int32)
    ib = np.asarray(b, np.uint16).astype(np.int32)
    return bool(np.all((np.abs(ia - ib) <= 1) | (R.bf2f(a) == R.bf2f(b))))


def test_replay_rmsnorm(g):
    for x, y, rs in zip(g["rms_x"], g["rms_y"], g["rms_rs"]):
        assert np.array_equal(R.rms_apply(x, g["rms_w"], rs), y)


def test_oracle_rmsnorm(oracle, g):
    L = oracle.lib()
    for x, y, rs in zip(g["rms_x"], g["rms_y"], g["rms_rs"]):
        o = np.zeros_like(y)
        L.pbo_rmsnorm(_p(np.ascontiguousarray(x)), _p(g["rms_w"]), _p(o), x.size, 1e-5)
        # 1/sqrt (correctly rounded) against CUDA's rsqrtf: within 2 ulp
        arg = R.rms_arg(x, np.float32(1e-5))
        assert _ulp_f32(np.float32(1.0) / np.sqrt(arg), rs) <= 2
        assert _within_one_bf16_ulp(o, y)
        assert np.mean(o != y) < 0.01


def test_replay_headnorm(g):
    assert np.array_equal(R.headnorm_apply(g["hn_x"], g["hn_w"], g["hn_rs"]), g["hn_y"])


def test_oracle_headnorm(oracle, g):
    x = np.ascontiguousarray(g["hn_x"]).copy()
    nh, hd = x.shape
    oracle.lib().pbo_headnorm(_p(x), _p(g["hn_w"]), nh, hd, 1e-5)
    assert _within_one_bf16_ulp(x, g["hn_y"])
    assert np.mean(x != g["hn_y"]) < 0.01


def test_replay_rope(g):
    for x, y, pos, rot, c, s in zip(g["rope_x"], g["rope_y"], g["rope_pos"], g["rope_rot"], g["rope_c"], g["rope_s"]):
        half = int(rot) // 2
        assert np.array_equal(R.rope_apply(x, c[:half], s[:half], int(rot)), y)


def test_oracle_rope(oracle, g):
    L = oracle.lib()
    for x, y, pos, rot, invf, c, s in zip(g["rope_x"], g["rope_y"], g["rope_pos"], g["rope_rot"], g["rope_invf"],
                                          g["rope_c"], g["rope_s"]):
        half = int(rot) // 2
        co, so = np.zeros(half, np.float32), np.zeros(half, np.float32)
        L.pbo_rope_cs(_p(np.ascontiguousarray(invf)), int(pos), half, _p(co), _p(so))
        assert np.all(_ulp_f32(co, c[:half]) <= 2) and np.all(_ulp_f32(so, s[:half]) <= 2)
        xo = np.ascontiguousarray(x).copy()
        L.pbo_rope(_p(xo), xo.shape[0], xo.shape[1], half, _p(co), _p(so))
        assert _within_one_bf16_ulp(xo, y)


def _attn_cases(g):
    for j in range(int(g["attn_n"])):
        npos, win = (int(v) for v in g["attn%d_cfg" % j])
        yield (npos, win, g["attn%d_q" % j], g["attn%d_kc" % j], g["attn%d_vc" % j], g["attn%d_out" % j],
               g["attn%d_e" % j])


def test_replay_attention(g):
    nh = int(g["shapes"][1])
    nkv = int(g["shapes"][2])
    for npos, win, q, kc, vc, out, e in _attn_cases(g):
        for h in range(nh):
            got = R.attn_apply(e[h], vc, h // (nh // nkv), npos, win)
            assert np.array_equal(got, out[h]), "head %d npos %d win %d" % (h, npos, win)


def test_oracle_attention(oracle, g):
    """the oracle's attention over an fp16 cache holding the same numbers (the
    fixtures' K/V values are exact in both bf16 and fp16)"""
    L = oracle.lib()
    nh, nkv, hd = (int(v) for v in g["shapes"][1:4])
    scaling = float(g["attn_scaling"])
    for npos, win, q, kc, vc, out, e in _attn_cases(g):
        k16 = R.bf2f(kc).astype(np.float16).view(np.uint16)
        v16 = R.bf2f(vc).astype(np.float16).view(np.uint16)
        assert np.array_equal(k16.view(np.float16).astype(np.float32), R.bf2f(kc))
        for h in range(nh):
            sc = R.attn_scores(q[h], kc, h // (nh // nkv), npos, win, scaling)
            args = R.attn_exp_args(sc)
            mine = np.array([L.pbo_expf(float(a)) for a in args], np.float32)
            assert np.all(_ulp_f32(mine, e[h]) <= 2)
            o = np.zeros(hd, np.uint16)
            L.pbo_attn_head(_p(np.ascontiguousarray(q[h])), _p(k16), _p(v16), h // (nh // nkv), nkv, hd, npos, win,
                            scaling, 0, 0, _p(o))
            assert _within_one_bf16_ulp(o, out[h]), "head %d npos %d win %d" % (h, npos, win)


def test_replay_silu_and_gate(g):
    assert np.array_equal(R.silu_apply(g["silu_a"], g["silu_b"], g["silu_ex"]), g["silu_y"])
    assert np.array_equal(R.gate_apply(g["gate_g"], g["gate_a"], g["gate_ex"]), g["gate_y"])


def test_oracle_silu_and_gate(oracle, g):
    L = oracle.lib()
    n = g["silu_a"].size
    y = np.zeros(n, np.uint16)
    L.pbo_silu_mul_bf(_p(g["silu_a"]), _p(g["silu_b"]), _p(y), n)
    assert _within_one_bf16_ulp(y, g["silu_y"])
    a = np.ascontiguousarray(g["gate_a"]).copy()
    L.pbo_sigmoid_gate(_p(g["gate_g"]), _p(a), a.shape[0], a.shape[1])
    assert _within_one_bf16_ulp(a, g["gate_y"])
    mine = np.array([L.pbo_expf(float(-v)) for v in R.bf2f(g["silu_a"])], np.float32)
    assert np.all(_ulp_f32(mine, g["silu_ex"]) <= 2)


def test_oracle_conv_mul_argmax_bitexact(oracle, g):
    L = oracle.lib()
    ring = np.ascontiguousarray(g["conv_ring"]).copy()
    H = ring.shape[1]
    y = np.zeros(H, np.uint16)
    L.pbo_conv_step(_p(ring), _p(g["conv_x"]), _p(g["conv_taps"]), 7, H, _p(y))
    assert np.array_equal(y, g["conv_y"]) and np.array_equal(ring, g["conv_ring_after"])
    mul = R.f2bf(R.bf2f(g["mul_a"]) * R.bf2f(g["mul_b"]))
    assert np.array_equal(mul, g["mul_y"])
    for j in range(3):
        lg = g["argmax%d_lg" % j]
        assert L.pbo_argmax(_p(lg), lg.size) == int(g["argmax%d_id" % j])


def test_oracle_q8_gemv_leaf_bitexact(oracle, g):
    """q8_partial + k_combine_bf with pick()'s chunking, the reference's own
    kernels: one 7680-code chunk (lane chains over blocks l, l+32, ... of the
    whole row, one tree), 2048-code chunks summed ascending, a short row"""
    if "q8g_n" not in g:
        pytest.skip("fixture predates the GEMV cases")
    for j in range(int(g["q8g_n"])):
        q, sc, x, y = g["q8g%d_q" % j], g["q8g%d_s" % j], g["q8g%d_x" % j], g["q8g%d_y" % j]
        want = oracle.f2bf(np.float32(0) + oracle.q8f_gemv(q, sc, x))
        assert np.array_equal(want, y), "case %d (K %d)" % (j, q.shape[1])


def test_oracle_bf16_head_bitexact(oracle, g):
    """k_gemv_bf16 (lm_head_bf16) of the reference against the oracle"""
    if "b16_w" not in g:
        pytest.skip("fixture predates the bf16 head")
    got = oracle.gemv_bf16(g["b16_w"], g["b16_x"])
    assert np.array_equal(got.view(np.uint32), np.ascontiguousarray(g["b16_y"]).view(np.uint32))
