"""Generates tests/golden/lfm3_layer.npz from the reference's OWN LFM3 layer
kernels (lfm3_nanode.cu: k_rmsnorm, k_headnorm, k_rope, k_attn_head,
k_silu_mul_bf, k_sigmoid_gate, k_mul_bf, k_shift_in + k_conv7, k_argmax),
compiled for sm_100a by oracle/build_ref.sh into oracle/_ref/libpb_refgpu.so
and run on a B200. TEST INFRASTRUCTURE ONLY.

It also holds the Q8 GEMV leaf (q8_partial + k_combine_bf, one-chunk and
chunked K) and the bf16 head (k_gemv_bf16) on seeded inputs.

Besides each kernel's seeded inputs and outputs, the file records the values
CUDA's rsqrtf / expf / cosf / sinf give for the arguments the kernels form
(the arguments are found by replaying the kernels' arithmetic in numpy,
lfm3_replay.py), so that the CPU test can replay every output bit for bit and
compare the oracle's own transcendentals with CUDA's.

Run on the GPU box from the repository root:
    python tests/golden/make_golden_lfm3.py [out.npz]
"""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
import lfm3_replay as R  # noqa: E402

LIB = os.path.join(ROOT, "oracle", "_ref", "libpb_refgpu.so")


def p(a):
    return a.ctypes.data_as(C.c_void_p)


def bf16(x):
    return R.f2bf(np.asarray(x, np.float32))


def bf16_f16_exact(rng, shape, scale=1.0):
    """bf16 values that fp16 also holds exactly (|v| >= 2^-14 or 0, |v| < 65504),
    so that the oracle's fp16 cache and the reference's bf16 cache hold the
    same numbers"""
    v = bf16(rng.standard_normal(shape) * scale)
    f = R.bf2f(v)
    v[(np.abs(f) < 2.0 ** -14)] = 0
    assert np.all(np.abs(R.bf2f(v)) < 60000)
    return v


def main(path):
    L = C.CDLL(LIB)
    vp, i, f = C.c_void_p, C.c_int, C.c_float
    for name, args in [("pbref_shapes", [vp]), ("pbref_gpu_rmsnorm", [vp, vp, vp, f]),
                       ("pbref_gpu_headnorm", [vp, vp, i, f]), ("pbref_gpu_rope", [vp, vp, i, i, i]),
                       ("pbref_gpu_attn", [vp, vp, vp, vp, i, i, f]), ("pbref_gpu_silu_mul", [vp, vp, vp, i]),
                       ("pbref_gpu_mul_bf", [vp, vp, vp, i]), ("pbref_gpu_sigmoid_gate", [vp, vp, i]),
                       ("pbref_gpu_conv", [vp, vp, vp, vp]), ("pbref_gpu_argmax", [vp, i, vp]),
                       ("pbref_gpu_expf", [vp, vp, i]), ("pbref_gpu_rsqrtf", [vp, vp, i]),
                       ("pbref_gpu_cossin", [vp, vp, vp, i]), ("pbref_gpu_q8_gemv", [vp, vp, vp, vp, i, i]),
                       ("pbref_gpu_gemv_bf16", [vp, vp, vp, i, i])]:
        getattr(L, name).argtypes = args
        getattr(L, name).restype = i
    sh = np.zeros(5, np.int32)
    L.pbref_shapes(p(sh))
    H, NH, NKV, HD, MAXTOK = (int(v) for v in sh)

    def dev(fn, x):
        x = np.ascontiguousarray(x, np.float32).reshape(-1)
        y = np.zeros_like(x)
        assert fn(p(x), p(y), x.size) == 0
        return y

    def rsq(x):
        return dev(L.pbref_gpu_rsqrtf, x)

    def ex(x):
        return dev(L.pbref_gpu_expf, x)

    def cossin(x):
        x = np.ascontiguousarray(x, np.float32).reshape(-1)
        c, s = np.zeros_like(x), np.zeros_like(x)
        assert L.pbref_gpu_cossin(p(x), p(c), p(s), x.size) == 0
        return c, s

    rng = np.random.default_rng(20261202)
    g = {"shapes": sh}
    eps = np.float32(1e-5)
    # rmsnorm: three magnitudes
    xs = np.stack([bf16(rng.standard_normal(H) * sc) for sc in (1.0, 37.0, 0.003)])
    w = (1.0 + 0.05 * rng.standard_normal(H)).astype(np.float32)
    ys, rss = [], []
    for x in xs:
        y = np.zeros(H, np.uint16)
        assert L.pbref_gpu_rmsnorm(p(x), p(w), p(y), eps) == 0
        ys.append(y)
        rss.append(rsq(R.rms_arg(x, eps))[0])
    g.update(rms_x=xs, rms_w=w, rms_y=np.stack(ys), rms_rs=np.array(rss, np.float32))
    # headnorm: NH heads
    hx = bf16(rng.standard_normal((NH, HD)) * 3.0)
    hw = (1.0 + 0.05 * rng.standard_normal(HD)).astype(np.float32)
    hy = hx.copy()
    assert L.pbref_gpu_headnorm(p(hy), p(hw), NH, eps) == 0
    g.update(hn_x=hx, hn_w=hw, hn_y=hy, hn_rs=rsq(R.headnorm_arg(hx, eps)))
    # rope: full layers (rotary over HD/2, theta 1e6) and sliding layers (all
    # of HD, theta 1e4), build_invf's tables (lfm3_nanode.cu:3719-3723,
    # :5486-5487) made by the oracle's restatement of it
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    Ol = O.lib()
    rope = []
    for base, part, rot in ((1e6, 0.5, HD // 2), (1e4, 1.0, HD)):
        invf = np.zeros(HD // 2, np.float32)
        Ol.pbo_rope_invf(p(invf), base, HD, part)
        for pos in (0, 7, 1023, MAXTOK - 1):
            x = bf16(rng.standard_normal((NH, HD)))
            y = x.copy()
            assert L.pbref_gpu_rope(p(y), p(invf), NH, pos, rot) == 0
            c, s = cossin(R.rope_angles(pos, invf, rot))
            rope.append(dict(invf=invf, pos=pos, rot=rot, x=x, y=y, c=c, s=s))
    for k in ("invf", "pos", "rot", "x", "y"):
        g["rope_" + k] = np.stack([np.asarray(r[k]) for r in rope])
    g["rope_c"] = np.stack([np.pad(r["c"], (0, HD // 2 - r["c"].size)) for r in rope])
    g["rope_s"] = np.stack([np.pad(r["s"], (0, HD // 2 - r["s"].size)) for r in rope])
    # attention: several spans, full and sliding window
    scaling = np.float32(1.0 / np.sqrt(np.float32(HD)))
    att = []
    for npos, win in ((1, 0), (37, 0), (300, 0), (1000, 0), (700, 256)):
        q = bf16_f16_exact(rng, (NH, HD), 1.0)
        kc = bf16_f16_exact(rng, (npos, NKV, HD), 1.0)
        vc = bf16_f16_exact(rng, (npos, NKV, HD), 2.0)
        out = np.zeros((NH, HD), np.uint16)
        assert L.pbref_gpu_attn(p(q), p(kc), p(vc), p(out), npos, win, scaling) == 0
        e = []
        for h in range(NH):
            sc = R.attn_scores(q[h], kc, h // (NH // NKV), npos, win, scaling)
            e.append(ex(R.attn_exp_args(sc)))
        att.append(dict(npos=npos, win=win, q=q, kc=kc, vc=vc, out=out, e=e))
    for j, a in enumerate(att):
        for k in ("q", "kc", "vc", "out"):
            g["attn%d_%s" % (j, k)] = a[k]
        g["attn%d_e" % j] = np.stack(a["e"])
        g["attn%d_cfg" % j] = np.array([a["npos"], a["win"]], np.int32)
    g["attn_n"] = np.array(len(att), np.int32)
    g["attn_scaling"] = np.array(scaling, np.float32)
    # silu * w3, sigmoid gate, B * x
    n = 8192
    sa, sb = bf16(rng.standard_normal(n) * 4.0), bf16(rng.standard_normal(n))
    sy = np.zeros(n, np.uint16)
    assert L.pbref_gpu_silu_mul(p(sa), p(sb), p(sy), n) == 0
    g.update(silu_a=sa, silu_b=sb, silu_y=sy, silu_ex=ex(-R.bf2f(sa)))
    gg = bf16(rng.standard_normal(NH) * 3.0)
    ga = bf16(rng.standard_normal((NH, HD)))
    gy = ga.copy()
    assert L.pbref_gpu_sigmoid_gate(p(gg), p(gy), NH) == 0
    g.update(gate_g=gg, gate_a=ga, gate_y=gy, gate_ex=ex(-R.bf2f(gg)))
    ma, mb = bf16(rng.standard_normal(4096) * 2), bf16(rng.standard_normal(4096) * 2)
    my = np.zeros(4096, np.uint16)
    assert L.pbref_gpu_mul_bf(p(ma), p(mb), p(my), 4096) == 0
    g.update(mul_a=ma, mul_b=mb, mul_y=my)
    # conv: a 7-slot ring, newest last
    ring = bf16(rng.standard_normal((7, H)))
    xin = bf16(rng.standard_normal(H))
    taps = (0.5 * rng.standard_normal((H, 7))).astype(np.float32)
    r2, cy = ring.copy(), np.zeros(H, np.uint16)
    assert L.pbref_gpu_conv(p(r2), p(xin), p(taps), p(cy)) == 0
    g.update(conv_ring=ring, conv_x=xin, conv_taps=taps, conv_y=cy, conv_ring_after=r2)
    # argmax over logits with a unique maximum
    am = []
    for nv in (1000, 65536, 128000):
        lg = rng.standard_normal(nv).astype(np.float32)
        lg[rng.integers(0, nv)] = 9.5
        o = np.zeros(1, np.int32)
        assert L.pbref_gpu_argmax(p(lg), nv, p(o)) == 0
        am.append((lg, int(o[0])))
    for j, (lg, o) in enumerate(am):
        g["argmax%d_lg" % j] = lg
        g["argmax%d_id" % j] = np.array(o, np.int32)
    # the Q8 GEMV leaf (q8_partial + k_combine_bf) with pick()'s chunking:
    # one 7680-code chunk (the reference model's w2), 2048-code chunks, and a
    # short one-chunk row; fp32 scales, bf16 input and output
    for j, (N, K) in enumerate(((24, 7680), (16, 8192), (40, 1024))):
        q = rng.integers(-127, 128, (N, K), dtype=np.int8)
        q[0, :32] = -128
        sc = (np.abs(rng.standard_normal((N, K // 32))) * 0.01).astype(np.float32)
        x = bf16(rng.standard_normal(K))
        y = np.zeros(N, np.uint16)
        assert L.pbref_gpu_q8_gemv(p(q), p(sc), p(x), p(y), N, K) == 0
        g.update({"q8g%d_q" % j: q, "q8g%d_s" % j: sc, "q8g%d_x" % j: x, "q8g%d_y" % j: y})
    g["q8g_n"] = np.array(3, np.int32)
    # the certified arm's bf16 head (k_gemv_bf16 via lm_head_bf16)
    wb = bf16(rng.standard_normal((64, 2048)) * 2.0)
    wb[3] = 0x8000
    xb = bf16(rng.standard_normal(2048))
    yb = np.zeros(64, np.float32)
    assert L.pbref_gpu_gemv_bf16(p(wb), p(xb), p(yb), 64, 2048) == 0
    g.update(b16_w=wb, b16_x=xb, b16_y=yb)
    np.savez_compressed(path, **g)
    print("wrote", path, "(%d arrays)" % len(g))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "lfm3_layer.npz"))
