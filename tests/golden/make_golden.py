"""Generates the golden fixtures in this folder from the REFERENCE's own CPU
functions, compiled from the reference sources by oracle/build_ref.sh into
oracle/_ref/libpb_refpins.so. Run here (where the reference tree exists):

    python tests/golden/make_golden.py

Fixtures (numpy .npz, inputs and the reference's outputs):
  q1_parity.npz     pq1_parity.c's seeded Q1_0 gate inputs (weights srand(31337),
                    Q8_K mk_q8k seed 99) at 256x4096 and the output of the
                    reference's pq1_split_repack + pq1_gemv_cpu (pq1_host.c:78-120)
  q8k_rms.npz       rms_ref (pq1_parity.c:119-147): RMS + Q8_K bytes for three
                    vectors (random, a tie at the block maximum, an all-zero block)
  q80_quant.npz     the Q8_0 activation quantizer q8() (fwd35_ref.c:333-344)
  q8f_tree.npz      REF_FLOAT GEMV outputs that the reference's own scalar
                    transcription cpuchk_run (lfm3_nanode.cu:4658-4684) accepts
                    with zero bitwise differences (single-chunk shapes, T = 1 and 4)
  q8_gemv_cpu.npz   the x86/C CPU GEMV gemv_q8 (.auto/lfm3/q8_gemv_cpu.c:29-60)
                    output, a different summation order: a tolerance fixture
  bonsai.npz        the Bonsai step pieces: fwd8.c's rms (:312-317), YaRN rope
                    table and rotation (:320-369, gcc's default contraction),
                    pq1_host.c's f16 flash-attention decode (:373-434) and silu
                    tail (:226), the last two with expf set to the oracle's
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402


def main():
    O.build()
    R = O.ref()
    if R is None:
        sys.exit("reference pins not built (needs the reference tree)")
    p = O._p
    # ---- Q1 parity gate inputs and the reference's output
    rows, K = 256, 4096
    q1 = np.zeros(rows * (K // 128) * 18, np.uint8)
    R.pbref_parity_q1_weights(p(q1), rows, K)
    xq = np.zeros((K // 256) * 292, np.uint8)
    R.pbref_mk_q8k(p(xq), K, 99)
    wb = np.zeros((rows, K // 32), np.uint32)
    sc = np.zeros((rows, K // 128), np.uint16)
    R.pbref_q1_repack(p(q1), rows, K, p(wb), p(sc))
    y = np.zeros(rows, np.float32)
    R.pbref_q1_gemv(rows, K, p(wb), p(sc), p(xq), p(y))
    np.savez_compressed(os.path.join(HERE, "q1_parity.npz"), q1=q1, xq=xq, rows=rows, K=K, y=y)

    # ---- RMS + Q8_K chain
    rng = np.random.default_rng(20261201)
    n = 1024
    xs = [rng.standard_normal(n).astype(np.float32) * 3]
    t = rng.standard_normal(n).astype(np.float32)
    t[17] = 9.0
    t[40] = -9.0          # same |x|: the first index must win
    xs.append(t)
    z = rng.standard_normal(n).astype(np.float32)
    z[256:512] = 0.0      # an all-zero Q8_K block after the norm
    xs.append(z)
    w = (1 + 0.1 * rng.standard_normal(n)).astype(np.float32)
    outs = []
    for x in xs:
        xx = x.copy()
        q = np.zeros((n // 256) * 292, np.uint8)
        R.pbref_rms_q8k(p(xx), None, p(w), n, p(q))
        outs.append(q)
    np.savez_compressed(os.path.join(HERE, "q8k_rms.npz"), x=np.stack(xs), w=w, xq=np.stack(outs))

    # ---- Q8_0 activation quantizer
    xa = (rng.standard_normal(2048) * 2).astype(np.float32)
    xa[64:96] = 0.0       # an all-zero block
    qr = np.zeros(2048, np.int8)
    dr = np.zeros(64, np.float32)
    R.pbref_q80_quant(p(xa), 2048, p(qr), p(dr))
    np.savez_compressed(os.path.join(HERE, "q80_quant.npz"), x=xa, q=qr, d=dr)

    # ---- REF_FLOAT GEMV, accepted bit for bit by cpuchk_run
    cases = {}
    for tag, (N, Kc, T) in {"a": (64, 2048, 4), "b": (32, 7680, 2), "c": (32, 1024, 1)}.items():
        codes = rng.integers(-127, 128, (N, Kc), dtype=np.int8)
        s16 = (np.abs(rng.standard_normal((N, Kc // 32))) * 0.01).astype(np.float16)
        s32 = s16.astype(np.float32)
        xb = O.f2bf(rng.standard_normal((T, Kc)).astype(np.float32))
        yo = O.q8f_gemv(codes, s32, xb).reshape(T, N)
        yb = O.f2bf(np.float32(0) + yo)
        bad = R.pbref_cpuchk(p(codes), p(s32), p(xb), p(yb), N, Kc, T, N)
        assert bad == 0, "cpuchk_run rejects the oracle (%d)" % bad
        cases[tag] = (codes, s16, xb, yb)
    np.savez_compressed(os.path.join(HERE, "q8f_tree.npz"),
                        **{"%s_%s" % (t, k): v for t, c in cases.items()
                           for k, v in zip(("codes", "s16", "x", "y"), c)})

    # ---- gemv_q8 (different order) for the tolerance check
    N, Kc = 128, 2048
    codes = rng.integers(-127, 128, (N, Kc), dtype=np.int8)
    s32 = (np.abs(rng.standard_normal((N, Kc // 32))) * 0.01).astype(np.float16).astype(np.float32)
    xb = O.f2bf(rng.standard_normal(Kc).astype(np.float32))
    xf = O.bf2f(xb)
    yr = np.zeros(N, np.float32)
    R.pbref_gemv_q8(p(codes), p(s32), p(xf), p(yr), N, Kc)
    np.savez_compressed(os.path.join(HERE, "q8_gemv_cpu.npz"), codes=codes, s=s32, x=xb, y=yr)

    # ---- Bonsai step pieces (fwd8.c rms and YaRN rope; pq1_host.c f16
    #      attention and silu tail, their expf pointed at the oracle's)
    np.savez_compressed(os.path.join(HERE, "bonsai.npz"), **bonsai_fixtures(R))
    print("golden fixtures written to", HERE)


def set_expf_hook(R, on):
    import ctypes as C
    h = C.c_void_p.in_dll(R, "pbref_expf_hook")
    h.value = C.cast(O.lib().pbo_expf, C.c_void_p).value if on else None


def bonsai_fixtures(R):
    p = O._p
    rng = np.random.default_rng(8)
    f = {}
    for n in (4096, 128):
        x = (rng.standard_normal(n) * 2).astype(np.float32)
        w = (1 + 0.05 * rng.standard_normal(n)).astype(np.float32)
        y = np.zeros(n, np.float32)
        R.pbref_bs_rms(p(x), p(w), n, p(y))
        f["rms%d_x" % n], f["rms%d_w" % n], f["rms%d_y" % n] = x, w, y
    pos = np.array([0, 1, 7, 100, 1023, 2047, 8191, 16383], np.int32)
    cs = np.zeros((len(pos), 128), np.float32)
    for i, ps in enumerate(pos):
        R.pbref_bs_rope_table(int(ps), p(cs[i]), p(cs[i, 64:]))
    f["rope_pos"], f["rope_cs"] = pos, cs
    xr = rng.standard_normal(4 * 128).astype(np.float32)
    yr = xr.copy()
    R.pbref_bs_rope(p(yr), 4, 37)
    f["rope_x"], f["rope_y"] = xr, yr
    set_expf_hook(R, True)
    for T in (1, 2, 31, 33, 97, 512):
        q = rng.standard_normal(128).astype(np.float32) * 3
        K = rng.standard_normal((T, 128)).astype(np.float16).view(np.uint16)
        V = rng.standard_normal((T, 128)).astype(np.float16).view(np.uint16)
        if T > 8:
            K[T // 2] = K[3]       # an exact tie of two scores
        out = np.zeros(128, np.float32)
        R.pbref_fa16_head(p(q), p(K), p(V), T, np.float32(0.0883883476), p(out))
        f["fa%d_q" % T], f["fa%d_k" % T], f["fa%d_v" % T], f["fa%d_out" % T] = q, K, V, out
    g = (rng.standard_normal(4096) * 4).astype(np.float32)
    u = rng.standard_normal(4096).astype(np.float32)
    o = u.copy()
    R.pbref_silu_mul(p(o), p(g), 4096)
    f["silu_g"], f["silu_u"], f["silu_out"] = g, u, o
    set_expf_hook(R, False)
    return f


if __name__ == "__main__":
    main()
