"""The Bonsai host hooks fwd8.c calls through pq1_fwd8_shim.h:24-60, driven
the way fwd8.c drives them (host Q1_0 weights and norms, the token's fp32
embedding row, the position's rope row), bit for bit against the oracle's
fwd8 token step: the logits each step writes to the host, pq1_head_top after
pq1_head_need(0), two interleaved sessions, the first token run on the host
with its K/V rows mirrored by pq1_attn_kv_put (fwd8.c's own flow), and the
calls that must decline; and the per-layer hooks pq1_attn_fused /
pq1_ffn_fused with their debug hooks, continued by pq1_token_fused on the
same cache."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _embed_row(blocks):
    """fwd8.c:438-452, the Q1_0 embedding row: x = bit ? sc : -sc, sc the
    block's fp16 scale widened, bits LSB first"""
    sc = blocks[:, 0:2].copy().view(np.float16).astype(np.float32)[:, 0]
    bits = np.unpackbits(blocks[:, 2:18], axis=1, bitorder="little").astype(bool)
    return np.where(bits, sc[:, None], -sc[:, None]).reshape(-1).astype(np.float32)


@pytest.mark.parametrize("kvtq", [0, 4])
def test_pq1_token_fused_sessions(oracle, pb, cuda, monkeypatch, kvtq):
    """PQ1_KVTQ=0: the f16 cache; 4: the TurboQuant cache (the reference's
    default), the host-run first token's rows coded by pq1_attn_kv_put"""
    monkeypatch.setenv("PQ1_KVTQ", str(kvtq))
    from pulsar_b200 import synth
    c = dict(synth.BONSAI_TINY)
    w = synth.make_bonsai_weights(c, seed=31)
    nl, H, F, NH, NKV, V = c["n_layers"], c["hidden"], c["inter"], c["n_heads"], c["n_kv"], c["vocab"]
    ctx = 64
    L = pb.lib()
    vp, i, fp = C.c_void_p, C.c_int, C.POINTER(C.c_float)
    L.pq1_kv_shape.argtypes = [i, i, i]
    L.pq1_token_fused.argtypes = [i, vp, vp, i, i, i, i, i, i, i, vp, vp, vp, vp]
    L.pq1_token_fused.restype = i
    L.pq1_head_need.argtypes = [i]
    L.pq1_head_top.argtypes = [fp]
    L.pq1_head_top.restype = i
    L.pq1_sess_init.argtypes = [i]
    L.pq1_sess_init.restype = i
    L.pq1_sess_select.argtypes = [i]
    L.pq1_attn_kv_put.argtypes = [i, i, i, i, i, vp, vp]
    L.pq1_attn_kv_put.restype = i
    L.pb_pq1_hooks_reset.restype = i
    assert L.pb_pq1_hooks_reset() == 0
    O = oracle.lib()
    O.pbo_bs_rope_table.argtypes = [i, C.c_float, i, C.c_float, vp, vp]
    keep = []
    wt = (vp * (7 * nl + 1))()
    nw = (vp * (4 * nl + 1))()
    for il, d in enumerate(w["layers"]):
        for k, name in enumerate(("q", "k", "v", "o", "gate", "up", "down")):
            a = np.ascontiguousarray(d[name])
            keep.append(a)
            wt[7 * il + k] = a.ctypes.data
        for k, name in enumerate(("attn_norm", "ffn_norm", "q_norm", "k_norm")):
            a = np.ascontiguousarray(d[name], np.float32)
            keep.append(a)
            nw[4 * il + k] = a.ctypes.data
    emb = np.ascontiguousarray(w["embed"])
    onorm = np.ascontiguousarray(w["out_norm"], np.float32)
    keep += [emb, onorm]
    wt[7 * nl] = emb.ctypes.data          # tied: output.weight is the table
    nw[4 * nl] = onorm.ctypes.data

    def step(tok, pos, head):
        rc_, rs_ = np.zeros(64, np.float32), np.zeros(64, np.float32)
        O.pbo_bs_rope_table(pos, c["rope_factor"], c["rope_orig_ctx"], c["rope_base"],
                            rc_.ctypes.data, rs_.ctypes.data)
        x = _embed_row(emb[tok])
        return L.pq1_token_fused(nl, wt, nw, NH, NKV, H, F, V, ctx, pos, rc_.ctypes.data, rs_.ctypes.data,
                                 x.ctypes.data, head.ctypes.data if head is not None else None), x

    # nothing runs before the cache shape is known
    head = np.zeros(V, np.float32)
    assert step(5, 0, head)[0] == -1
    L.pq1_kv_shape(nl, NKV, ctx)
    assert L.pq1_sess_init(2) == 0
    oms = [oracle.BsModel(c, w, ctx, kv_bits=kvtq), oracle.BsModel(c, w, ctx, kv_bits=kvtq)]
    rng = np.random.default_rng(8)
    toks = [rng.integers(0, V, 16), rng.integers(0, V, 16)]
    nxt = [0, 0]

    def run(sess, n, need=True):
        L.pq1_sess_select(sess)
        L.pq1_head_need(1 if need else 0)
        for _ in range(n):
            pos = nxt[sess]
            tok = int(toks[sess][pos])
            head = np.full(V, np.nan, np.float32)
            rc, x = step(tok, pos, head)
            assert rc == 0, "session %d position %d declined: %s" % (sess, pos, pb.last_error())
            want, lg, _ = oms[sess].decode(tok, pos, x_in=x, want_logits=True)
            if need:
                assert np.array_equal(_bits(head), _bits(lg)), "session %d position %d" % (sess, pos)
            else:
                assert np.all(np.isnan(head)), "logits copied although not needed"
            v = C.c_float()
            assert L.pq1_head_top(C.byref(v)) == want
            assert _bits(np.float32(v.value)) == _bits(lg[want])
            assert L.pq1_head_top(C.byref(v)) == -1      # consumed
            nxt[sess] += 1

    # session 0 as fwd8.c runs a sequence: the first token on the host (here
    # the oracle), its K/V rows mirrored layer by layer, the fused path after
    L.pq1_sess_select(0)
    tok0 = int(toks[0][0])
    oms[0].decode(tok0, 0, x_in=_embed_row(emb[tok0]))
    for il in range(nl):
        k0 = np.ascontiguousarray(oms[0].kv(il, 0)[:, 0, :])
        v0 = np.ascontiguousarray(oms[0].kv(il, 1)[:, 0, :])
        assert L.pq1_attn_kv_put(il, nl, NKV, ctx, 1, k0.ctypes.data, v0.ctypes.data) == -1   # not its next position
        assert L.pq1_attn_kv_put(il, nl, NKV, ctx, 0, k0.ctypes.data, v0.ctypes.data) == 0
    nxt[0] = 1
    run(0, 6)
    run(1, 4)
    run(0, 3, need=False)
    run(1, 2)
    # a position the session's cache does not continue, and a changed shape, decline
    L.pq1_sess_select(1)
    assert step(int(toks[1][0]), nxt[1] + 1, head)[0] == -1
    L.pq1_kv_shape(nl, NKV, ctx * 2)
    assert step(int(toks[1][0]), nxt[1], head)[0] == -1
    L.pq1_kv_shape(nl, NKV, ctx)
    run(1, 1)
    # sessions are fixed once a step has run
    assert L.pq1_sess_init(3) == -1


def _q1_ref(blocks, rows, K, xq, oracle):
    wb, sc = oracle.q1_repack(np.ascontiguousarray(blocks), rows, K)
    return oracle.q1_gemv(wb, sc, xq, K)[1]


def _f16(a):
    return np.ascontiguousarray(a, np.float32).astype(np.float16).view(np.uint16)


@pytest.mark.parametrize("kvtq", [0, 4])
def test_pq1_layer_hooks(oracle, pb, cuda, monkeypatch, kvtq):
    """fwd8.c's per-layer flow (fwd8.c:812-883): host RMS norm and Q8_K, then
    pq1_attn_fused and pq1_ffn_fused per layer (the first token's attention
    on the host with its rows mirrored, as fwd8 runs it), each output and the
    PQ1_ATT_CHECK / PQ1_FFN_CHECK debug values bit for bit against the
    oracle's restatement of attn_cpu and the FFN tail; then pq1_token_fused
    continues the same cache. PQ1_KVTQ=0: the f16 cache; 4: the TurboQuant
    cache (rows coded at their store, attention over the codes; no f16 rows
    for pq1_attn_dbg, as in the reference)."""
    monkeypatch.setenv("PQ1_KVTQ", str(kvtq))
    from pulsar_b200 import synth
    c = dict(synth.BONSAI_TINY)
    w = synth.make_bonsai_weights(c, seed=47)
    nl, H, F, NH, NKV, V = c["n_layers"], c["hidden"], c["inter"], c["n_heads"], c["n_kv"], c["vocab"]
    QD, KD, G, ctx = NH * 128, NKV * 128, NH // NKV, 64
    L = pb.lib()
    vp, i, ul = C.c_void_p, C.c_int, C.c_ulong
    L.pb_pq1_hooks_reset.restype = i
    L.pq1_kv_shape.argtypes = [i, i, i]
    L.pq1_attn_kv_put.argtypes = [i, i, i, i, i, vp, vp]
    L.pq1_attn_kv_put.restype = i
    L.pq1_attn_fused.argtypes = [i, vp, vp, vp, vp, vp, vp, i, i, i, i, i, vp, vp, vp, vp]
    L.pq1_attn_fused.restype = i
    L.pq1_ffn_fused.argtypes = [vp, vp, vp, i, i, vp, vp]
    L.pq1_ffn_fused.restype = i
    L.pq1_attn_dbg.argtypes = [i, i, vp, vp, vp, vp, i]
    L.pq1_ffn_dbg_xq.argtypes = [vp, ul]
    L.pq1_token_fused.argtypes = [i, vp, vp, i, i, i, i, i, i, i, vp, vp, vp, vp]
    L.pq1_token_fused.restype = i
    L.pq1_head_need.argtypes = [i]
    assert L.pb_pq1_hooks_reset() == 0
    lw = [{k: np.ascontiguousarray(v) for k, v in d.items()} for d in w["layers"]]
    for d in lw:
        for k in ("attn_norm", "ffn_norm", "q_norm", "k_norm"):
            d[k] = np.ascontiguousarray(d[k], np.float32)
    emb = np.ascontiguousarray(w["embed"])
    onorm = np.ascontiguousarray(w["out_norm"], np.float32)
    kc = [np.zeros((NKV, ctx, 128), np.uint16) for _ in range(nl)]
    vc = [np.zeros((NKV, ctx, 128), np.uint16) for _ in range(nl)]

    def attn(il, x, pos, rc_, rs_, on_device):
        d = lw[il]
        xq = oracle.q8k_quant(oracle.bs_rms(x, d["attn_norm"]))
        qf = _q1_ref(d["q"], QD, H, xq, oracle)
        kf = _q1_ref(d["k"], KD, H, xq, oracle)
        vf = _q1_ref(d["v"], KD, H, xq, oracle)
        qf = np.concatenate([oracle.bs_rms(qf[h * 128:(h + 1) * 128], d["q_norm"]) for h in range(NH)])
        kf = np.concatenate([oracle.bs_rms(kf[h * 128:(h + 1) * 128], d["k_norm"]) for h in range(NKV)])
        qf, kf = oracle.bs_rope(qf, rc_, rs_), oracle.bs_rope(kf, rc_, rs_)
        kr, vr = _f16(kf).reshape(NKV, 128), _f16(vf).reshape(NKV, 128)
        kc[il][:, pos], vc[il][:, pos] = kr, vr
        if kvtq:
            tkc, tks = oracle.tq_rows(kc[il][:, :pos + 1].reshape(-1, 128), kvtq)
            tvc, tvs = oracle.tq_rows(vc[il][:, :pos + 1].reshape(-1, 128), kvtq)
            tkc, tvc = tkc.reshape(NKV, pos + 1, -1), tvc.reshape(NKV, pos + 1, -1)
            tks, tvs = tks.reshape(NKV, pos + 1), tvs.reshape(NKV, pos + 1)
            at = np.concatenate([oracle.tq_attn(qf[kh * 512:(kh + 1) * 512].reshape(4, 128), kvtq, kvtq, tkc[kh],
                                                tks[kh], tvc[kh], tvs[kh], pos + 1).reshape(-1)
                                 for kh in range(NKV)])
        else:
            at = np.concatenate([oracle.bs_fa16_head(qf[h * 128:(h + 1) * 128], kc[il][h // G, :pos + 1],
                                                     vc[il][h // G, :pos + 1]) for h in range(NH)])
        ao = _q1_ref(d["o"], H, QD, oracle.q8k_quant(at), oracle)
        if not on_device:
            assert L.pq1_attn_kv_put(il, nl, NKV, ctx, pos, np.ascontiguousarray(kr).ctypes.data,
                                     np.ascontiguousarray(vr).ctypes.data) == 0
            return ao
        got = np.full(H, np.nan, np.float32)
        assert L.pq1_attn_fused(il, d["q"].ctypes.data, d["k"].ctypes.data, d["v"].ctypes.data, d["o"].ctypes.data,
                                d["q_norm"].ctypes.data, d["k_norm"].ctypes.data, NH, NKV, H, ctx, pos,
                                rc_.ctypes.data, rs_.ctypes.data, xq.ctypes.data, got.ctypes.data) == 0, \
            pb.last_error()
        assert np.array_equal(_bits(got), _bits(ao)), "attention output, layer %d position %d" % (il, pos)
        if kvtq:
            return got
        kd, vd = np.zeros((NKV, 128), np.uint16), np.zeros((NKV, 128), np.uint16)
        qd, od = np.zeros(QD, np.float32), np.zeros(QD, np.float32)
        L.pq1_attn_dbg(il, pos, kd.ctypes.data, vd.ctypes.data, qd.ctypes.data, od.ctypes.data, NH)
        assert np.array_equal(kd, kr) and np.array_equal(vd, vr), "K/V rows, layer %d position %d" % (il, pos)
        assert np.array_equal(_bits(qd), _bits(qf)), "post-rope q, layer %d position %d" % (il, pos)
        assert np.array_equal(_bits(od), _bits(at)), "attention, layer %d position %d" % (il, pos)
        return got

    def ffn(il, x):
        d = lw[il]
        xq = oracle.q8k_quant(oracle.bs_rms(x, d["ffn_norm"]))
        u = oracle.bs_silu_mul(_q1_ref(d["gate"], F, H, xq, oracle), _q1_ref(d["up"], F, H, xq, oracle))
        dq = oracle.q8k_quant(u)
        fo = _q1_ref(d["down"], H, F, dq, oracle)
        got = np.full(H, np.nan, np.float32)
        assert L.pq1_ffn_fused(d["gate"].ctypes.data, d["up"].ctypes.data, d["down"].ctypes.data, F, H,
                               xq.ctypes.data, got.ctypes.data) == 0, pb.last_error()
        assert np.array_equal(_bits(got), _bits(fo)), "FFN output, layer %d" % il
        xd = np.zeros(dq.size, np.uint8)
        L.pq1_ffn_dbg_xq(xd.ctypes.data, xd.size)
        for b in range(F // 256):   # fwd8's ffn_check compares d and qs (the first 260 bytes)
            assert np.array_equal(xd[b * 292:b * 292 + 260], dq[b * 292:b * 292 + 260]), "down activation block %d" % b
        return got

    rng = np.random.default_rng(12)
    toks = rng.integers(0, V, 12)
    xs = [_embed_row(emb[int(t)]) for t in toks]
    d0 = lw[0]
    x = xs[0].copy()
    rc0, rs0 = oracle.bs_rope_table(0)
    # before the cache shape is known the attention hook declines
    xq0 = oracle.q8k_quant(oracle.bs_rms(x, d0["attn_norm"]))
    ao0 = np.zeros(H, np.float32)
    assert L.pq1_attn_fused(0, d0["q"].ctypes.data, d0["k"].ctypes.data, d0["v"].ctypes.data, d0["o"].ctypes.data,
                            d0["q_norm"].ctypes.data, d0["k_norm"].ctypes.data, NH, NKV, H, ctx, 1,
                            rc0.ctypes.data, rs0.ctypes.data, xq0.ctypes.data, ao0.ctypes.data) == -1
    L.pq1_kv_shape(nl, NKV, ctx)
    npos_layer = 6
    for pos in range(npos_layer):
        rc_, rs_ = oracle.bs_rope_table(pos)
        x = xs[pos].copy()
        for il in range(nl):
            if pos == 1 and il == 0:   # a position the layer's cache does not continue declines
                d = lw[0]
                assert L.pq1_attn_fused(0, d["q"].ctypes.data, d["k"].ctypes.data, d["v"].ctypes.data,
                                        d["o"].ctypes.data, d["q_norm"].ctypes.data, d["k_norm"].ctypes.data,
                                        NH, NKV, H, ctx, 2, rc_.ctypes.data, rs_.ctypes.data, xq0.ctypes.data,
                                        ao0.ctypes.data) == -1
            x = x + attn(il, x, pos, rc_, rs_, on_device=pos > 0)
            x = x + ffn(il, x)
    # the whole-token hook continues the cache the per-layer hooks wrote
    om = oracle.BsModel(c, w, ctx, kv_bits=kvtq)
    for il in range(nl):
        om.set_kv(il, 0, kc[il])
        om.set_kv(il, 1, vc[il])
    om.tq_recode(npos_layer)
    wt = (vp * (7 * nl + 1))()
    nw = (vp * (4 * nl + 1))()
    for il, d in enumerate(lw):
        for k, name in enumerate(("q", "k", "v", "o", "gate", "up", "down")):
            wt[7 * il + k] = d[name].ctypes.data
        for k, name in enumerate(("attn_norm", "ffn_norm", "q_norm", "k_norm")):
            nw[4 * il + k] = d[name].ctypes.data
    wt[7 * nl] = emb.ctypes.data
    nw[4 * nl] = onorm.ctypes.data
    L.pq1_head_need(1)
    for pos in range(npos_layer, npos_layer + 4):
        rc_, rs_ = oracle.bs_rope_table(pos)
        head = np.full(V, np.nan, np.float32)
        assert L.pq1_token_fused(nl, wt, nw, NH, NKV, H, F, V, ctx, pos, rc_.ctypes.data, rs_.ctypes.data,
                                 xs[pos].ctypes.data, head.ctypes.data) == 0, pb.last_error()
        _, lg, _ = om.decode(int(toks[pos]), pos, x_in=xs[pos], want_logits=True)
        assert np.array_equal(_bits(head), _bits(lg)), "token path after the per-layer hooks, position %d" % pos
    assert L.pb_pq1_hooks_reset() == 0
