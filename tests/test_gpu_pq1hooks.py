"""The Bonsai host hooks fwd8.c calls through pq1_fwd8_shim.h:24-60, driven
the way fwd8.c drives them (host Q1_0 weights and norms, the token's fp32
embedding row, the position's rope row), bit for bit against the oracle's
fwd8 token step: the logits each step writes to the host, pq1_head_top after
pq1_head_need(0), two interleaved sessions, the first token run on the host
with its K/V rows mirrored by pq1_attn_kv_put (fwd8.c's own flow), and the
calls that must decline."""
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


def test_pq1_token_fused_sessions(oracle, pb, cuda):
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
    oms = [oracle.BsModel(c, w, ctx), oracle.BsModel(c, w, ctx)]
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
