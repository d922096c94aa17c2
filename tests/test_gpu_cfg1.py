"""Parity at the benchmarked configuration itself (cfg1: hidden 2048, 24
layers, FFN 8192, 32/8 heads x 64, conv width 3, vocab 65536), through the
persistent decode kernel that the bench times, against the CPU oracle's
restatement of layer_body + head + argmax (lfm3_nanode.cu:3739-3856,
:3634-3664, :942-964), bit for bit.

The first test seeds both states with the same random fp16 K/V rows for
positions below 1020 and the same conv-ring history, then decodes 8 tokens at
positions 1020..1027 (attention spans up to 1028 keys, the FFN-8192 schedule,
the 65536-row head with its 148-CTA argmax) and compares every step's logits,
final residual and id, then the K/V rows and rings. The second compares 256
greedy ids from position 0 at the cfg1 shape."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

P0 = 1020          # first decoded position of the seeded-cache test
NSTEP = 8
MAX_CTX = 1032


@pytest.fixture(scope="module")
def cfg1(tmp_path_factory, oracle, pb, cuda):
    from pulsar_b200 import synth
    c = dict(synth.LFM3_CFG1)
    w = synth.make_weights(c, seed=2024)
    path = str(tmp_path_factory.mktemp("cfg1") / "cfg1.lfm3q8")
    synth.write_model(path, c, w)
    m = pb.Model(path)
    return c, w, m


def _bits32(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _seed_state(c, s, om, rng, p0):
    """same KV rows (positions < p0) and ring history in the device state and
    the oracle; device KV [attn layer][2][max_ctx][n_kv][hd], rings
    [conv layer][W][H] with slot = position mod W"""
    torch = pytest.importorskip("torch")
    from pulsar_b200 import _view_device
    NKV, HD, H, W = c["n_kv"], c["head_dim"], c["hidden"], c["conv_w"]
    per = MAX_CTX * NKV * HD
    kv_all = np.zeros((len(c["attn_layers"]), 2, per), np.uint16)
    for ai, L in enumerate(c["attn_layers"]):
        for which in (0, 1):
            a = (rng.standard_normal((MAX_CTX, NKV, HD)) * (0.5 + which)).astype(np.float16).view(np.uint16)
            a[p0:] = 0
            kv_all[ai, which] = a.reshape(-1)
            om.set_kv(L, which, a)
    p, n = s.debug_ptr(0)
    assert n == kv_all.nbytes
    _view_device(p, n).copy_(torch.from_numpy(kv_all.view(np.uint8).reshape(-1)).cuda())
    conv = [L for L in range(c["n_layers"]) if L not in c["attn_layers"]]
    rings = np.zeros((len(conv), W, H), np.uint16)
    for ci, L in enumerate(conv):
        hist = np.asarray(rng.standard_normal((W, H)), np.float32)
        hb = oracle_f2bf(hist)                 # row k: position p0 - W + k
        om.set_ring(L, hb)
        for k in range(W):
            rings[ci, (p0 - W + k) % W] = hb[k]
    p, n = s.debug_ptr(1)
    assert n == rings.nbytes
    _view_device(p, n).copy_(torch.from_numpy(rings.view(np.uint8).reshape(-1)).cuda())
    torch.cuda.synchronize()


def oracle_f2bf(a):
    import oracle as O
    return O.f2bf(a)


def test_cfg1_seeded_cache_steps_bitexact(cfg1, oracle, pb, cuda):
    torch = cuda
    from pulsar_b200 import synth
    c, w, m = cfg1
    s = m.new_state(MAX_CTX)
    om = oracle.Model(synth.oracle_cfg(c, MAX_CTX), w)
    rng = np.random.default_rng(31)
    _seed_state(c, s, om, rng, P0)
    logits = torch.empty(c["vocab"], dtype=torch.float32, device="cuda")
    tok = int(rng.integers(0, c["vocab"]))
    for step in range(NSTEP):
        pos = P0 + step
        got = s.decode_token(tok, pos, logits=logits)
        want, lg, x = om.decode(tok, pos, want_logits=True)
        torch.cuda.synchronize()
        assert np.array_equal(_bits32(logits.cpu().numpy()), _bits32(lg)), "logits differ at pos %d" % pos
        res = s.debug_tensor(2, torch.int16).cpu().numpy().view(np.uint16)
        assert np.array_equal(res, x), "residual differs at pos %d" % pos
        assert got == want, "id differs at pos %d" % pos
        tok = got
    s.status()
    NKV, HD = c["n_kv"], c["head_dim"]
    per = MAX_CTX * NKV * HD
    kv = s.debug_tensor(0, torch.int16).cpu().numpy().view(np.uint16)
    end = (P0 + NSTEP) * NKV * HD
    for ai, L in enumerate(c["attn_layers"]):
        for which in (0, 1):
            dev = kv[(ai * 2 + which) * per:(ai * 2 + which) * per + end]
            assert np.array_equal(dev, om.kv(L, which, P0 + NSTEP)), "KV layer %d" % L
    W, H = c["conv_w"], c["hidden"]
    rings = s.debug_tensor(1, torch.int16).cpu().numpy().view(np.uint16).reshape(-1, W, H)
    conv = [L for L in range(c["n_layers"]) if L not in c["attn_layers"]]
    last = P0 + NSTEP - 1
    for ci, L in enumerate(conv):
        want = om.ring(L)                      # row k: position last - (W - 1) + k
        for k in range(W):
            assert np.array_equal(rings[ci, (last - (W - 1) + k) % W], want[k]), "ring layer %d" % L


def test_cfg1_greedy_256_ids_identical(cfg1, oracle, pb, cuda):
    torch = cuda
    from pulsar_b200 import synth
    c, w, m = cfg1
    n = 256
    s = m.new_state(n + 8)
    om = oracle.Model(synth.oracle_cfg(c, n + 8), w)
    ids = torch.full((n,), -1, dtype=torch.int32, device="cuda")
    s.decode_greedy(4321, 0, n, ids)
    torch.cuda.synchronize()
    s.status()
    got = ids.cpu().numpy()
    tok, want = 4321, []
    for pos in range(n):
        tok, _, _ = om.decode(tok, pos)
        want.append(tok)
    assert got.tolist() == want
