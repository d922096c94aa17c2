"""The Bonsai Q1_0 decoder (fwd8.c token step) against the CPU oracle, bit for
bit: every step's logits, greedy id, residual stream and K/V rows, on a tiny
model over many positions, on the Bonsai-8B layer shapes (full vocabulary) at
a 2048-position context, through the greedy loop, through the caller-row
input (pq1_token_fused's contract) and through the serial fallback of the RMS
norm."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def _pair(pb, oracle, cfg, seed, max_ctx):
    from pulsar_b200 import synth
    w = synth.make_bonsai_weights(cfg, seed=seed)
    return pb.Bonsai(cfg, w), oracle.BsModel(cfg, w, max_ctx), w


def test_bonsai_tiny_steps(oracle, pb, cuda):
    torch = cuda
    from pulsar_b200 import synth
    c = dict(synth.BONSAI_TINY)
    max_ctx = 96
    m, om, _ = _pair(pb, oracle, c, 21, max_ctx)
    s = m.new_state(max_ctx)
    rng = np.random.default_rng(3)
    toks = rng.integers(0, c["vocab"], 70)
    lg = torch.empty(c["vocab"], dtype=torch.float32, device="cuda")
    xr = torch.empty(c["hidden"], dtype=torch.float32, device="cuda")
    for pos, tok in enumerate(toks):
        got = s.decode(int(tok), pos, logits=lg)
        want, lw, xw = om.decode(int(tok), pos, want_logits=True)
        s.residual(xr)
        torch.cuda.synchronize()
        assert np.array_equal(_bits(lg.cpu().numpy()), _bits(lw)), "logits differ at position %d" % pos
        assert np.array_equal(_bits(xr.cpu().numpy()), _bits(xw)), "residual differs at position %d" % pos
        assert got == want
    s.status()
    n = len(toks)
    for L in range(c["n_layers"]):
        for which in (0, 1):
            dev = s.kv(L, which).cpu().numpy().view(np.uint16)
            assert np.array_equal(dev[:, :n], om.kv(L, which)[:, :n]), "KV layer %d" % L


def test_bonsai_8b_layers_ctx2048(oracle, pb, cuda):
    """Bonsai-8B shapes (hidden 4096, 32/8 heads, FFN 12288, vocab 151936), two
    layers, the step at position 2047 over a filled f16 cache"""
    torch = cuda
    from pulsar_b200 import synth
    c = dict(synth.BONSAI_CFG3)
    c["n_layers"] = 2
    max_ctx = 2048
    m, om, _ = _pair(pb, oracle, c, 5, max_ctx)
    s = m.new_state(max_ctx)
    rng = np.random.default_rng(9)
    first = max_ctx - 2     # positions first and first + 1: the last step reads 2048 rows
    for L in range(c["n_layers"]):
        for which in (0, 1):
            kv = (rng.standard_normal((c["n_kv"], max_ctx, 128)) * (1.0 + which)).astype(np.float16).view(np.uint16)
            kv[:, first:] = 0
            om.set_kv(L, which, kv)
            s.kv(L, which).copy_(torch.from_numpy(kv.view(np.int16)).cuda())
    lg = torch.empty(c["vocab"], dtype=torch.float32, device="cuda")
    for step, tok in enumerate([1234, 77]):
        p = first + step
        got = s.decode(tok, p, logits=lg)
        want, lw, _ = om.decode(tok, p, want_logits=True)
        torch.cuda.synchronize()
        assert np.array_equal(_bits(lg.cpu().numpy()), _bits(lw)), "logits differ at position %d" % p
        assert got == want
    s.status()
    for L in range(c["n_layers"]):
        for which in (0, 1):
            dev = s.kv(L, which).cpu().numpy().view(np.uint16)
            assert np.array_equal(dev, om.kv(L, which)), "KV layer %d" % L


def test_bonsai_greedy_and_caller_row(oracle, pb, cuda):
    torch = cuda
    from pulsar_b200 import synth
    c = dict(synth.BONSAI_TINY)
    max_ctx = 64
    m, om, _ = _pair(pb, oracle, c, 33, max_ctx)
    s = m.new_state(max_ctx)
    ids = torch.empty(24, dtype=torch.int32, device="cuda")
    s.decode_greedy(11, 0, 24, ids)
    want, tok = [], 11
    for pos in range(24):
        tok, _, _ = om.decode(tok, pos)
        want.append(tok)
    assert ids.cpu().tolist() == want
    # the caller supplies the input row (pq1_token_fused): here a row whose
    # serial double sum of squares stops exactly on a float rounding midpoint
    # (2^40 + 2^16; the 2^-60 terms vanish below its ulp) while the exact sum
    # lies just above it, so neither certificate holds and the device runs the
    # serial chain
    s2, om2 = m.new_state(max_ctx), oracle.BsModel(c, synth.make_bonsai_weights(c, seed=33), max_ctx)
    x = np.full(c["hidden"], 2.0 ** -30, np.float32)
    x[0], x[1] = 2.0 ** 20, 2.0 ** 8
    lg = torch.empty(c["vocab"], dtype=torch.float32, device="cuda")
    before = s2.fallbacks()
    got = s2.decode(0, 0, x=torch.from_numpy(x).cuda(), logits=lg)
    want_id, lw, _ = om2.decode(0, 0, x_in=x, want_logits=True)
    torch.cuda.synchronize()
    assert s2.fallbacks() > before
    assert np.array_equal(_bits(lg.cpu().numpy()), _bits(lw))
    assert got == want_id


@pytest.mark.parametrize("bits", [4, 3, 43])
def test_bonsai_turboquant_cache(oracle, pb, cuda, bits):
    """the decoder with a TurboQuant K/V cache (pb_bonsai_state_create_tq, the
    reference glue's default PQ1_KVTQ=4) against the oracle's token step with
    the same cache, bit for bit: logits and greedy ids over 300 positions
    (beyond one 256-position chunk of the V sum)"""
    torch = cuda
    from pulsar_b200 import synth
    c = dict(synth.BONSAI_TINY)
    max_ctx = 320
    w = synth.make_bonsai_weights(c, seed=77)
    m, om = pb.Bonsai(c, w), oracle.BsModel(c, w, max_ctx, kv_bits=bits)
    s = m.new_state(max_ctx, kv_bits=bits)
    rng = np.random.default_rng(bits)
    toks = rng.integers(0, c["vocab"], 300)
    lg = torch.empty(c["vocab"], dtype=torch.float32, device="cuda")
    for pos, tok in enumerate(toks):
        got = s.decode(int(tok), pos, logits=lg)
        want, lw, _ = om.decode(int(tok), pos, want_logits=True)
        torch.cuda.synchronize()
        assert np.array_equal(_bits(lg.cpu().numpy()), _bits(lw)), "logits differ at position %d" % pos
        assert got == want
    s.status()
    with pytest.raises(pb.PBError):
        s.kv(0, 0)     # no f16 cache to view
