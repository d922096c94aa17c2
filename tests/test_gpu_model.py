"""Whole-model parity on the B200: the fused decode step (CUDA graph, PDL)
against the CPU oracle's restatement of layer_body + head + argmax, bit for bit
(logits, final residual, KV cache, conv rings) and greedy ids over 256 steps."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny(tmp_path_factory, oracle, pb, cuda):
    from pulsar_b200 import synth
    c = dict(synth.LFM3_TINY)
    w = synth.make_weights(c, seed=77)
    path = str(tmp_path_factory.mktemp("m") / "tiny.lfm3q8")
    synth.write_model(path, c, w)
    return c, w, path


def _bits32(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_decode_bitexact_with_oracle(tiny, oracle, pb, cuda):
    torch = cuda
    c, w, path = tiny
    from pulsar_b200 import synth
    max_ctx = 64
    m = pb.Model(path)
    s = m.new_state(max_ctx)
    om = oracle.Model(synth.oracle_cfg(c, max_ctx), w)
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, c["vocab"], 12)
    logits = torch.empty(c["vocab"], dtype=torch.float32, device="cuda")
    tok = int(prompt[0])
    for pos in range(40):
        if pos < len(prompt):
            tok = int(prompt[pos])
        got = s.decode_token(tok, pos, logits=logits)
        want, lg, x = om.decode(tok, pos, want_logits=True)
        torch.cuda.synchronize()
        assert np.array_equal(_bits32(logits.cpu().numpy()), _bits32(lg)), "logits differ at pos %d" % pos
        res = s.debug_tensor(2, torch.int16).cpu().numpy().view(np.uint16)
        assert np.array_equal(res, x), "residual differs at pos %d" % pos
        assert got == want
        tok = got
    # state: KV caches of both attention layers, conv rings
    kv = s.debug_tensor(0, torch.int16).cpu().numpy().view(np.uint16)
    per = max_ctx * c["n_kv"] * c["head_dim"]
    for ai, L in enumerate(c["attn_layers"]):
        for which in (0, 1):
            dev = kv[(ai * 2 + which) * per:(ai * 2 + which) * per + 40 * c["n_kv"] * c["head_dim"]]
            assert np.array_equal(dev, om.kv(L, which, 40))


def test_greedy_256_ids_identical(tiny, oracle, pb, cuda):
    torch = cuda
    c, w, path = tiny
    from pulsar_b200 import synth
    n = 256
    m = pb.Model(path)
    s = m.new_state(n + 8)
    om = oracle.Model(synth.oracle_cfg(c, n + 8), w)
    ids = torch.full((n,), -1, dtype=torch.int32, device="cuda")
    s.decode_greedy(11, 0, n, ids)
    torch.cuda.synchronize()
    got = ids.cpu().numpy()
    tok, want = 11, []
    for pos in range(n):
        tok, _, _ = om.decode(tok, pos)
        want.append(tok)
    assert got.tolist() == want


def test_prompt_feed_matches_token_by_token(tiny, pb, cuda):
    torch = cuda
    c, w, path = tiny
    m = pb.Model(path)
    rng = np.random.default_rng(8)
    prompt = rng.integers(0, c["vocab"], 20).astype(np.int32)
    s1 = m.new_state(64)
    ids = torch.full((20,), -1, dtype=torch.int32, device="cuda")
    s1.decode_prompt(torch.from_numpy(prompt).cuda(), 0, ids)
    torch.cuda.synchronize()
    s2 = m.new_state(64)
    want = [s2.decode_token(int(t), p) for p, t in enumerate(prompt)]
    assert ids.cpu().numpy().tolist() == want


def test_layer_step_matches_decode(tiny, oracle, pb, cuda):
    """pb_layer_step over every layer from the embedding row = the oracle's
    residual after the last layer (position 0)"""
    torch = cuda
    c, w, path = tiny
    from pulsar_b200 import synth
    m = pb.Model(path)
    s = m.new_state(16)
    tok = 123
    codes, sc = w["embed"]
    emb = oracle.f2bf(codes[tok].astype(np.float32) * np.repeat(sc[tok].astype(np.float32), 32))
    x = torch.from_numpy(emb.view(np.int16).copy()).cuda()
    for L in range(c["n_layers"]):
        s.layer_step(L, 0, x)
    torch.cuda.synchronize()
    om = oracle.Model(synth.oracle_cfg(c, 16), w)
    _, _, want = om.decode(tok, 0)
    assert np.array_equal(x.cpu().numpy().view(np.uint16), want)


def test_fp32_scale_blob(tmp_path, oracle, pb, cuda):
    """the reference's certified blob format (dtype 1, fp32 scales)"""
    torch = cuda
    from pulsar_b200 import synth
    c = dict(synth.LFM3_TINY, n_layers=2, attn_layers=(1,), vocab=1024)
    w = synth.make_weights(c, seed=99)
    path = str(tmp_path / "f32.lfm3q8")
    synth.write_model(path, c, w, fp32_scales=True)
    m = pb.Model(path)
    s = m.new_state(32)
    om = oracle.Model(synth.oracle_cfg(c, 32), w)
    tok = 5
    for pos in range(6):
        got = s.decode_token(tok, pos)
        want, _, _ = om.decode(tok, pos)
        assert got == want
        tok = got


def test_corrupt_blob_rejected_on_device_open(tmp_path, pb, cuda):
    from pulsar_b200 import synth
    c = dict(synth.LFM3_TINY, n_layers=1, attn_layers=(), vocab=256)
    w = synth.make_weights(c, seed=1)
    path = str(tmp_path / "bad.lfm3q8")
    synth.write_model(path, c, w)
    with open(path, "r+b") as f:
        f.seek(-100, 2)
        f.write(b"\x00\x01\x02\x03")
    with pytest.raises(pb.PBError) as e:
        pb.Model(path)
    assert e.value.code == -5


def test_full_and_sliding_attention_layers(tmp_path, oracle, pb, cuda):
    """per-layer attention types as the reference builds them
    (lfm3_nanode.cu:3753-3785): a full-attention layer rotating half of the
    head dims with base 1e6 over every key, and a sliding-attention layer
    rotating all of them with base 1e4 over the last 8 keys; 40 positions, so
    the window slides, through the persistent kernel; bit-exact"""
    torch = cuda
    from pulsar_b200 import synth
    c = dict(synth.LFM3_TINY, n_layers=4, attn_layers=(1, 3), slide_layers=(3,), rope_partial=0.5,
             slide_window=8, slide_theta=1e4, slide_partial=1.0, vocab=1024)
    w = synth.make_weights(c, seed=404)
    path = str(tmp_path / "slide.lfm3q8")
    synth.write_model(path, c, w)
    m = pb.Model(path)
    max_ctx = 48
    s = m.new_state(max_ctx)
    om = oracle.Model(synth.oracle_cfg(c, max_ctx), w)
    logits = torch.empty(c["vocab"], dtype=torch.float32, device="cuda")
    tok = 17
    for pos in range(40):
        got = s.decode_token(tok, pos, logits=logits)
        want, lg, _ = om.decode(tok, pos, want_logits=True)
        torch.cuda.synchronize()
        assert np.array_equal(_bits32(logits.cpu().numpy()), _bits32(lg)), "logits differ at pos %d" % pos
        assert got == want
        tok = got
