"""The reference engine's own model shape (lfm3_nanode.cu:74-101) on every
decode path, bit for bit against the oracle: hidden 2048, FFN 7680 (w2's
K = 7680 is reduced as ONE chunk per row: pick(), lfm3_nanode.cu:1763-1768),
16 query / 4 KV heads of 128, a 7-tap gated short conv, full-attention layers
rotating half of each head with base 1e6 over every key and sliding-attention
layers rotating all of it with base 1e4 over a key window
(lfm3_nanode.cu:3753-3785). Four layers and a 4096-entry vocabulary instead of
24 and 128000 keep the oracle quick; every matrix, head and conv shape is the
reference's. The window is 16 keys here (256 in the shipped config) so that it
slides within the test's positions."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REF_SHAPE = dict(hidden=2048, inter=7680, n_layers=4, n_heads=16, n_kv=4, head_dim=128, vocab=4096, conv_w=7,
                 rope_theta=1e6, rope_partial=0.5, norm_eps=1e-5, sliding_window=0, attn_layers=(1, 3),
                 slide_layers=(3,), slide_window=16, slide_theta=1e4, slide_partial=1.0)


def _bits32(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.fixture(scope="module")
def refm(tmp_path_factory, pb, cuda):
    from pulsar_b200 import synth
    c = dict(REF_SHAPE)
    w = synth.make_weights(c, seed=2026)
    path = str(tmp_path_factory.mktemp("ref") / "refshape.lfm3q8")
    synth.write_model(path, c, w)
    return c, w, path


def _decode_and_check(pb, torch, oracle, c, w, path, n, max_ctx=64):
    from pulsar_b200 import synth
    m = pb.Model(path)
    s = m.new_state(max_ctx)
    om = oracle.Model(synth.oracle_cfg(c, max_ctx), w)
    logits = torch.empty(c["vocab"], dtype=torch.float32, device="cuda")
    tok = 101
    for pos in range(n):
        got = s.decode_token(tok, pos, logits=logits)
        want, lg, x = om.decode(tok, pos, want_logits=True)
        torch.cuda.synchronize()
        assert np.array_equal(_bits32(logits.cpu().numpy()), _bits32(lg)), "logits differ at pos %d" % pos
        res = s.debug_tensor(2, torch.int16).cpu().numpy().view(np.uint16)
        assert np.array_equal(res, x), "residual differs at pos %d" % pos
        assert got == want
        tok = got
    # KV caches of both attention layers
    kv = s.debug_tensor(0, torch.int16).cpu().numpy().view(np.uint16)
    per = max_ctx * c["n_kv"] * c["head_dim"]
    for ai, L in enumerate(c["attn_layers"]):
        for which in (0, 1):
            dev = kv[(ai * 2 + which) * per:(ai * 2 + which) * per + n * c["n_kv"] * c["head_dim"]]
            assert np.array_equal(dev, om.kv(L, which, n)), "KV layer %d" % L
    s.status()


def test_refshape_persistent_decode(refm, oracle, pb, cuda, monkeypatch):
    """the persistent kernel's head_dim-128, conv-7 build with the one-chunk
    w2: 36 positions, so the sliding window moves"""
    monkeypatch.delenv("PB_DECODE_MODE", raising=False)
    c, w, path = refm
    _decode_and_check(pb, cuda, oracle, c, w, path, 36)


def test_refshape_graph_decode(refm, oracle, pb, cuda, monkeypatch):
    """the per-kernel CUDA-graph path (k_step's one-chunk rows)"""
    monkeypatch.setenv("PB_DECODE_MODE", "graph")
    c, w, path = refm
    _decode_and_check(pb, cuda, oracle, c, w, path, 24)


def test_refshape_prefill_and_batch_integer_path(refm, oracle, pb, cuda):
    """chunked prefill (32 positions) and one batched step of 16 sequences on
    the tensor-core integer path, against the oracle's integer mode"""
    torch = cuda
    from pulsar_b200 import synth
    c, w, path = refm
    max_ctx = 64
    m = pb.Model(path)
    T = 32
    rng = np.random.default_rng(21)
    tokens = rng.integers(0, c["vocab"], T).astype(np.int32)
    s = m.new_state(max_ctx)
    om = oracle.Model(synth.oracle_cfg(c, max_ctx), w, int_path=True)
    ids = torch.empty(T, dtype=torch.int32, device="cuda")
    logits = torch.empty((T, c["vocab"]), dtype=torch.float32, device="cuda")
    s.prefill_chunk(torch.from_numpy(tokens).cuda(), 0, ids, logits)
    torch.cuda.synchronize()
    lg_dev, id_dev = logits.cpu().numpy(), ids.cpu().numpy()
    for t in range(T):
        want, lg, _ = om.decode(int(tokens[t]), t, want_logits=True)
        assert np.array_equal(_bits32(lg_dev[t]), _bits32(lg)), "prefill logits differ at position %d" % t
        assert int(id_dev[t]) == want
    # batched decode: 16 sequences, each after its own 16-position prefill
    B = 16
    states, oms, last = [], [], []
    ids1 = torch.empty(16, dtype=torch.int32, device="cuda")
    for b in range(B):
        sb = m.new_state(max_ctx)
        ob = oracle.Model(synth.oracle_cfg(c, max_ctx), w, int_path=True)
        prompt = rng.integers(0, c["vocab"], 16).astype(np.int32)
        sb.prefill_chunk(torch.from_numpy(prompt).cuda(), 0, ids1)
        for p, t in enumerate(prompt):
            want, _, _ = ob.decode(int(t), p)
        torch.cuda.synchronize()
        assert int(ids1[15].item()) == want
        states.append(sb)
        oms.append(ob)
        last.append(want)
    tk = torch.tensor(last, dtype=torch.int32, device="cuda")
    pos = torch.full((B,), 16, dtype=torch.int32, device="cuda")
    bid = torch.empty(B, dtype=torch.int32, device="cuda")
    blg = torch.empty((B, c["vocab"]), dtype=torch.float32, device="cuda")
    m.decode_batch(states, tk, pos, bid, blg)
    torch.cuda.synchronize()
    lg_dev, id_dev = blg.cpu().numpy(), bid.cpu().numpy()
    for b in range(B):
        want, lg, _ = oms[b].decode(last[b], 16, want_logits=True)
        assert np.array_equal(_bits32(lg_dev[b]), _bits32(lg)), "batched logits differ for sequence %d" % b
        assert int(id_dev[b]) == want


def test_bf16_head_kernel(oracle, pb, cuda):
    """k_gemv_bf16 over the re-laid table (pb_bf16_relayout + pb_bf16_gemv)
    bit for bit against the oracle's restatement, including a row of -0
    weights and the largest finite bf16"""
    torch = cuda
    import ctypes as C
    rng = np.random.default_rng(9)
    N, K = 1000, 2048
    w = oracle.f2bf((rng.standard_normal((N, K)) * 3).astype(np.float32))
    w[5] = 0x8000                 # a row of -0 weights
    w[7, :8] = 0x7F7F             # the largest finite bf16
    x = oracle.f2bf(rng.standard_normal(K).astype(np.float32))
    want = oracle.gemv_bf16(w, x)
    src = torch.from_numpy(w.view(np.int16)).cuda()
    dst = torch.empty_like(src)
    L = pb.lib()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.pb_bf16_relayout(C.c_void_p(src.data_ptr()), C.c_void_p(dst.data_ptr()), N, K, stream) == 0
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    y = torch.empty(N, dtype=torch.float32, device="cuda")
    assert L.pb_bf16_gemv(C.c_void_p(dst.data_ptr()), N, K, C.c_void_p(xd.data_ptr()), C.c_void_p(y.data_ptr()),
                          stream) == 0
    torch.cuda.synchronize()
    assert np.array_equal(_bits32(y.cpu().numpy()), _bits32(want))


def test_bf16_embedding_model(tmp_path, oracle, pb, cuda, monkeypatch):
    """the certified arm (blob dtype 3): embedding rows copied from the bf16
    table and the k_gemv_bf16 head, at the reference shape; persistent kernel,
    graph path and the chunked prefill, bit-exact"""
    torch = cuda
    from pulsar_b200 import synth
    c = dict(REF_SHAPE, emb_bf16=True, n_layers=2, attn_layers=(1,), slide_layers=())
    w = synth.make_weights(c, seed=3)
    path = str(tmp_path / "b16.lfm3q8")
    synth.write_model(path, c, w)
    monkeypatch.delenv("PB_DECODE_MODE", raising=False)
    _decode_and_check(pb, torch, oracle, c, w, path, 20)
    monkeypatch.setenv("PB_DECODE_MODE", "graph")
    _decode_and_check(pb, torch, oracle, c, w, path, 12)
    m = pb.Model(path)
    s = m.new_state(64)
    om = oracle.Model(synth.oracle_cfg(c, 64), w, int_path=True)
    T = 16
    tokens = np.random.default_rng(4).integers(0, c["vocab"], T).astype(np.int32)
    ids = torch.empty(T, dtype=torch.int32, device="cuda")
    logits = torch.empty((T, c["vocab"]), dtype=torch.float32, device="cuda")
    s.prefill_chunk(torch.from_numpy(tokens).cuda(), 0, ids, logits)
    torch.cuda.synchronize()
    lg_dev, id_dev = logits.cpu().numpy(), ids.cpu().numpy()
    for t in range(T):
        want, lg, _ = om.decode(int(tokens[t]), t, want_logits=True)
        assert np.array_equal(_bits32(lg_dev[t]), _bits32(lg)), "prefill logits differ at position %d" % t
        assert int(id_dev[t]) == want
