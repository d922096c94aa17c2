"""Chunked prefill on the integer path (tensor-core GEMMs) against the CPU
oracle's integer mode, bit for bit: every position's logits and greedy id,
the KV caches and the conv rings after each chunk of 32 positions."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bits32(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.mark.parametrize("T", [32, 16])
def test_prefill_chunks_match_integer_oracle(tmp_path, oracle, pb, cuda, T):
    torch = cuda
    from pulsar_b200 import synth
    c = dict(synth.LFM3_TINY)
    w = synth.make_weights(c, seed=78)
    path = str(tmp_path / "tiny.lfm3q8")
    synth.write_model(path, c, w)
    max_ctx = 96
    m = pb.Model(path)
    s = m.new_state(max_ctx)
    om = oracle.Model(synth.oracle_cfg(c, max_ctx), w, int_path=True)
    rng = np.random.default_rng(11)
    n = 2 * T
    tokens = rng.integers(0, c["vocab"], n).astype(np.int32)
    ids = torch.empty(T, dtype=torch.int32, device="cuda")
    logits = torch.empty((T, c["vocab"]), dtype=torch.float32, device="cuda")
    for ch in range(2):
        tk = torch.from_numpy(tokens[ch * T:(ch + 1) * T].copy()).cuda()
        s.prefill_chunk(tk, ch * T, ids, logits)
        torch.cuda.synchronize()
        lg_dev, id_dev = logits.cpu().numpy(), ids.cpu().numpy()
        for t in range(T):
            pos = ch * T + t
            want, lg, _ = om.decode(int(tokens[pos]), pos, want_logits=True)
            assert np.array_equal(_bits32(lg_dev[t]), _bits32(lg)), "logits differ at position %d" % pos
            assert int(id_dev[t]) == want
    # KV caches of the attention layers, rows 0 .. n-1
    kv = s.debug_tensor(0, torch.int16).cpu().numpy().view(np.uint16)
    per = max_ctx * c["n_kv"] * c["head_dim"]
    for ai, L in enumerate(c["attn_layers"]):
        for which in (0, 1):
            dev = kv[(ai * 2 + which) * per:(ai * 2 + which) * per + n * c["n_kv"] * c["head_dim"]]
            assert np.array_equal(dev, om.kv(L, which, n)), "KV layer %d" % L
    # conv rings: device slot p mod W holds position p; the oracle's ring is oldest first
    rings = s.debug_tensor(1, torch.int16).cpu().numpy().view(np.uint16)
    W, H = c["conv_w"], c["hidden"]
    conv_layers = [L for L in range(c["n_layers"]) if L not in c["attn_layers"]]
    for ci, L in enumerate(conv_layers):
        want = om.ring(L)
        dev = rings[ci * W * H:(ci + 1) * W * H].reshape(W, H)
        for k in range(W):
            p = n - W + k
            assert np.array_equal(dev[p % W], want[k]), "ring layer %d position %d" % (L, p)
