"""Batched decode of independent sequences (one integer-path GEMM per
projection over the batch, tensor cores) against the CPU oracle's integer
mode, sequence by sequence and bit for bit: logits and greedy ids over
several steps, from ragged contexts filled by the chunked prefill."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _bits32(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_batched_decode_matches_integer_oracle(tmp_path, oracle, pb, cuda):
    torch = cuda
    from pulsar_b200 import synth
    c = dict(synth.LFM3_TINY)
    w = synth.make_weights(c, seed=79)
    path = str(tmp_path / "tiny.lfm3q8")
    synth.write_model(path, c, w)
    B, max_ctx, steps = 16, 80, 3
    m = pb.Model(path)
    rng = np.random.default_rng(12)
    ctx = rng.choice([16, 32, 48], B)
    states, oms, last = [], [], []
    ids1 = torch.empty(48, dtype=torch.int32, device="cuda")
    for b in range(B):
        s = m.new_state(max_ctx)
        om = oracle.Model(synth.oracle_cfg(c, max_ctx), w, int_path=True)
        prompt = rng.integers(0, c["vocab"], int(ctx[b])).astype(np.int32)
        s.prefill_chunk(torch.from_numpy(prompt).cuda(), 0, ids1[:len(prompt)])
        for p, t in enumerate(prompt):
            want, _, _ = om.decode(int(t), p)
        torch.cuda.synchronize()
        assert int(ids1[len(prompt) - 1].item()) == want
        states.append(s)
        oms.append(om)
        last.append(want)
    tokens = torch.tensor(last, dtype=torch.int32, device="cuda")
    pos = torch.tensor(ctx, dtype=torch.int32, device="cuda")
    ids = torch.empty(B, dtype=torch.int32, device="cuda")
    logits = torch.empty((B, c["vocab"]), dtype=torch.float32, device="cuda")
    for step in range(steps):
        m.decode_batch(states, tokens, pos, ids, logits)
        torch.cuda.synchronize()
        lg_dev, id_dev = logits.cpu().numpy(), ids.cpu().numpy()
        for b in range(B):
            want, lg, _ = oms[b].decode(int(tokens[b].item()), int(ctx[b]) + step, want_logits=True)
            assert np.array_equal(_bits32(lg_dev[b]), _bits32(lg)), "sequence %d step %d" % (b, step)
            assert int(id_dev[b]) == want
        tokens = ids.clone()
        pos = pos + 1
    for s in states:
        s.status()
