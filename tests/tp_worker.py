"""One rank of the row-sharded decode check (launched by test_gpu_tp.py under
torchrun): the tiny LFM3 model decoded with every GEMV's rows split over the
ranks and all-gathered; every position's logits and greedy id must equal the
CPU oracle's bit for bit on every rank."""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(HERE, "..", "pulsar-asm_b200"), os.path.join(HERE, "..", "oracle")]


def main():
    import torch
    import pulsar_b200 as pb
    from pulsar_b200 import dist, synth
    rank, world, local = dist.env_rank()
    torch.cuda.set_device(local)
    dist.init(backend="gloo", timeout_s=60)
    c = dict(synth.LFM3_TINY)
    w = synth.make_weights(c, seed=91)
    path = os.path.join(os.environ.get("PB_TP_DIR", "/tmp"), "tp_tiny_r%d.lfm3q8" % rank)
    synth.write_model(path, c, w)
    max_ctx = 64
    m = pb.Model(path, device=local)
    s = m.new_state(max_ctx)
    uid = dist.share_from_rank0(pb.nccl_unique_id)
    s.shard(rank, world, uid)
    import oracle
    om = oracle.Model(synth.oracle_cfg(c, max_ctx), w)
    rng = np.random.default_rng(5)
    toks = rng.integers(0, c["vocab"], 40)
    lg = torch.empty(c["vocab"], dtype=torch.float32, device="cuda")
    bad = 0
    for pos, tok in enumerate(toks):
        got = s.decode_token(int(tok), pos, logits=lg)
        want, lw, _ = om.decode(int(tok), pos, want_logits=True)
        torch.cuda.synchronize()
        if got != want or not np.array_equal(lg.cpu().numpy().view(np.uint32), lw.view(np.uint32)):
            bad += 1
    # greedy continuation, ids fed back on the device
    ids = torch.empty(16, dtype=torch.int32, device="cuda")
    first = int(toks[-1])
    s.decode_greedy(first, len(toks), 16, ids)
    s.status()
    want_ids, t = [], first
    for i in range(16):
        t, _, _ = om.decode(t, len(toks) + i)
        want_ids.append(t)
    if ids.cpu().tolist() != want_ids:
        bad += 1000
    kpt = s.kernels_per_token()
    s.destroy()
    m.close()
    ok = dist.sum_over_ranks(float(bad == 0))
    dist.finish()
    if rank == 0:
        print("TP_RESULT world=%d ok_ranks=%d kernels_per_token=%d bad=%d" % (world, int(ok), kpt, bad), flush=True)
    sys.exit(0 if bad == 0 else 1)


if __name__ == "__main__":
    main()
