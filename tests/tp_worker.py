"""One rank of the row-sharded decode check (launched by test_gpu_tp.py under
torchrun): the tiny LFM3 model decoded with every GEMV's rows split over the
ranks and all-gathered; every position's logits and greedy id must equal the
CPU oracle's (computed once by the test, expected.npz) bit for bit on every
rank."""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.join(HERE, "..", "pulsar-asm_b200")]


def _mark(rank, what):
    if os.environ.get("PB_TP_TRACE"):
        print("rank %d: %s" % (rank, what), file=sys.stderr, flush=True)


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
    _mark(rank, "model loaded")
    uid = dist.share_from_rank0(pb.nccl_unique_id)
    _mark(rank, "id shared")
    s.shard(rank, world, uid)
    _mark(rank, "sharded")
    exp = np.load(os.path.join(os.environ["PB_TP_DIR"], "expected.npz"))
    toks, want_lg, want_id, want_greedy = exp["toks"], exp["logits"], exp["ids"], exp["greedy"]
    lg = torch.empty(c["vocab"], dtype=torch.float32, device="cuda")
    bad = 0
    for pos, tok in enumerate(toks):
        got = s.decode_token(int(tok), pos, logits=lg)
        torch.cuda.synchronize()
        _mark(rank, "position %d" % pos)
        if got != int(want_id[pos]) or not np.array_equal(lg.cpu().numpy().view(np.uint32),
                                                          want_lg[pos].view(np.uint32)):
            bad += 1
    # greedy continuation, ids fed back on the device
    ng = len(want_greedy)
    ids = torch.empty(ng, dtype=torch.int32, device="cuda")
    s.decode_greedy(int(toks[-1]), len(toks), ng, ids)
    s.status()
    _mark(rank, "greedy done")
    if ids.cpu().tolist() != [int(x) for x in want_greedy]:
        bad += 1000
    kpt = s.kernels_per_token()
    s.destroy()
    m.close()
    _mark(rank, "destroyed")
    ok = dist.sum_over_ranks(float(bad == 0))
    dist.finish()
    if rank == 0:
        print("TP_RESULT world=%d ok_ranks=%d kernels_per_token=%d bad=%d" % (world, int(ok), kpt, bad), flush=True)
    sys.exit(0 if bad == 0 else 1)


if __name__ == "__main__":
    main()
