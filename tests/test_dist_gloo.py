"""The benchmark's multi-rank plumbing on CPU ranks (gloo, world size 2):
rendezvous on 127.0.0.1, max/sum reductions over ranks, and a rank that fails
before the reduction surfacing as an error on the other rank instead of a hang."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, fail_rank):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "pulsar-asm_b200"))
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from pulsar_b200 import dist
    try:
        dist.init(backend="gloo", timeout_s=10)
        lo, hi = dist.shard_range(64, rank, world)
        if rank == fail_rank:
            raise RuntimeError("injected failure on rank %d" % rank)
        mx = dist.max_over_ranks(float(rank + 1) * 1.5)
        tot = dist.sum_over_ranks(hi - lo)
        dist.barrier()
        q.put((rank, "ok", mx, tot))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "err", repr(e), None))
    finally:
        try:
            dist.finish()
        except Exception:
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in ps:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(out)


def test_max_and_sum_over_two_ranks():
    out = _run(2)
    assert [o[1] for o in out] == ["ok", "ok"]
    assert all(o[2] == 3.0 and o[3] == 64 for o in out)


def test_failed_rank_is_an_error_not_a_hang():
    out = _run(2, fail_rank=1)
    status = {o[0]: o[1] for o in out}
    assert status[1] == "err"
    assert status[0] == "err"      # the survivor's collective times out or aborts


def _uid_worker(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "pulsar-asm_b200"))
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from pulsar_b200 import dist
    try:
        dist.init(backend="gloo", timeout_s=20)
        calls = []

        def make():
            calls.append(rank)
            return bytes([7, rank, 9]) * 42 + b"xy"
        v = dist.share_from_rank0(make)
        q.put((rank, v, calls))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e), None))
    finally:
        try:
            dist.finish()
        except Exception:
            pass


def test_share_from_rank0_gloo():
    """the row-sharded state's NCCL id: made once on rank 0, the same bytes on every rank"""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_uid_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = sorted(q.get(timeout=120) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
    want = bytes([7, 0, 9]) * 42 + b"xy"
    assert out[0] == (0, want, [0]) and out[1] == (1, want, [])


def _shard_worker(rank, world, port, q):
    """the row sharding of pb_state_shard restated on CPU ranks: rank r computes
    rows [r N/world, (r+1) N/world) of each GEMV whole (the reference's
    reduction order inside a row is untouched), an all-gather assembles the
    output; also the SwiGLU pairs (rows 2i, 2i+1 stay on one rank) and the
    batched decode's sequence split"""
    import sys
    import numpy as np
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "pulsar-asm_b200"))
    sys.path.insert(0, os.path.join(root, "oracle"))
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch
    import torch.distributed as tdist
    import oracle
    from pulsar_b200 import dist
    try:
        dist.init(backend="gloo", timeout_s=30)
        res = {}
        for N, K in ((512, 2048), (256, 7680), (128, 8192)):
            rng = np.random.default_rng(N + K)
            codes = rng.integers(-127, 128, (N, K), dtype=np.int8)
            sc = (np.abs(rng.standard_normal((N, K // 32))) * 0.01).astype(np.float32)
            x = oracle.f2bf(rng.standard_normal(K).astype(np.float32))
            rows = N // world
            part = oracle.q8f_gemv(codes[rank * rows:(rank + 1) * rows], sc[rank * rows:(rank + 1) * rows], x)
            got = [torch.empty(rows, dtype=torch.float32) for _ in range(world)]
            tdist.all_gather(got, torch.from_numpy(np.ascontiguousarray(part)))
            full = torch.cat(got).numpy()
            res["gemv_%d_%d" % (N, K)] = bool(np.array_equal(full.view(np.uint32),
                                                             oracle.q8f_gemv(codes, sc, x).view(np.uint32)))
        # SwiGLU pairs: an even share of rows keeps every (w1, w3) pair on one rank
        N = 2 * 96
        lo, hi = rank * (N // world), (rank + 1) * (N // world)
        res["pairs"] = lo % 2 == 0 and hi % 2 == 0
        # the batched decode's split: every sequence on exactly one rank
        B = 64
        mine = list(range(*dist.shard_range(B, rank, world)))
        allm = [None] * world
        tdist.all_gather_object(allm, mine)
        flat = sorted(s for m in allm for s in m)
        res["batch"] = flat == list(range(B))
        q.put((rank, "ok", res))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "err", repr(e)))
    finally:
        try:
            dist.finish()
        except Exception:
            pass


def test_row_shard_math_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_shard_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = sorted(q.get(timeout=180) for _ in range(2))
    for p in ps:
        p.join(timeout=60)
    for rank, status, res in out:
        assert status == "ok", res
        assert all(res.values()), res
