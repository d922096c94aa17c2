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
