"""Row-sharded decode over two GPUs (one process per GPU, NCCL all-gather of
every GEMV's output): bit-exact to the CPU oracle on every rank. Needs two
GPUs; skipped otherwise."""
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _expected(oracle, path):
    """the oracle's logits and ids for the workers' token sequence (same seeds
    as tp_worker.py), computed here once with every host thread"""
    import numpy as np
    from pulsar_b200 import synth
    c = dict(synth.LFM3_TINY)
    w = synth.make_weights(c, seed=91)
    om = oracle.Model(synth.oracle_cfg(c, 64), w)
    toks = np.random.default_rng(5).integers(0, c["vocab"], 24)
    lgs, ids = [], []
    for pos, tok in enumerate(toks):
        i, lg, _ = om.decode(int(tok), pos, want_logits=True)
        lgs.append(lg)
        ids.append(i)
    greedy, t = [], int(toks[-1])
    for i in range(8):
        t, _, _ = om.decode(t, len(toks) + i)
        greedy.append(t)
    np.savez(path, toks=toks, logits=np.stack(lgs), ids=np.array(ids), greedy=np.array(greedy))


def test_row_sharded_decode_two_gpus(cuda, oracle, tmp_path):
    torch = cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("row-sharded decode needs two GPUs")
    _expected(oracle, str(tmp_path / "expected.npz"))
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, PB_TP_DIR=str(tmp_path), NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(here, "tp_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert "TP_RESULT world=2 ok_ranks=2" in r.stdout
