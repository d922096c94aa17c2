"""pb_sample_topkpp (fwd8.c:465-521 on the device, one CTA per row) against
the oracle's restatement with the same expf, bit for bit: every row's id and
advanced generator state, over Bonsai's 151936-entry vocabulary and cfg4's
batch of 64 rows, ties and signed zeros, greedy rows, top-k beyond n, strided
rows, chained draws and a row holding a NaN."""
import importlib.util
import os

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu


def _gen():
    p = os.path.join(ROOT, "tests", "golden", "make_golden_sample.py")
    spec = importlib.util.spec_from_file_location("make_golden_sample", p)
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


PARAMS = [  # temp, topp, topk, minp
    (0.7, 0.95, 40, 0.05), (1.0, 1.0, 0, 0.0), (0.3, 0.5, 1024, 0.0), (1.6, 0.9, 7, 0.3),
    (0.8, 0.0, 40, 0.0), (1.0, 0.9, 1, 0.0), (0.0, 0.9, 40, 0.0),
]


def _run(pb, torch, lg, params, seeds, ld=None):
    B, n = lg.shape
    if ld is None:
        d = torch.from_numpy(lg).cuda()
    else:
        big = torch.full((B, ld), float("nan"), dtype=torch.float32, device="cuda")
        big[:, :n] = torch.from_numpy(lg).cuda()
        d = big[:, :n]
    rng = torch.from_numpy(np.asarray(seeds, np.uint64).view(np.int64)).cuda()
    ids = torch.empty(B, dtype=torch.int32, device="cuda")
    temp, topp, topk, minp = params
    pb.sample_topkpp(d, temp, topp, topk, minp, rng, ids)
    torch.cuda.synchronize()
    return ids.cpu().numpy(), rng.cpu().numpy().view(np.uint64)


@pytest.mark.parametrize("n,B", [(151936, 12), (2048, 64), (3, 4)])
def test_sampler_rows(oracle, pb, cuda, n, B):
    torch = cuda
    g = _gen()
    rs0 = np.random.default_rng(n).integers(0, 2**63, B, dtype=np.uint64)
    lg = np.stack([g.case_logits(1000 + b, n, b % 4) for b in range(B)])
    for params in PARAMS:
        ids, rs = _run(pb, torch, lg, params, rs0)
        for b in range(B):
            want = oracle.sample_topkpp(lg[b], *params, int(rs0[b]))
            assert (int(ids[b]), int(rs[b])) == want, (params, b)


def test_sampler_strided_chained_and_nan(oracle, pb, cuda):
    torch = cuda
    g = _gen()
    B, n, ld = 8, 5000, 5120
    lg = np.stack([g.case_logits(7 + b, n, 1) for b in range(B)])
    lg[3, 123] = np.nan
    rs = np.random.default_rng(3).integers(0, 2**63, B, dtype=np.uint64)
    d = torch.full((B, ld), float("nan"), dtype=torch.float32, device="cuda")
    d[:, :n] = torch.from_numpy(lg).cuda()
    rng = torch.from_numpy(rs.view(np.int64)).cuda()
    ids = torch.empty(B, dtype=torch.int32, device="cuda")
    want_rs = [int(x) for x in rs]
    for step in range(3):   # three draws in a row: each row's state chains
        pb.sample_topkpp(d[:, :n], 0.9, 0.9, 64, 0.02, rng, ids)
        torch.cuda.synchronize()
        got_ids, got_rs = ids.cpu().numpy(), rng.cpu().numpy().view(np.uint64)
        for b in range(B):
            wid, want_rs[b] = oracle.sample_topkpp(lg[b], 0.9, 0.9, 64, 0.02, want_rs[b])
            assert int(got_ids[b]) == wid and int(got_rs[b]) == want_rs[b], (step, b)
    assert int(got_ids[3]) == -1 and int(got_rs[3]) == int(rs[3])   # the NaN row: no draw
    # greedy without generator states
    pb.sample_topkpp(d[:, :n], 0.0, 1.0, 0, 0.0, None, ids)
    torch.cuda.synchronize()
    got = ids.cpu().numpy()
    for b in range(B):
        assert int(got[b]) == (-1 if b == 3 else int(np.argmax(lg[b]))), b
