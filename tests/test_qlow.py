"""The low-bit (Q4 / Q5) GEMV's oracle (lfm3_qlow.cuh's k_qlow + k_qlow_combine
as qlow_gemv launches them, lfm3_nanode.cu:1894-1915), pinned: bit for bit the
outputs that the reference's own kernels produced on a B200 for seeded
tensors (tests/golden/qlow.npz: Q4 and Q5, K slices of 2 and 4, N from 32)."""
import importlib.util
import os

import numpy as np
import pytest

from conftest import ROOT

GOLDEN = os.path.join(ROOT, "tests", "golden")


def _gen():
    spec = importlib.util.spec_from_file_location("make_golden_qlow", os.path.join(GOLDEN, "make_golden_qlow.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def test_oracle_qlow_matches_reference_kernels(oracle):
    path = os.path.join(GOLDEN, "qlow.npz")
    g = _gen()
    z = np.load(path)
    assert len(z.files) == len(g.CASES)
    for bits, N, K, seed in g.CASES:
        codes, scales, x = g.case_inputs(bits, N, K, seed)
        want = z["q%d_%d_%d_%d" % (bits, N, K, seed)]
        got = oracle.qlow_gemv(codes, scales, bits, N, K, x)
        assert np.array_equal(got, want), (bits, N, K, seed, int(np.sum(got != want)))


def test_oracle_qlow_positions_are_independent(oracle):
    """T positions give each position's one-position result (the reference's
    prefill loops qlow_gemv over positions, lfm3_nanode.cu:4847)"""
    g = _gen()
    codes, scales, x0 = g.case_inputs(5, 64, 512, 11)
    xs = np.stack([x0, x0[::-1].copy(), (x0 ^ 0x8000).astype(np.uint16)])
    y = oracle.qlow_gemv(codes, scales, 5, 64, 512, xs)
    for t in range(3):
        assert np.array_equal(y[t], oracle.qlow_gemv(codes, scales, 5, 64, 512, xs[t]))
