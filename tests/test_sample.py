"""The sampler's oracle (sample_topkpp + frand01, pulsar_arm/bonsai2/fwd8.c:
465-521), pinned: with the C library's expf (the reference's) it returns the
ids and generator states that the reference's own compiled function returned
on 160 seeded cases (tests/golden/sample_topkpp.json: ties, signed zeros,
dominant values, vocabularies up to 151936, greedy, top-k beyond the list and
beyond n, min-p and top-p), and the same against the compiled function live
where oracle/_ref is built. With the device's expf it is the checker of the
GPU sampler."""
import ctypes as C
import importlib.util
import json
import os

import numpy as np
import pytest

from conftest import ROOT

GOLDEN = os.path.join(ROOT, "tests", "golden")


def _gen():
    spec = importlib.util.spec_from_file_location("make_golden_sample", os.path.join(GOLDEN, "make_golden_sample.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def test_oracle_sampler_matches_reference_golden(oracle):
    g = _gen()
    cases = json.load(open(os.path.join(GOLDEN, "sample_topkpp.json")))
    assert len(cases) == 160
    for cs in cases:
        lg = g.case_logits(cs["seed"], cs["n"], cs["kind"])
        tid, rs = oracle.sample_topkpp(lg, cs["temp"], cs["topp"], cs["topk"], cs["minp"], cs["rs"], libm_exp=True)
        assert (tid, rs) == (cs["id"], cs["rs_out"]), cs
        if cs["temp"] <= 0:
            assert rs == cs["rs"]   # greedy leaves the generator alone


def test_oracle_sampler_matches_reference_live(oracle):
    lib = os.path.join(ROOT, "oracle", "_ref", "libpb_sample.so")
    if not os.path.exists(lib):
        pytest.skip("fwd8.c's sampler not built (no reference tree)")
    L = C.CDLL(lib)
    L.pbref_sample_topkpp.restype = C.c_int
    L.pbref_sample_topkpp.argtypes = [C.c_void_p, C.c_int, C.c_float, C.c_float, C.c_int, C.c_float,
                                      C.POINTER(C.c_uint64)]
    rng = np.random.default_rng(77)
    for _ in range(60):
        n = int(rng.choice([2, 17, 1500, 32000]))
        lg = (rng.standard_normal(n) * 2).astype(np.float32)
        lg[rng.integers(0, n, 4)] = lg[0]            # exact ties with the first entry
        temp, topp = float(rng.uniform(0.05, 2.0)), float(rng.uniform(0.0, 1.0))
        topk, minp = int(rng.integers(-1, 1100)), float(rng.choice([0.0, rng.uniform(0, 0.5)]))
        seed = int(rng.integers(0, 2**63))
        st = C.c_uint64(seed)
        want = L.pbref_sample_topkpp(lg.ctypes.data, n, temp, topp, topk, minp, C.byref(st))
        assert oracle.sample_topkpp(lg, temp, topp, topk, minp, seed, libm_exp=True) == (want, st.value)


def test_oracle_sampler_nan_row(oracle):
    lg = np.zeros(100, np.float32)
    lg[37] = np.nan
    assert oracle.sample_topkpp(lg, 0.8, 0.9, 40, 0.0, 5) == (-1, 5)
    assert oracle.sample_topkpp(lg, 0.0, 0.9, 40, 0.0, 5) == (-1, 5)
