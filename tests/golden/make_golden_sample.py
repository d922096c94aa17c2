"""Generates tests/golden/sample_topkpp.json: seeded sampler cases and the ids
and generator states that the REFERENCE's own sample_topkpp (pulsar_arm/
bonsai2/fwd8.c:465-521, compiled unmodified into oracle/_ref/libpb_sample.so
by oracle/build_ref.sh) returns for them. TEST INFRASTRUCTURE:
tests/test_sample.py checks the oracle's restatement against these values
(and against the library itself where it is built). The logits of a case are
regenerated from its seed by case_logits(); only the parameters and the
answers are committed.

    bash oracle/build_ref.sh && python tests/golden/make_golden_sample.py
"""
import ctypes as C
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "sample_topkpp.json")


def case_logits(seed, n, kind):
    """kind 0: plain normal logits; 1: quantised to quarters (many ties);
    2: ties plus signed zeros; 3: a few dominant values"""
    rng = np.random.default_rng(seed)
    lg = (rng.standard_normal(n) * (0.5 + 4.0 * rng.random())).astype(np.float32)
    if kind in (1, 2):
        lg = (np.round(lg * 4) / 4).astype(np.float32)
    if kind == 2:
        lg[rng.integers(0, n, 8)] = np.float32(-0.0)
        lg[rng.integers(0, n, 8)] = np.float32(0.0)
    if kind == 3:
        lg[rng.integers(0, n, 3)] += np.float32(12.0)
    return lg


def cases():
    rng = np.random.default_rng(20261202)
    out = []
    for c in range(160):
        out.append(dict(seed=int(rng.integers(0, 2**31)), n=int(rng.choice([3, 40, 1000, 4096, 65536, 151936])),
                        kind=int(c % 4), temp=float(rng.choice([0.0, 0.25, 0.7, 1.0, 1.6])),
                        topp=float(rng.choice([0.05, 0.5, 0.9, 0.95, 1.0])),
                        topk=int(rng.choice([0, 1, 7, 40, 1024, 3000])),
                        minp=float(rng.choice([0.0, 0.01, 0.05, 0.3])), rs=int(rng.integers(0, 2**63))))
    return out


def main():
    L = C.CDLL(os.path.join(ROOT, "oracle", "_ref", "libpb_sample.so"))
    L.pbref_sample_topkpp.restype = C.c_int
    L.pbref_sample_topkpp.argtypes = [C.c_void_p, C.c_int, C.c_float, C.c_float, C.c_int, C.c_float,
                                      C.POINTER(C.c_uint64)]
    res = []
    for cs in cases():
        lg = case_logits(cs["seed"], cs["n"], cs["kind"])
        st = C.c_uint64(cs["rs"])
        tid = L.pbref_sample_topkpp(lg.ctypes.data, cs["n"], cs["temp"], cs["topp"], cs["topk"], cs["minp"],
                                    C.byref(st))
        res.append(dict(cs, id=int(tid), rs_out=int(st.value)))
    json.dump(res, open(OUT, "w"), indent=0)
    print("wrote %d cases to %s" % (len(res), OUT))


if __name__ == "__main__":
    main()
