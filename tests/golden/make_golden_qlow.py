"""Generates tests/golden/qlow.npz: the outputs of the REFERENCE's own low-bit
GEMV kernels (pulsar_arm/asm/lfm3_qlow.cuh: k_qlow + k_qlow_combine, compiled
where they lie into oracle/_ref/libpb_refqlow.so by oracle/build_ref.sh and
launched as qlow_gemv launches them) on seeded Q4 and Q5 tensors. TEST
INFRASTRUCTURE: tests/test_qlow.py checks the oracle's restatement against
these outputs. Runs on a GPU box (the library is sm_100a code); the inputs of
a case are regenerated from its seed by case_inputs(), only the outputs are
committed.

    bash oracle/build_ref.sh && python tests/golden/make_golden_qlow.py
"""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "qlow.npz")

# (bits, N, K, seed): K slices of 2 and 4, tiny and ragged group counts
CASES = [(4, 256, 2048, 1), (5, 256, 2048, 2), (4, 96, 4096, 3), (5, 128, 8192, 4), (4, 64, 256, 5),
         (5, 32, 768, 6), (5, 160, 4096, 7)]


def case_inputs(bits, N, K, seed):
    sys.path.insert(0, os.path.join(ROOT, "pulsar-asm_b200"))
    from pulsar_b200 import synth
    rng = np.random.default_rng(seed)
    codes, scales = synth.qlow_payload(rng, N, K, bits)
    xf = rng.standard_normal(K).astype(np.float32)
    u = xf.view(np.uint32)
    x = ((u + np.uint32(0x7FFF) + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return codes, scales, x


def main():
    L = C.CDLL(os.path.join(ROOT, "oracle", "_ref", "libpb_refqlow.so"))
    L.pbref_gpu_qlow.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int]
    out = {}
    for bits, N, K, seed in CASES:
        codes, scales, x = case_inputs(bits, N, K, seed)
        y = np.zeros(N, np.uint16)
        rc = L.pbref_gpu_qlow(codes.ctypes.data, scales.ctypes.data, bits, x.ctypes.data, y.ctypes.data, N, K)
        assert rc == 0, "reference kernel failed"
        out["q%d_%d_%d_%d" % (bits, N, K, seed)] = y
    np.savez(OUT, **out)
    print("wrote", OUT, sorted(out))


if __name__ == "__main__":
    main()
