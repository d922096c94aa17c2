"""Times the reference's own GPU kernels, compiled by oracle/build_ref.sh into
oracle/_ref (libpb_refgpu.so: q8_partial + k_combine_bf; libpb_refqlow.so:
k_qlow + k_qlow_combine), against this library's kernels at the same shapes
on the same GPU: each side over rotating weight copies larger than L2, CUDA
events, mean microseconds per call. Prints one line per shape and, for the
Q8 GEMV, what the reference's per-name GEMVs of one cfg1 token (18 conv
layers, 6 attention layers, the head) would take. TEST INFRASTRUCTURE
(context for the benchmark, not part of it); GPU box only.

    bash oracle/build_ref.sh && python oracle/time_ref_kernels.py
"""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "pulsar-asm_b200"))
L2 = 126 * 2 ** 20


def main():
    import torch
    import pulsar_b200 as pb
    from pulsar_b200 import synth
    st = torch.cuda.Stream()

    def trot(fns, reps):
        for f in fns:
            f()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        for _ in range(reps):
            for f in fns:
                f()
        e1.record(st)
        e1.synchronize()
        return e0.elapsed_time(e1) * 1e3 / (reps * len(fns))

    R = C.CDLL(os.path.join(HERE, "_ref", "libpb_refgpu.so"))
    R.pbref_gpu_q8_gemv_time.restype = C.c_float
    R.pbref_gpu_q8_gemv_time.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int]
    Q = C.CDLL(os.path.join(HERE, "_ref", "libpb_refqlow.so"))
    Q.pbref_gpu_qlow_time.restype = C.c_float
    Q.pbref_gpu_qlow_time.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]
    rng = np.random.default_rng(1)
    res = {}
    print("Q8 GEMV (fp32 scales, bf16 x and y): reference q8_partial + k_combine_bf | pb_q8_gemv")
    with torch.cuda.stream(st):
        for N, K in [(6144, 2048), (2048, 2048), (8192, 2048), (16384, 2048), (2048, 8192), (512, 2048), (32, 2048),
                     (65536, 2048)]:
            nb = N * K + N * K // 32 * 4 + K * 2 + N * 2
            ncp = int(2 * L2 // nb) + 1
            q = rng.integers(-127, 128, (N, K), dtype=np.int8)
            s = (rng.random((N, K // 32)) * 0.01).astype(np.float32)
            ref = R.pbref_gpu_q8_gemv_time(q.ctypes.data, s.ctypes.data, N, K, ncp, 20)
            dq, ds = torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()
            ws = [pb.Q8Tensor(dq, ds, stream=st) for _ in range(ncp)]
            x = torch.randn(K, device="cuda").to(torch.bfloat16).view(torch.int16)
            y = torch.empty(N, dtype=torch.int16, device="cuda")
            ours = trot([lambda w=w: w.gemv(x, y, stream=st) for w in ws], 20)
            del ws
            res[(N, K)] = ref
            print("%6d x %5d  reference %7.2f us %5.0f GB/s | ours %6.2f us %5.0f GB/s | x%.2f"
                  % (N, K, ref, nb / ref / 1e3, ours, nb / ours / 1e3, ref / ours), flush=True)
        conv = res[(6144, 2048)] + res[(2048, 2048)] + 2 * res[(8192, 2048)] + res[(2048, 8192)]
        attn = (2 * res[(2048, 2048)] + 2 * res[(512, 2048)] + res[(32, 2048)] + 2 * res[(8192, 2048)] +
                res[(2048, 8192)])
        print("reference GEMVs of one cfg1 token: %.1f us" % (18 * conv + 6 * attn + res[(65536, 2048)]))
        print("Q4 / Q5 GEMV: reference k_qlow + k_qlow_combine | pb_qlow_gemv")
        for bits in (4, 5):
            for N, K in [(8192, 2048), (2048, 8192), (65536, 2048)]:
                nb = N * K // 32 * (20 if bits == 5 else 16) + N * K // 32 * 4 + K * 2 + N * 2
                ncp = int(2 * L2 // nb) + 1
                qc, qs = synth.qlow_payload(np.random.default_rng(bits), N, K, bits)
                ref = Q.pbref_gpu_qlow_time(qc.ctypes.data, qs.ctypes.data, bits, N, K, ncp, 20)
                dc, dsc = torch.from_numpy(qc).cuda(), torch.from_numpy(qs.view(np.int16)).cuda()
                ws = [pb.QlowTensor(dc, dsc, bits, N, K, stream=st) for _ in range(ncp)]
                x = torch.randn(K, device="cuda").to(torch.bfloat16).view(torch.int16)
                y = torch.empty(N, dtype=torch.int16, device="cuda")
                ours = trot([lambda w=w: w.gemv(x, y, stream=st) for w in ws], 20)
                del ws
                print("Q%d %6d x %5d  reference %6.2f us %5.0f GB/s | ours %6.2f us %5.0f GB/s | x%.2f"
                      % (bits, N, K, ref, nb / ref / 1e3, ours, nb / ours / 1e3, ref / ours), flush=True)


if __name__ == "__main__":
    main()
