"""Benchmark: decode tok/s of the LFM3-style Q8_0 backbone (BASELINE.json
configs[1]) on B200, with achieved HBM GB/s of the dominant kernel against the
measured roofline, an end-to-end number through the C ABI with host buffers,
and the CPU baseline on the box's host cores.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One process per GPU (torchrun for N > 1). Each rank decodes its own sequence on
its own replica of the model (the path shards by sequence: no data-path
collective); `value` is the tokens of all ranks over the slowest rank's device
time. Weights are synthetic with the configuration's distributions (seeded);
every token streams 1.8 GB of weights, far more than the 126 MB L2, so no L2
flush is needed between steps.
"""
import argparse
import json
import numpy as np
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "pulsar-asm_b200"))

METRIC = "decode tok/s + achieved HBM GB/s vs ~8 TB/s (Q8_0/Q1_0 GEMV) at 1/2/4/8 B200"
WORKLOAD = ("cfg1: LFM3-style backbone decode T=1, hidden 2048, 24 layers (18 gated short-conv "
            "k=3 + 6 GQA 32q/8kv hd64), SwiGLU 8192, vocab 65536 tied Q8_0 head, fp16 KV at ctx 1024")
SEED = 20261201


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ctx", type=int, default=1024)
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-kernels", action="store_true", help="skip the per-kernel GB/s suite")
    ap.add_argument("--no-tp", action="store_true", help="skip the row-sharded decode at N > 1")
    ap.add_argument("--blob", default=os.environ.get("PB_BENCH_BLOB", "/tmp/pb_cfg1.lfm3q8"))
    ap.add_argument("--phase-trace", action="store_true",
                    help="print the persistent decode kernel's per-phase time breakdown (one GPU) and exit")
    ap.add_argument("--bonsai-only", type=int, default=-1, metavar="KV_BITS",
                    help="profiling only: run just the cfg3 Bonsai decode (K/V cache 0 = f16, 3, 4, 43 = TurboQuant) "
                         "for --warmup + --steps tokens, print its line and exit")
    ap.add_argument("--batch-only", action="store_true",
                    help="profiling only: run just the cfg4 batched decode (greedy, then sampled) on the cfg1 "
                         "model, print its line and exit")
    ap.add_argument("--layers", type=int, default=0,
                    help="profiling only: a shallower model of the same shapes (0 = the 24-layer cfg1)")
    return ap.parse_args()


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs"), "measured"
    return 6650.0, "fallback"


def ncu_traffic():
    """dram bytes per token of the roofline kernel from the committed ncu summary"""
    p = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    if os.path.exists(p):
        try:
            return json.load(open(p)).get("traffic_bytes_per_token")
        except Exception:
            return None
    return None


CPU_SAMPLE = ("%d decode steps of the full cfg1 model at positions %d.. over seeded fp16 KV rows and conv "
              "rings (the oracle's restatement of layer_body + head + argmax, C, OpenMP over rows)")
CLOCK_ROLL_S = 0.15   # identical untimed launches before and after the timed one


def clock_roll(state, tok, pos, n, ids, stream, seconds):
    """back-to-back launches of the timed workload (n greedy tokens from pos)
    on a second state for `seconds`: the clock record around the timed launch"""
    t_end = time.time() + seconds
    while time.time() < t_end:
        state.decode_greedy(tok, pos, n, ids, stream=stream)
        stream.synchronize()


class Clocks:
    """nvidia-smi sampling around the timed region (SM clock and throttle
    reasons). The sampler is started and seen to print before the window
    begins; every sample carries nvidia-smi's own timestamp, and only samples
    taken between the window's start and end count. The window is the timed
    launch plus identical untimed launches before and after it (clock_roll),
    because a K-token launch lasts less than one 25 ms sampler period; the
    summary also says how many samples fell inside the timed launch itself."""

    Q = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index, period_ms=25):
        self.index, self.period, self.p, self.lines = index, period_ms, None, []
        self.t0 = self.t1 = None
        self.r0 = self.r1 = None

    def region_start(self):
        self.r0 = time.time()

    def region_end(self):
        self.r1 = time.time()

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.Q,
                                       "--format=csv,noheader,nounits", "-lms", str(self.period)],
                                      stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t = time.time()
            while not self.lines and time.time() - t < 10:
                time.sleep(0.005)
        except Exception:
            self.p = None
        self.t0 = time.time()
        return self

    def _read(self):
        for line in self.p.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        self.t1 = time.time()
        if self.p:
            time.sleep(2 * self.period / 1000.0)   # samples of the region's last instants
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except Exception:
                self.p.kill()
            self.t.join(timeout=2)

    @staticmethod
    def _when(stamp):
        import datetime
        try:
            return datetime.datetime.strptime(stamp, "%Y/%m/%d %H:%M:%S.%f").timestamp()
        except ValueError:
            return None

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        in_region = 0
        for ln in list(self.lines):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 10:
                continue
            w = self._when(f[0])
            if w is None or self.t0 is None or not (self.t0 <= w <= self.t1):
                continue
            if self.r0 is not None and self.r1 is not None and self.r0 <= w <= self.r1:
                in_region += 1
            try:
                sm.append(float(f[2]))
                mx = float(f[3])
            except ValueError:
                continue
            for n, v in zip(names, f[6:10]):
                if v.lower() == "active":
                    reasons.add(n)
        out = {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
               "reasons": sorted(reasons), "samples": len(sm)}
        if self.t0 is not None and self.t1 is not None:
            out["window_ms"] = round((self.t1 - self.t0) * 1e3, 1)
        if self.r0 is not None and self.r1 is not None:
            out["samples_in_timed_launch"] = in_region
        return out


def bench_cfg(layers):
    from pulsar_b200 import synth
    c = dict(synth.LFM3_CFG1)
    if layers:
        c["n_layers"] = layers
        c["attn_layers"] = tuple(L for L in c["attn_layers"] if L < layers) or (layers - 1,)
    return c


def make_blob(path, c):
    from pulsar_b200 import synth
    if os.path.exists(path) and os.path.exists(path + ".ok"):
        return c, None
    w = synth.make_weights(c, seed=SEED)
    tmp = path + ".tmp%d" % os.getpid()
    synth.write_model(tmp, c, w)
    os.replace(tmp, path)
    open(path + ".ok", "w").write("seed %d\n" % SEED)
    return c, w


def cpu_baseline(c, weights, ctx, seconds):
    """the oracle's decode step (C, OpenMP over rows) on the host cores, over a
    bounded sample at the timed workload's own positions: the KV caches hold
    ctx seeded fp16 rows and the conv rings a seeded history (so each step
    reads the same context the GPU's timed steps read), then whole decode
    steps at positions ctx, ctx+1, ... are timed until `seconds` pass."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import oracle as O
    from pulsar_b200 import synth
    if weights is None:
        weights = synth.make_weights(c, seed=SEED)
    max_ctx = ctx + 64
    om = O.Model(synth.oracle_cfg(c, max_ctx), weights)
    rng = np.random.default_rng(SEED)
    for L in range(c["n_layers"]):
        if L in c["attn_layers"]:
            for which in (0, 1):
                a = (rng.standard_normal((max_ctx, c["n_kv"], c["head_dim"])) * 0.5).astype(np.float16)
                a[ctx:] = 0
                om.set_kv(L, which, a.view(np.uint16))
        else:
            om.set_ring(L, O.f2bf(rng.standard_normal((c["conv_w"], c["hidden"])).astype(np.float32)))
    tok = int(rng.integers(0, c["vocab"]))
    t0 = time.time()
    n, pos = 0, ctx
    while True:
        tok, _, _ = om.decode(tok, pos)
        pos += 1
        n += 1
        if (time.time() - t0 > seconds and n >= 2) or pos >= max_ctx:
            break
    dt = time.time() - t0
    return n / dt, O.lib().pbo_threads(), n, pos


def config_dict(ctx, world):
    """the workload's config, the same in both arms"""
    return {"workload": WORKLOAD, "ctx": ctx, "seqs_per_gpu": 1,
            "weights": "Q8_0 int8 codes + fp16 scales per 32, activations bf16",
            "l2": "inputs larger than L2 (1.8 GB of weights per token)",
            "parallelism": "sequence split, one replica per GPU (dp%d)" % world}


def cpu_model():
    try:
        for ln in subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout.splitlines():
            if ln.startswith("Model name:"):
                return ln.split(":", 1)[1].strip()
    except Exception:
        pass
    return None


def cpu_reference_gemv(seconds=2.0):
    """the reference's own x86/C CPU Q8 GEMV (.auto/lfm3/q8_gemv_cpu.c, built
    unmodified by oracle/build_ref.sh at -O3 and -O3 -march=x86-64-v3) at the
    cfg0 shape (8192 x 2048, fp32 x, fp32 scales): GB/s of codes + scales + x +
    y, with every host core and with one; null where it was not built"""
    import ctypes as C
    import numpy as np
    out = {}
    ncores = len(os.sched_getaffinity(0))
    N, K = 8192, 2048
    rng = np.random.default_rng(SEED)
    q = rng.integers(-127, 128, (N, K), dtype=np.int8)
    sc = (np.abs(rng.standard_normal((N, K // 32))) * 0.01).astype(np.float16).astype(np.float32)
    x = rng.standard_normal(K).astype(np.float32)
    y = np.zeros(N, np.float32)
    nbytes = N * K + N * (K // 32) * 4 + K * 4 + N * 4
    for arm in ("O3", "v3"):
        path = os.path.join(ROOT, "oracle", "_ref", "libpb_q8cpu_%s.so" % arm)
        if not os.path.exists(path):
            continue
        L = C.CDLL(path)
        vp = C.c_void_p
        L.pbref_gemv_q8.argtypes = [vp, vp, vp, vp, C.c_int, C.c_int]
        L.pbref_set_threads.argtypes = [C.c_int]
        res = {}
        for th in (ncores, 1):
            L.pbref_set_threads(th)
            args = [q.ctypes.data_as(vp), sc.ctypes.data_as(vp), x.ctypes.data_as(vp), y.ctypes.data_as(vp), N, K]
            for _ in range(3):
                L.pbref_gemv_q8(*args)
            best = float("inf")
            t_end = time.time() + seconds
            while time.time() < t_end:
                t0 = time.perf_counter()
                L.pbref_gemv_q8(*args)
                best = min(best, time.perf_counter() - t0)
            res["threads_%d" % th] = {"ms": best * 1e3, "gbs": nbytes / best / 1e9}
        out["-O3" if arm == "O3" else "-O3 -march=x86-64-v3"] = res
    return {"kernel": ".auto/lfm3/q8_gemv_cpu.c gemv_q8 (the reference's x86/C path), cfg0 8192x2048",
            "cpu": cpu_model(), "cores": ncores, "arms": out} if out else None


def _time_rotating(torch, stream, fns, reps):
    """mean ms per call of fns (rotating over distinct weight copies whose
    total exceeds L2), after a warm-up pass, by CUDA events on `stream`"""
    for f in fns:
        f()
    stream.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        for f in fns:
            f()
    e1.record(stream)
    e1.synchronize()
    return e0.elapsed_time(e1) / (reps * len(fns))


def kernel_suite(torch, pb, peak, stream):
    """the GEMV/GEMM kernels of the other configs, each over rotating copies
    larger than L2: cfg0 Q8_0 integer GEMV, cfg3 Q1_0 GEMV (gate|up shape),
    cfg2/cfg4 integer GEMMs on the tensor cores (one layer's projections at
    T = 32 and T = 64). Bytes are algorithmic (Q8_0 scales 2 B per block,
    Q1_0 18 B per 128 weights)."""
    out = {}
    g = torch.Generator(device="cuda").manual_seed(SEED)
    L2 = 126 * 2 ** 20

    def q8_dev(N, K):
        c = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda", generator=g)
        s = (torch.randn((N, K // 32), device="cuda", generator=g).abs() * 0.01).half()
        return c, s

    with torch.cuda.stream(stream):
        # cfg0: W 8192x2048 Q8_0, x quantised per 32-block, y fp32
        N, K = 8192, 2048
        nbytes = N * K + N * (K // 32) * 2 + K + (K // 32) * 2 + N * 4
        ncp = int(2 * L2 // nbytes) + 1
        ws = []
        for _ in range(ncp):
            c, sc = q8_dev(N, K)
            ws.append(pb.Q8Tensor(c, sc, stream=stream))
        x = torch.randn(K, device="cuda", generator=g)
        qx = torch.empty(K, dtype=torch.int8, device="cuda")
        dx = torch.empty(K // 32, dtype=torch.int16, device="cuda")
        pb.q80_quantize(x, qx, dx, stream=stream)
        y = torch.empty(N, dtype=torch.float32, device="cuda")
        ms = _time_rotating(torch, stream, [lambda w=w: w.gemv_int(qx, dx, y, stream=stream) for w in ws], 20)
        gbs = nbytes / (ms / 1e3) / 1e9
        out["cfg0_q80_gemv"] = {"shape": [N, K], "us": ms * 1e3, "bytes": nbytes, "GB/s": gbs,
                                "frac": gbs / peak, "copies": ncp}
        del ws
        # cfg0 shape on the low-bit formats (blob dtypes 6 / 7): Q4 and Q5, bf16
        # x and y; and one conv layer's four projections at T = 32 in Q4
        from pulsar_b200 import synth as _synth
        for bits in (4, 5):
            N, K = 8192, 2048
            nbytes = N * K // 32 * (20 if bits == 5 else 16) + N * K // 32 * 4 + K * 2 + N * 2
            ncp = int(2 * L2 // nbytes) + 1
            rng = np.random.default_rng(bits)
            qc, qs = _synth.qlow_payload(rng, N, K, bits)
            qls = [pb.QlowTensor(torch.from_numpy(qc).cuda(), torch.from_numpy(qs.view(np.int16)).cuda(), bits, N, K,
                                 stream=stream) for _ in range(ncp)]
            xb = torch.randn(K, device="cuda", generator=g).to(torch.bfloat16).view(torch.int16)
            yb = torch.empty(N, dtype=torch.int16, device="cuda")
            ms = _time_rotating(torch, stream, [lambda w=w: w.gemv(xb, yb, stream=stream) for w in qls], 20)
            gbs = nbytes / (ms / 1e3) / 1e9
            out["cfg0_q%d_gemv" % bits] = {"shape": [N, K], "us": ms * 1e3, "bytes": nbytes, "GB/s": gbs,
                                           "frac": gbs / peak, "copies": ncp,
                                           "path": "k_qlow_tile (lfm3_qlow.cuh arithmetic, blob dtype %d)" % (
                                               7 if bits == 5 else 6)}
            del qls
        shapes = [(6144, 2048), (2048, 2048), (16384, 2048), (2048, 8192)]
        T = 32
        lay_bytes = sum(n * k // 32 * 16 + n * k // 32 * 4 + T * (k + n) * 2 for n, k in shapes)
        ncp = int(2 * L2 // lay_bytes) + 1
        rng = np.random.default_rng(7)
        lays = []
        for _ in range(ncp):
            lay = []
            for n, k in shapes:
                qc, qs = _synth.qlow_payload(rng, n, k, 4)
                lay.append(pb.QlowTensor(qc, qs, 4, n, k, stream=stream))
            lays.append(lay)
        xs = {k: torch.randn((T, k), device="cuda", generator=g).to(torch.bfloat16).view(torch.int16)
              for k in (2048, 8192)}
        ys = {n: torch.empty((T, n), dtype=torch.int16, device="cuda") for n, _ in shapes}

        def q4_layer(lay):
            for (n, k), w in zip(shapes, lay):
                w.gemm(xs[k], ys[n], stream=stream)
        ms = _time_rotating(torch, stream, [lambda lay=lay: q4_layer(lay) for lay in lays], 10)
        out["cfg2_q4_gemm_T32"] = {"layer_gemms": [list(x) for x in shapes], "T": T, "us_per_layer": ms * 1e3,
                                   "bytes": lay_bytes, "GB/s": lay_bytes / (ms / 1e3) / 1e9,
                                   "frac": lay_bytes / (ms / 1e3) / 1e9 / peak, "copies": ncp,
                                   "path": "k_qlow_tile, 4 positions per tile read (blob dtype 6)"}
        del lays
        # cfg3: Q1_0 gate|up 24576x4096, Q8_K activation, y fp32
        N, K = 24576, 4096
        nbytes = N * K // 8 + N * (K // 128) * 2 + (K // 256) * 292 + N * 4
        ncp = int(2 * L2 // nbytes) + 1
        q1s = []
        for _ in range(ncp):
            blk = torch.randint(0, 256, (N, (K // 128) * 18), dtype=torch.uint8, device="cuda", generator=g)
            sc = (torch.randn((N, K // 128), device="cuda", generator=g).abs() * 0.02).half()
            blk.view(N, K // 128, 18)[:, :, :2].copy_(sc.view(torch.uint8).view(N, K // 128, 2))
            q1s.append(pb.Q1Tensor(blk, N, K, stream=stream))
        xq = torch.empty((K // 256) * 292, dtype=torch.uint8, device="cuda")
        pb.q8k_quantize(torch.randn(K, device="cuda", generator=g), xq, stream=stream)
        y = torch.empty(N, dtype=torch.float32, device="cuda")
        ms = _time_rotating(torch, stream, [lambda w=w: w.gemv(xq, y, stream=stream) for w in q1s], 20)
        gbs = nbytes / (ms / 1e3) / 1e9
        out["cfg3_q1_gemv"] = {"shape": [N, K], "us": ms * 1e3, "bytes": nbytes, "GB/s": gbs,
                               "frac": gbs / peak, "copies": ncp}
        del q1s
        # cfg2 / cfg4: one conv layer's projections as integer GEMMs on the tensor cores
        shapes = [(6144, 2048), (2048, 2048), (16384, 2048), (2048, 8192)]
        lay_bytes = sum(n * k + n * (k // 32) * 2 for n, k in shapes)
        ncp = int(2 * L2 // lay_bytes) + 1
        layers = [[pb.Q8Tensor(*q8_dev(n, k), stream=stream, tensor_cores=True) for n, k in shapes]
                  for _ in range(ncp)]
        for T, key in ((32, "cfg2_q80_gemm_tc_T32"), (64, "cfg4_q80_gemm_tc_T64")):
            acts = {}
            for n, k in shapes:
                if k not in acts:
                    xa = torch.randn((T, k), device="cuda", generator=g)
                    qa = torch.empty((T, k), dtype=torch.int8, device="cuda")
                    da = torch.empty((T, k // 32), dtype=torch.int16, device="cuda")
                    pb.q80_quantize(xa, qa, da, stream=stream)
                    acts[k] = (qa, da)
            ys = {n: torch.empty((T, n), dtype=torch.float32, device="cuda") for n, _ in shapes}

            def layer(ws=None):
                for w, (n, k) in zip(ws, shapes):
                    w.gemm_int(acts[k][0], acts[k][1], ys[n], stream=stream)
            ms = _time_rotating(torch, stream, [lambda ws=ws: layer(ws) for ws in layers], 10)
            pb.Q8Tensor.gemm_int_status(stream)
            nbytes = lay_bytes + sum(T * k + T * (k // 32) * 2 + T * n * 4 for n, k in shapes)
            ops = sum(2 * n * k * T for n, k in shapes)
            gbs = nbytes / (ms / 1e3) / 1e9
            out[key] = {"layer_gemms": shapes, "T": T, "us_per_layer": ms * 1e3, "bytes": nbytes,
                        "GB/s": gbs, "frac": gbs / peak, "int8_TOPS": ops / (ms / 1e3) / 1e12, "copies": ncp}
        del layers
        # cfg2, float path (the reference's REF_FLOAT numerics, pf_gemv_T): the
        # same layer's projections at T = 32 through the position-tiled
        # streaming kernel, bf16 in and out
        T = 32
        layers = [[pb.Q8Tensor(*q8_dev(n, k), stream=stream) for n, k in shapes] for _ in range(ncp)]
        xs = {k: torch.randn((T, k), device="cuda", generator=g).to(torch.bfloat16).view(torch.int16)
              for _, k in shapes}
        ys = {n: torch.empty((T, n), dtype=torch.int16, device="cuda") for n, _ in shapes}

        def flayer(ws=None):
            for w, (n, k) in zip(ws, shapes):
                w.gemm(xs[k], ys[n], stream=stream)
        ms = _time_rotating(torch, stream, [lambda ws=ws: flayer(ws) for ws in layers], 10)
        nbytes = lay_bytes + sum(T * k * 2 + T * n * 2 for n, k in shapes)
        flops = sum(2 * n * k * T for n, k in shapes)
        gbs = nbytes / (ms / 1e3) / 1e9
        out["cfg2_q8f_gemm_T32"] = {"layer_gemms": shapes, "T": T, "us_per_layer": ms * 1e3, "bytes": nbytes,
                                    "GB/s": gbs, "frac": gbs / peak, "fp32_TFLOPS": flops / (ms / 1e3) / 1e12,
                                    "copies": ncp, "path": "float (REF_FLOAT leaf per position, k_q8f_tiled)"}
        del layers
    torch.cuda.synchronize()
    return out


def prefill_bench(torch, model, prompt, stream, T=32):
    """cfg2: the 1024-token prompt in chunks of T positions through the whole
    backbone on the integer path (tensor-core GEMMs), timed by CUDA events
    after one untimed pass (which also builds the tensor-core weight copies)"""
    n = (prompt.numel() // T) * T
    st = model.new_state(n + 8)
    ids = torch.empty(T, dtype=torch.int32, device="cuda")
    with torch.cuda.stream(stream):
        for c in range(0, n, T):
            st.prefill_chunk(prompt[c:c + T], c, ids, stream=stream)
        stream.synchronize()
        st.reset(stream=stream)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for c in range(0, n, T):
            st.prefill_chunk(prompt[c:c + T], c, ids, stream=stream)
        e1.record(stream)
        e1.synchronize()
    st.status(stream)
    ms = e0.elapsed_time(e1)
    st.destroy()
    return {"tokens": n, "chunk": T, "ms": ms, "tok/s": n / (ms / 1e3), "ms_per_chunk": ms / (n // T),
            "path": "integer (Q8_0 activations, tcgen05 kind::i8 GEMMs)"}


def batch_bench(torch, model, c, stream, B=64, steps=10):
    """cfg4: B independent sequences with ragged contexts drawn uniformly from
    [16, 2048] (seeded, rounded up to multiples of 16 for the chunked prefill
    that fills them), then `steps` batched decode steps (one integer-path
    tensor-core GEMM per projection over the batch), timed by CUDA events"""
    rng = np.random.default_rng(SEED + 4)
    ctx = ((rng.integers(16, 2049, B) + 15) // 16) * 16
    g = torch.Generator().manual_seed(SEED + 5)
    states = []
    with torch.cuda.stream(stream):
        for b in range(B):
            st = model.new_state(int(ctx[b]) + 2 * steps + 16)   # the greedy and the sampled steps
            toks = torch.randint(0, c["vocab"], (int(ctx[b]),), generator=g, dtype=torch.int32).cuda()
            for p0 in range(0, int(ctx[b]), 64):
                n = min(64, int(ctx[b]) - p0)
                st.prefill_chunk(toks[p0:p0 + n], p0, stream=stream)
            states.append(st)
        stream.synchronize()
        tokens = torch.randint(0, c["vocab"], (B,), generator=g, dtype=torch.int32).cuda()
        pos = torch.from_numpy(ctx.astype(np.int32)).cuda()
        ids = torch.empty(B, dtype=torch.int32, device="cuda")
        model.decode_batch(states, tokens, pos, ids, stream=stream)      # warm-up step
        pos += 1
        tokens = ids.clone()
        stream.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            model.decode_batch(states, tokens, pos, ids, stream=stream)
            pos += 1
            tokens.copy_(ids)
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        # the same steps with each sequence's next id drawn on the device by
        # fwd8.c's sampler (temperature 0.7, top-p 0.9, top-k 40, one LCG state
        # per sequence) from the step's logits, instead of the greedy id
        import pulsar_b200 as pbm
        logits = torch.empty((B, c["vocab"]), dtype=torch.float32, device="cuda")
        rs = torch.arange(1, B + 1, dtype=torch.int64, device="cuda") * 7919
        marks = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        # one untimed sampled step: the sampler's first launch loads its module
        model.decode_batch(states, tokens, pos, ids, logits, stream=stream)
        pbm.sample_topkpp(logits, 0.7, 0.9, 40, 0.0, rs, tokens, stream=stream)
        pos += 1
        stream.synchronize()
        e2 = torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("cfg4_sampled_steps")   # a profiler's capture range; no-op otherwise
        e2.record(stream)
        for k in range(steps):
            model.decode_batch(states, tokens, pos, ids, logits, stream=stream)
            marks[k][0].record(stream)
            pbm.sample_topkpp(logits, 0.7, 0.9, 40, 0.0, rs, tokens, stream=stream)
            marks[k][1].record(stream)
            pos += 1
        torch.cuda.nvtx.range_pop()
        marks[-1][1].synchronize()
        ms_sampled = e2.elapsed_time(marks[-1][1])
        ms_sample = sum(a.elapsed_time(b) for a, b in marks)
    for st in states:
        st.status(stream)
        st.destroy()
    return {"sequences": B, "steps": steps, "mean_ctx": float(ctx.mean()), "ms_per_step": ms / steps,
            "tok/s": B * steps / (ms / 1e3), "path": "integer (Q8_0 activations, tcgen05 kind::i8 GEMMs, N = 64)",
            "sampled": {"ms_per_step": ms_sampled / steps, "tok/s": B * steps / (ms_sampled / 1e3),
                        "sampler_us_per_step": ms_sample * 1e3 / steps,
                        "path": "logits [64][vocab] from the batched step, pb_sample_topkpp (fwd8.c:465-521) "
                                "on the device"}}


def bonsai_bench(torch, pb, peak, stream, steps=20, warmup=3, kv_bits=0):
    """cfg3: the Bonsai-8B-shaped Q1_0 decoder (36 layers, hidden 4096, 32/8
    heads x 128, FFN 12288, vocab 151936, tied head) over an f16 K/V cache
    filled to just below 2048 positions; `warmup` + `steps` greedy tokens end
    at position 2047 (each step's CUDA graph: 364 kernels). Weights are
    seeded on the device (uniform sign bits, fp16 scales |N(0,1)|*0.02), the
    cache with N(0,1) f16 rows. Also timed end to end through the public
    call with a host token in and the host id out per step. kv_bits 4: the
    same with the TurboQuant cache the reference's glue uses by default (its
    positions below pos0 hold zero codes: the kernels' work does not depend on
    the code values)."""
    from pulsar_b200 import synth
    max_ctx = 2048
    pos0 = max_ctx - (warmup + steps)
    c, m, s = bonsai_setup(torch, pb, stream, max_ctx, pos0, kv_bits=kv_bits)
    ids = torch.empty(warmup + steps, dtype=torch.int32, device="cuda")
    with torch.cuda.stream(stream):
        s.decode_greedy(7, pos0, warmup, ids[:warmup], stream=stream)
        nxt = int(ids[warmup - 1].item())
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        s.decode_greedy(nxt, pos0 + warmup, steps, ids[warmup:], stream=stream)
        e1.record(stream)
        e1.synchronize()
        ms = e0.elapsed_time(e1)
        # end to end: the same positions again through the per-token public call
        tok = nxt
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2.record(stream)
        for i in range(steps):
            tok = s.decode(tok, pos0 + warmup + i, stream=stream)
        e3.record(stream)
        e3.synchronize()
        ms_e2e = e2.elapsed_time(e3)
    fb = s.fallbacks()
    ctx_mean = pos0 + warmup + (steps + 1) / 2.0
    nbytes = synth.bonsai_bytes_per_token(c, ctx_mean, kv_bits=kv_bits)
    step_s = ms / 1e3 / steps
    s.destroy()
    m.close()
    return {"model": "Bonsai-8B shape, Q1_0, 36 layers, vocab 151936", "steps": steps, "warmup": warmup,
            "positions": [pos0 + warmup, pos0 + warmup + steps - 1], "mean_ctx": ctx_mean,
            "ms_per_token": ms / steps, "tok/s": steps / (ms / 1e3),
            "e2e_tok/s": steps / (ms_e2e / 1e3), "bytes_per_token": nbytes,
            "GB/s": nbytes / step_s / 1e9, "frac": nbytes / step_s / 1e9 / peak,
            "kernels_per_token": 36 * (14 if kv_bits else 10) + 4, "rms_serial_fallbacks": fb,
            "path": ("CUDA graph of PDL launches: Q1_0 x Q8_K GEMVs, TurboQuant %d-bit K/V cache "
                     "(store, scores, softmax, chunked rotated-domain P.V, inverse rotation)" % kv_bits) if kv_bits else
                    "CUDA graph of PDL launches: Q1_0 x Q8_K GEMVs, f16 flash-attention decode in fork order"}


def bonsai_setup(torch, pb, stream, max_ctx, pos0, n_layers=None, kv_bits=0):
    """the cfg3 model with seeded device weights and a state whose K/V cache
    holds N(0,1) f16 rows at positions < pos0"""
    from pulsar_b200 import synth
    c = dict(synth.BONSAI_CFG3)
    if n_layers:
        c["n_layers"] = n_layers
    g = torch.Generator(device="cuda").manual_seed(SEED + 3)
    H, F, NH, NKV = c["hidden"], c["inter"], c["n_heads"], c["n_kv"]
    m = pb.Bonsai(c)

    def q1(rows, K):
        b = torch.randint(0, 256, (rows, K // 128, 18), dtype=torch.uint8, device="cuda", generator=g)
        sc = (torch.randn((rows, K // 128), device="cuda", generator=g).abs() * 0.02).half()
        b[:, :, :2].copy_(sc.view(torch.uint8).view(rows, K // 128, 2))
        return b

    def norm(n):
        return (1.0 + 0.05 * torch.randn(n, generator=torch.Generator().manual_seed(n))).numpy()
    st = pb._stream(stream)
    shapes = {0: (NH * 128, H), 1: (NKV * 128, H), 2: (NKV * 128, H), 3: (H, NH * 128),
              4: (F, H), 5: (F, H), 6: (H, F)}
    for L in range(c["n_layers"]):
        for slot, (r, k) in shapes.items():
            m.set_q1(L, slot, q1(r, k), st)
        for slot, n in ((0, H), (1, H), (2, 128), (3, 128)):
            m.set_norm(L, slot, norm(n), st)
    m.set_q1(-1, 16, q1(c["vocab"], H), st)
    m.set_norm(-1, 16, norm(H), st)
    s = m.new_state(max_ctx, kv_bits=kv_bits)
    if not kv_bits:
        for L in range(c["n_layers"]):
            for which in (0, 1):
                kv = s.kv(L, which)
                kv.copy_(torch.randn(kv.shape, device="cuda", generator=g).half().view(torch.int16))
                kv[:, pos0:].zero_()
    torch.cuda.synchronize()
    return c, m, s


def phase_trace(torch, model, prompt, stream, ctx):
    """Per-phase breakdown of one decode token (token 0 of a 4-token launch of
    the persistent kernel, after two warm launches) from the kernel's own
    globaltimer marks (PB_DECODE_TRACE): per CTA and phase the entry, the end
    of the prologue (the previous phase's tagged output arrived and the GEMV
    input built), the end of the work and the phase's closing CTA barrier, plus
    warp 0's data waits, slot releases (with refill issues) and chain
    arithmetic inside the GEMV stage loops. Times are means over the CTAs (over
    the head CTAs for attention phases), in microseconds."""
    import numpy as np
    os.environ["PB_DECODE_TRACE"] = "1"
    st = model.new_state(ctx + 64)
    ids = torch.empty(4, dtype=torch.int32, device="cuda")
    with torch.cuda.stream(stream):
        st.decode_prompt(prompt, 0, stream=stream)
        for _ in range(3):
            st.decode_greedy(int(prompt[-1].item()), ctx, 4, ids, stream=stream)
        stream.synchronize()
    tr = st.debug_tensor(5, torch.int64).cpu().numpy().astype(np.int64)
    st.destroy()
    del os.environ["PB_DECODE_TRACE"]
    G = torch.cuda.get_device_properties(0).multi_processor_count
    nph = tr.size // (G * 8)
    tr = tr.reshape(G, nph, 8).astype(np.float64) / 1e3
    gemv = (tr[:, :, 1] != 0).any(axis=0)
    nh = int(model.info["n_heads"])
    mean = lambda a: a.mean(axis=0)
    pro = mean(tr[:, :, 1] - tr[:, :, 0])
    work_g = mean(tr[:, :, 3] - tr[:, :, 1])
    work_a = (tr[:nh, :, 3] - tr[:nh, :, 0]).mean(axis=0)
    close = mean(tr[:, :, 4] - tr[:, :, 3])
    attn = ~gemv
    # GEMV inputs: when thread 0's poll saw the previous phase's tagged output
    # (mark 2), against when the last producer CTA ended its work (mark 3)
    polled = (tr[:, :, 2] != 0).all(axis=0)
    prev_last = np.concatenate([[np.nan], tr[:, :-1, 3].max(axis=0)])
    prev_first = np.concatenate([[np.nan], tr[:, :-1, 3].min(axis=0)])
    detect = mean(tr[:, :, 2]) - prev_last
    out = {"phases": int(nph), "gemv_phases": int(gemv.sum()), "attention_phases": int(attn.sum()),
           "token_us": float(tr[:, -1, 4].max() - tr[:, 0, 0].min()),
           "gemv_prologue_with_input_wait_us": float(pro[gemv].sum()),
           "gemv_input_wait_us": float(mean(tr[:, :, 2] - tr[:, :, 0])[polled].sum()),
           "gemv_input_after_last_producer_us": float(detect[polled].sum()),
           "producer_end_spread_us": float((prev_last - prev_first)[polled].sum()),
           "gemv_norm_and_x_us": float(mean(tr[:, :, 1] - tr[:, :, 2])[polled].sum()),
           "gemv_work_us": float(work_g[gemv].sum()),
           "attention_work_us_head_ctas": float(work_a[attn].sum()),
           "phase_close_us": float(close.sum()),
           # slots 5 to 7 are written only by a library built with
           # EXTRA=-DPB_TRACE_STAGE_LOOP (null otherwise)
           "warp0_data_wait_us": float(mean(tr[:, :, 6])[gemv].sum()) if tr[:, :, 6].any() else None,
           "warp0_release_issue_us": float(mean(tr[:, :, 5])[gemv].sum()) if tr[:, :, 5].any() else None,
           "warp0_chains_trees_us": float(mean(tr[:, :, 7])[gemv].sum()) if tr[:, :, 7].any() else None,
           "first_phases": [{"phase": p, "kind": "gemv" if gemv[p] else "attention",
                             "prologue_us": round(float(pro[p]), 2) if gemv[p] else None,
                             "work_us": round(float(work_g[p] if gemv[p] else work_a[p]), 2),
                             "close_us": round(float(close[p]), 2),
                             "span_us": round(float(tr[:, p, 4].max() - tr[:, p, 0].min()), 2)}
                            for p in range(min(nph, 12))]}
    return out


def tp_bench(torch, pb, model, prompt, stream, rank, world, steps=32, warmup=3):
    """one sequence decoded with every GEMV's rows split over the ranks and
    each output all-gathered over NVLink (pb_state_shard); the same prompt as
    the replica measurement, then `steps` greedy tokens timed by CUDA events,
    max over ranks"""
    from pulsar_b200 import dist
    ctx = int(prompt.numel())
    st = model.new_state(ctx + warmup + steps + 8)
    uid = dist.share_from_rank0(pb.nccl_unique_id)
    st.shard(rank, world, uid)
    ids = torch.empty(warmup + steps, dtype=torch.int32, device="cuda")
    with torch.cuda.stream(stream):
        st.decode_prompt(prompt, 0, stream=stream)
        st.decode_greedy(int(prompt[-1].item()), ctx, warmup, ids[:warmup], stream=stream)
        stream.synchronize()
        nxt = int(ids[warmup - 1].item())
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        st.decode_greedy(nxt, ctx + warmup, steps, ids[warmup:], stream=stream)
        e1.record(stream)
        e1.synchronize()
    st.status(stream)
    ms = dist.max_over_ranks(e0.elapsed_time(e1), device="cuda")
    kpt = st.kernels_per_token()
    st.destroy()
    return {"ranks": world, "steps": steps, "ms_per_token": ms / steps, "tok/s": steps / (ms / 1e3),
            "kernels_per_token": kpt,
            "path": "row-sharded GEMVs (rank r computes rows [r N/world, (r+1) N/world)), in-place NCCL "
                    "all-gather of every output, CUDA graph per token; one sequence over all GPUs"}


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU implementation of this path (the
    oracle port: the reference's decode engine has no CPU form) on this box's
    host cores, rank 0 only."""
    if rank != 0:
        return
    # torchrun sets OMP_NUM_THREADS=1 for N > 1; the reference arm uses every host core
    os.environ["OMP_NUM_THREADS"] = str(len(os.sched_getaffinity(0)))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.build() if not os.path.exists(O.LIB_PATH) else None
    from pulsar_b200 import synth
    c = synth.LFM3_CFG1
    w = synth.make_weights(c, seed=SEED)
    per_step = max(2.0, min(20.0, 120.0 / max(1, args.steps + args.warmup)))
    tps, cores, n, _ = cpu_baseline(c, w, args.ctx, per_step * max(1, min(args.steps, 6)))
    line = {"impl": "reference", "metric": METRIC, "value": tps, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 / tps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic", "config": config_dict(args.ctx, world),
            "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": cores, "kind": "port", "cpu": cpu_model(),
                             "sample": CPU_SAMPLE % (n, args.ctx)},
            "cpu_reference": cpu_reference_gemv(),
            "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    from pulsar_b200 import dist
    rank, world, local = dist.env_rank()
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    import torch
    import pulsar_b200 as pb
    from pulsar_b200 import synth
    torch.cuda.set_device(local)
    dist.init(timeout_s=900)
    if not os.path.exists(pb.LIB_PATH):
        pb.build()
    if args.bonsai_only >= 0:
        if rank == 0:
            peak, _ = measured_peaks()
            print(json.dumps({"cfg3_decode": bonsai_bench(torch, pb, peak, torch.cuda.Stream(), steps=args.steps,
                                                          warmup=args.warmup, kv_bits=args.bonsai_only)}))
        dist.finish()
        return
    c = bench_cfg(args.layers)
    blob = args.blob if not args.layers else args.blob.replace(".lfm3q8", "_L%d.lfm3q8" % args.layers)
    weights = None
    if rank == 0:
        c, weights = make_blob(blob, c)
    dist.barrier()
    model = pb.Model(blob, device=local)
    max_ctx = args.ctx + args.warmup + 2 * args.steps + 8
    st = model.new_state(max_ctx)
    stream = torch.cuda.Stream()
    rng = torch.Generator().manual_seed(SEED + rank)
    prompt = torch.randint(0, c["vocab"], (args.ctx,), generator=rng, dtype=torch.int32).cuda()
    if args.batch_only:
        if rank == 0:
            print(json.dumps({"cfg4_batched_decode": batch_bench(torch, model, c, stream)}))
        st.destroy()
        dist.finish()
        return
    if args.phase_trace:
        if rank == 0:
            print(json.dumps({"phase_trace": phase_trace(torch, model, prompt, stream, args.ctx),
                              "config": {"workload": "cfg1", "ctx": args.ctx}}))
        st.destroy()
        dist.finish()
        return
    with torch.cuda.stream(stream):
        # prefill the KV cache and conv rings: `ctx` teacher-forced tokens
        st.decode_prompt(prompt, 0, stream=stream)
        ids = torch.empty(args.warmup + args.steps, dtype=torch.int32, device="cuda")
        first = int(prompt[-1].item())
        pos = args.ctx
        # warm-up steps (greedy)
        st.decode_greedy(first, pos, args.warmup, ids[:args.warmup], stream=stream)
        stream.synchronize()
        pos += args.warmup
        nxt = int(ids[args.warmup - 1].item()) if args.warmup else first
        # a second state at the same positions runs identical launches around
        # the timed one, so that the clock record spans many sampler periods
        # (a K-token launch is shorter than one)
        aux = model.new_state(max_ctx)
        aux.decode_prompt(prompt, 0, stream=stream)
        aux_ids = torch.empty(args.steps, dtype=torch.int32, device="cuda")
        stream.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with Clocks(local) as clk:
            clock_roll(aux, nxt, pos, args.steps, aux_ids, stream, CLOCK_ROLL_S)
            clk.region_start()
            launches0 = pb.launch_count()
            e0.record(stream)
            st.decode_greedy(nxt, pos, args.steps, ids[args.warmup:], stream=stream)
            e1.record(stream)
            e1.synchronize()
            launches = pb.launch_count() - launches0
            clk.region_end()
            clock_roll(aux, nxt, pos, args.steps, aux_ids, stream, CLOCK_ROLL_S)
        aux.destroy()
        dist.barrier()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        ms_max = dist.max_over_ranks(ms, device="cuda")
        pos += args.steps
        # end to end through the public API with host buffers: per step the
        # token goes host->device (pinned control block) and the greedy id
        # comes back device->host, all inside the timed region
        e2e_steps = max(10, args.steps // 2)
        tok = int(ids[-1].item())
        dist.barrier()
        torch.cuda.synchronize()
        e2 = torch.cuda.Event(enable_timing=True)
        e3 = torch.cuda.Event(enable_timing=True)
        e2.record(stream)
        for i in range(e2e_steps):
            tok = st.decode_token(tok, pos + i, stream=stream)
        e3.record(stream)
        e3.synchronize()
        ms_e2e = dist.max_over_ranks(e2.elapsed_time(e3), device="cuda")
        # per-kernel path, for reference: the fused w1|w3 GEMV kernel alone
        # (34.6 MB per launch) cycling over the 24 layers' distinct weights
        k_ms, k_bytes = st.time_step_kernel(2, 96, stream=stream)
        kpt = st.kernels_per_token()
    tokens = args.steps * world
    value = tokens / (ms_max / 1000.0)
    peak, peak_kind = measured_peaks()
    wb = model.info["weight_bytes"]
    ctx_mid = args.ctx + args.warmup + args.steps // 2
    kvb = synth.kv_bytes_per_token(c, ctx_mid)
    step_s = ms / 1000.0 / args.steps
    persistent = kpt == 1
    if persistent:
        # the decode kernel: one cooperative launch for the K timed tokens; its
        # algorithmic bytes are every token's weights plus the KV it reads
        achieved = (wb + kvb) / step_s / 1e9
        rk = {"kernel": "k_decode (persistent: TMA bulk weight ring, tagged phase hand-off, fused prologues)",
              "bytes_per_launch": (wb + kvb) * args.steps, "ms_per_launch": ms,
              "bytes_per_token": wb + kvb}
    else:
        achieved = k_bytes / (k_ms / 1000.0) / 1e9
        rk = {"kernel": "k_step<1,fp16 scales,SiLU epilogue> (w1|w3 GEMV, 16384x2048)",
              "bytes_per_launch": k_bytes, "ms_per_launch": k_ms}
    # ncu's dram bytes per token (one captured launch), scaled to this launch
    tpt = ncu_traffic()
    traffic = tpt * args.steps if (tpt and persistent) else None
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": config_dict(args.ctx, world),
            "decode_path": "persistent" if persistent else "graph",
            "e2e": {"value": e2e_steps * world / (ms_e2e / 1000.0), "unit": "tok/s",
                    "h2d_bytes_per_step": 40, "d2h_bytes_per_step": 4},
            "gpu_launches": launches,
            "kernels_per_token": kpt,
            "roofline": dict({"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                              "frac": achieved / peak, "traffic": traffic,
                              "peak_source": "measured hbm_gbs (MEASURED_PEAKS.json)" if peak_kind == "measured"
                              else "fallback 6.65 TB/s"}, **rk),
            "step_kernel_gbs": k_bytes / (k_ms / 1000.0) / 1e9,
            "clocks": clk.summary()}
    if world > 1 and not args.no_tp:
        line["tp_decode"] = tp_bench(torch, pb, model, prompt, stream, rank, world)
    if world > 1 and not args.no_kernels:
        # cfg4 over the ranks: each rank decodes its own share of the sequences
        # (a multiple of 16, the batched step's granule), no data-path
        # collective; the step time is the maximum over ranks
        br = max(16, (64 // world + 15) // 16 * 16)
        b = batch_bench(torch, model, c, stream, B=br)
        msb = dist.max_over_ranks(b["ms_per_step"], device="cuda")
        line["cfg4_batched_decode_split"] = {
            "ranks": world, "sequences_per_rank": br, "sequences": br * world, "steps": b["steps"],
            "ms_per_step": msb, "tok/s": br * world / (msb / 1e3), "scaling": "sequence split, weak",
            "path": b["path"]}
    if rank == 0 and world == 1 and not args.no_kernels:
        line["kernels"] = kernel_suite(torch, pb, peak, stream)
        line["kernels"]["cfg2_prefill"] = prefill_bench(torch, model, prompt, stream)
        line["kernels"]["cfg4_batched_decode"] = batch_bench(torch, model, c, stream)
        line["kernels"]["cfg3_decode"] = bonsai_bench(torch, pb, peak, stream)
        line["kernels"]["cfg3_decode_tq4"] = bonsai_bench(torch, pb, peak, stream, kv_bits=4)
    if rank == 0 and world == 1 and not args.no_cpu:
        tps, cores, n, _ = cpu_baseline(c, weights, args.ctx, args.cpu_seconds)
        line["cpu_baseline"] = {"value": tps, "unit": "tok/s", "cores": cores, "kind": "port", "cpu": cpu_model(),
                                "sample": CPU_SAMPLE % (n, args.ctx)}
        line["cpu_reference"] = cpu_reference_gemv()
    if rank == 0:
        print(json.dumps(line), flush=True)
    st.destroy()
    model.close()
    dist.finish()


if __name__ == "__main__":
    main()
