"""Kernel parity on the B200: every CUDA entry point against the CPU oracle on
the same seeded inputs. Integer results (block dots, quantised bytes) and the
float path (the reference's fixed reduction order) must match bit for bit."""
import os

import numpy as np
import pytest

from conftest import GOLDEN

pytestmark = pytest.mark.gpu


def _dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if a.dtype == np.float32 else np.uint16)


@pytest.mark.parametrize("N,K", [(512, 2048), (3104, 2048), (16384, 2048), (2048, 8192), (1000, 4096),
                                 (96, 1024), (64, 7680), (32, 512), (37, 2048)])
@pytest.mark.parametrize("scales", ["f16", "f32"])
def test_q8_gemv_bitexact(cuda, oracle, pb, N, K, scales):
    torch = cuda
    rng = np.random.default_rng(N * 7 + K)
    codes = rng.integers(-127, 128, (N, K), dtype=np.int8)
    s16 = (np.abs(rng.standard_normal((N, K // 32))) * 0.01).astype(np.float16)
    s = s16.astype(np.float32) if scales == "f32" else s16
    xb = oracle.f2bf(rng.standard_normal(K).astype(np.float32))
    want = oracle.q8f_gemv(codes, s16.astype(np.float32), xb)
    w = pb.Q8Tensor(_dev(torch, codes), _dev(torch, s))
    x = _dev(torch, xb.view(np.int16))
    yb = torch.empty(N, dtype=torch.int16, device="cuda")
    yf = torch.empty(N, dtype=torch.float32, device="cuda")
    w.gemv(x, yb)
    w.gemv(x, yf)
    torch.cuda.synchronize()
    assert np.array_equal(yb.cpu().numpy().view(np.uint16), oracle.f2bf(np.float32(0) + want))
    assert np.array_equal(_bits(yf.cpu().numpy()), _bits(np.float32(0) + want))


@pytest.mark.parametrize("N,K,T", [(256, 2048, 4), (128, 1024, 5), (64, 8192, 3), (96, 7680, 21), (300, 2048, 40),
                                   (40, 16384, 3), (70, 4096, 9)])
def test_q8_gemm_positions(cuda, oracle, pb, N, K, T):
    """T positions of a streaming tensor in one position-tiled launch: every
    position's output equals the single-position GEMV's (pf_gemv_T)"""
    torch = cuda
    rng = np.random.default_rng(T)
    codes = rng.integers(-127, 128, (N, K), dtype=np.int8)
    s16 = (np.abs(rng.standard_normal((N, K // 32))) * 0.01).astype(np.float16)
    xb = oracle.f2bf(rng.standard_normal((T, K)).astype(np.float32))
    want = oracle.q8f_gemv(codes, s16.astype(np.float32), xb)
    w = pb.Q8Tensor(_dev(torch, codes), _dev(torch, s16))
    y = torch.empty((T, N), dtype=torch.int16, device="cuda")
    w.gemm(_dev(torch, xb.view(np.int16)), y)
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy().view(np.uint16), oracle.f2bf(np.float32(0) + want))


def test_q8_gemv_golden_tree(cuda, oracle, pb):
    """the fixture accepted bit for bit by the reference's cpuchk_run"""
    torch = cuda
    g = np.load(os.path.join(GOLDEN, "q8f_tree.npz"))
    for t in ("a", "b", "c"):
        codes, s16, x, y = g[t + "_codes"], g[t + "_s16"], g[t + "_x"], g[t + "_y"]
        w = pb.Q8Tensor(_dev(torch, codes), _dev(torch, s16))
        out = torch.empty((x.shape[0], codes.shape[0]), dtype=torch.int16, device="cuda")
        w.gemm(_dev(torch, x.view(np.int16)), out)
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy().view(np.uint16), y)


def test_q8_gemv_edge_values(cuda, oracle, pb):
    """zero scales, zero x, extreme codes, huge and tiny activations"""
    torch = cuda
    N, K = 256, 2048
    rng = np.random.default_rng(1)
    codes = rng.integers(-127, 128, (N, K), dtype=np.int8)
    codes[:8] = 127
    codes[8:16] = -128
    s16 = (np.abs(rng.standard_normal((N, K // 32))) * 0.01).astype(np.float16)
    s16[16:32] = 0
    s16[32:40] = np.float16(65504)
    for xv in [np.zeros(K, np.float32), rng.standard_normal(K).astype(np.float32) * 1e30,
               rng.standard_normal(K).astype(np.float32) * 1e-30]:
        xb = oracle.f2bf(xv)
        want = oracle.q8f_gemv(codes, s16.astype(np.float32), xb)
        w = pb.Q8Tensor(codes, s16)     # host source: exercises the upload path too
        yf = torch.empty(N, dtype=torch.float32, device="cuda")
        w.gemv(_dev(torch, xb.view(np.int16)), yf)
        torch.cuda.synchronize()
        got = yf.cpu().numpy()
        nan = np.isnan(want)
        assert np.array_equal(np.isnan(got), nan)
        assert np.array_equal(_bits(got[~nan]), _bits(np.float32(0) + want[~nan]))


def test_q80_integer_path_cfg0(cuda, oracle, pb):
    """config 0: W 8192x2048 Q8_0, x N(0,1) quantised per 32-block; block dots
    exact, the fold in block order bit for bit"""
    torch = cuda
    N, K = 8192, 2048
    rng = np.random.default_rng(0)
    codes = rng.integers(-127, 128, (N, K), dtype=np.int8)
    s16 = (np.abs(rng.standard_normal((N, K // 32))) * 0.01).astype(np.float16)
    x = rng.standard_normal(K).astype(np.float32)
    x[:32] = 0      # an all-zero activation block
    qx_o, dx_o = oracle.q80_quant_act(x)
    isum_o, y_o = oracle.q80_gemv(codes, s16.view(np.uint16), qx_o, dx_o)
    qx = torch.empty(K, dtype=torch.int8, device="cuda")
    dx = torch.empty(K // 32, dtype=torch.int16, device="cuda")
    pb.q80_quantize(_dev(torch, x), qx, dx)
    w = pb.Q8Tensor(_dev(torch, codes), _dev(torch, s16))
    y = torch.empty(N, dtype=torch.float32, device="cuda")
    isum = torch.empty((N, K // 32), dtype=torch.int32, device="cuda")
    w.gemv_int(qx, dx, y, isum)
    torch.cuda.synchronize()
    assert np.array_equal(qx.cpu().numpy(), qx_o)
    assert np.array_equal(dx.cpu().numpy().view(np.uint16), dx_o)
    assert np.array_equal(isum.cpu().numpy(), isum_o)
    assert np.array_equal(_bits(y.cpu().numpy()), _bits(y_o))


@pytest.mark.parametrize("N,K,T", [(300, 2048, 16), (300, 2048, 32), (300, 2048, 64), (2048, 8192, 32),
                                   (16384, 2048, 32), (640, 2048, 48), (128, 256, 64), (200, 512, 128)])
def test_q80_gemm_tensor_cores(cuda, oracle, pb, N, K, T):
    """tcgen05 kind::i8 integer GEMM (prefill chunk / batched decode): every
    position's block dots exact and its fold bit for bit = the oracle's
    single-position integer path"""
    torch = cuda
    rng = np.random.default_rng(N + K + T)
    codes = rng.integers(-127, 128, (N, K), dtype=np.int8)
    codes[0, :32] = -128          # the int8 extreme
    s16 = (np.abs(rng.standard_normal((N, K // 32))) * 0.01).astype(np.float16)
    x = rng.standard_normal((T, K)).astype(np.float32)
    x[1, 32:64] = 0               # an all-zero activation block
    qx = torch.empty((T, K), dtype=torch.int8, device="cuda")
    dx = torch.empty((T, K // 32), dtype=torch.int16, device="cuda")
    pb.q80_quantize(_dev(torch, x), qx, dx)
    w = pb.Q8Tensor(_dev(torch, codes), _dev(torch, s16), tensor_cores=True)
    y = torch.full((T, N), float("nan"), dtype=torch.float32, device="cuda")
    isum = torch.empty((T, N, K // 32), dtype=torch.int32, device="cuda")
    w.gemm_int(qx, dx, y, isum)
    pb.Q8Tensor.gemm_int_status()
    yh, ih = y.cpu().numpy(), isum.cpu().numpy()
    qxh, dxh = qx.cpu().numpy(), dx.cpu().numpy().view(np.uint16)
    for t in range(T):
        qo, do = oracle.q80_quant_act(x[t])
        assert np.array_equal(qxh[t], qo) and np.array_equal(dxh[t], do)
        io, yo = oracle.q80_gemv(codes, s16.view(np.uint16), qo, do)
        assert np.array_equal(ih[t], io), "position %d block dots" % t
        assert np.array_equal(_bits(yh[t]), _bits(yo)), "position %d outputs" % t


def test_q80_gemm_tensor_cores_f32_scales(cuda, oracle, pb):
    """fp32 block scales (.lfm3q8 dtype 1): the fold in numpy float32, block order"""
    torch = cuda
    N, K, T = 256, 512, 32
    rng = np.random.default_rng(5)
    codes = rng.integers(-127, 128, (N, K), dtype=np.int8)
    s32 = (np.abs(rng.standard_normal((N, K // 32))) * 0.01).astype(np.float32)
    x = rng.standard_normal((T, K)).astype(np.float32)
    qx = torch.empty((T, K), dtype=torch.int8, device="cuda")
    dx = torch.empty((T, K // 32), dtype=torch.int16, device="cuda")
    pb.q80_quantize(_dev(torch, x), qx, dx)
    w = pb.Q8Tensor(_dev(torch, codes), _dev(torch, s32), tensor_cores=True)
    y = torch.empty((T, N), dtype=torch.float32, device="cuda")
    w.gemm_int(qx, dx, y)
    pb.Q8Tensor.gemm_int_status()
    q = qx.cpu().numpy().astype(np.int32)
    d = dx.cpu().numpy().view(np.float16).astype(np.float32)
    isum = np.einsum("nbj,tbj->tnb", codes.reshape(N, K // 32, 32).astype(np.int32), q.reshape(T, K // 32, 32))
    acc = np.zeros((T, N), np.float32)
    for b in range(K // 32):
        acc = acc + (s32[None, :, b] * d[:, None, b]) * isum[:, :, b].astype(np.float32)
    assert np.array_equal(_bits(y.cpu().numpy()), _bits(acc))


def test_q80_golden_quantizer(cuda, oracle, pb):
    torch = cuda
    g = np.load(os.path.join(GOLDEN, "q80_quant.npz"))
    qx = torch.empty(2048, dtype=torch.int8, device="cuda")
    dx = torch.empty(64, dtype=torch.int16, device="cuda")
    pb.q80_quantize(_dev(torch, g["x"]), qx, dx)
    torch.cuda.synchronize()
    assert np.array_equal(qx.cpu().numpy(), g["q"])
    assert np.array_equal(oracle.h2f_vec(dx.cpu().numpy().view(np.uint16)), g["d"])


def test_q1_golden_parity(cuda, oracle, pb):
    """pq1_parity.c's gate inputs: device output bit for bit = the reference's
    pq1_gemv_cpu output"""
    torch = cuda
    g = np.load(os.path.join(GOLDEN, "q1_parity.npz"))
    rows, K = int(g["rows"]), int(g["K"])
    w = pb.Q1Tensor(_dev(torch, g["q1"]), rows, K)
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    w.gemv(_dev(torch, g["xq"]), y)
    torch.cuda.synchronize()
    assert np.array_equal(_bits(y.cpu().numpy()), _bits(g["y"]))


@pytest.mark.parametrize("rows,K", [(6144, 4096), (4096, 12288), (512, 12288), (300, 4096)])
def test_q1_gemv_cfg3_shapes(cuda, oracle, pb, rows, K):
    torch = cuda
    rng = np.random.default_rng(rows + K)
    nb = K // 128
    blocks = rng.integers(0, 256, (rows, nb, 18), dtype=np.uint8)
    sc = (np.abs(rng.standard_normal((rows, nb))) * 0.02).astype(np.float16)
    blocks[:, :, 0:2] = sc.view(np.uint8).reshape(rows, nb, 2)
    blocks = blocks.reshape(-1)
    x = rng.standard_normal(K).astype(np.float32)
    xq = oracle.q8k_quant(x)
    wb, ws = oracle.q1_repack(blocks, rows, K)
    isum_o, y_o = oracle.q1_gemv(wb, ws, xq, K)
    w = pb.Q1Tensor(_dev(torch, blocks), rows, K)
    xq_d = torch.empty(len(xq), dtype=torch.uint8, device="cuda")
    pb.q8k_quantize(_dev(torch, x), xq_d)
    y = torch.empty(rows, dtype=torch.float32, device="cuda")
    isum = torch.empty((rows, nb), dtype=torch.int32, device="cuda")
    w.gemv(xq_d, y, isum)
    torch.cuda.synchronize()
    assert np.array_equal(xq_d.cpu().numpy(), xq)
    assert np.array_equal(isum.cpu().numpy(), isum_o)
    assert np.array_equal(_bits(y.cpu().numpy()), _bits(y_o))


def test_q8k_golden_rms_chain(cuda, oracle, pb):
    torch = cuda
    g = np.load(os.path.join(GOLDEN, "q8k_rms.npz"))
    n = g["x"].shape[1]
    mask = np.ones((n // 256) * 292, bool)
    for b in range(n // 256):
        mask[b * 292 + 260:b * 292 + 292] = False
    for x, want in zip(g["x"], g["xq"]):
        _, y, _ = oracle.q1_rms_q8k(x, g["w"])      # the norm is host-side in the Q1 engine
        xq = torch.empty(len(want), dtype=torch.uint8, device="cuda")
        pb.q8k_quantize(_dev(torch, y), xq)
        torch.cuda.synchronize()
        assert np.array_equal(xq.cpu().numpy()[mask], want[mask])


def test_q1_compat_host_abi(cuda, oracle, pb):
    g = np.load(os.path.join(GOLDEN, "q1_parity.npz"))
    rows, K = int(g["rows"]), int(g["K"])
    y = np.zeros(rows, np.float32)
    pb.compat_gemv(rows, K, g["q1"], g["xq"], y)
    assert np.array_equal(_bits(y), _bits(g["y"]))
    pb.compat_gemv(rows, K, g["q1"], g["xq"], y)   # cached second call
    assert np.array_equal(_bits(y), _bits(g["y"]))


def test_grid_wait_gives_up_and_reports(cuda, pb):
    """The decode kernel's grid wait is bounded: on a counter that nothing
    advances it gives up after its poll limit and reports it (the kernel then
    records an error code and leaves); the context stays usable. A counter
    that has reached the target passes at once."""
    torch = cuda
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert pb.device_grid_wait(counter, 1, 1 << 12) == 1
    counter.fill_(5)
    assert pb.device_grid_wait(counter, 5, 1 << 12) == 2
    x = torch.ones(4, device="cuda")
    assert float((x * 2).sum().item()) == 8.0


def test_device_expf_matches_oracle_and_cuda(cuda, oracle, pb):
    torch = cuda
    xs = np.concatenate([np.linspace(-104, 89, 400001), np.linspace(-2, 2, 10001)]).astype(np.float32)
    x = _dev(torch, xs)
    y = torch.empty_like(x)
    pb.device_expf(x, y)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    want = np.array([oracle.lib().pbo_expf(float(v)) for v in xs[::7]], np.float32)
    assert np.array_equal(_bits(got[::7]), _bits(want))
    ref = torch.exp(x).cpu().numpy().astype(np.float64)          # CUDA's own expf
    ok = (ref > 1.2e-38) & (ref < 3.4e38)
    ulp = np.abs(got[ok] - ref[ok]) / np.spacing(ref[ok].astype(np.float32))
    assert ulp.max() <= 3
