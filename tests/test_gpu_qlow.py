"""pb_qlow_gemv / pb_qlow_gemm (the Q4 / Q5 backbone GEMV of lfm3_qlow.cuh on
the B200) bit for bit against the oracle, whose arithmetic is pinned to the
reference's own kernels: Q4 and Q5, K slices of 2 and 4, the cfg0 and cfg1
shapes, T positions (codes read once per tile of positions), a ragged last
tile of positions, and the overlap check."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _case(bits, N, K, seed, T=1):
    from pulsar_b200 import synth
    rng = np.random.default_rng(seed)
    codes, scales = synth.qlow_payload(rng, N, K, bits)
    xf = rng.standard_normal((T, K)).astype(np.float32)
    u = xf.view(np.uint32)
    x = ((u + np.uint32(0x7FFF) + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return codes, scales, x


@pytest.mark.parametrize("bits,N,K", [(4, 8192, 2048), (5, 8192, 2048), (4, 2048, 8192), (5, 2048, 8192),
                                      (4, 96, 4096), (5, 32, 768), (4, 64, 256), (5, 6144, 2048),
                                      (4, 65536, 2048), (5, 16384, 4096)])
def test_qlow_gemv(oracle, pb, cuda, bits, N, K):
    torch = cuda
    codes, scales, x = _case(bits, N, K, N + K + bits)
    w = pb.QlowTensor(codes, scales, bits, N, K)
    xd = torch.from_numpy(x[0].view(np.int16)).cuda()
    y = torch.empty(N, dtype=torch.int16, device="cuda")
    w.gemv(xd, y)
    torch.cuda.synchronize()
    want = oracle.qlow_gemv(codes, scales, bits, N, K, x[0])
    assert np.array_equal(y.cpu().numpy().view(np.uint16), want)


@pytest.mark.parametrize("bits,N,K,T", [(4, 2048, 2048, 32), (5, 2048, 8192, 5), (5, 512, 4096, 7), (4, 256, 16384, 3)])
def test_qlow_gemm_positions(oracle, pb, cuda, bits, N, K, T):
    torch = cuda
    codes, scales, x = _case(bits, N, K, 3 * N + T, T)
    w = pb.QlowTensor(torch.from_numpy(codes).cuda(), torch.from_numpy(scales.view(np.int16)).cuda(), bits, N, K)
    xd = torch.from_numpy(x.view(np.int16)).cuda()
    y = torch.empty((T, N), dtype=torch.int16, device="cuda")
    w.gemm(xd, y)
    torch.cuda.synchronize()
    want = oracle.qlow_gemv(codes, scales, bits, N, K, x)
    assert np.array_equal(y.cpu().numpy().view(np.uint16), want)


def test_qlow_rejects_overlap_and_bad_shapes(pb, cuda):
    torch = cuda
    codes, scales, x = _case(4, 256, 256, 1)
    w = pb.QlowTensor(codes, scales, 4, 256, 256)
    buf = torch.zeros(512, dtype=torch.int16, device="cuda")
    with pytest.raises(pb.PBError):
        w.gemv(buf[:256], buf[100:356])      # y overlaps x
    with pytest.raises(pb.PBError):
        w.gemv(buf[1:257], torch.empty(256, dtype=torch.int16, device="cuda"))   # x not 16-byte aligned
    with pytest.raises(pb.PBError):
        pb.QlowTensor(codes, scales, 4, 250, 256)   # N not a multiple of 32
    with pytest.raises(pb.PBError):
        pb.QlowTensor(codes, scales, 6, 256, 256)   # 4 or 5 bits only


def test_model_with_lowbit_records(oracle, pb, cuda, tmp_path):
    """a model holding Q4 / Q5 records loads in per-tensor mode: pb_model_gemv
    dispatches each named matrix by its record (the reference's gemv(),
    lfm3_nanode.cu:1916-1922), bit for bit; the fused decode declines it"""
    torch = cuda
    import importlib.util
    import os
    from conftest import ROOT
    from pulsar_b200 import blob, synth
    spec = importlib.util.spec_from_file_location("t_abi", os.path.join(ROOT, "tests", "test_abi.py"))
    t_abi = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(t_abi)
    tensors = t_abi._lowbit_blob(tmp_path)
    path = str(tmp_path / "low.lfm3q8")
    blob.write_blob(path, synth.hf_cfg(dict(synth.LFM3_TINY)), tensors)
    m = pb.Model(path)
    rng = np.random.default_rng(5)
    for name, kind, payload in tensors:
        if kind == "f32":
            continue
        if kind == "q8":
            N, K = payload[0].shape
        else:
            N, K = payload[0]
        xf = rng.standard_normal(K).astype(np.float32)
        u = xf.view(np.uint32)
        x = ((u + np.uint32(0x7FFF) + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        y = torch.empty(N, dtype=torch.int16, device="cuda")
        m.gemv(name, torch.from_numpy(x.view(np.int16)).cuda(), y)
        torch.cuda.synchronize()
        got = y.cpu().numpy().view(np.uint16)
        if kind == "q8":
            want = oracle.f2bf(oracle.q8f_gemv(payload[0], payload[1], x))
        else:
            want = oracle.qlow_gemv(payload[1], payload[2], 4 if kind == "q4" else 5, N, K, x)
        assert np.array_equal(got, want), name
    with pytest.raises(pb.PBError):
        m.new_state(64)
