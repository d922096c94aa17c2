"""TurboQuant K/V cache on the device (pb_tq_store, pb_tq_attention) bit for
bit against the oracle's restatement of pq1_swar_sm53.cu's kernels, whose
orders are pinned to the reference's own kernels (tests/test_tq.py): every
code word and scale of 3-bit and 4-bit rows (outlier channels, an all-zero
row), and the attention outputs over 1 to 2048 positions (one and several
256-position chunks), for 3-bit, 4-bit and 4-bit-K/3-bit-V caches."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

BITS = [(3, 3, 3), (4, 4, 4), (43, 4, 3)]


def _rows(n, nkv, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((n, 2 * nkv, 128)).astype(np.float32)
    x[:, :nkv, [3, 64, 100]] *= 8.0
    x[min(5, n - 1)] = 0.0
    return x.astype(np.float16).view(np.uint16)


@pytest.mark.parametrize("bits,bk,bv", BITS)
def test_tq_store_and_attention(oracle, pb, cuda, bits, bk, bv):
    torch = cuda
    nkv, ctx = 8, 2048
    rows = _rows(ctx, nkv, 7 + bits)
    cwk, cwv = oracle.tq_cw(bk), oracle.tq_cw(bv)
    kc = torch.zeros((nkv, ctx, cwk), dtype=torch.int32, device="cuda")
    vc = torch.zeros((nkv, ctx, cwv), dtype=torch.int32, device="cuda")
    ks = torch.zeros((nkv, ctx), dtype=torch.float32, device="cuda")
    vs = torch.zeros((nkv, ctx), dtype=torch.float32, device="cuda")
    dr = torch.from_numpy(rows.view(np.int16)).cuda()
    for t in range(ctx):
        pb.tq_store(bits, dr[t], t, kc, ks, vc, vs, nkv, ctx)
    torch.cuda.synchronize()
    okc, oks = oracle.tq_rows(rows[:, :nkv].reshape(-1, 128), bk)
    ovc, ovs = oracle.tq_rows(rows[:, nkv:].reshape(-1, 128), bv)
    okc = okc.reshape(ctx, nkv, cwk).transpose(1, 0, 2)
    ovc = ovc.reshape(ctx, nkv, cwv).transpose(1, 0, 2)
    oks, ovs = oks.reshape(ctx, nkv).T, ovs.reshape(ctx, nkv).T
    assert np.array_equal(kc.cpu().numpy().view(np.uint32), okc), "K code words"
    assert np.array_equal(vc.cpu().numpy().view(np.uint32), ovc), "V code words"
    assert np.array_equal(ks.cpu().numpy().view(np.uint32), np.ascontiguousarray(oks).view(np.uint32)), "K scales"
    assert np.array_equal(vs.cpu().numpy().view(np.uint32), np.ascontiguousarray(ovs).view(np.uint32)), "V scales"
    assert float(ks[0, 5]) == 0.0 and float(vs[0, 5]) == 0.0   # the all-zero row
    rng = np.random.default_rng(bits)
    for T in (1, 37, 256, 257, 700, 2048):
        q = (rng.standard_normal((4 * nkv, 128)) * 1.5).astype(np.float32)
        at = torch.empty((4 * nkv, 128), dtype=torch.float32, device="cuda")
        pb.tq_attention(bits, torch.from_numpy(q).cuda(), kc, ks, vc, vs, nkv, ctx, T, at)
        torch.cuda.synchronize()
        got = at.cpu().numpy()
        for kh in range(nkv):
            want = oracle.tq_attn(q[4 * kh:4 * kh + 4], bk, bv, okc[kh], oks[kh], ovc[kh], ovs[kh], T)
            assert np.array_equal(got[4 * kh:4 * kh + 4].view(np.uint32), want.view(np.uint32)), (T, kh)
