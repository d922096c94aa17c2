"""Replays of the reference's LFM3 layer kernels (lfm3_nanode.cu) in numpy
float32, operation by operation, with the transcendental values (rsqrtf,
expf, cosf, sinf) supplied from outside. TEST INFRASTRUCTURE: the golden
generator (make_golden_lfm3.py) uses it to form the arguments whose device
transcendentals it records, and tests/test_oracle_lfm3.py replays the
reference's outputs from those values bit for bit, which pins every reduction
order and rounding step of the kernels.

numpy evaluates each float32 +, *, / separately with round-to-nearest-even
(no fused multiply-add, no wider intermediates), as the kernels' __fadd_rn /
__fmul_rn / __fdiv_rn do.
"""
import numpy as np

F = np.float32


def bf2f(h):
    return (np.asarray(h, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f2bf(x):
    """f2bf, lfm3_nanode.cu:116-121: round to nearest even, inf/nan truncated"""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32)
    special = ((u >> 23) & 0xFF) == 0xFF
    r = ((u + np.uint32(0x7FFF) + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(special, (u >> 16).astype(np.uint16), r)


def tree_down(v):
    """lane 0 of a shuffle-down tree over the last axis (32 or 8 lanes):
    v[l] += v[l + o] for o = n/2 .. 1"""
    v = np.array(v, np.float32, copy=True)
    o = v.shape[-1] // 2
    while o >= 1:
        v[..., :o] = v[..., :o] + v[..., o:2 * o]
        o //= 2
    return v[..., 0]


def pairwise(v):
    """((v0+v1)+(v2+v3))+... over the last axis (a power of two)"""
    v = np.array(v, np.float32, copy=True)
    while v.shape[-1] > 1:
        v = v[..., 0::2] + v[..., 1::2]
    return v[..., 0]


# ---- rmsnorm_body (lfm3_nanode.cu:383-440): 256 threads x 8, warp trees,
#      8 partials ascending; rs = rsqrtf(tot * (1/H) + eps)
def rms_arg(x, eps):
    H = x.shape[-1]
    xf = bf2f(x).reshape(256, H // 256)
    part = pairwise(xf * xf)
    w8 = tree_down(part.reshape(8, 32))
    tot = w8[0]
    for i in range(1, 8):
        tot = F(tot + w8[i])
    return F(F(tot * (F(1.0) / F(H))) + F(eps))


def rms_apply(x, w, rs):
    return f2bf(np.asarray(w, np.float32) * bf2f(f2bf(bf2f(x) * F(rs))))


# ---- k_headnorm (:460-479): 32 lanes x 4, "+ 0", shuffle-down tree
def headnorm_arg(x, eps):
    """x [heads][hd] -> the argument of rsqrtf per head"""
    nh, hd = x.shape
    xf = bf2f(x).reshape(nh, 32, hd // 32)
    s = pairwise(xf * xf) + F(0.0)
    s = tree_down(s)
    return (s * (F(1.0) / F(hd)) + F(eps)).astype(np.float32)


def headnorm_apply(x, w, rs):
    return f2bf(np.asarray(w, np.float32)[None, :] * bf2f(f2bf(bf2f(x) * rs[:, None])))


# ---- k_rope (:483-498): pairs (i, i + hd/2) for i < rot/2
def rope_angles(pos, invf, rot):
    half = rot // 2
    return (F(pos) * np.asarray(invf[:half], np.float32)).astype(np.float32)


def rope_apply(x, c, s, rot):
    x = np.array(x, np.uint16, copy=True)
    hd = x.shape[-1]
    half = rot // 2
    lo = bf2f(x[..., :half])
    hi = bf2f(x[..., hd // 2:hd // 2 + half])
    x[..., :half] = f2bf(lo * c + (-hi) * s)
    x[..., hd // 2:hd // 2 + half] = f2bf(hi * c + lo * s)
    return x


# ---- k_attn_head (:503-602) for one q head over a bf16 cache
def attn_scores(q, kc, kvh, npos, win, scaling):
    """q [HD] bf16; kc [ctx][nkv][HD] bf16 -> scores [np] (lo .. npos-1)"""
    hd = q.shape[0]
    E = hd // 32
    lo = npos - win if (win > 0 and npos > win) else 0
    qf = bf2f(q).reshape(32, E)
    kf = bf2f(kc[lo:npos, kvh]).reshape(npos - lo, 32, E)
    s = np.zeros((npos - lo, 32), np.float32)
    for j in range(E):
        s = s + qf[None, :, j] * kf[:, :, j]
    return tree_down(s) * F(scaling)


def attn_exp_args(sc):
    m = F(-1e30)
    if sc.size:
        m = max(m, F(sc.max()))
    return (sc + (-m)).astype(np.float32)


def attn_apply(e, vc, kvh, npos, win):
    """e: the exponentials [np]; vc [ctx][nkv][HD] bf16 -> out [HD] bf16"""
    hd = vc.shape[-1]
    lo = npos - win if (win > 0 and npos > win) else 0
    np_ = npos - lo
    th = np.zeros(256, np.float32)
    for i in range(np_):
        th[i & 255] = th[i & 255] + e[i]
    tot = tree_down(tree_down(th.reshape(8, 32)))
    inv = F(1.0) / F(tot)
    vf = bf2f(vc[lo:npos, kvh])                     # [np][HD]
    seg = np.zeros((8, hd), np.float32)
    for p in range(np_):
        seg[p & 7] = seg[p & 7] + (e[p] * inv) * vf[p]
    return f2bf(pairwise(seg.T))


# ---- k_silu_mul_bf (:821-829) and k_sigmoid_gate (:852-859)
def silu_apply(a, b, ex):
    """ex = expf(-a) as the device computes it"""
    af = bf2f(a)
    sg = F(1.0) / (F(1.0) + ex)
    return f2bf((af * sg) * bf2f(b))


def gate_apply(g, attn, ex):
    """ex = expf(-g) per head; attn [nh][hd]"""
    sg = (F(1.0) / (F(1.0) + ex)).astype(np.float32)
    return f2bf(bf2f(attn) * sg[:, None])
