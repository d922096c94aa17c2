"""Seeded synthetic models and inputs with the shapes and value distributions of
the benchmark configurations (no checkpoint or dataset is available offline):
Q8_0 codes uniform integers in [-127, 127]; fp16 scales |N(0,1)| * 0.01; norm
weights 1 + 0.05 N(0,1); conv taps 0.5 N(0,1); Q1_0 signs uniform, fp16 scales
|N(0,1)| * 0.02.
"""
import numpy as np

from . import blob

LFM3_CFG1 = dict(hidden=2048, inter=8192, n_layers=24, n_heads=32, n_kv=8, head_dim=64,
                 vocab=65536, conv_w=3, rope_theta=1e6, rope_partial=1.0, norm_eps=1e-5,
                 sliding_window=0, attn_layers=(2, 6, 10, 14, 18, 22))

# small model for parity tests: same kernels (K multiple of 2048), quick oracle
LFM3_TINY = dict(hidden=2048, inter=2048, n_layers=4, n_heads=32, n_kv=8, head_dim=64,
                 vocab=4096, conv_w=3, rope_theta=1e6, rope_partial=1.0, norm_eps=1e-5,
                 sliding_window=0, attn_layers=(1, 3))


def layer_types(c):
    """conv, full_attention, or sliding_attention (layers listed in slide_layers)"""
    slide = set(c.get("slide_layers", ()))
    return [("sliding_attention" if i in slide else "full_attention") if i in c["attn_layers"] else "conv"
            for i in range(c["n_layers"])]


def hf_cfg(c):
    """the blob header's cfg object (HF-style keys the loader reads)."""
    d = dict(hidden_size=c["hidden"], intermediate_size=c["inter"],
             num_hidden_layers=c["n_layers"], num_attention_heads=c["n_heads"],
             num_key_value_heads=c["n_kv"], head_dim=c["head_dim"], vocab_size=c["vocab"],
             conv_L_cache=c["conv_w"], rope_theta=c["rope_theta"],
             partial_rotary_factor=c["rope_partial"], norm_eps=c["norm_eps"],
             layer_types=layer_types(c))
    if c.get("slide_layers"):
        d.update(sliding_window=c.get("slide_window", 256), sliding_rope_theta=c.get("slide_theta", 1e4),
                 sliding_partial_rotary_factor=c.get("slide_partial", 1.0))
    return d


def oracle_cfg(c, max_ctx):
    d = dict(c)
    d["max_ctx"] = max_ctx
    d["layer_types"] = layer_types(c)
    return d


def q8(rng, N, K, scale=0.01):
    codes = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    sc = (np.abs(rng.standard_normal((N, K // 32), dtype=np.float32)) * np.float32(scale)).astype(np.float16)
    return codes, sc


def make_weights(c, seed=1234):
    rng = np.random.default_rng(seed)
    H, F, NH, NKV, HD, W = c["hidden"], c["inter"], c["n_heads"], c["n_kv"], c["head_dim"], c["conv_w"]

    def norm(n):
        return (1.0 + 0.05 * rng.standard_normal(n)).astype(np.float32)

    layers = []
    for L in range(c["n_layers"]):
        d = {}
        if L in c["attn_layers"]:
            d["q"] = q8(rng, NH * HD, H)
            d["k"] = q8(rng, NKV * HD, H)
            d["v"] = q8(rng, NKV * HD, H)
            d["gate"] = q8(rng, NH, H)
            d["o"] = q8(rng, H, NH * HD)
            d["q_norm"] = norm(HD)
            d["k_norm"] = norm(HD)
        else:
            d["in_proj"] = q8(rng, 3 * H, H)
            d["out_proj"] = q8(rng, H, H)
            d["taps"] = (0.5 * rng.standard_normal((H, W))).astype(np.float32)
        d["w1"] = q8(rng, F, H)
        d["w3"] = q8(rng, F, H)
        d["w2"] = q8(rng, H, F)
        for k in ("op_norm", "post_op_norm", "ffn_norm", "post_ffn_norm"):
            d[k] = norm(H)
        layers.append(d)
    if c.get("emb_bf16"):
        # the certified arm's bf16 table (blob dtype 3): N(0, 1) values as bf16 bits
        e = rng.standard_normal((c["vocab"], H), dtype=np.float32)
        u = e.view(np.uint32)
        e16 = ((u + np.uint32(0x7FFF) + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        return dict(layers=layers, embed_bf16=e16, final_norm=norm(H))
    return dict(layers=layers, embed=q8(rng, c["vocab"], H), final_norm=norm(H))


NAMES_Q8 = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj",
            "gate": "self_attn.gate_proj", "o": "self_attn.o_proj", "in_proj": "conv.in_proj",
            "out_proj": "conv.out_proj", "w1": "feed_forward.w1", "w3": "feed_forward.w3",
            "w2": "feed_forward.w2"}
NAMES_F = {"q_norm": "self_attn.q_norm", "k_norm": "self_attn.k_norm", "op_norm": "operator_norm",
           "post_op_norm": "post_operator_norm", "ffn_norm": "ffn_norm",
           "post_ffn_norm": "post_ffn_norm"}


def write_model(path, c, w, fp32_scales=False):
    ts = []
    for L, d in enumerate(w["layers"]):
        p = "lfm.model.layers.%d." % L
        for k, nm in NAMES_Q8.items():
            if k in d:
                codes, sc = d[k]
                ts.append((p + nm + ".weight", "q8", (codes, sc.astype(np.float32) if fp32_scales else sc)))
        for k, nm in NAMES_F.items():
            if k in d:
                ts.append((p + nm + ".weight", "f32", d[k]))
        if "taps" in d:
            ts.append((p + "conv.conv.weight", "f32", d["taps"].reshape(c["hidden"], 1, c["conv_w"])))
    if "embed_bf16" in w:
        ts.append(("lfm.model.embed_tokens.weight", "bf16", w["embed_bf16"]))
    else:
        codes, sc = w["embed"]
        ts.append(("lfm.model.embed_tokens.weight", "q8", (codes, sc.astype(np.float32) if fp32_scales else sc)))
    ts.append(("lfm.model.embedding_norm.weight", "f32", w["final_norm"]))
    return blob.write_blob(path, hf_cfg(c), ts)


def weight_bytes_per_token(c, fp32_scales=False):
    """algorithmic bytes one decode token streams: every Q8 tensor (codes +
    scales), every fp32 vector, one embedding row."""
    H, F, NH, NKV, HD, V, W = (c["hidden"], c["inter"], c["n_heads"], c["n_kv"], c["head_dim"],
                               c["vocab"], c["conv_w"])
    sb = 4 if fp32_scales else 2

    def q(N, K):
        return N * K + N * (K // 32) * sb
    tot = 0
    for L in range(c["n_layers"]):
        if L in c["attn_layers"]:
            tot += q(NH * HD, H) + 2 * q(NKV * HD, H) + q(NH, H) + q(H, NH * HD) + 2 * HD * 4
        else:
            tot += q(3 * H, H) + q(H, H) + H * W * 4
        tot += 2 * q(F, H) + q(H, F) + 4 * H * 4
    if c.get("emb_bf16"):
        tot += V * H * 2 + H * 4 + H * 2          # bf16 head, final norm, one embedding row
    else:
        tot += q(V, H) + H * 4 + H + (H // 32) * sb
    return tot


def kv_bytes_per_token(c, ctx):
    """fp16 K and V read by the attention layers at context ctx."""
    n_attn = len(c["attn_layers"])
    return n_attn * 2 * ctx * c["n_kv"] * c["head_dim"] * 2


# ------------------------------------------------------------------ Bonsai ----
# Bonsai-8B shape (fwd8.c:35-57): YaRN factor 4 over an original 16384-token
# context, base 1e6, attention scale 1/sqrt(128) as fwd8.c:566 writes it
BONSAI_CFG3 = dict(hidden=4096, inter=12288, n_layers=36, n_heads=32, n_kv=8, vocab=151936,
                   rope_factor=4.0, rope_orig_ctx=16384, rope_base=1e6, attn_scale=0.0883883476)
# small model for parity tests: same kernels, quick oracle
BONSAI_TINY = dict(hidden=1024, inter=2048, n_layers=2, n_heads=8, n_kv=2, vocab=2048,
                   rope_factor=4.0, rope_orig_ctx=16384, rope_base=1e6, attn_scale=0.0883883476)


def qlow_payload(rng, N, K, bits):
    """a seeded Q4 / Q5 tensor [N, K] in the exporter's tiled payload
    (lfm3_qlow.cuh:5-13): (codes uint8 [N*K/32*(16|20)], scales uint16
    [N*K/32*2] = fp16 (d' = 128 d, mn) per row and group). Every code pattern
    is a valid tensor, so the codes and planes are uniform random bytes; d' is
    positive and mn about -d' q_mid / 128, so w = d q + mn is centred."""
    G = K // 32
    codes = rng.integers(0, 256, N * K // 32 * (20 if bits == 5 else 16), dtype=np.uint8)
    dp = rng.uniform(0.02, 0.25, (N // 32, G, 32)).astype(np.float32)
    mn = (-dp * (2 ** (bits - 1)) / 128 + rng.normal(0, 0.002, dp.shape)).astype(np.float32)
    sc = np.stack([dp.astype(np.float16), mn.astype(np.float16)], axis=-1).view(np.uint16).reshape(-1)
    return codes, np.ascontiguousarray(sc)


def q1_blocks(rng, rows, K, scale=0.02):
    """Q1_0 18-byte blocks [rows][K/128]: fp16 scale |N(0,1)|*scale, then 16
    bytes of uniform sign bits"""
    nb = K // 128
    b = rng.integers(0, 256, size=(rows, nb, 18), dtype=np.uint8)
    sc = (np.abs(rng.standard_normal((rows, nb), dtype=np.float32)) * np.float32(scale)).astype(np.float16)
    b[:, :, 0:2] = sc.view(np.uint8).reshape(rows, nb, 2)
    return b


def make_bonsai_weights(c, seed=4321, tied=True):
    rng = np.random.default_rng(seed)
    H, F, NH, NKV = c["hidden"], c["inter"], c["n_heads"], c["n_kv"]

    def norm(n):
        return (1.0 + 0.05 * rng.standard_normal(n)).astype(np.float32)
    layers = []
    for _ in range(c["n_layers"]):
        layers.append(dict(q=q1_blocks(rng, NH * 128, H), k=q1_blocks(rng, NKV * 128, H),
                           v=q1_blocks(rng, NKV * 128, H), o=q1_blocks(rng, H, NH * 128),
                           gate=q1_blocks(rng, F, H), up=q1_blocks(rng, F, H), down=q1_blocks(rng, H, F),
                           attn_norm=norm(H), ffn_norm=norm(H), q_norm=norm(128), k_norm=norm(128)))
    emb = q1_blocks(rng, c["vocab"], H)
    return dict(layers=layers, embed=emb, head=None if tied else q1_blocks(rng, c["vocab"], H),
                out_norm=norm(H))


def bonsai_bytes_per_token(c, ctx, kv_bits=0):
    """algorithmic bytes of one decode token at context ctx: every Q1_0 tensor
    (18 B per 128 weights), the norm vectors, the head once, and the K and V
    rows the attention reads (f16: 256 B per row; TurboQuant: 48 or 64 B of
    codes and a 4 B scale)"""
    H, F, NH, NKV, L = c["hidden"], c["inter"], c["n_heads"], c["n_kv"], c["n_layers"]

    def q(rows, K):
        return rows * (K // 128) * 18
    layer = q((NH + 2 * NKV) * 128, H) + q(H, NH * 128) + 2 * q(F, H) + q(H, F) + (2 * H + 256) * 4
    if kv_bits:
        bk, bv = (4, 3) if kv_bits == 43 else (kv_bits, kv_bits)
        kv = NKV * ctx * ((12 if bk == 3 else 16) * 4 + 4 + (12 if bv == 3 else 16) * 4 + 4)
    else:
        kv = 2 * NKV * ctx * 128 * 2
    return L * (layer + kv) + q(c["vocab"], H) + H * 4
