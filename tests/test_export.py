"""The .lfm3q8 exporter and the GGUF reader, on the CPU.

* pulsar_b200.export writes, from the committed tiny checkpoint, the very bytes
  the reference exporter (export_lfm3_q8.py, run unmodified by
  tests/golden/make_golden_export.py) wrote: both the Q8-embedding and the
  bf16-embedding (certified) arms, digests in export_tiny/reference_blobs.json.
* the certified quantiser's edge cases: an all-zero group, exact halves
  (round half to even), the clamp.
* an exported LFM3-shaped checkpoint passes the loader's validate-only open.
* pulsar_b200.gguf round-trips the Bonsai weights and finds every tensor at
  the offset fwd8.c's own gguf_table finds (compiled by oracle/build_ref.sh).
"""
import ctypes as C
import hashlib
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
TINY = os.path.join(HERE, "golden", "export_tiny")
ROOT = os.path.dirname(HERE)


def test_export_bytes_match_reference_exporter(tmp_path):
    from pulsar_b200 import export
    ref = json.load(open(os.path.join(TINY, "reference_blobs.json")))
    for arm, bf in (("q8", False), ("emb_bf16", True)):
        out = str(tmp_path / (arm + ".lfm3q8"))
        export.export(TINY, out, emb_bf16=bf, log=None)
        b = open(out, "rb").read()
        assert len(b) == ref[arm]["bytes"]
        assert hashlib.sha256(b).hexdigest() == ref[arm]["sha256"], arm
        assert export.selfcheck(TINY, out) == []


def test_quantizer_edge_cases():
    from pulsar_b200 import export
    w = np.zeros((3, 64), np.float32)
    w[0, :32] = np.arange(32) - 15.5          # max 15.5 -> s = 15.5/127
    w[1, 32:] = 0.0                           # all-zero group
    w[1, :32] = np.linspace(-1, 1, 32)
    w[2, :32] = 1e-30                         # tiny values: scale tiny, codes 127
    c, s = export.quantize_q8(w)
    assert s.dtype == np.float32 and c.dtype == np.int8
    assert s[1, 1] == 0 and np.all(c[1, 32:] == 0)
    sc = np.float32(15.5) / np.float32(127.0)
    want = np.clip(np.round((w[0, :32] / sc).astype(np.float32)), -128, 127).astype(np.int8)
    assert np.array_equal(c[0, :32], want)
    assert np.all(np.abs(c) <= 127)
    assert np.all(c[2, :32] == 127)


def _lfm3_checkpoint(d, H=256, F=512, NH=4, NKV=2, HD=64, V=512, W=3, seed=5):
    """a seeded LFM3-style checkpoint (bf16) the loader accepts: layer 0 conv,
    layer 1 full attention"""
    from pulsar_b200 import export
    rng = np.random.default_rng(seed)
    cfg = {"hidden_size": H, "intermediate_size": F, "num_hidden_layers": 2, "num_attention_heads": NH,
           "num_key_value_heads": NKV, "head_dim": HD, "vocab_size": V, "conv_L_cache": W,
           "layer_types": ["conv", "full_attention"], "rope_theta": 1e6, "partial_rotary_factor": 1.0,
           "norm_eps": 1e-5}

    def m(n, k, sc=0.05):
        return (rng.standard_normal((n, k)) * sc).astype(np.float32)

    def nv(n):
        return (1 + 0.05 * rng.standard_normal(n)).astype(np.float32)
    t = []
    p0, p1 = "lfm.model.layers.0.", "lfm.model.layers.1."
    t += [(p0 + "conv.in_proj.weight", m(3 * H, H)), (p0 + "conv.out_proj.weight", m(H, H)),
          (p0 + "conv.conv.weight", m(H, W, 0.5).reshape(H, 1, W))]
    t += [(p1 + "self_attn.q_proj.weight", m(NH * HD, H)), (p1 + "self_attn.k_proj.weight", m(NKV * HD, H)),
          (p1 + "self_attn.v_proj.weight", m(NKV * HD, H)), (p1 + "self_attn.o_proj.weight", m(H, NH * HD)),
          (p1 + "self_attn.gate_proj.weight", m(NH, H)), (p1 + "self_attn.q_norm.weight", nv(HD)),
          (p1 + "self_attn.k_norm.weight", nv(HD))]
    for p in (p0, p1):
        t += [(p + "feed_forward.w1.weight", m(F, H)), (p + "feed_forward.w3.weight", m(F, H)),
              (p + "feed_forward.w2.weight", m(H, F))]
        for nm in ("operator_norm", "post_operator_norm", "ffn_norm", "post_ffn_norm"):
            t.append((p + nm + ".weight", nv(H)))
    t += [("lfm.model.embed_tokens.weight", m(V, H)), ("lfm.model.embedding_norm.weight", nv(H))]
    os.makedirs(d, exist_ok=True)
    export.write_safetensors(os.path.join(d, "model.safetensors"), t)
    json.dump({"lfm": cfg}, open(os.path.join(d, "config.json"), "w"))
    return cfg


def test_exported_checkpoint_loads(pb, tmp_path):
    from pulsar_b200 import export
    d = str(tmp_path / "ckpt")
    _lfm3_checkpoint(d)
    for bf in (False, True):
        out = str(tmp_path / ("m%d.lfm3q8" % bf))
        export.export(d, out, emb_bf16=bf, log=None)
        assert pb.lib().pb_open(out.encode(), -1, C.byref(C.c_void_p())) == 0


def test_gguf_round_trip_and_fwd8_offsets(tmp_path):
    from pulsar_b200 import gguf, synth
    c = dict(synth.BONSAI_TINY, n_layers=2)
    for tied in (True, False):
        w = synth.make_bonsai_weights(c, seed=12, tied=tied)
        path = str(tmp_path / ("b%d.gguf" % tied))
        gguf.write_bonsai(path, c, w)
        r = gguf.bonsai_weights(path, c)
        assert np.array_equal(r["embed"], w["embed"]) and np.array_equal(r["out_norm"], w["out_norm"])
        assert (r["head"] is None) == tied
        if not tied:
            assert np.array_equal(r["head"], w["head"])
        for a, b in zip(r["layers"], w["layers"]):
            for k in b:
                assert np.array_equal(a[k], b[k]), k
        lib = os.path.join(ROOT, "oracle", "_ref", "libpb_gguf.so")
        if not os.path.exists(lib):
            pytest.skip("fwd8.c's table reader not built (no reference tree)")
        L = C.CDLL(lib)
        L.pbref_gguf_offset.argtypes = [C.c_char_p, C.c_char_p, C.POINTER(C.c_ulonglong)]
        g = gguf.GGUF(path)
        for name, (dims, tt, off) in g.tensors.items():
            o = C.c_ulonglong()
            assert L.pbref_gguf_offset(path.encode(), name.encode(), C.byref(o)) == 0
            assert o.value == off, name
