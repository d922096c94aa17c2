"""Generates tests/golden/export_tiny/: a tiny seeded LFM3-style checkpoint
(config.json with an "lfm" object, model.safetensors in bf16) and the digests
of the .lfm3q8 blobs the REFERENCE exporter (pulsar_asm/lfm3/tools/
export_lfm3_q8.py, run unmodified) writes from it, with and without
--emb-bf16. TEST INFRASTRUCTURE: tests/test_export.py checks that
pulsar_b200.export writes the same bytes. Needs /root/reference, torch and
safetensors (this container); the committed files are all the test reads.

    python tests/golden/make_golden_export.py
"""
import hashlib
import json
import os
import struct
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "export_tiny")
REF = "/root/reference/pulsar_asm/lfm3/tools/export_lfm3_q8.py"


def bf16_bits(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def write_safetensors(path, tensors):
    """tensors: list of (name, uint16 bf16 bits array)"""
    hdr, off, blobs = {}, 0, []
    for name, a in tensors:
        b = np.ascontiguousarray(a).tobytes()
        hdr[name] = {"dtype": "BF16", "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    hj = json.dumps(hdr, separators=(",", ":")).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)


def main():
    rng = np.random.default_rng(20261203)
    H, F, NH, NKV, HD, V, W = 64, 96, 2, 1, 32, 80, 3
    cfg = {"hidden_size": H, "intermediate_size": F, "num_hidden_layers": 2, "num_attention_heads": NH,
           "num_key_value_heads": NKV, "head_dim": HD, "vocab_size": V, "conv_L_cache": W,
           "layer_types": ["conv", "full_attention"], "rope_theta": 1e6, "norm_eps": 1e-5}

    def mat(n, k, sc=0.05):
        m = (rng.standard_normal((n, k)) * sc).astype(np.float32)
        return m

    t = []
    p0, p1 = "lfm.model.layers.0.", "lfm.model.layers.1."
    in_proj = mat(3 * H, H)
    in_proj[5, 32:64] = 0.0                      # an all-zero group: codes 0, scale 0
    in_proj[6, :32] = np.arange(32) - 15.5       # a group with many exact halves
    t += [(p0 + "conv.in_proj.weight", in_proj), (p0 + "conv.out_proj.weight", mat(H, H)),
          (p0 + "conv.conv.weight", mat(H, 1, 0.5).repeat(W, 1).reshape(H, 1, W))]
    t += [(p1 + "self_attn.q_proj.weight", mat(NH * HD, H)), (p1 + "self_attn.k_proj.weight", mat(NKV * HD, H)),
          (p1 + "self_attn.v_proj.weight", mat(NKV * HD, H)), (p1 + "self_attn.o_proj.weight", mat(H, NH * HD)),
          (p1 + "self_attn.gate_proj.weight", mat(NH, H)),
          (p1 + "self_attn.q_norm.weight", 1 + mat(1, HD)[0]), (p1 + "self_attn.k_norm.weight", 1 + mat(1, HD)[0])]
    for p in (p0, p1):
        t += [(p + "feed_forward.w1.weight", mat(F, H)), (p + "feed_forward.w3.weight", mat(F, H)),
              (p + "feed_forward.w2.weight", mat(H, F))]
        for nm in ("operator_norm", "post_operator_norm", "ffn_norm", "post_ffn_norm"):
            t.append((p + nm + ".weight", 1 + mat(1, H)[0]))
    t += [("lfm.model.embed_tokens.weight", mat(V, H)), ("lfm.model.embedding_norm.weight", 1 + mat(1, H)[0])]
    os.makedirs(OUT, exist_ok=True)
    write_safetensors(os.path.join(OUT, "model.safetensors"), [(n, bf16_bits(a)) for n, a in t])
    json.dump({"lfm": cfg}, open(os.path.join(OUT, "config.json"), "w"))
    digests = {}
    with tempfile.TemporaryDirectory() as td:
        for arm, extra in (("q8", []), ("emb_bf16", ["--emb-bf16"])):
            blob = os.path.join(td, arm + ".lfm3q8")
            subprocess.check_call([sys.executable, REF, "--model", OUT, "--out", blob] + extra)
            b = open(blob, "rb").read()
            digests[arm] = {"bytes": len(b), "sha256": hashlib.sha256(b).hexdigest()}
    json.dump(digests, open(os.path.join(OUT, "reference_blobs.json"), "w"), indent=1)
    print(digests)


if __name__ == "__main__":
    main()
