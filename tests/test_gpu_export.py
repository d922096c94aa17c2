"""A checkpoint exported by pulsar_b200.export (the certified quantiser, fp32
scales) decodes on the B200 bit for bit like the oracle fed with the blob's
own payloads: the Q8 embedding and the bf16 embedding arms."""
import json
import os

import numpy as np
import pytest

from test_export import _lfm3_checkpoint

pytestmark = pytest.mark.gpu

Q8 = {"self_attn.q_proj": "q", "self_attn.k_proj": "k", "self_attn.v_proj": "v", "self_attn.gate_proj": "gate",
      "self_attn.o_proj": "o", "conv.in_proj": "in_proj", "conv.out_proj": "out_proj", "feed_forward.w1": "w1",
      "feed_forward.w3": "w3", "feed_forward.w2": "w2"}
F32 = {"self_attn.q_norm": "q_norm", "self_attn.k_norm": "k_norm", "operator_norm": "op_norm",
       "post_operator_norm": "post_op_norm", "ffn_norm": "ffn_norm", "post_ffn_norm": "post_ffn_norm"}


def _weights_from_blob(path, n_layers):
    from pulsar_b200 import blob
    hdr, base = blob.read_header(path)
    raw = open(path, "rb").read()
    layers = [dict() for _ in range(n_layers)]
    w = {"layers": layers}
    for e in hdr["table"]:
        p = raw[base + e["off"]:base + e["off"] + e["ncodes"] + e["nscales"]]
        nm = e["name"]
        if e["dtype"] == 1:
            N, K = e["ne"]
            val = (np.frombuffer(p[:e["ncodes"]], np.int8).reshape(N, K).copy(),
                   np.frombuffer(p[e["ncodes"]:], np.float32).reshape(N, K // 32).copy())
        elif e["dtype"] == 3:
            val = np.frombuffer(p, np.uint16).reshape(e["ne"]).copy()
        else:
            val = np.frombuffer(p, np.float32).copy()
        if nm == "lfm.model.embed_tokens.weight":
            w["embed_bf16" if e["dtype"] == 3 else "embed"] = val
        elif nm == "lfm.model.embedding_norm.weight":
            w["final_norm"] = val
        else:
            L = int(nm.split(".")[3])
            key = nm.split(".", 4)[4].rsplit(".weight", 1)[0]
            if key in Q8:
                layers[L][Q8[key]] = val
            elif key in F32:
                layers[L][F32[key]] = val
            elif key == "conv.conv":
                layers[L]["taps"] = val.reshape(-1, e["ne"][2])
    return w


@pytest.mark.parametrize("emb_bf16", [False, True])
def test_exported_model_decodes_bitexact(tmp_path, oracle, pb, cuda, monkeypatch, emb_bf16):
    torch = cuda
    from pulsar_b200 import export
    d = str(tmp_path / "ckpt")
    hf = _lfm3_checkpoint(d)
    out = str(tmp_path / "m.lfm3q8")
    export.export(d, out, emb_bf16=emb_bf16, log=None)
    w = _weights_from_blob(out, 2)
    c = dict(hidden=hf["hidden_size"], inter=hf["intermediate_size"], n_layers=2, n_heads=hf["num_attention_heads"],
             n_kv=hf["num_key_value_heads"], head_dim=hf["head_dim"], vocab=hf["vocab_size"], conv_w=hf["conv_L_cache"],
             rope_theta=hf["rope_theta"], rope_partial=1.0, norm_eps=hf["norm_eps"], sliding_window=0,
             attn_layers=(1,), max_ctx=32, layer_types=hf["layer_types"])
    m = pb.Model(out)
    s = m.new_state(32)
    om = oracle.Model(c, w)
    logits = torch.empty(c["vocab"], dtype=torch.float32, device="cuda")
    tok = 7
    for pos in range(12):
        got = s.decode_token(tok, pos, logits=logits)
        want, lg, _ = om.decode(tok, pos, want_logits=True)
        torch.cuda.synchronize()
        assert np.array_equal(logits.cpu().numpy().view(np.uint32), lg.view(np.uint32)), "pos %d" % pos
        assert got == want
        tok = got
