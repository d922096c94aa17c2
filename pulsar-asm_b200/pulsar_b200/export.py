"""Float checkpoint -> .lfm3q8 blob, in the certified arm's numerics, without
torch. Follows the reference exporter (pulsar_asm/lfm3/tools/export_lfm3_q8.py:
50-210): every backbone tensor ("lfm." prefix) in name order; the projection
matrices (Q8_PATTERNS) and the tied embedding quantised to Q8 with fp32 scales
(dtype 1), or the embedding kept as bf16 (dtype 3, the certified arm); every
other tensor (norms, the [H,1,W] conv taps) stored as fp32 (dtype 2); CRC-32
of each payload; the JSON header with the checkpoint's "lfm" config.

The quantiser is the certified one (quantize_q8, :50-67): per 32-value group
s = max|w| / 127 in fp32, codes = round-half-to-even(w / s) clamped to
[-128, 127], and an all-zero group writes codes 0 and scale 0.

The checkpoint is read by a small safetensors parser of our own (8-byte header
length, JSON header, raw little-endian payloads; BF16, F16 and F32).

    python -m pulsar_b200.export --model DIR --out FILE [--emb-bf16] [--selfcheck]

DIR holds config.json (with an "lfm" object) and model.safetensors.
"""
import argparse
import json
import os
import struct
import sys
import zlib

import numpy as np

MAGIC = b"LFM3Q8\x01\x00"
T_Q8, T_F32, T_BF16 = 1, 2, 3
BACKBONE = "lfm."
Q8_PATTERNS = ("conv.in_proj", "conv.out_proj", "feed_forward.w1", "feed_forward.w2", "feed_forward.w3",
               "self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
               "self_attn.gate_proj")

_ST_DTYPES = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16, "I8": np.int8, "U8": np.uint8,
              "I32": np.int32, "I64": np.int64}


class SafeTensors:
    """A safetensors file: .names(), .shape(name), .dtype(name), .get(name)
    (numpy array in the stored dtype; BF16 as its uint16 bits)."""

    def __init__(self, path):
        self.f = open(path, "rb")
        n = struct.unpack("<Q", self.f.read(8))[0]
        hdr = json.loads(self.f.read(n))
        self.meta = hdr.pop("__metadata__", {})
        self.hdr = hdr
        self.base = 8 + n

    def names(self):
        return sorted(self.hdr)

    def shape(self, name):
        return list(self.hdr[name]["shape"])

    def dtype(self, name):
        return self.hdr[name]["dtype"]

    def get(self, name):
        e = self.hdr[name]
        if e["dtype"] not in _ST_DTYPES:
            raise ValueError("%s: safetensors dtype %s not supported" % (name, e["dtype"]))
        b0, b1 = e["data_offsets"]
        self.f.seek(self.base + b0)
        a = np.frombuffer(self.f.read(b1 - b0), dtype=_ST_DTYPES[e["dtype"]])
        return a.reshape(e["shape"])

    def get_f32(self, name):
        """the tensor as fp32 (bf16 and fp16 widen exactly)"""
        a = self.get(name)
        if self.dtype(name) == "BF16":
            return (a.astype(np.uint32) << 16).view(np.float32)
        return a.astype(np.float32)


def write_safetensors(path, tensors, bf16=True):
    """a checkpoint file from (name, fp32 array) pairs, stored as bf16 (round
    to nearest even) or fp32"""
    hdr, off, blobs = {}, 0, []
    for name, a in tensors:
        if bf16:
            b, dt = _f32_to_bf16_bits(a).tobytes(), "BF16"
        else:
            b, dt = np.ascontiguousarray(a, np.float32).tobytes(), "F32"
        hdr[name] = {"dtype": dt, "shape": list(np.shape(a)), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    hj = json.dumps(hdr, separators=(",", ":")).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)


def quantize_q8(w):
    """[N, K] fp32 -> (codes int8 [N, K], scales fp32 [N, K/32]), the certified
    quantiser (export_lfm3_q8.py:50-67)"""
    w = np.ascontiguousarray(w, np.float32)
    N, K = w.shape
    if K % 32:
        raise ValueError("Q8_0 needs K % 32 == 0, got K=%d" % K)
    g = w.reshape(N, K // 32, 32)
    m = np.abs(g).max(axis=-1)
    s = (m / np.float32(127.0)).astype(np.float32)
    safe = np.where(s == 0, np.float32(1.0), s)[:, :, None]
    c = np.clip(np.round(g / safe), -128.0, 127.0).astype(np.int8)   # np.round: half to even
    c = np.where(s[:, :, None] == 0, np.int8(0), c)
    return np.ascontiguousarray(c.reshape(N, K)), np.ascontiguousarray(s.reshape(N, K // 32))


def _f32_to_bf16_bits(a):
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    special = ((u >> 23) & 0xFF) == 0xFF
    r = ((u + np.uint32(0x7FFF) + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(special, (u >> 16).astype(np.uint16), r)


def export(model_dir, out, emb_bf16=False, log=print):
    """write the blob; returns its header (dict)"""
    cfg = json.load(open(os.path.join(model_dir, "config.json")))["lfm"]
    st = SafeTensors(os.path.join(model_dir, "model.safetensors"))
    keys = [k for k in st.names() if k.startswith(BACKBONE)]
    if not keys:
        raise ValueError("no %s* tensors in the checkpoint" % BACKBONE)
    hit = {p: 0 for p in Q8_PATTERNS}
    hit["embed_tokens"] = 0
    entries, blobs, off = [], [], 0
    for k in keys:
        shp = st.shape(k)
        is_emb = "embed_tokens" in k
        if is_emb and emb_bf16:
            if len(shp) != 2:
                raise ValueError("%s is %d-D" % (k, len(shp)))
            hit["embed_tokens"] += 1
            w = st.get(k) if st.dtype(k) == "BF16" else _f32_to_bf16_bits(st.get_f32(k))
            b = np.ascontiguousarray(w, np.uint16).tobytes()
            entries.append(dict(name=k, dtype=T_BF16, ne=shp, off=off, ncodes=len(b), nscales=0,
                                crc=zlib.crc32(b) & 0xFFFFFFFF))
            blobs.append(b)
            off += len(b)
            continue
        if is_emb or any(p in k for p in Q8_PATTERNS):
            if len(shp) != 2:
                raise ValueError("%s is %d-D; the Q8 quantiser is 2-D only" % (k, len(shp)))
            for p in (["embed_tokens"] if is_emb else [p for p in Q8_PATTERNS if p in k]):
                hit[p] += 1
            codes, scales = quantize_q8(st.get_f32(k))
            cb, sb = codes.tobytes(), scales.tobytes()
            entries.append(dict(name=k, dtype=T_Q8, ne=shp, off=off, ncodes=len(cb), nscales=len(sb),
                                crc=zlib.crc32(sb, zlib.crc32(cb)) & 0xFFFFFFFF))
            blobs += [cb, sb]
            off += len(cb) + len(sb)
        else:
            if len(shp) not in (1, 2, 3):
                raise ValueError("%s is %d-D" % (k, len(shp)))
            b = np.ascontiguousarray(st.get_f32(k)).tobytes()
            entries.append(dict(name=k, dtype=T_F32, ne=shp, off=off, ncodes=len(b), nscales=0,
                                crc=zlib.crc32(b) & 0xFFFFFFFF))
            blobs.append(b)
            off += len(b)
    empty = [p for p, c in hit.items() if c == 0]
    if empty:
        raise ValueError("Q8 patterns matched no tensors: %s" % empty)
    want_conv = cfg["num_hidden_layers"] - sum(1 for lt in cfg["layer_types"] if lt != "conv")
    nconv = sum(1 for e in entries if e["name"].endswith("conv.conv.weight"))
    if nconv != want_conv:
        raise ValueError("expected %d conv.conv.weight, got %d" % (want_conv, nconv))
    hdr = dict(magic=MAGIC.decode(), cfg=cfg, n_tensors=len(entries), vocab_size=cfg["vocab_size"],
               hidden_size=cfg["hidden_size"], data_bytes=off, table=entries)
    hj = json.dumps(hdr, separators=(",", ":")).encode()
    with open(out, "wb") as fh:
        fh.write(MAGIC)
        fh.write(struct.pack("<I", len(hj)))
        fh.write(hj)
        for b in blobs:
            fh.write(b)
    if log:
        log("wrote %s: %.1f MB, %d tensors" % (out, (len(hj) + off) / 1e6, len(entries)))
    return hdr


def selfcheck(model_dir, out):
    """re-read the blob, check every payload's CRC and re-derive it from the
    checkpoint; returns the names that disagree"""
    st = SafeTensors(os.path.join(model_dir, "model.safetensors"))
    with open(out, "rb") as f:
        f.read(len(MAGIC))
        n = struct.unpack("<I", f.read(4))[0]
        hdr = json.loads(f.read(n))
        base = f.tell()
        bad = []
        for e in hdr["table"]:
            f.seek(base + e["off"])
            raw = f.read(e["ncodes"] + e["nscales"])
            if zlib.crc32(raw) & 0xFFFFFFFF != e["crc"]:
                bad.append(e["name"] + ":load")
                continue
            if e["dtype"] == T_Q8:
                c, s = quantize_q8(st.get_f32(e["name"]))
                ref = c.tobytes() + s.tobytes()
            elif e["dtype"] == T_BF16:
                w = st.get(e["name"]) if st.dtype(e["name"]) == "BF16" else _f32_to_bf16_bits(st.get_f32(e["name"]))
                ref = np.ascontiguousarray(w, np.uint16).tobytes()
            else:
                ref = np.ascontiguousarray(st.get_f32(e["name"])).tobytes()
            if ref != raw:
                bad.append(e["name"] + ":quant")
    return bad


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--model", required=True, help="directory with config.json and model.safetensors")
    ap.add_argument("--out", required=True)
    ap.add_argument("--emb-bf16", action="store_true", help="keep the tied embedding as bf16 (dtype 3)")
    ap.add_argument("--selfcheck", action="store_true", help="re-read the blob and re-derive every tensor")
    a = ap.parse_args(argv)
    export(a.model, a.out, emb_bf16=a.emb_bf16)
    if a.selfcheck:
        bad = selfcheck(a.model, a.out)
        print("SELFCHECK %s (%d bad)%s" % ("OK" if not bad else "FAIL", len(bad), "" if not bad else " " + str(bad[:8])))
        return 0 if not bad else 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
