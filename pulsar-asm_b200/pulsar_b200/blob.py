""".lfm3q8 blob writer and reader.

Layout (the reference writer is pulsar_asm/lfm3/tools/export_lfm3_q8.py:38-210,
its reader lfm3_nanode.cu:1404-1733): 8-byte magic "LFM3Q8\\x01\\x00", a u32
little-endian header length, a JSON header
  {"magic", "cfg", "n_tensors", "vocab_size", "hidden_size", "data_bytes",
   "table": [{"name", "dtype", "ne", "off", "ncodes", "nscales", "crc"}, ...]}
then the payloads back to back (offsets relative to the end of the header).
A Q8 payload is its codes followed by its scales. crc is zlib's CRC-32 of the
payload bytes (the reference's writer uses zlib.crc32 too, :69-80).

dtype: 1 = Q8 codes + fp32 scales (the reference's certified format),
       2 = fp32, 3 = bf16, 8 = Q8_0 codes + fp16 scales (ggml-style; this
       build's addition for fp16-scale checkpoints).
"""
import json
import struct
import zlib

import numpy as np

MAGIC = b"LFM3Q8\x01\x00"
T_Q8_F32S, T_F32, T_BF16, T_Q4, T_Q5, T_Q8_F16S = 1, 2, 3, 6, 7, 8


def write_blob(path, cfg, tensors):
    """tensors: list of (name, kind, payload) with kind "q8" -> (codes int8 [N,K],
    scales fp16/fp32 [N,K/32]), "bf16" -> uint16 bf16 bits, "q4" / "q5" ->
    ((N, K), tiled codes uint8, half2 scales as uint16), or "f32" -> ndarray."""
    table, blobs, off = [], [], 0
    for name, kind, payload in tensors:
        if kind == "q8":
            codes, scales = payload
            codes = np.ascontiguousarray(codes, np.int8)
            if scales.dtype == np.float32:
                dt = T_Q8_F32S
                sc = np.ascontiguousarray(scales, np.float32)
            else:
                dt = T_Q8_F16S
                sc = np.ascontiguousarray(scales).view(np.uint16)
            cb, sb = codes.tobytes(), sc.tobytes()
            crc = zlib.crc32(sb, zlib.crc32(cb)) & 0xFFFFFFFF
            table.append(dict(name=name, dtype=dt, ne=list(codes.shape), off=off,
                              ncodes=len(cb), nscales=len(sb), crc=crc))
            blobs += [cb, sb]
            off += len(cb) + len(sb)
        elif kind == "bf16":
            # the certified arm's embedding: bf16 bits verbatim, no scales
            # (export_lfm3_q8.py:96-110)
            a = np.ascontiguousarray(payload, np.uint16)
            b = a.tobytes()
            table.append(dict(name=name, dtype=T_BF16, ne=list(a.shape), off=off, ncodes=len(b),
                              nscales=0, crc=zlib.crc32(b) & 0xFFFFFFFF))
            blobs.append(b)
            off += len(b)
        elif kind in ("q4", "q5"):
            # the low-bit records (lfm3_nanode.cu:1494-1501): the exporter's
            # tiled codes, then the half2 (128 d, mn) scales; ne = [N, K]
            (N, K), codes, scales = payload
            cb = np.ascontiguousarray(codes, np.uint8).tobytes()
            sb = np.ascontiguousarray(scales, np.uint16).tobytes()
            table.append(dict(name=name, dtype=T_Q4 if kind == "q4" else T_Q5, ne=[int(N), int(K)], off=off,
                              ncodes=len(cb), nscales=len(sb), crc=zlib.crc32(sb, zlib.crc32(cb)) & 0xFFFFFFFF))
            blobs += [cb, sb]
            off += len(cb) + len(sb)
        elif kind == "f32":
            a = np.ascontiguousarray(payload, np.float32)
            b = a.tobytes()
            table.append(dict(name=name, dtype=T_F32, ne=list(a.shape), off=off, ncodes=len(b),
                              nscales=0, crc=zlib.crc32(b) & 0xFFFFFFFF))
            blobs.append(b)
            off += len(b)
        else:
            raise ValueError(kind)
    hdr = dict(magic=MAGIC.decode("latin-1"), cfg=cfg, n_tensors=len(table),
               vocab_size=cfg.get("vocab_size"), hidden_size=cfg.get("hidden_size"),
               data_bytes=off, table=table)
    hj = json.dumps(hdr, separators=(",", ":")).encode()
    with open(path, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<I", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)
    return off


def read_header(path):
    with open(path, "rb") as f:
        if f.read(8) != MAGIC:
            raise ValueError("bad magic")
        n = struct.unpack("<I", f.read(4))[0]
        hdr = json.loads(f.read(n))
    return hdr, 12 + n
