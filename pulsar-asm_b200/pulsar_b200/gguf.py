"""GGUF (v3) reader for the Bonsai Q1_0 decoder's weights, and a minimal
writer (tests, round trips).

The reader walks the file as fwd8.c's gguf_table does (pulsar_arm/bonsai2/
fwd8.c:210-263): magic "GGUF", u32 version, u64 tensor count, u64 key count;
each key a u64-length string, an i32 value type and the value (strings and
arrays skipped by their lengths); each tensor a name, an i32 dimension count,
u64 dimensions, an i32 type and a u64 offset; tensor data starting at the next
multiple of the file's alignment (general.alignment, 32 by default) after the
table. Tensors are found by name: blk.{i}.attn_q.weight ... ffn_down.weight,
the norms, output_norm.weight, token_embd.weight and output.weight (absent
when the head is tied to the table, fwd8.c:258-263).

Q1_0 tensors (18-byte blocks: an fp16 scale and 16 bytes of LSB-first sign
bits per 128 weights, pq1_wrap.h:24-35) come from the PrismML ggml fork,
whose type number is not vendored here; like fwd8.c, the reader does not rely
on it: a weight tensor is accepted when its bytes up to the next tensor (or
the file's end) hold rows x K/128 blocks. Norms are F32 (type 0).
"""
import mmap
import os
import struct

import numpy as np

GGUF_MAGIC = b"GGUF"
T_F32 = 0
Q1_0_BLOCK = 18
_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}


class GGUF:
    """.meta: key -> value (arrays as lists); .tensors: name -> (dims, type,
    absolute file offset); .raw(name, nbytes)"""

    def __init__(self, path):
        self.path = path
        with open(path, "rb") as f:
            # mapped, not read: an 8B model's file is over a gigabyte
            self.buf = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) if os.fstat(f.fileno()).st_size else b""
        b = self.buf
        if b[:4] != GGUF_MAGIC:
            raise ValueError("%s: not a GGUF file" % path)
        self.version, nt, nkv = struct.unpack_from("<IQQ", b, 4)
        p = 24
        self.meta = {}
        for _ in range(nkv):
            key, p = self._str(p)
            t = struct.unpack_from("<i", b, p)[0]
            p += 4
            self.meta[key], p = self._val(t, p)
        self.tensors = {}
        order = []
        for _ in range(nt):
            name, p = self._str(p)
            nd = struct.unpack_from("<i", b, p)[0]
            p += 4
            dims = list(struct.unpack_from("<%dQ" % nd, b, p))
            p += 8 * nd
            tt, off = struct.unpack_from("<iQ", b, p)
            p += 12
            self.tensors[name] = [dims, tt, off]
            order.append(name)
        align = int(self.meta.get("general.alignment", 32))
        self.data_start = (p + align - 1) // align * align
        for name in order:
            self.tensors[name][2] += self.data_start
        ends = sorted(v[2] for v in self.tensors.values()) + [len(b)]
        self._end = {}
        for name in order:
            o = self.tensors[name][2]
            self._end[name] = min(e for e in ends if e > o) if any(e > o for e in ends) else len(b)

    def _str(self, p):
        n = struct.unpack_from("<Q", self.buf, p)[0]
        return self.buf[p + 8:p + 8 + n].decode("utf-8", "replace"), p + 8 + n

    def _val(self, t, p):
        if t == 8:
            return self._str(p)
        if t == 9:
            et, n = struct.unpack_from("<iQ", self.buf, p)
            p += 12
            out = []
            for _ in range(n):
                v, p = self._val(et, p)
                out.append(v)
            return out, p
        if t not in _SCALAR:
            raise ValueError("bad GGUF value type %d" % t)
        fmt = _SCALAR[t]
        return struct.unpack_from(fmt, self.buf, p)[0], p + struct.calcsize(fmt)

    def raw(self, name, nbytes):
        dims, tt, off = self.tensors[name]
        if off + nbytes > self._end[name]:
            raise ValueError("%s: %d bytes do not fit before the next tensor" % (name, nbytes))
        return np.frombuffer(self.buf, np.uint8, nbytes, off)

    def q1(self, name, rows, K):
        """Q1_0 blocks [rows][K/128][18]"""
        if K % 128:
            raise ValueError("%s: K=%d is not a multiple of 128" % (name, K))
        return self.raw(name, rows * (K // 128) * Q1_0_BLOCK).reshape(rows, K // 128, Q1_0_BLOCK).copy()

    def f32(self, name, n):
        return self.raw(name, 4 * n).view(np.float32).copy()


LAYER_Q1 = (("q", "attn_q.weight"), ("k", "attn_k.weight"), ("v", "attn_v.weight"), ("o", "attn_output.weight"),
            ("gate", "ffn_gate.weight"), ("up", "ffn_up.weight"), ("down", "ffn_down.weight"))
LAYER_NORMS = (("attn_norm", "attn_norm.weight"), ("ffn_norm", "ffn_norm.weight"),
               ("q_norm", "attn_q_norm.weight"), ("k_norm", "attn_k_norm.weight"))


def bonsai_weights(path, cfg):
    """the Bonsai decoder's weights (shaped like synth.make_bonsai_weights)
    from a GGUF file; cfg: hidden, inter, n_layers, n_heads, n_kv, vocab"""
    g = GGUF(path)
    H, F, NH, NKV, V = cfg["hidden"], cfg["inter"], cfg["n_heads"], cfg["n_kv"], cfg["vocab"]
    shapes = {"q": (NH * 128, H), "k": (NKV * 128, H), "v": (NKV * 128, H), "o": (H, NH * 128),
              "gate": (F, H), "up": (F, H), "down": (H, F)}
    layers = []
    for il in range(cfg["n_layers"]):
        d = {}
        for key, nm in LAYER_Q1:
            rows, K = shapes[key]
            d[key] = g.q1("blk.%d.%s" % (il, nm), rows, K)
        for key, nm in LAYER_NORMS:
            d[key] = g.f32("blk.%d.%s" % (il, nm), 128 if key in ("q_norm", "k_norm") else H)
        layers.append(d)
    head = g.q1("output.weight", V, H) if "output.weight" in g.tensors else None
    return dict(layers=layers, embed=g.q1("token_embd.weight", V, H), head=head,
                out_norm=g.f32("output_norm.weight", H))


def write(path, meta, tensors, q1_type=41, align=32):
    """a GGUF v3 file: meta (str -> int / float / str), tensors: list of
    (name, dims in GGUF order, type, bytes); Q1_0 tensors take q1_type"""
    def s(x):
        e = x.encode()
        return struct.pack("<Q", len(e)) + e
    out = bytearray(GGUF_MAGIC + struct.pack("<IQQ", 3, len(tensors), len(meta)))
    for k, v in meta.items():
        out += s(k)
        if isinstance(v, str):
            out += struct.pack("<i", 8) + s(v)
        elif isinstance(v, float):
            out += struct.pack("<if", 6, v)
        else:
            out += struct.pack("<iI", 4, v)
    off, offs = 0, []
    for name, dims, tt, data in tensors:
        offs.append(off)
        off += (len(data) + align - 1) // align * align
    for (name, dims, tt, data), o in zip(tensors, offs):
        out += s(name) + struct.pack("<i", len(dims)) + struct.pack("<%dQ" % len(dims), *dims)
        out += struct.pack("<iQ", tt, o)
    out += b"\0" * ((align - len(out) % align) % align)
    for (name, dims, tt, data), o in zip(tensors, offs):
        out += data + b"\0" * ((align - len(data) % align) % align)
    with open(path, "wb") as f:
        f.write(out)


def write_bonsai(path, cfg, w, q1_type=41):
    """the Bonsai weights (synth.make_bonsai_weights form) as a GGUF file with
    fwd8.c's tensor names (GGUF dims: fastest first)"""
    t = [("token_embd.weight", [cfg["hidden"], cfg["vocab"]], q1_type, np.ascontiguousarray(w["embed"]).tobytes())]
    for il, d in enumerate(w["layers"]):
        for key, nm in LAYER_Q1:
            a = np.ascontiguousarray(d[key])
            t.append(("blk.%d.%s" % (il, nm), [a.shape[1] * 128, a.shape[0]], q1_type, a.tobytes()))
        for key, nm in LAYER_NORMS:
            a = np.ascontiguousarray(d[key], np.float32)
            t.append(("blk.%d.%s" % (il, nm), [a.size], T_F32, a.tobytes()))
    if w.get("head") is not None:
        t.append(("output.weight", [cfg["hidden"], cfg["vocab"]], q1_type, np.ascontiguousarray(w["head"]).tobytes()))
    t.append(("output_norm.weight", [cfg["hidden"]], T_F32, np.ascontiguousarray(w["out_norm"], np.float32).tobytes()))
    meta = {"general.architecture": "qwen3", "general.alignment": 32, "qwen3.block_count": cfg["n_layers"],
            "qwen3.embedding_length": cfg["hidden"], "qwen3.feed_forward_length": cfg["inter"],
            "qwen3.attention.head_count": cfg["n_heads"], "qwen3.attention.head_count_kv": cfg["n_kv"]}
    write(path, meta, t, q1_type)
