"""The C ABI library without a GPU: it loads, exports every function that
include/*.h declares, and the loader's format checks (validate-only open,
device < 0) reject corrupt blobs with the documented status codes."""
import ctypes as C
import glob
import os
import re
import struct

import numpy as np
import pytest

from conftest import ROOT


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        src = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        for m in re.finditer(r"^\s*(?:[A-Za-z_][\w\s\*]*?)\b((?:pb|pq1)_\w+)\s*\(", src, re.M):
            names.add(m.group(1))
    return sorted(names)


def test_exports_every_declared_symbol(pb):
    L = pb.lib()
    names = declared_functions()
    assert len(names) > 20
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_version_and_error_channel(pb):
    assert pb.lib().pb_version() >= 10000
    rc = pb.lib().pb_open(b"/nonexistent/blob.lfm3q8", -1, C.byref(C.c_void_p()))
    assert rc == -4
    assert "cannot open" in pb.last_error()


def _tiny_blob(tmp_path, **over):
    from pulsar_b200 import synth
    c = dict(synth.LFM3_TINY)
    c.update(vocab=256, n_layers=2, attn_layers=(1,), inter=2048)
    c.update(over)
    w = synth.make_weights(c, seed=3)
    path = str(tmp_path / "m.lfm3q8")
    synth.write_model(path, c, w)
    return path


def _open_validate(pb, path):
    return pb.lib().pb_open(path.encode(), -1, C.byref(C.c_void_p()))


def test_validate_good_blob(pb, tmp_path):
    assert _open_validate(pb, _tiny_blob(tmp_path)) == 0


def test_corrupt_payload_is_crc_error(pb, tmp_path):
    path = _tiny_blob(tmp_path)
    with open(path, "r+b") as f:
        f.seek(-5000, os.SEEK_END)
        b = f.read(1)
        f.seek(-5000, os.SEEK_END)
        f.write(bytes([b[0] ^ 0x40]))
    assert _open_validate(pb, path) == -5
    assert "CRC" in pb.last_error()


def test_truncated_blob_is_io_error(pb, tmp_path):
    path = _tiny_blob(tmp_path)
    n = os.path.getsize(path)
    with open(path, "r+b") as f:
        f.truncate(n - 100)
    assert _open_validate(pb, path) == -4


def test_bad_magic_and_header(pb, tmp_path):
    p = tmp_path / "bad.lfm3q8"
    p.write_bytes(b"GGUF\x03\x00\x00\x00" + b"\x00" * 64)
    assert _open_validate(pb, str(p)) == -6
    p.write_bytes(b"LFM3Q8\x01\x00" + struct.pack("<I", 10) + b"{not json}")
    assert _open_validate(pb, str(p)) == -6


def test_missing_tensor_is_format_error(pb, tmp_path):
    from pulsar_b200 import blob, synth
    c = dict(synth.LFM3_TINY)
    c.update(vocab=256, n_layers=1, attn_layers=(), inter=2048)
    w = synth.make_weights(c, seed=4)
    del w["layers"][0]["w2"]
    path = str(tmp_path / "m.lfm3q8")
    synth.write_model(path, c, w)
    assert _open_validate(pb, path) == -6
    assert "w2" in pb.last_error()


def test_misshapen_tensor_is_format_error(pb, tmp_path):
    from pulsar_b200 import synth
    c = dict(synth.LFM3_TINY)
    c.update(vocab=256, n_layers=1, attn_layers=(), inter=2048)
    w = synth.make_weights(c, seed=4)
    codes, sc = w["layers"][0]["out_proj"]
    w["layers"][0]["out_proj"] = (codes[:1024], sc[:1024])
    path = str(tmp_path / "m.lfm3q8")
    synth.write_model(path, c, w)
    assert _open_validate(pb, path) == -6


def test_shim_host_silu_mul(pb):
    """pq1_silu_mul (the shim's host helper, pq1_host.c:196-227) runs without a
    GPU: lu = (g * (1/(1+expf(-g)))) * lu, each operation rounded to fp32, with
    the C library's expf, on edge values (0, -0, large magnitudes, subnormal)"""
    L = pb.lib()
    L.pq1_silu_mul.argtypes = [C.c_void_p, C.c_void_p, C.c_int]
    libm = C.CDLL("libm.so.6")
    libm.expf.argtypes = [C.c_float]
    libm.expf.restype = C.c_float
    rng = np.random.default_rng(5)
    g = np.concatenate([rng.standard_normal(4093).astype(np.float32) * 6,
                        np.array([0.0, -0.0, 88.0, -88.0, 103.0, -103.0, 1e-40], np.float32)])
    u = rng.standard_normal(g.size).astype(np.float32)
    out = u.copy()
    L.pq1_silu_mul(out.ctypes.data, g.ctypes.data, g.size)
    f = np.float32
    want = np.array([f(f(gi * f(f(1.0) / f(f(1.0) + f(libm.expf(f(-gi)))))) * ui) for gi, ui in zip(g, u)], np.float32)
    assert np.array_equal(out.view(np.uint32), want.view(np.uint32))


def _lowbit_blob(tmp_path, corrupt=None):
    """a model holding Q4 / Q5 records next to a Q8 one (the speech server's
    low-bit backbone, lfm3_nanode.cu:1494-1501)"""
    from pulsar_b200 import synth
    c = dict(synth.LFM3_TINY)
    rng = np.random.default_rng(3)
    q4c, q4s = synth.qlow_payload(rng, 256, 512, 4)
    q5c, q5s = synth.qlow_payload(rng, 64, 256, 5)
    if corrupt == "size":
        q5s = q5s[:-2]
    q8 = (rng.integers(-127, 128, (128, 256), dtype=np.int8), (rng.random((128, 8)) * 0.01).astype(np.float32))
    tensors = [("lfm.model.layers.0.feed_forward.w1.weight", "q4", ((256, 512), q4c, q4s)),
               ("lfm.model.layers.0.feed_forward.w2.weight", "q5", ((64, 256), q5c, q5s)),
               ("lfm.model.layers.0.conv.out_proj.weight", "q8", q8),
               ("lfm.model.embedding_norm.weight", "f32", np.ones(c["hidden"], np.float32))]
    return tensors


def test_lowbit_records(pb, tmp_path):
    """pb_open takes Q4 / Q5 records (the reference's record checks) into its
    per-tensor mode; a record with inconsistent sizes is a format error, a
    corrupt payload a CRC error"""
    from pulsar_b200 import blob, synth
    c = dict(synth.LFM3_TINY)
    cfg = synth.hf_cfg(c)
    path = str(tmp_path / "low.lfm3q8")
    blob.write_blob(path, cfg, _lowbit_blob(tmp_path))
    assert _open_validate(pb, path) == 0
    bad = str(tmp_path / "bad.lfm3q8")
    blob.write_blob(bad, cfg, _lowbit_blob(tmp_path, corrupt="size"))
    assert _open_validate(pb, bad) == -6          # PB_EFORMAT
    raw = bytearray(open(path, "rb").read())
    raw[-40] ^= 0xFF
    open(bad, "wb").write(bytes(raw))
    assert _open_validate(pb, bad) == -5          # PB_ECRC
