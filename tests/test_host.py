"""Host-side logic: synthetic model accounting, blob round trip, sharding."""
import numpy as np

from pulsar_b200 import blob, dist, synth


def test_cfg1_bytes_per_token_matches_the_plan():
    # conv layer 71,360,512 B; attn layer 64,721,408 B + 2 MiB of KV at ctx 1024;
    # tied head 142,606,336 B; 1,828,017,280 B per token in total
    c = synth.LFM3_CFG1
    w = synth.weight_bytes_per_token(c)
    assert w + synth.kv_bytes_per_token(c, 1024) == 1_828_017_280


def test_blob_header_round_trip(tmp_path):
    c = dict(synth.LFM3_TINY, vocab=128, n_layers=1, attn_layers=(0,))
    w = synth.make_weights(c, seed=9)
    path = str(tmp_path / "t.lfm3q8")
    n = synth.write_model(path, c, w)
    hdr, base = blob.read_header(path)
    assert hdr["data_bytes"] == n and hdr["cfg"]["layer_types"] == ["full_attention"]
    rec = [t for t in hdr["table"] if t["name"].endswith("q_proj.weight")][0]
    with open(path, "rb") as f:
        f.seek(base + rec["off"])
        codes = np.frombuffer(f.read(rec["ncodes"]), np.int8).reshape(rec["ne"])
        sc = np.frombuffer(f.read(rec["nscales"]), np.float16)
    assert np.array_equal(codes, w["layers"][0]["q"][0])
    assert np.array_equal(sc.reshape(w["layers"][0]["q"][1].shape), w["layers"][0]["q"][1])
    assert rec["dtype"] == blob.T_Q8_F16S


def test_synth_distributions():
    import numpy as np
    rng = np.random.default_rng(0)
    codes, sc = synth.q8(rng, 256, 2048)
    assert codes.min() >= -127 and codes.max() <= 127
    assert sc.dtype == np.float16 and (sc >= 0).all()


def test_shard_range_partitions():
    for n in (0, 1, 7, 64, 65):
        for world in (1, 2, 3, 8):
            parts = [dist.shard_range(n, r, world) for r in range(world)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(world - 1))
            assert max(b - a for a, b in parts) - min(b - a for a, b in parts) <= 1


def test_bench_clock_samples_only_inside_the_timed_region():
    """The bench's nvidia-smi sampler keeps only the samples whose own
    timestamps fall inside the timed region, and reads clock and throttle
    fields by position after the timestamp."""
    import datetime
    import os
    import sys
    import time
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import bench
    c = bench.Clocks(0)
    now = time.time()
    c.t0, c.t1 = now - 1.0, now + 1.0

    def stamp(t):
        return datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    quiet = "Not Active, Not Active, Not Active, Not Active"
    c.lines = [stamp(now - 5) + ", 0, 900, 1965, 100.0, 0x1, Active, Not Active, Not Active, Not Active",
               stamp(now - 0.5) + ", 0, 1965, 1965, 300.0, 0x0, " + quiet,
               stamp(now) + ", 0, 1900, 1965, 320.0, 0x4, Not Active, Not Active, Not Active, Active",
               stamp(now + 5) + ", 0, 800, 1965, 100.0, 0x0, " + quiet,
               "garbage line"]
    s = c.summary()
    assert s["samples"] == 2
    assert s["sm_mhz"] == (1965.0 + 1900.0) / 2 and s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["sw_power_cap"]
