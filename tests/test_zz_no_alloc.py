"""pb_layer_step_noalloc: the layer step for callers that cannot allocate
device memory (their runtime owns every allocation, or allocation is forbidden
after start-up). Its intermediates live in a static device array; its output
must equal pb_layer_step's bit for bit, on two calls in a row (the array keeps
the previous call's contents, which must not leak into the next call).

Collected last on purpose (file name), so that a run that stops at the first
failure has already run every other test."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_noalloc_layer_step_matches_layer_step(tmp_path, pb, cuda):
    torch = cuda
    from pulsar_b200 import synth
    c = dict(synth.LFM3_TINY, n_layers=2, attn_layers=(1,), vocab=512)
    w = synth.make_weights(c, seed=21)
    path = str(tmp_path / "noalloc.lfm3q8")
    synth.write_model(path, c, w)
    m = pb.Model(path)
    s_ref = m.new_state(8)
    s_new = m.new_state(8)
    rng = np.random.default_rng(4)
    x0 = (rng.standard_normal(c["hidden"]) * 2).astype(np.float32)
    xb = ((x0.view(np.uint32) + 0x7FFF + ((x0.view(np.uint32) >> 16) & 1)) >> 16).astype(np.uint16)
    x_ref = torch.from_numpy(xb.view(np.int16).copy()).cuda()
    x_new = x_ref.clone()
    # calls in a row: the conv layer then the attention layer, at four
    # positions; after the first position (warm: modules loaded, the array's
    # address looked up) the calls take no device memory
    free0 = None
    for pos in (0, 1, 2, 3):
        for layer in (0, 1):
            s_ref.layer_step(layer, pos, x_ref)
            s_new.layer_step_noalloc(layer, pos, x_new)
            torch.cuda.synchronize()
            assert torch.equal(x_ref, x_new), "layer %d pos %d" % (layer, pos)
        if pos == 0:
            free0 = torch.cuda.mem_get_info()[0]
    free1 = torch.cuda.mem_get_info()[0]
    kv_ref = s_ref.debug_tensor(0, torch.int16)
    kv_new = s_new.debug_tensor(0, torch.int16)
    ring_ref = s_ref.debug_tensor(1, torch.int16)
    ring_new = s_new.debug_tensor(1, torch.int16)
    assert torch.equal(kv_ref, kv_new) and torch.equal(ring_ref, ring_new)
    assert free1 == free0
    s_ref.destroy()
    s_new.destroy()
    m.close()
