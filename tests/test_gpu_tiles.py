"""The decode kernel's weight-tile ring (TMA boxes of 128 bytes x 32 or 64
rows, 128-byte swizzle) against the per-thread weight loads and the oracle.

The tile ring changes only how the weight bytes reach the FMA chains of the
reference's row dot (src/int8_expert.rs:380-458 INT8, :473-649 INT4), so
every output is compared bit for bit.  The single-launch kernel takes the
tiles for single-token launches (batch-1 decode); shapes cover a last stage
that is only partly inside the row (OOB bytes zero-filled by TMA and never
used), a down tile that runs past H, INT8 and INT4 weights, single layers
and stacks.  A multi-token launch of tile-capable layers keeps per-thread
loads and still equals the oracle.  MOE_DECODE_TILES=0 at set-layer time
keeps a layer on the per-thread loads.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests import helpers

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import doantotnghiepmoe_b200 as M  # noqa: E402
from doantotnghiepmoe_b200 import _lib  # noqa: E402


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def make_layer(seed, layer, H, I, E, K, norm, int4):
    lw = O.synth_layer(seed, layer, H, I, E, K, norm)
    if not int4:
        return lw
    rng = np.random.default_rng(1000 * seed + layer)
    packed = rng.integers(0, 256, size=(E, 3 * H * I // 2), dtype=np.uint8)
    return O.LayerWeights(H, I, E, K, norm, lw.router, packed, (lw.scales * 16.0).astype(np.float32),
                          int4=True)


def run(lw, h, tiles, monkeypatch):
    monkeypatch.setenv("MOE_DECODE_TILES", "1" if tiles else "0")
    T = h.shape[0]
    eng = M.MoeLayerEngine(M.MoeConfig(lw.H, lw.I, lw.E, lw.K, lw.norm_topk_prob, T, 1))
    eng.set_path(_lib.MOE_PATH_GEMV)
    eng.set_layer_packed(0, *helpers.to_device(lw))
    hd = torch.from_numpy(h).cuda()
    out = torch.empty_like(hd)
    ids = torch.empty((T, lw.K), dtype=torch.int32, device="cuda")
    eng.profile(True)
    eng.forward(0, hd, out, ids=ids)
    eng.sync_status()
    prof = eng.profile_read()
    return out.cpu().numpy(), ids.cpu().numpy().astype(np.uint32), prof


@pytest.mark.parametrize("int4", [False, True])
@pytest.mark.parametrize("H,I,T", [(1056, 544, 1), (2048, 1024, 1), (128, 256, 1),
                                   (1056, 544, 7)])
def test_tiles_equal_thread_loads_and_oracle(H, I, T, int4, monkeypatch):
    """H = 1056: the last 128-byte stage of a row is partly outside it, and
    the last 64-row down tile runs past H.  (128, 256): INT4 rows of 64
    bytes are shorter than a stage, so that layer stays on thread loads.
    T = 7: a multi-token launch (per-thread loads)."""
    lw = make_layer(221, 0, H, I, 16, 4, T == 7, int4)
    h = O.synth_hidden(221, T, H)
    ref = O.layer_forward(lw, h)
    ot, it, pt = run(lw, h, True, monkeypatch)
    op, ip, pp = run(lw, h, False, monkeypatch)
    assert "fused_decode" in pt and "fused_decode" in pp, (pt, pp)
    assert np.array_equal(it, ref.ids) and np.array_equal(ip, ref.ids)
    assert np.array_equal(bits(ot), bits(ref.out))
    assert np.array_equal(bits(op), bits(ot))


@pytest.mark.parametrize("int4", [False, True])
def test_tile_stack(int4, monkeypatch):
    """Three stacked layers, batch-1, on the tile ring (one launch; the
    ring's stage counter runs on across layers) equal the oracle bit for
    bit."""
    monkeypatch.setenv("MOE_DECODE_TILES", "1")
    H, I, E, K, T = 1024, 512, 16, 4, 1
    layers = [make_layer(223, l, H, I, E, K, False, int4) for l in range(3)]
    x0 = O.synth_hidden(223, T, H)
    ref_x, _, _ = O.stack_forward(layers, x0)
    eng = M.MoeLayerEngine(M.MoeConfig(H, I, E, K, False, T, 3))
    eng.set_path(_lib.MOE_PATH_GEMV)
    keep = []
    for l, lw in enumerate(layers):
        dev = helpers.to_device(lw)
        keep.append(dev)
        eng.set_layer_packed(l, *dev)
    x = torch.from_numpy(x0).cuda()
    eng.stack_forward(0, 3, x, 1e-5)
    eng.sync_status()
    assert np.array_equal(bits(x.cpu().numpy()), bits(ref_x))
