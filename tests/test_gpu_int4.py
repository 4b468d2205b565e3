"""INT4 nibble experts on the exact GEMV paths (src/int8_expert.rs:473-649,
:785-952): the single-launch decode kernel (one route and multi-route per
expert), the per-phase launches, odd shapes (leftover 8-chunks and scalar
tails), stacks of INT4 layers and stacks mixing formats, checkpoint loading
-- all bit-identical to the oracle's restatement of the reference's INT4
AVX2 path.  The tensor-core path takes INT8 layers only."""
import numpy as np
import pytest

from oracle import oracle as O
from tests import helpers
from tests.helpers import write_safetensors

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import doantotnghiepmoe_b200 as M  # noqa: E402
from doantotnghiepmoe_b200 import _lib  # noqa: E402


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def int4_layer(seed, layer, H, I, E, K, norm):
    lw = O.synth_layer(seed, layer, H, I, E, K, norm)
    rng = np.random.default_rng(1000 * seed + layer)
    packed = rng.integers(0, 256, size=(E, 3 * H * I // 2), dtype=np.uint8)
    # scales sized for nibble weights (|q| <= 8)
    scales = (lw.scales * 16.0).astype(np.float32)
    return O.LayerWeights(H, I, E, K, norm, lw.router, packed, scales, int4=True)


def run_layer(lw, h, path=_lib.MOE_PATH_AUTO):
    T = h.shape[0]
    eng = M.MoeLayerEngine(M.MoeConfig(lw.H, lw.I, lw.E, lw.K, lw.norm_topk_prob, T, 1))
    eng.set_path(path)
    ex, sc, rt = helpers.to_device(lw)
    eng.set_layer_packed(0, ex, sc, rt)
    hd = torch.from_numpy(h).cuda()
    out = torch.empty_like(hd)
    ids = torch.empty((T, lw.K), dtype=torch.int32, device="cuda")
    eng.forward(0, hd, out, ids=ids)
    eng.sync_status()
    return out.cpu().numpy(), ids.cpu().numpy().astype(np.uint32), eng


@pytest.mark.parametrize("T,path", [(1, _lib.MOE_PATH_AUTO), (8, _lib.MOE_PATH_AUTO),
                                    (3, _lib.MOE_PATH_GEMV_PHASED),
                                    (200, _lib.MOE_PATH_AUTO)])
def test_int4_olmoe_layer_bit_exact(T, path):
    """OLMoE shape (H=2048, I=1024, E=64, K=8); T=200 would take the tensor
    cores for INT8 and stays on the exact GEMV here."""
    lw = int4_layer(201, 0, 2048, 1024, 64, 8, False)
    h = O.synth_hidden(201, T, 2048)
    ref = O.layer_forward(lw, h)
    out, ids, _ = run_layer(lw, h, path)
    assert np.array_equal(ids, ref.ids)
    assert np.array_equal(bits(out), bits(ref.out))


@pytest.mark.parametrize("H,I", [(76, 36), (40, 24), (72, 40)])
def test_int4_odd_shapes(H, I):
    """H, I even but not multiples of 32 (leftover 8-chunks) or of 8 (tails)."""
    lw = int4_layer(203, 0, H, I, 8, 2, True)
    h = O.synth_hidden(203, 5, H)
    ref = O.layer_forward(lw, h)
    for path in (_lib.MOE_PATH_AUTO, _lib.MOE_PATH_GEMV_PHASED):
        out, ids, _ = run_layer(lw, h, path)
        assert np.array_equal(ids, ref.ids)
        assert np.array_equal(bits(out), bits(ref.out)), path


def test_int4_rejected_by_tensor_path():
    lw = int4_layer(205, 0, 256, 128, 16, 4, False)
    with pytest.raises(M.MoeError) as ei:
        run_layer(lw, O.synth_hidden(205, 4, 256), _lib.MOE_PATH_TENSOR)
    assert ei.value.status == _lib.MOE_ERR_STATE


@pytest.mark.parametrize("mixed", [False, True])
def test_int4_stacks(mixed):
    """Stacked decode over INT4 layers (one launch) and over INT8 / INT4
    layers mixed (one launch per phase): bit-exact against the oracle."""
    H, I, E, K, T = 512, 256, 16, 4, 4
    layers = []
    for l in range(3):
        if mixed and l == 1:
            layers.append(O.synth_layer(207, l, H, I, E, K, False))
        else:
            layers.append(int4_layer(207, l, H, I, E, K, False))
    x0 = O.synth_hidden(207, T, H)
    ref_x, _, _ = O.stack_forward(layers, x0)
    eng = M.MoeLayerEngine(M.MoeConfig(H, I, E, K, False, T, 3))
    keep = []
    for l, lw in enumerate(layers):
        dev = helpers.to_device(lw)
        keep.append(dev)
        eng.set_layer_packed(l, *dev)
    x = torch.from_numpy(x0).cuda()
    eng.stack_forward(0, 3, x, 1e-5)
    eng.sync_status()
    if mixed:
        # the default path runs the INT8 layer on the digit decode launch:
        # within the tolerance; the exact path is bit-exact
        assert helpers.rel_err(x.cpu().numpy(), ref_x) < 1e-3
        eng.set_path(_lib.MOE_PATH_GEMV)
        x = torch.from_numpy(x0).cuda()
        eng.stack_forward(0, 3, x, 1e-5)
        eng.sync_status()
    assert np.array_equal(bits(x.cpu().numpy()), bits(ref_x))


def test_int4_checkpoint_load(tmp_path):
    H, I, E, K = 256, 128, 8, 2
    lw = int4_layer(209, 0, H, I, E, K, False)
    t = [("model.layers.0.mlp.gate.weight", "F32", lw.router)]
    for e in range(E):
        t.append((f"model.layers.0.mlp.experts.{e}.merged_weight", "U8", lw.experts[e]))
        t.append((f"model.layers.0.mlp.experts.{e}.qs", "F32", lw.scales[e]))
    write_safetensors(tmp_path / "m.safetensors", t)
    eng = M.MoeLayerEngine(M.MoeConfig(H, I, E, K, False, 6, 1))
    eng.load_layer(M.Checkpoint(str(tmp_path)), 0)
    h = O.synth_hidden(209, 6, H)
    ref = O.layer_forward(lw, h)
    hd = torch.from_numpy(h).cuda()
    out = torch.empty_like(hd)
    eng.forward(0, hd, out)
    eng.sync_status()
    assert np.array_equal(bits(out.cpu().numpy()), bits(ref.out))
