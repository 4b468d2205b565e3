"""moe_load_layer: merged-INT8 checkpoint layers straight into device memory.

A checkpoint written here in the converter's layout (tools/prepare_olmoe.py:
85-94) is loaded into engine slots and run: routing and outputs are
bit-identical to the oracle on the same weights, for an f32 router, a BF16
router kept as BF16 and the same widened to f32.  The loader's checks
(src/int8_expert.rs:90-170) reject missing tensors, formats mixed within a
layer and non-positive scales; a slot set again by the caller releases the
loaded copy.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests import helpers
from tests.helpers import write_safetensors

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import doantotnghiepmoe_b200 as M  # noqa: E402
from doantotnghiepmoe_b200 import _lib  # noqa: E402

H, I, E, K = 256, 128, 8, 2


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def layer_tensors(l, lw, router_dtype):
    t = []
    if router_dtype == "BF16":
        t.append((f"model.layers.{l}.mlp.gate.weight", "BF16", lw.router))
    else:
        t.append((f"model.layers.{l}.mlp.gate.weight", "F32", lw.router))
    for e in range(lw.E):
        t.append((f"model.layers.{l}.mlp.experts.{e}.merged_weight", "I8", lw.experts[e]))
        t.append((f"model.layers.{l}.mlp.experts.{e}.qs", "F32", lw.scales[e]))
    return t


def bf16_layer(lw):
    bits16 = (lw.router.view(np.uint32) >> 16).astype(np.uint16)
    return O.LayerWeights(lw.H, lw.I, lw.E, lw.K, lw.norm_topk_prob, bits16, lw.experts,
                          lw.scales, router_bf16=True)


def run(eng, layer, h):
    T = h.shape[0]
    hd = torch.from_numpy(h).cuda()
    out = torch.empty_like(hd)
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    eng.forward(layer, hd, out, ids=ids)
    eng.sync_status()
    return out.cpu().numpy(), ids.cpu().numpy().astype(np.uint32)


def test_loaded_layers_bit_exact(tmp_path):
    lw0 = O.synth_layer(71, 0, H, I, E, K, False)
    lw1 = bf16_layer(O.synth_layer(71, 1, H, I, E, K, False))
    write_safetensors(tmp_path / "model-00000.safetensors", layer_tensors(0, lw0, "F32"))
    write_safetensors(tmp_path / "model-00001.safetensors", layer_tensors(1, lw1, "BF16"))
    ck = M.Checkpoint(str(tmp_path))
    eng = M.MoeLayerEngine(M.MoeConfig(H, I, E, K, False, 6, 3))
    eng.set_path(_lib.MOE_PATH_GEMV)
    eng.load_layer(ck, 0)
    eng.load_layer(ck, 1)                      # router kept as BF16
    eng.load_layer(ck, 1, layer=2, keep_bf16=False)  # widened to f32: the same values
    h = O.synth_hidden(72, 6, H)
    for layer, lw in ((0, lw0), (1, lw1)):
        ref = O.layer_forward(lw, h)
        out, ids = run(eng, layer, h)
        assert np.array_equal(ids, ref.ids)
        assert np.array_equal(bits(out), bits(ref.out))
    out2, ids2 = run(eng, 2, h)
    ref1 = O.layer_forward(lw1, h)
    assert np.array_equal(ids2, ref1.ids)
    assert np.array_equal(bits(out2), bits(ref1.out))
    # the caller replaces a loaded slot: the engine releases its copy
    ex, sc, rt = helpers.to_device(lw0)
    eng.set_layer_packed(2, ex, sc, rt)
    out3, _ = run(eng, 2, h)
    assert np.array_equal(bits(out3), bits(O.layer_forward(lw0, h).out))


def test_loader_rejects_bad_layers(tmp_path):
    lw = O.synth_layer(73, 0, H, I, E, K, False)
    eng = M.MoeLayerEngine(M.MoeConfig(H, I, E, K, False, 4, 1))
    # INT8 and INT4 experts mixed in one layer
    d = tmp_path / "mixed"
    d.mkdir()
    t = [(f"model.layers.0.mlp.gate.weight", "F32", lw.router)]
    for e in range(E):
        w = lw.experts[e][: 3 * I * H // 2].view(np.uint8) if e == 3 else lw.experts[e]
        t.append((f"model.layers.0.mlp.experts.{e}.merged_weight", "U8" if e == 3 else "I8", w))
        t.append((f"model.layers.0.mlp.experts.{e}.qs", "F32", lw.scales[e]))
    write_safetensors(d / "m.safetensors", t)
    with pytest.raises(M.MoeError) as ei:
        eng.load_layer(M.Checkpoint(str(d)), 0)
    assert ei.value.status == _lib.MOE_ERR_INVALID and "layout" in ei.value.message
    # a zero scale
    d = tmp_path / "scale"
    d.mkdir()
    sc = lw.scales.copy()
    sc[3, 5] = 0.0
    bad = O.LayerWeights(H, I, E, K, False, lw.router, lw.experts, sc)
    write_safetensors(d / "m.safetensors", layer_tensors(0, bad, "F32"))
    with pytest.raises(M.MoeError) as ei:
        eng.load_layer(M.Checkpoint(str(d)), 0)
    assert "positive" in ei.value.message
    # a missing expert
    d = tmp_path / "missing"
    d.mkdir()
    write_safetensors(d / "m.safetensors", layer_tensors(0, lw, "F32")[:-2])
    with pytest.raises(M.MoeError) as ei:
        eng.load_layer(M.Checkpoint(str(d)), 0)
    assert "missing tensor" in ei.value.message


@pytest.mark.parametrize("path", [_lib.MOE_PATH_GEMV, _lib.MOE_PATH_GEMV_PHASED])
def test_loaded_stack_with_post_attention_norm(tmp_path, path):
    """x <- x + MoE_l(RMSNorm(x) * w_l) over a 3-layer stack whose checkpoint
    carries `post_attention_layernorm.weight`: the single launch and the
    phased launches both equal the oracle bit for bit."""
    Hs, Is, Es, Ks, T = 512, 256, 16, 4, 3
    layers = []
    tensors = []
    rng = np.random.default_rng(77)
    for l in range(3):
        lw = O.synth_layer(75, l, Hs, Is, Es, Ks, False)
        lw.norm_w = (1.0 + 0.25 * rng.standard_normal(Hs)).astype(np.float32)
        layers.append(lw)
        tensors += layer_tensors(l, lw, "F32")
        tensors.append((f"model.layers.{l}.post_attention_layernorm.weight", "F32", lw.norm_w))
    write_safetensors(tmp_path / "m.safetensors", tensors)
    ck = M.Checkpoint(str(tmp_path))
    x0 = O.synth_hidden(76, T, Hs)
    for norm in (False, True):  # norm_topk_prob is per engine (a model setting)
        for lw in layers:
            lw.norm_topk_prob = norm
        ref_x, _, _ = O.stack_forward(layers, x0)
        eng = M.MoeLayerEngine(M.MoeConfig(Hs, Is, Es, Ks, norm, T, 3))
        eng.set_path(path)
        for l in range(3):
            eng.load_layer(ck, l)
        x = torch.from_numpy(x0).cuda()
        eng.stack_forward(0, 3, x, 1e-5)
        eng.sync_status()
        assert np.array_equal(bits(x.cpu().numpy()), bits(ref_x)), (path, norm)
        # without the gains the result is different (the gain is applied)
        for l in range(3):
            eng.set_layer_norm(l, None)
        x = torch.from_numpy(x0).cuda()
        eng.stack_forward(0, 3, x, 1e-5)
        eng.sync_status()
        assert not np.array_equal(bits(x.cpu().numpy()), bits(ref_x))
