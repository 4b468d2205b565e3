"""Launch-graph replay (moe_set_graphs): a replayed call must compute on the
buffers' current contents and equal direct launches bit for bit, across the
tensor-core path, the exact GEMV path and stacks; changing a layer's weights
must drop the captured graphs."""
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


@pytest.mark.parametrize("path,T", [(_lib.MOE_PATH_TENSOR, 256), (_lib.MOE_PATH_GEMV, 3),
                                    (_lib.MOE_PATH_GEMV_PHASED, 40), (_lib.MOE_PATH_DIGITS, 3),
                                    (_lib.MOE_PATH_DIGITS, 1)])
def test_replay_equals_direct(path, T):
    H, I, E, K = 512, 256, 32, 4
    lw = O.synth_layer(501, 0, H, I, E, K, True)
    eng = M.MoeLayerEngine(M.MoeConfig(H, I, E, K, True, T, 1))
    t = helpers.to_device(lw)
    eng.set_layer_packed(0, *t)
    eng.set_path(path)
    hd = torch.empty((T, H), dtype=torch.float32, device="cuda")
    out = torch.empty_like(hd)
    for rep in range(3):  # capture, then replays on new data in the same buffers
        h = O.synth_hidden(510 + rep, T, H)
        hd.copy_(torch.from_numpy(h))
        eng.set_graphs(True)
        eng.forward(0, hd, out)
        eng.sync_status()
        g = out.cpu().numpy().copy()
        eng.set_graphs(False)
        eng.forward(0, hd, out)
        eng.sync_status()
        d = out.cpu().numpy()
        assert np.array_equal(bits(g), bits(d)), rep
        ref = O.layer_forward(lw, h)
        if path in (_lib.MOE_PATH_TENSOR, _lib.MOE_PATH_DIGITS):
            assert helpers.rel_err(g, ref.out) < 1e-3
        else:
            assert np.array_equal(bits(g), bits(ref.out))


def test_replay_follows_new_weights_and_stacks():
    H, I, E, K, T = 512, 256, 16, 4, 2
    layers = [O.synth_layer(520 + l, 0, H, I, E, K, False) for l in range(2)]
    eng = M.MoeLayerEngine(M.MoeConfig(H, I, E, K, False, T, 1))
    eng.set_path(_lib.MOE_PATH_GEMV)
    x0 = O.synth_hidden(530, T, H)
    hd = torch.from_numpy(x0).cuda()
    out = torch.empty_like(hd)
    keep = []
    for lw in layers:  # same buffers, new weights: the captured graph must go
        t = helpers.to_device(lw)
        keep.append(t)
        eng.set_layer_packed(0, *t)
        for _ in range(2):
            eng.forward(0, hd, out)
        eng.sync_status()
        assert np.array_equal(bits(out.cpu().numpy()), bits(O.layer_forward(lw, x0).out))
    # a two-layer stack replayed twice from the same input
    eng2 = M.MoeLayerEngine(M.MoeConfig(H, I, E, K, False, T, 2))
    eng2.set_path(_lib.MOE_PATH_GEMV)
    for l, t in enumerate(keep):
        eng2.set_layer_packed(l, *t)
    ref_x, _, _ = O.stack_forward(layers, x0)
    x = torch.empty_like(hd)
    for _ in range(2):
        x.copy_(hd)
        eng2.stack_forward(0, 2, x, 1e-5)
        eng2.sync_status()
        assert np.array_equal(bits(x.cpu().numpy()), bits(ref_x))
