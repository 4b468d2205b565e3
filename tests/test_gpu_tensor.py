"""GPU tests of the tensor-core (tcgen05) expert path used for prefill-sized
batches: routing stays bit-exact (it is the same router), the layer output
must stay within the 1e-3 relative tolerance of the CPU path."""
import numpy as np
import pytest

from oracle import oracle as O
from tests import helpers

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import doantotnghiepmoe_b200 as M  # noqa: E402
from doantotnghiepmoe_b200 import _lib  # noqa: E402

TOL = 1e-3


def run_tensor(lw, h, resid=None, path=_lib.MOE_PATH_TENSOR):
    T = h.shape[0]
    eng = M.MoeLayerEngine(M.MoeConfig(lw.H, lw.I, lw.E, lw.K, lw.norm_topk_prob, T, 1))
    ex, sc, rt = helpers.to_device(lw)
    eng.set_layer_packed(0, ex, sc, rt)
    eng.set_path(path)
    hd = torch.from_numpy(h).cuda()
    rd = None if resid is None else torch.from_numpy(resid).cuda()
    out = torch.empty_like(hd)
    ids = torch.empty((T, lw.K), dtype=torch.int32, device="cuda")
    eng.forward(0, hd, out, resid=rd, ids=ids)
    eng.sync_status()
    return out.cpu().numpy(), ids.cpu().numpy().astype(np.uint32), eng


@pytest.mark.parametrize("T", [512, 37])
def test_olmoe_prefill_tensor_path(T):
    lw = O.synth_layer(101, 0, 2048, 1024, 64, 8, False)
    h = O.synth_hidden(101, T, 2048)
    ref = O.layer_forward(lw, h, nthreads=8)
    out, ids, _ = run_tensor(lw, h)
    assert np.array_equal(ids, ref.ids)
    err = helpers.rel_err(out, ref.out)
    assert err < TOL, err


def test_qwen3_prefill_tensor_path_with_residual():
    lw = O.synth_layer(103, 0, 2048, 768, 128, 8, True)
    h = O.synth_hidden(103, 256, 2048)
    resid = O.synth_hidden(104, 256, 2048)
    ref = O.layer_forward(lw, h, resid=resid, nthreads=8)
    out, ids, _ = run_tensor(lw, h, resid)
    assert np.array_equal(ids, ref.ids)
    err = helpers.rel_err(out - resid, ref.out - resid)  # the MoE part alone
    assert err < TOL, err


@pytest.mark.parametrize("T,E,K", [(256, 64, 8), (2100, 16, 4)])
def test_tensor_path_tile_list_from_permutation(T, E, K):
    """The permutation writes the tensor-core tile list itself: one CTA up to
    2048 routes (here exactly 2048), the multi-CTA sort above (8400 routes,
    about 9 tiles per expert); the per-token digit planes land at every
    route's sorted row."""
    lw = O.synth_layer(107, 0, 256, 128, E, K, False)
    h = O.synth_hidden(107, T, 256)
    ref = O.layer_forward(lw, h, nthreads=8)
    out, ids, _ = run_tensor(lw, h)
    assert np.array_equal(ids, ref.ids)
    err = helpers.rel_err(out, ref.out)
    assert err < TOL, err


def test_auto_path_picks_tensor_cores_for_prefill():
    lw = O.synth_layer(105, 0, 256, 128, 16, 4, False)
    h = O.synth_hidden(105, 256, 256)
    ref = O.layer_forward(lw, h)
    out, ids, eng = run_tensor(lw, h, path=_lib.MOE_PATH_AUTO)
    eng.profile(True)
    hd = torch.from_numpy(h).cuda()
    o2 = torch.empty_like(hd)
    eng.forward(0, hd, o2)
    prof = eng.profile_read()
    assert "gate_up_tc" in prof and "down_tc" in prof
    assert np.array_equal(ids, ref.ids)
    assert helpers.rel_err(out, ref.out) < TOL


def test_tensor_path_unavailable_is_an_error():
    # I = 8 is not a multiple of 16: no tensor map, so forcing the path fails
    meta, layers = helpers.load_fixture("olmoe_unnormalized-mha")
    lw, case = layers[0]
    with pytest.raises(M.MoeError) as ei:
        run_tensor(lw, case["h"])
    assert ei.value.status == _lib.MOE_ERR_STATE
