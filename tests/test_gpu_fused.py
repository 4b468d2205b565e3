"""GPU tests of the single-launch exact decode kernel (MOE_PATH_GEMV).  It
uses the phased kernels' arithmetic, so everything is compared bit for bit:
against the oracle and against MOE_PATH_GEMV_PHASED."""
import numpy as np
import pytest

from oracle import oracle as O
from tests import helpers

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import doantotnghiepmoe_b200 as M  # noqa: E402
from doantotnghiepmoe_b200 import _lib  # noqa: E402

KERNELS = [(_lib.MOE_PATH_GEMV, "fused_decode")]


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def layer_out(eng, h, path, resid=None):
    eng.set_path(path)
    hd = torch.from_numpy(h).cuda()
    out = torch.empty_like(hd)
    ids = torch.empty((h.shape[0], eng.cfg.top_k), dtype=torch.int32, device="cuda")
    gates = torch.empty((h.shape[0], eng.cfg.top_k), dtype=torch.float32, device="cuda")
    rd = None if resid is None else torch.from_numpy(resid).cuda()
    eng.profile(True)
    eng.forward(0, hd, out, resid=rd, ids=ids, gates=gates)
    eng.sync_status()
    prof = eng.profile_read()
    eng.profile(False)
    return out.cpu().numpy(), ids.cpu().numpy().astype(np.uint32), gates.cpu().numpy(), prof


def check_layer(lw, h, resid, path, kernel, cfg):
    ref = O.layer_forward(lw, h, resid=resid)
    eng = M.MoeLayerEngine(cfg)
    t = helpers.to_device(lw)
    eng.set_layer_packed(0, *t)
    of, idf, gf, pf = layer_out(eng, h, path, resid)
    assert kernel in pf, pf
    assert np.array_equal(idf, ref.ids)
    assert np.array_equal(bits(gf), bits(ref.gates))
    assert np.array_equal(bits(of), bits(ref.out))
    return eng, of


@pytest.mark.parametrize("path,kernel", KERNELS)
@pytest.mark.parametrize("T", [1, 5, 16])
def test_single_launch_equals_phased_and_oracle(T, path, kernel):
    lw = O.synth_layer(201, 0, 2048, 1024, 64, 8, T == 5)
    h = O.synth_hidden(201, T, 2048)
    resid = O.synth_hidden(202, T, 2048) if T == 16 else None
    cfg = M.MoeConfig(2048, 1024, 64, 8, T == 5, T, 1)
    eng, of = check_layer(lw, h, resid, path, kernel, cfg)
    op, _, _, pp = layer_out(eng, h, _lib.MOE_PATH_GEMV_PHASED, resid)
    assert "fused_decode" not in pp
    assert np.array_equal(bits(of), bits(op))


_QWEN = {}


def qwen_stack():
    if not _QWEN:
        layers = [O.synth_layer(211, l, 2048, 768, 128, 8, True) for l in range(2)]
        x0 = O.synth_hidden(211, 64, 2048)
        ref_x, _, _ = O.stack_forward(layers, x0, nthreads=8)
        _QWEN.update(layers=layers, x0=x0, ref=ref_x)
    return _QWEN


@pytest.mark.parametrize("path,kernel", KERNELS)
def test_qwen3_stack_t64(path, kernel):
    """Qwen3-shaped decode (H=2048, I=768, E=128, K=8, normalized), T=64, two
    stacked layers with RMSNorm + residual: bit-exact after both layers."""
    q = qwen_stack()
    eng = M.MoeLayerEngine(M.MoeConfig(2048, 768, 128, 8, True, 64, 2))
    keep = []
    for l, lw in enumerate(q["layers"]):
        t = helpers.to_device(lw)
        keep.append(t)
        eng.set_layer_packed(l, *t)
    eng.set_path(path)
    x = torch.from_numpy(q["x0"]).cuda()
    eng.profile(True)
    eng.stack_forward(0, 2, x, 1e-5)
    eng.sync_status()
    assert kernel in eng.profile_read()
    xg = x.cpu().numpy()
    assert helpers.rel_err(xg, q["ref"]) < 1e-3
    assert np.array_equal(bits(xg), bits(q["ref"]))


@pytest.mark.parametrize("path,kernel", KERNELS)
def test_router_variant_and_repeat_calls(path, kernel):
    """Router::select_top_k semantics through the single-launch kernels, and
    repeated calls (counters must come back clean)."""
    lw = O.synth_layer(221, 0, 256, 128, 16, 4, True)
    eng = M.MoeLayerEngine(M.MoeConfig(256, 128, 16, 4, True, 8, 1))
    ex, sc, rt = helpers.to_device(lw)
    eng.set_layer_packed(0, ex, sc, rt)
    eng.set_route_mode(_lib.MOE_ROUTE_TOPK_SOFTMAX)
    for rep in range(3):
        h = O.synth_hidden(222 + rep, 8, 256)
        _, ids, gates, prof = layer_out(eng, h, path)
        assert kernel in prof
        for t in range(8):
            scores = np.array([O.lib().oracle_dot_seq(lw.router[e].ctypes.data,
                                                      h[t].ctypes.data, 256)
                               for e in range(16)], np.float32)
            rid, rg = O.select_topk_then_softmax(scores, 4)
            assert np.array_equal(ids[t], rid)
            assert np.array_equal(bits(gates[t]), bits(rg))
