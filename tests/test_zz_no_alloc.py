"""The allocation-free layer entry point (moe_layer_forward_noalloc).

It exists for callers that may not allocate GPU memory themselves -- a host
whose own allocator or VRAM budget accounts for every byte, or a decode loop
that cannot afford the device synchronisation cudaMalloc/cudaFree can cause.
This test calls it through the C ABI twice in a row (the fixed scratch array
is reused and keeps the previous call's contents) and checks each result
against the regular, allocating moe_layer_forward on the same inputs, with
the tolerance the other parity tests use.  The file is named to be collected
last, so a stop-at-first-failure run has already run every other test; it
also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests import helpers

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import doantotnghiepmoe_b200 as M  # noqa: E402
from doantotnghiepmoe_b200 import _lib  # noqa: E402

TOL = 1e-3


def _noalloc(dims, ex, sc, rt, h, resid, out, router_dtype=_lib.MOE_ROUTER_F32):
    err = ctypes.create_string_buffer(256)
    st = _lib.lib().moe_layer_forward_noalloc(
        ctypes.byref(dims), ex.data_ptr(), sc.data_ptr(), rt.data_ptr(), router_dtype,
        h.data_ptr(), None if resid is None else resid.data_ptr(), out.data_ptr(), h.shape[0],
        None, err, len(err))
    return st, err.value.decode()


def _check_twice(H, I, E, K, T, norm, seed, bf16_router=False):
    """Two calls in a row (the second with a residual), each against
    moe_layer_forward on the exact GEMV path: within TOL and bit for bit."""
    lw = O.synth_layer(seed, 0, H, I, E, K, norm)
    if bf16_router:
        rb = (lw.router.view(np.uint32) >> 16).astype(np.uint16)
        lw = O.LayerWeights(H, I, E, K, norm, rb, lw.experts, lw.scales, router_bf16=True)
    ex, sc, rt = helpers.to_device(lw)
    dims = _lib.MoeDims(H, I, E, K, int(norm), T, 1)
    eng = M.MoeLayerEngine(M.MoeConfig(H, I, E, K, norm, T, 1))
    eng.set_path(_lib.MOE_PATH_GEMV)
    eng.set_layer_packed(0, ex, sc, rt)
    rdt = _lib.MOE_ROUTER_BF16 if bf16_router else _lib.MOE_ROUTER_F32
    for call, (hseed, use_resid) in enumerate([(seed + 1, False), (seed + 2, True)]):
        h = torch.from_numpy(O.synth_hidden(hseed, T, H)).cuda()
        resid = torch.from_numpy(O.synth_hidden(hseed + 100, T, H)).cuda() if use_resid else None
        want = torch.empty_like(h)
        eng.forward(0, h, want, resid=resid)
        eng.sync_status()
        got = torch.full_like(h, float("nan"))
        st, msg = _noalloc(dims, ex, sc, rt, h, resid, got, rdt)
        assert st == _lib.MOE_OK, (call, st, msg)
        g, w = got.cpu().numpy(), want.cpu().numpy()
        assert helpers.rel_err(g, w) < TOL, call
        assert np.array_equal(g.view(np.uint32), w.view(np.uint32)), call


def test_noalloc_matches_allocating_entry_point_twice():
    assert torch.cuda.is_available()
    _check_twice(2048, 1024, 64, 8, 4, False, 77)


def test_noalloc_largest_olmoe_batch():
    """T = 84 is the largest OLMoE-shaped batch the fixed scratch holds (the
    pipelined router kernel runs from T = 16 on)."""
    _check_twice(2048, 1024, 64, 8, 84, False, 81)


def test_noalloc_bf16_router_and_odd_shapes():
    """A bf16 router, and a shape whose rows are not 8-byte multiples (the
    GEMV kernels' scalar-load variant), normalized top-k."""
    _check_twice(2048, 1024, 64, 8, 3, False, 91, bf16_router=True)
    _check_twice(250, 98, 16, 4, 5, True, 93)


def test_noalloc_rejects_oversized_call():
    H, I, E, K = 2048, 1024, 64, 8
    T = 85  # one token more than the fixed scratch holds at this shape
    dims = _lib.MoeDims(H, I, E, K, 0, T, 1)
    z8 = torch.zeros(E * 3 * I * H, dtype=torch.int8, device="cuda")
    zs = torch.zeros(E * (2 * I + H), dtype=torch.float32, device="cuda")
    zr = torch.zeros(E * H, dtype=torch.float32, device="cuda")
    h = torch.zeros((T, H), dtype=torch.float32, device="cuda")
    out = torch.empty_like(h)
    st, msg = _noalloc(dims, z8, zs, zr, h, None, out)
    assert st == _lib.MOE_ERR_INVALID
    assert "scratch" in msg
