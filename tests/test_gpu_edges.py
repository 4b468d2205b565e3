"""Empty batches through every entry point.

The reference accepts empty slices: `GpuExpertKernels::forward` /
`forward_pairs` pass their count checks with no experts and launch nothing
(src/gpu_expert.rs:366-403).  The C ABI does the same for T = 0 with valid
pointers -- a Rust caller's empty `Vec` has a non-null pointer -- on every
path: it returns MOE_OK, launches nothing and writes nothing.  Null
pointers stay an argument error even then.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests import helpers

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import doantotnghiepmoe_b200 as M  # noqa: E402
from doantotnghiepmoe_b200 import _lib  # noqa: E402

H, I, E, K = 256, 128, 16, 4


@pytest.mark.parametrize("path", [_lib.MOE_PATH_AUTO, _lib.MOE_PATH_GEMV,
                                  _lib.MOE_PATH_GEMV_PHASED, _lib.MOE_PATH_DIGITS,
                                  _lib.MOE_PATH_TENSOR])
def test_empty_batch_is_a_no_op(path):
    lw = O.synth_layer(231, 0, H, I, E, K, False)
    eng = M.MoeLayerEngine(M.MoeConfig(H, I, E, K, False, 4, 1))
    eng.set_path(path)
    dev = helpers.to_device(lw)
    eng.set_layer_packed(0, *dev)
    L = _lib.lib()
    x = torch.full((1, H), 7.0, device="cuda")
    out = torch.full((1, H), -3.0, device="cuda")
    ids = torch.full((1, K), 99, dtype=torch.int32, device="cuda")
    gates = torch.full((1, K), -1.0, device="cuda")
    eng.profile(True)
    assert L.moe_layer_forward(eng._h, 0, x.data_ptr(), None, out.data_ptr(), 0,
                               ids.data_ptr(), gates.data_ptr(), None) == _lib.MOE_OK
    assert L.moe_stack_forward(eng._h, 0, 1, out.data_ptr(), 0, 1e-5, None) == _lib.MOE_OK
    assert L.moe_route(eng._h, 0, x.data_ptr(), 0, ids.data_ptr(), gates.data_ptr(), None,
                       None) == _lib.MOE_OK
    hx = np.full((1, H), 7.0, np.float32)
    ho = np.full((1, H), -3.0, np.float32)
    assert L.moe_layer_forward_host(eng._h, 0, hx.ctypes.data, None, ho.ctypes.data, 0,
                                    None, None) == _lib.MOE_OK
    eng.sync_status()
    torch.cuda.synchronize()
    assert eng.profile_read() == {}  # nothing launched
    eng.profile(False)
    assert bool((out == -3.0).all()) and bool((ids == 99).all()) and bool((gates == -1.0).all())
    assert np.all(ho == -3.0)
    # null pointers are still an argument error at T = 0
    assert L.moe_layer_forward(eng._h, 0, None, None, out.data_ptr(), 0, None, None,
                               None) == _lib.MOE_ERR_INVALID


def test_expert_kernels_with_no_experts():
    """forward / forward_pairs with no experts return without a launch."""
    k = M.GpuExpertKernels.init(H, I, 4)
    x = np.ones(H, np.float32)
    k.forward([], x, [])
    k.forward_pairs([], [], [])
    k.close()
