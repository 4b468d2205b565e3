"""GPU tests of the digit decode path (MOE_PATH_DIGITS, the default for T < 12).

Routing must equal the CPU oracle bit for bit (ids and gates); outputs must be
within the 1e-3 tolerance of the oracle and bit-identical to the tensor-core
path (MOE_PATH_TENSOR), which multiplies the same int8 digit planes on the
tensor cores.  Token counts cover the single-token down phase (T = 1), the
in-CTA top-k (T <= 8) and the grid-distributed top-k (T > 8)."""
import numpy as np
import pytest

from oracle import oracle as O
from tests import helpers

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import doantotnghiepmoe_b200 as M  # noqa: E402
from doantotnghiepmoe_b200 import _lib  # noqa: E402

TOL = 1e-3


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def run(eng, h, path, resid=None):
    eng.set_path(path)
    hd = torch.from_numpy(h).cuda()
    out = torch.full_like(hd, float("nan"))
    T, K = h.shape[0], eng.cfg.top_k
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    gates = torch.empty((T, K), dtype=torch.float32, device="cuda")
    rd = None if resid is None else torch.from_numpy(resid).cuda()
    eng.profile(True)
    eng.forward(0, hd, out, resid=rd, ids=ids, gates=gates)
    eng.sync_status()
    prof = eng.profile_read()
    eng.profile(False)
    return (out.cpu().numpy(), ids.cpu().numpy().astype(np.uint32), gates.cpu().numpy(), prof)


def check(lw, h, resid=None, route_mode=None):
    T = h.shape[0]
    eng = M.MoeLayerEngine(M.MoeConfig(lw.H, lw.I, lw.E, lw.K, lw.norm_topk_prob, T, 1))
    dev = helpers.to_device(lw)
    eng.set_layer_packed(0, *dev)
    if route_mode is not None:
        eng.set_route_mode(route_mode)
    od, idd, gd, prof = run(eng, h, _lib.MOE_PATH_DIGITS, resid)
    assert "digit_decode" in prof, prof
    ot, idt, _, proft = run(eng, h, _lib.MOE_PATH_TENSOR, resid)
    assert "gate_up_tc" in proft
    if route_mode is None:
        ref = O.layer_forward(lw, h, resid=resid, nthreads=8)
        assert np.array_equal(idd, ref.ids)
        assert np.array_equal(bits(gd), bits(ref.gates))
        assert helpers.rel_err(od, ref.out) < TOL
    assert np.array_equal(idd, idt)
    assert np.array_equal(bits(od), bits(ot))
    return od


@pytest.mark.parametrize("T", [1, 2, 5, 8, 9, 16, 64])
def test_olmoe_layer(T):
    lw = O.synth_layer(601, 0, 2048, 1024, 64, 8, T % 2 == 0)
    h = O.synth_hidden(602 + T, T, 2048)
    resid = O.synth_hidden(603 + T, T, 2048) if T in (1, 9) else None
    check(lw, h, resid)


@pytest.mark.parametrize("T", [1, 64])
def test_qwen3_layer(T):
    lw = O.synth_layer(611, 0, 2048, 768, 128, 8, True)
    check(lw, O.synth_hidden(612, T, 2048))


def test_bf16_router_and_small_shapes():
    lw = O.synth_layer(621, 0, 512, 256, 16, 4, False)
    rb = (lw.router.view(np.uint32) >> 16).astype(np.uint16)
    lw = O.LayerWeights(512, 256, 16, 4, False, rb, lw.experts, lw.scales, router_bf16=True)
    check(lw, O.synth_hidden(622, 3, 512))
    lw2 = O.synth_layer(623, 0, 256, 160, 32, 2, True)  # I = 160: partial 16-byte chunks
    check(lw2, O.synth_hidden(624, 12, 256), resid=O.synth_hidden(625, 12, 256))


@pytest.mark.parametrize("T,want", [(1, "digit_decode"), (11, "digit_decode"),
                                    (12, "gate_up_tc"), (64, "gate_up_tc")])
def test_auto_path_switches_at_twelve_tokens(T, want):
    """MOE_PATH_AUTO: the single-launch digit decode below 12 tokens, the
    tensor-core GEMMs from 12 (the measured crossover on B200)."""
    lw = O.synth_layer(651, 0, 512, 256, 16, 4, True)
    eng = M.MoeLayerEngine(M.MoeConfig(512, 256, 16, 4, True, T, 1))
    eng.set_layer_packed(0, *helpers.to_device(lw))
    _, _, _, prof = run(eng, O.synth_hidden(652, T, 512), _lib.MOE_PATH_AUTO)
    assert want in prof, prof
    other = "gate_up_tc" if want == "digit_decode" else "digit_decode"
    assert other not in prof, prof


@pytest.mark.parametrize("T,want", [(4, "digit_decode"), (16, "gate_up_tc")])
def test_auto_stack_path_switches_at_twelve_tokens(T, want):
    """moe_stack_forward under MOE_PATH_AUTO follows the same switch: one
    digit launch for the stack below 12 tokens, the tensor-core layers from
    12 (never the slower exact single launch)."""
    layers = [O.synth_layer(653, l, 512, 256, 16, 4, True) for l in range(2)]
    eng = M.MoeLayerEngine(M.MoeConfig(512, 256, 16, 4, True, T, 2))
    keep = [helpers.to_device(lw) for lw in layers]
    for l, t in enumerate(keep):
        eng.set_layer_packed(l, *t)
    eng.set_path(_lib.MOE_PATH_AUTO)
    x0 = O.synth_hidden(654, T, 512)
    x = torch.from_numpy(x0).cuda()
    eng.profile(True)
    eng.stack_forward(0, 2, x, 1e-5)
    eng.sync_status()
    prof = eng.profile_read()
    eng.profile(False)
    assert want in prof and "fused_decode" not in prof, prof
    ref_x, _, _ = O.stack_forward(layers, x0, nthreads=8)
    assert helpers.rel_err(x.cpu().numpy(), ref_x) < TOL


def test_router_variant_routes_like_the_tensor_path():
    lw = O.synth_layer(631, 0, 512, 256, 16, 4, True)
    h = O.synth_hidden(632, 4, 512)
    check(lw, h, route_mode=_lib.MOE_ROUTE_TOPK_SOFTMAX)


def test_unsupported_layers_fall_back_or_refuse():
    """INT4 experts are not on the digit path: AUTO runs them on the exact
    GEMV, an explicit MOE_PATH_DIGITS refuses with MOE_ERR_STATE."""
    lw = O.synth_layer(641, 0, 256, 128, 16, 4, False)
    w4 = ((lw.experts[:, 0::2].astype(np.int16) >> 4) & 0xF) | \
         (((lw.experts[:, 1::2].astype(np.int16) >> 4) & 0xF) << 4)
    eng = M.MoeLayerEngine(M.MoeConfig(256, 128, 16, 4, False, 2, 1))
    ex = torch.from_numpy(w4.astype(np.uint8)).cuda()
    sc = torch.from_numpy(lw.scales * 16).cuda()
    rt = torch.from_numpy(lw.router).cuda()
    eng.set_layer_packed(0, ex, sc, rt)  # uint8 experts: INT4
    h = O.synth_hidden(642, 2, 256)
    _, _, _, prof = run(eng, h, _lib.MOE_PATH_AUTO)
    assert "digit_decode" not in prof
    with pytest.raises(M.MoeError) as ei:
        run(eng, h, _lib.MOE_PATH_DIGITS)
    assert ei.value.status == _lib.MOE_ERR_STATE


_STACK = {}


def olmoe_layers(n):
    if len(_STACK.get("layers", [])) < n:
        _STACK["layers"] = [O.synth_layer(651, l, 2048, 1024, 64, 8, False) for l in range(n)]
    return _STACK["layers"][:n]


@pytest.mark.parametrize("T", [1, 8, 32])
def test_olmoe_stack_16_layers(T):
    """The configs[2] stack (16 layers, RMSNorm + residual) in one launch:
    bit-identical to the tensor-core stack, within 1e-3 of the oracle after
    16 layers, and each layer routes the oracle's own input bit-exactly."""
    layers = olmoe_layers(16)
    x0 = O.synth_hidden(660 + T, T, 2048)
    eng = M.MoeLayerEngine(M.MoeConfig(2048, 1024, 64, 8, False, T, 16))
    keep = [helpers.to_device(lw) for lw in layers]
    for l, t in enumerate(keep):
        eng.set_layer_packed(l, *t)
    out = {}
    for path in (_lib.MOE_PATH_DIGITS, _lib.MOE_PATH_TENSOR):
        eng.set_path(path)
        x = torch.from_numpy(x0).cuda()
        eng.profile(True)
        eng.stack_forward(0, 16, x, 1e-5)
        eng.sync_status()
        prof = eng.profile_read()
        eng.profile(False)
        assert ("digit_decode" in prof) == (path == _lib.MOE_PATH_DIGITS), prof
        out[path] = x.cpu().numpy()
    assert np.array_equal(bits(out[_lib.MOE_PATH_DIGITS]), bits(out[_lib.MOE_PATH_TENSOR]))
    ref_x, _, _ = O.stack_forward(layers, x0, nthreads=8)
    assert helpers.rel_err(out[_lib.MOE_PATH_DIGITS], ref_x) < TOL
    # per layer, on the oracle's own input: routing bit-exact
    eng.set_path(_lib.MOE_PATH_DIGITS)
    xl = x0.copy()
    ids = torch.empty((T, 8), dtype=torch.int32, device="cuda")
    for l, lw in enumerate(layers):
        h = np.stack([O.rms_norm(row, 1e-5) for row in xl])
        ref = O.layer_forward(lw, h, resid=xl, nthreads=8)
        hd = torch.from_numpy(h).cuda()
        od = torch.empty_like(hd)
        eng.forward(l, hd, od, resid=torch.from_numpy(xl).cuda(), ids=ids)
        eng.sync_status()
        assert np.array_equal(ids.cpu().numpy().astype(np.uint32), ref.ids), l
        assert helpers.rel_err(od.cpu().numpy(), ref.out) < TOL, l
        xl = ref.out


def test_topk_ties_and_router_kat_on_the_digit_path():
    """The reference's top-k tie cases (src/olmoe.rs:6496-6543) and the
    learned-router KAT (src/router.rs:118-140) through the digit launch's own
    router and rank-based top-k.  Rows are padded to 16 with zeros: the
    hidden state is e_0 (plus the KAT's second component), so the logits are
    the cases' values exactly."""
    H, I = 16, 16
    cases = helpers.unit_cases()
    for case in cases["topk_ties"]:
        vals = np.array(case["values"], np.float32)
        router = np.zeros((64, H), np.float32)
        router[:, 0] = vals
        lw = O.LayerWeights(H, I, 64, 8, False, router, np.zeros((64, 3 * H * I), np.int8),
                            np.ones((64, 2 * I + H), np.float32))
        eng = M.MoeLayerEngine(M.MoeConfig(H, I, 64, 8, False, 1, 1))
        eng.set_layer_packed(0, *helpers.to_device(lw))
        h = np.zeros((1, H), np.float32)
        h[0, 0] = 1.0
        _, ids, _, prof = run(eng, h, _lib.MOE_PATH_DIGITS)
        assert "digit_decode" in prof
        assert list(ids[0]) == case["expected"]
    kat = cases["router_kat"]
    router = np.zeros((3, H), np.float32)
    router[:, :2] = np.array(kat["weights"], np.float32).reshape(3, 2)
    lw = O.LayerWeights(H, I, 3, 2, False, router, np.zeros((3, 3 * H * I), np.int8),
                        np.ones((3, 2 * I + H), np.float32))
    eng = M.MoeLayerEngine(M.MoeConfig(H, I, 3, 2, False, 1, 1))
    eng.set_layer_packed(0, *helpers.to_device(lw))
    eng.set_route_mode(_lib.MOE_ROUTE_TOPK_SOFTMAX)
    h = np.zeros((1, H), np.float32)
    h[0, :2] = kat["hidden"]
    _, ids, gates, _ = run(eng, h, _lib.MOE_PATH_DIGITS)
    assert list(ids[0]) == kat["ids"]
    assert np.array_equal(bits(gates[0]), bits(np.array(kat["gates"], np.float32)))
