"""GPU parity tests: the CUDA path (through the C ABI) against the oracle and
the committed golden vectors.  Bit-exact for routing and for the GEMV expert
path; the reference tolerance (max relative error 1e-3 over the layer output,
defined as max|gpu - cpu| / max|cpu| as in src/gpu_expert.rs:566-575) is
asserted as well so a failure says by how much."""
import ctypes

import os

import numpy as np
import pytest

from oracle import oracle as O
from tests import helpers
from tests.golden import generators as G

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import doantotnghiepmoe_b200 as M  # noqa: E402
from doantotnghiepmoe_b200 import _lib  # noqa: E402

TOL = 1e-3


def engine_for(lw, max_tokens, num_layers=1, path=_lib.MOE_PATH_GEMV):
    """An engine on the exact path by default: these tests compare bits."""
    cfg = M.MoeConfig(lw.H, lw.I, lw.E, lw.K, lw.norm_topk_prob, max_tokens, num_layers)
    eng = M.MoeLayerEngine(cfg)
    eng.set_path(path)
    return eng


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    assert torch.cuda.is_available(), "GPU tests need CUDA"
    torch.cuda.init()


def test_device_expf_equals_host_expf():
    """The softmax exponential on the GPU equals libm expf bit for bit, on
    contiguous runs of float inputs spread over the softmax domain [-104, 0]
    (the exhaustive CPU comparison of the same method is in golden/pins.json)."""
    chunk = 1 << 24
    out = torch.empty(chunk, dtype=torch.float32, device="cuda")
    for start in (0x80000000, 0xBC000000, 0xBF000000, 0xBF800000, 0xC0800000, 0xC1F00000,
                  0xC2B00000, 0xC2C80000):
        assert _lib.lib().moe_debug_expf(start, chunk, out.data_ptr(), None) == 0
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        ref = O.expf_libm_range(start, chunk)
        bad = np.flatnonzero(bits(got) != bits(ref))
        assert bad.size == 0, (hex(start), bad[:5])


@pytest.mark.parametrize("name", helpers.FIXTURES)
def test_fixture_layers_bit_exact(name):
    meta, layers = helpers.load_fixture(name)
    for lw, case in layers:
        T = case["h"].shape[0]
        eng = engine_for(lw, T)
        ex, sc, rt = helpers.to_device(lw)
        eng.set_layer_packed(0, ex, sc, rt)
        h = torch.from_numpy(case["h"]).cuda()
        out = torch.empty_like(h)
        ids = torch.empty((T, lw.K), dtype=torch.int32, device="cuda")
        gates = torch.empty((T, lw.K), dtype=torch.float32, device="cuda")
        eng.forward(0, h, out, ids=ids, gates=gates)
        eng.sync_status()
        assert np.array_equal(ids.cpu().numpy().astype(np.uint32), case["ids"])
        assert np.array_equal(bits(gates.cpu().numpy()), bits(case["gates"]))
        o = out.cpu().numpy()
        assert helpers.rel_err(o, case["out"]) < TOL
        assert np.array_equal(bits(o), bits(case["out"]))
        # permutation (expert_uses) is index work: bit-exact
        seg = torch.empty(lw.E + 1, dtype=torch.int32, device="cuda")
        rtok = torch.empty(T * lw.K, dtype=torch.int32, device="cuda")
        rslot = torch.empty(T * lw.K, dtype=torch.int32, device="cuda")
        eng.route_permute(0, h, ids, gates, seg, rtok, rslot)
        torch.cuda.synchronize()
        assert np.array_equal(seg.cpu().numpy(), case["seg_off"])
        assert np.array_equal(rtok.cpu().numpy(), case["use_token"])
        assert np.array_equal(rslot.cpu().numpy(), case["use_slot"])


@pytest.mark.parametrize("T,norm", [(1, False), (8, False), (3, True)])
def test_olmoe_layer_bit_exact(T, norm):
    """OLMoE-shaped layer (H=2048, I=1024, E=64, K=8), seeded synthetic inputs."""
    lw = O.synth_layer(11, 0, 2048, 1024, 64, 8, norm)
    h = O.synth_hidden(11, T, 2048)
    ref = O.layer_forward(lw, h)
    eng = engine_for(lw, T)
    ex, sc, rt = helpers.to_device(lw)
    eng.set_layer_packed(0, ex, sc, rt)
    hd = torch.from_numpy(h).cuda()
    out = torch.empty_like(hd)
    ids = torch.empty((T, 8), dtype=torch.int32, device="cuda")
    gates = torch.empty((T, 8), dtype=torch.float32, device="cuda")
    eng.forward(0, hd, out, ids=ids, gates=gates)
    eng.sync_status()
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), ref.ids)
    assert np.array_equal(bits(gates.cpu().numpy()), bits(ref.gates))
    o = out.cpu().numpy()
    assert helpers.rel_err(o, ref.out) < TOL
    assert np.array_equal(bits(o), bits(ref.out))


def test_device_synth_matches_host_generator():
    H, I = 256, 96
    w = torch.empty(3 * H * I, dtype=torch.int8, device="cuda")
    s = torch.empty(2 * I + H, dtype=torch.float32, device="cuda")
    M.synth_expert(5, 2, 3, H, I, w, s)
    torch.cuda.synchronize()
    hw, hs = O.synth_expert(5, 2, 3, H, I)
    assert np.array_equal(w.cpu().numpy(), hw)
    assert np.array_equal(bits(s.cpu().numpy()), bits(hs))


@pytest.mark.parametrize("h,i", [(2048, 1024), (16, 8), (6, 10)])
def test_gpu_expert_kernels_match_cpu(h, i):
    """src/gpu_expert.rs:532-581 replayed: GpuExpertKernels::forward vs CPU
    Int8Expert::forward, rel < 1e-4 (here: bit-exact), and a wrong output
    count is rejected."""
    k = M.GpuExpertKernels.init(h, i, 2)
    x = G.gpu_expert_input(h)
    experts, expected, keep = [], [], []
    for seed in (1, 2):
        w, s = G.gpu_expert_weights(h, i, seed + h)
        wd = torch.from_numpy(w).cuda()
        sd = torch.from_numpy(s).cuda()
        keep += [wd, sd]
        experts.append(M.GpuExpertWeights.from_tensors(wd, sd))
        expected.append(O.expert_forward(w, s, h, i, x)[1])
    outs = [np.zeros(h, np.float32) for _ in range(2)]
    k.forward(experts, x, outs)
    for got, exp in zip(outs, expected):
        assert helpers.rel_err(got, exp) < 1e-4
        assert np.array_equal(bits(got), bits(exp))
    with pytest.raises(M.MoeError):
        k.forward(experts, x, outs[:1])
    # pairs with distinct inputs (the prefill use, src/olmoe.rs:3534-3566)
    x2 = [x, (x * np.float32(0.5)).astype(np.float32)]
    k.forward_pairs(experts, x2, outs)
    for j in range(2):
        w, s = G.gpu_expert_weights(h, i, j + 1 + h)
        assert np.array_equal(bits(outs[j]), bits(O.expert_forward(w, s, h, i, x2[j])[1]))
    k.close()


@pytest.mark.parametrize("h,i,seed", [(7, 5, 17), (32, 9, 73), (33, 17, 991), (2048, 1024, 17)])
def test_xorshift64_cases_bit_exact(h, i, seed):
    """Odd shapes of src/int8_expert.rs:1284-1300 (tails, leftover 8-chunks)."""
    z = np.load(helpers.os.path.join(helpers.GOLDEN, "expert_cases.npz"))
    w, s, x = G.gate_up_case(h, i, seed)
    k = M.GpuExpertKernels.init(h, i, 1)
    wd, sd = torch.from_numpy(w).cuda(), torch.from_numpy(s).cuda()
    out = [np.zeros(h, np.float32)]
    k.forward([M.GpuExpertWeights.from_tensors(wd, sd)], x, out)
    assert np.array_equal(bits(out[0]), bits(z[f"x64_{h}_{i}_{seed}"]))
    k.close()


def test_topk_ties_and_router_variant():
    cases = helpers.unit_cases()
    for case in cases["topk_ties"]:
        vals = np.array(case["values"], np.float32)
        # H = 1, h = [1]: logits equal the values exactly
        lw = O.LayerWeights(1, 1, 64, 8, False, vals.reshape(64, 1).copy(),
                            np.ones((64, 3), np.int8), np.ones((64, 3), np.float32))
        eng = engine_for(lw, 1)
        ex, sc, rt = helpers.to_device(lw)
        eng.set_layer_packed(0, ex, sc, rt)
        hd = torch.ones((1, 1), dtype=torch.float32, device="cuda")
        ids = torch.empty((1, 8), dtype=torch.int32, device="cuda")
        gates = torch.empty((1, 8), dtype=torch.float32, device="cuda")
        eng.route(0, hd, ids, gates)
        torch.cuda.synchronize()
        assert list(ids.cpu().numpy()[0]) == case["expected"]
    kat = cases["router_kat"]
    lw = O.LayerWeights(2, 1, 3, 2, False, np.array(kat["weights"], np.float32).reshape(3, 2),
                        np.ones((3, 6), np.int8), np.ones((3, 4), np.float32))
    eng = engine_for(lw, 1)
    ex, sc, rt = helpers.to_device(lw)
    eng.set_layer_packed(0, ex, sc, rt)
    eng.set_route_mode(_lib.MOE_ROUTE_TOPK_SOFTMAX)
    hd = torch.tensor([kat["hidden"]], dtype=torch.float32, device="cuda")
    ids = torch.empty((1, 2), dtype=torch.int32, device="cuda")
    gates = torch.empty((1, 2), dtype=torch.float32, device="cuda")
    eng.route(0, hd, ids, gates)
    torch.cuda.synchronize()
    assert list(ids.cpu().numpy()[0]) == kat["ids"]
    assert np.array_equal(bits(gates.cpu().numpy()[0]), bits(np.array(kat["gates"], np.float32)))


def test_topk_softmax_variant_random():
    lw = O.synth_layer(21, 0, 128, 32, 16, 4, True)
    h = O.synth_hidden(21, 6, 128)
    eng = engine_for(lw, 6)
    ex, sc, rt = helpers.to_device(lw)
    eng.set_layer_packed(0, ex, sc, rt)
    eng.set_route_mode(_lib.MOE_ROUTE_TOPK_SOFTMAX)
    ids = torch.empty((6, 4), dtype=torch.int32, device="cuda")
    gates = torch.empty((6, 4), dtype=torch.float32, device="cuda")
    eng.route(0, torch.from_numpy(h).cuda(), ids, gates)
    torch.cuda.synchronize()
    for t in range(6):
        scores = np.array([O.lib().oracle_dot_seq(lw.router[e].ctypes.data, h[t].ctypes.data, 128)
                           for e in range(16)], np.float32)
        rid, rg = O.select_topk_then_softmax(scores, 4)
        assert np.array_equal(ids.cpu().numpy()[t].astype(np.uint32), rid)
        assert np.array_equal(bits(gates.cpu().numpy()[t]), bits(rg))


def test_stacked_decode_bit_exact():
    """Four OLMoE-shaped layers, T=8: x <- x + MoE(RMSNorm(x)) per layer."""
    layers = [O.synth_layer(31, l, 2048, 1024, 64, 8, False) for l in range(4)]
    x0 = O.synth_hidden(31, 8, 2048)
    ref_x, ref_ids, _ = O.stack_forward(layers, x0)
    cfg = M.MoeConfig(2048, 1024, 64, 8, False, 8, 4)
    eng = M.MoeLayerEngine(cfg)
    eng.set_path(_lib.MOE_PATH_GEMV)
    keep = []
    for l, lw in enumerate(layers):
        ex, sc, rt = helpers.to_device(lw)
        keep.append((ex, sc, rt))
        eng.set_layer_packed(l, ex, sc, rt)
    x = torch.from_numpy(x0).cuda()
    eng.stack_forward(0, 4, x, 1e-5)
    eng.sync_status()
    xg = x.cpu().numpy()
    assert helpers.rel_err(xg, ref_x) < TOL
    assert np.array_equal(bits(xg), bits(ref_x))


def test_host_variant_and_residual():
    lw = O.synth_layer(41, 0, 512, 256, 16, 4, True)
    h = O.synth_hidden(41, 5, 512)
    resid = O.synth_hidden(42, 5, 512)
    ref = O.layer_forward(lw, h, resid=resid)
    eng = engine_for(lw, 5)
    ex, sc, rt = helpers.to_device(lw)
    eng.set_layer_packed(0, ex, sc, rt)
    out, ids, gates = eng.forward_host(0, h, resid)
    assert np.array_equal(ids, ref.ids)
    assert np.array_equal(bits(out), bits(ref.out))


def test_host_buffers_pinned_and_staged():
    """moe_layer_forward_host DMAs pinned buffers directly and stages pageable
    ones in chunks (2.4 MB here: three chunks); every mix gives the device
    call's bits."""
    lw = O.synth_layer(43, 0, 2048, 256, 8, 2, False)
    T = 300
    h = O.synth_hidden(43, T, 2048)
    resid = O.synth_hidden(44, T, 2048)
    eng = engine_for(lw, T, path=_lib.MOE_PATH_AUTO)
    ex, sc, rt = helpers.to_device(lw)
    eng.set_layer_packed(0, ex, sc, rt)
    hd, rd = torch.from_numpy(h).cuda(), torch.from_numpy(resid).cuda()
    od = torch.empty_like(hd)
    idd = torch.empty((T, 2), dtype=torch.int32, device="cuda")
    eng.forward(0, hd, od, resid=rd, ids=idd)
    eng.sync_status()
    want, want_ids = od.cpu().numpy(), idd.cpu().numpy().astype(np.uint32)
    ref = O.layer_forward(lw, h, resid=resid)
    assert np.array_equal(want_ids, ref.ids)
    assert helpers.rel_err(want, ref.out) < 1e-3

    def pinned(a):
        return torch.from_numpy(np.ascontiguousarray(a)).pin_memory().numpy()

    def lib_pinned(a):
        buf = M.host_empty(a.shape, a.dtype)
        buf[:] = a
        return buf

    for pin_in, pin_out in ((False, False), (True, True), (True, False), (False, True),
                            (lib_pinned, lib_pinned)):
        mk_in = pin_in if callable(pin_in) else (pinned if pin_in else np.copy)
        mk_out = pin_out if callable(pin_out) else (pinned if pin_out else np.copy)
        hi, ri = mk_in(h), mk_in(resid)
        out = mk_out(np.zeros_like(h))
        ids_buf = mk_out(np.zeros((T, 2), np.uint32))
        got, ids, _ = eng.forward_host(0, hi, ri, out=out, ids=ids_buf)
        assert got is out and ids is ids_buf
        assert np.array_equal(ids, want_ids)
        assert np.array_equal(bits(got), bits(want)), (pin_in, pin_out)
    with pytest.raises(ValueError):
        eng.forward_host(0, h, out=np.zeros((T, 2047), np.float32))


def test_host_call_in_token_chunks_matches_whole_batch():
    """At T >= 2048 the host-buffer call pipelines token chunks (copy in,
    layer, copy out on three streams).  Chunks of a token-independent layer
    give the whole batch's bits: 4000 tokens in three chunks, the last one
    shorter, pinned and pageable buffers, with a residual."""
    lw = O.synth_layer(45, 0, 2048, 256, 8, 2, True)
    T = 4000
    h = O.synth_hidden(45, T, 2048)
    resid = O.synth_hidden(46, T, 2048)
    eng = engine_for(lw, T, path=_lib.MOE_PATH_AUTO)
    ex, sc, rt = helpers.to_device(lw)
    eng.set_layer_packed(0, ex, sc, rt)
    hd, rd = torch.from_numpy(h).cuda(), torch.from_numpy(resid).cuda()
    od = torch.empty_like(hd)
    idd = torch.empty((T, 2), dtype=torch.int32, device="cuda")
    gd = torch.empty((T, 2), dtype=torch.float32, device="cuda")
    eng.forward(0, hd, od, resid=rd, ids=idd, gates=gd)
    eng.sync_status()
    whole_launches = eng.last_launch_count()
    want = od.cpu().numpy()
    want_ids = idd.cpu().numpy().astype(np.uint32)
    want_gates = gd.cpu().numpy()
    rows = np.arange(0, T, 97)
    ref = O.layer_forward(lw, h[rows], resid=resid[rows])
    assert np.array_equal(want_ids[rows], ref.ids)
    assert helpers.rel_err(want[rows], ref.out) < 1e-3
    chunked = os.environ.get("MOE_HOST_CHUNK", "1024") != "0"
    for pin in (True, False):
        def mk(a):
            if not pin:
                return np.copy(a)
            buf = M.host_empty(a.shape, a.dtype)
            buf[:] = a
            return buf
        out = mk(np.zeros_like(h))
        for _ in range(2):  # the second call replays the chunks' graphs
            got, ids, gates = eng.forward_host(0, mk(h), mk(resid), out=out,
                                               ids=mk(np.zeros((T, 2), np.uint32)),
                                               gates=mk(np.zeros((T, 2), np.float32)))
            assert np.array_equal(ids, want_ids)
            assert np.array_equal(bits(gates), bits(want_gates))
            assert np.array_equal(bits(got), bits(want)), pin
            if chunked:  # three layer calls (a chunk's route may take fewer launches)
                assert eng.last_launch_count() > 2 * whole_launches


def test_nonfinite_input_is_reported():
    lw = O.synth_layer(51, 0, 64, 32, 8, 2, False)
    h = O.synth_hidden(51, 2, 64)
    h[1, 5] = np.nan
    eng = engine_for(lw, 2)
    ex, sc, rt = helpers.to_device(lw)
    eng.set_layer_packed(0, ex, sc, rt)
    with pytest.raises(M.MoeError) as ei:
        eng.forward_host(0, h)
    assert ei.value.status == _lib.MOE_ERR_NONFINITE
    # the handle stays usable after the error
    h[1, 5] = 0.0
    out, ids, _ = eng.forward_host(0, h)
    ref = O.layer_forward(lw, h)
    assert np.array_equal(bits(out), bits(ref.out))


def test_invalid_arguments_rejected_before_launch():
    lw = O.synth_layer(61, 0, 64, 32, 8, 2, False)
    eng = engine_for(lw, 2)
    h = torch.zeros((3, 64), dtype=torch.float32, device="cuda")
    out = torch.empty_like(h)
    with pytest.raises(M.MoeError) as ei:
        eng.forward(0, h, out)  # layer weights never set
    assert ei.value.status == _lib.MOE_ERR_STATE
    ex, sc, rt = helpers.to_device(lw)
    eng.set_layer_packed(0, ex, sc, rt)
    with pytest.raises(M.MoeError) as ei:
        eng.forward(0, h, out)  # T=3 > max_tokens=2
    assert ei.value.status == _lib.MOE_ERR_INVALID
    with pytest.raises(M.MoeError):
        eng.forward(5, h[:2], out[:2])  # layer out of range


@pytest.mark.parametrize("bf16", [False, True])
def test_route_tiled_ragged_shapes(bf16):
    """T >= 16 takes the register-tiled router; E not a multiple of the tile,
    H with a ragged tail (H % 8 != 0), f32 and bf16 routers: bit-exact."""
    T, H, E, K = 50, 1030, 20, 3
    router = O.synth_normal(61, O.KIND_ROUTER, 0, E * H, 0.02).reshape(E, H)
    if bf16:
        bits16 = (router.view(np.uint32) >> 16).astype(np.uint16)
        router = bits16.reshape(E, H)
    lw = O.LayerWeights(H, 8, E, K, True, np.ascontiguousarray(router),
                        np.zeros((E, 3 * 8 * H), np.int8), np.ones((E, 2 * 8 + H), np.float32),
                        router_bf16=bf16)
    h = O.synth_hidden(62, T, H)
    eng = engine_for(lw, T)
    ex, sc, rt = helpers.to_device(lw)
    eng.set_layer_packed(0, ex, sc, rt)
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    gates = torch.empty((T, K), dtype=torch.float32, device="cuda")
    probs = torch.empty((T, E), dtype=torch.float32, device="cuda")
    eng.route(0, torch.from_numpy(h).cuda(), ids, gates, probs=probs)
    torch.cuda.synchronize()
    for t in range(T):
        lg = np.empty(E, np.float32)
        O.lib().oracle_router_logits(lw.router.ctypes.data, int(bf16), E, H, h[t].ctypes.data,
                                     lg.ctypes.data)
        p = O.softmax(lg)
        rid, rg = O.topk(p, K, True)
        assert np.array_equal(bits(probs.cpu().numpy()[t]), bits(p)), t
        assert np.array_equal(ids.cpu().numpy()[t].astype(np.uint32), rid), t
        assert np.array_equal(bits(gates.cpu().numpy()[t]), bits(rg)), t


@pytest.mark.parametrize("T,E", [(50, 20), (600, 36), (4010, 20), (2310, 200)])
def test_route_pipelined_blocks(T, E):
    """f32 routers with H % 4 == 0 take the pipelined register-blocked logits
    kernel; these (T, E) pick its 16x16 and 32x16 tiles, each with ragged
    token and expert edges, and H % 8 == 4 leaves a folded tail:
    probabilities, ids and gates bit-exact."""
    H, K = 1036, 3
    router = O.synth_normal(63, O.KIND_ROUTER, 0, E * H, 0.02).reshape(E, H)
    lw = O.LayerWeights(H, 8, E, K, True, np.ascontiguousarray(router),
                        np.zeros((E, 3 * 8 * H), np.int8), np.ones((E, 2 * 8 + H), np.float32))
    h = O.synth_hidden(64, T, H)
    eng = engine_for(lw, T)
    ex, sc, rt = helpers.to_device(lw)
    eng.set_layer_packed(0, ex, sc, rt)
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    gates = torch.empty((T, K), dtype=torch.float32, device="cuda")
    probs = torch.empty((T, E), dtype=torch.float32, device="cuda")
    eng.route(0, torch.from_numpy(h).cuda(), ids, gates, probs=probs)
    eng.sync_status()
    g_probs, g_ids, g_gates = probs.cpu().numpy(), ids.cpu().numpy(), gates.cpu().numpy()
    lg = np.empty(E, np.float32)
    for t in range(T):
        O.lib().oracle_router_logits(lw.router.ctypes.data, 0, E, H, h[t].ctypes.data,
                                     lg.ctypes.data)
        p = O.softmax(lg)
        rid, rg = O.topk(p, K, True)
        assert np.array_equal(bits(g_probs[t]), bits(p)), t
        assert np.array_equal(g_ids[t].astype(np.uint32), rid), t
        assert np.array_equal(bits(g_gates[t]), bits(rg)), t


def test_route_nonfinite_input_flagged_by_blocked_kernel():
    """The blocked kernel has no separate input scan: a non-finite input
    element makes every logit of its token non-finite, which is reported."""
    H, E, K, T = 512, 64, 4, 300
    lw = O.synth_layer(65, 0, H, 64, E, K, False)
    h = O.synth_hidden(65, T, H)
    h[217, 333] = np.inf
    eng = engine_for(lw, T)
    ex, sc, rt = helpers.to_device(lw)
    eng.set_layer_packed(0, ex, sc, rt)
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    gates = torch.empty((T, K), dtype=torch.float32, device="cuda")
    eng.route(0, torch.from_numpy(h).cuda(), ids, gates)
    with pytest.raises(M.MoeError) as ei:
        eng.sync_status()
    assert ei.value.status == _lib.MOE_ERR_NONFINITE


@pytest.mark.parametrize("T,E,K", [(600, 128, 8), (2100, 64, 4)])
def test_route_permute_large_multi_cta(T, E, K):
    """Route counts above 2048 take the multi-CTA permutation (tile
    histograms, per-expert scan, scatter): same segments and the same
    token-ascending order inside each expert as the oracle's expert_uses."""
    lw = O.synth_layer(41, 0, 256, 128, E, K, False)
    h = O.synth_hidden(41, T, 256)
    ref = O.layer_forward(lw, h, nthreads=8)
    eng = engine_for(lw, T)
    ex, sc, rt = helpers.to_device(lw)
    eng.set_layer_packed(0, ex, sc, rt)
    hd = torch.from_numpy(h).cuda()
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    gates = torch.empty((T, K), dtype=torch.float32, device="cuda")
    seg = torch.empty(E + 1, dtype=torch.int32, device="cuda")
    rtok = torch.empty(T * K, dtype=torch.int32, device="cuda")
    rslot = torch.empty(T * K, dtype=torch.int32, device="cuda")
    eng.route_permute(0, hd, ids, gates, seg, rtok, rslot)
    torch.cuda.synchronize()
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), ref.ids)
    assert np.array_equal(seg.cpu().numpy(), ref.seg_off)
    assert np.array_equal(rtok.cpu().numpy(), ref.use_token)
    assert np.array_equal(rslot.cpu().numpy(), ref.use_slot)
