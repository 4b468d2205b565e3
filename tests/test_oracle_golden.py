"""CPU tests: the oracle against the committed golden vectors and the
reference's own unit-test expectations (no GPU)."""
import numpy as np
import pytest

from oracle import oracle as O
from tests import helpers
from tests.golden import generators as G


@pytest.mark.parametrize("name", helpers.FIXTURES)
def test_fixture_layers_bit_exact(name):
    meta, layers = helpers.load_fixture(name)
    for lw, case in layers:
        r = O.layer_forward(lw, case["h"])
        assert np.array_equal(r.ids, case["ids"])
        assert np.array_equal(r.gates.view(np.uint32), case["gates"].view(np.uint32))
        assert np.array_equal(r.out.view(np.uint32), case["out"].view(np.uint32))
        assert np.array_equal(r.seg_off, case["seg_off"])
        assert np.array_equal(r.use_token, case["use_token"])
        assert np.array_equal(r.use_slot, case["use_slot"])
        # Transformers' own MoE block on the same input (fp32, other order)
        assert helpers.rel_err(r.out, case["hf_out"]) < 1e-5


def test_kat_int8_loader():
    # tests/int8_loader.rs:40-62: y = [2a, -1.5a], a = silu(1.5) * 0.75, |err| < 1e-6
    kat = helpers.unit_cases()["kat_int8_loader"]
    _, y = O.expert_forward(np.array(kat["weights"], np.int8), np.array(kat["scales"], np.float32),
                            2, 1, np.array(kat["x"], np.float32))
    g = np.float32(1.5)
    a = g / (np.float32(1) + np.exp(-g)) * np.float32(0.75)
    assert abs(y[0] - 2 * a) < 1e-6 and abs(y[1] + 1.5 * a) < 1e-6
    assert np.array_equal(y, np.array(kat["y"], np.float32))
    with pytest.raises(O.OracleError):
        O.expert_forward(np.array(kat["weights"], np.int8), np.array(kat["scales"], np.float32),
                         2, 1, np.array([np.nan, 1.0], np.float32))


def test_topk_ties_match_full_sort():
    for case in helpers.unit_cases()["topk_ties"]:
        ids, _ = O.topk(np.array(case["values"], np.float32), 8, False)
        assert list(ids) == case["expected"]


def test_router_kat():
    kat = helpers.unit_cases()["router_kat"]
    W = np.array(kat["weights"], np.float32).reshape(3, 2)
    scores = np.array([O.lib().oracle_dot_seq(W[e].ctypes.data,
                                              np.array(kat["hidden"], np.float32).ctypes.data, 2)
                       for e in range(3)], np.float32)
    ids, gates = O.select_topk_then_softmax(scores, 2)
    assert list(ids) == [0, 1] and abs(float(gates.sum()) - 1) < 1e-6


@pytest.mark.parametrize("cols", [1, 2, 7, 8, 9, 15, 16, 17, 1024, 2048, 2051])
def test_matvec_vs_f64(cols):
    # src/int8_expert.rs:1160-1183
    w, s, x = G.matvec_data(11, cols)
    for r in range(11):
        q = w[r * cols:(r + 1) * cols]
        got = O.dot_i8(q, x) * s[r]
        exp = float(np.dot(q.astype(np.float64), x.astype(np.float64)) * np.float64(s[r]))
        assert abs(float(got) - exp) <= 2e-5 * (1 + abs(exp))


def test_expert_cases_golden():
    z = np.load(helpers.os.path.join(helpers.GOLDEN, "expert_cases.npz"))
    for (h, i) in [(16, 8), (6, 10)]:
        x = G.gpu_expert_input(h)
        for seed in (1, 2):
            w, s = G.gpu_expert_weights(h, i, seed + h)
            _, y = O.expert_forward(w, s, h, i, x)
            assert np.array_equal(y, z[f"x32_{h}_{i}_{seed}"])
    for (h, i) in [(7, 5), (32, 9), (33, 17)]:
        for seed in (17, 73, 991):
            w, s, x = G.gate_up_case(h, i, seed)
            _, y = O.expert_forward(w, s, h, i, x)
            assert np.array_equal(y, z[f"x64_{h}_{i}_{seed}"])
            # scalar fallback vs AVX2 path: the reference's < 2e-5 bound
            _, ys = O.expert_forward(w, s, h, i, x, scalar=True)
            assert np.abs(ys - y).max() < 2e-5


def test_expf_table_equals_libm_sampled():
    # exhaustive check is recorded in golden/pins.json; sample here to stay fast
    assert O.lib().oracle_expf_table_mismatches(0x80000000, 0xC2D00000, 97) == 0
    assert O.lib().oracle_expf_table_mismatches(0x00000000, 0x42B17217, 97) == 0
    assert O.lib().oracle_expf_table_mismatches(0xC2D00000, 0xFF800000, 9973) == 0


def test_threaded_schedule_identical():
    L = O.synth_layer(7, 0, 128, 64, 16, 4, True)
    h = O.synth_hidden(7, 9, 128)
    a = O.layer_forward(L, h)
    for nt in (2, 4):
        b = O.layer_forward(L, h, nthreads=nt)
        assert np.array_equal(a.out, b.out) and np.array_equal(a.ids, b.ids)


def test_stack_matches_layerwise():
    layers = [O.synth_layer(3, l, 64, 32, 8, 2, False) for l in range(3)]
    x0 = O.synth_hidden(3, 4, 64)
    x, ids, gates = O.stack_forward(layers, x0)
    xr = x0.copy()
    for l, L in enumerate(layers):
        h = np.stack([O.rms_norm(xr[t], 1e-5) for t in range(xr.shape[0])])
        r = O.layer_forward(L, h, resid=xr)
        assert np.array_equal(r.ids, ids[l])
        xr = r.out
    assert np.array_equal(x, xr)
