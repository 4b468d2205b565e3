"""INT4 experts in the oracle, pinned to the reference's own INT4 tests.

* src/int8_expert.rs:1727-1749: the AVX2 dot equals the scalar fallback
  within 1e-4 (1 + |x|) at 16 lengths, including odd ones, on the
  reference's generators.
* src/int8_expert.rs:1785-1819: the gate/up pair kernel equals the single
  dots (here: the same per-row arithmetic, so bit-equal).
* src/int8_expert.rs:1822-1855: an INT4 expert (H=64, I=32) on the
  reference's generators; its output is checked against a float64
  evaluation of the same nibbles, and the decode and prefill schedules of
  the layer driver agree bit for bit.
"""
import numpy as np
import pytest

from oracle import oracle as O

LENS = [1, 2, 3, 7, 8, 9, 15, 16, 31, 32, 33, 64, 127, 128, 1024, 2048]


def nibbles(q: np.ndarray, n: int) -> np.ndarray:
    q = q.astype(np.uint8)
    lo = ((q & 0x0F).astype(np.int8) << 4) >> 4
    hi = (q.astype(np.int8) >> 4)
    out = np.empty(2 * q.size, np.int8)
    out[0::2], out[1::2] = lo, hi
    return out[:n]


@pytest.mark.parametrize("n", LENS)
def test_dot_i4_simd_matches_scalar(n):
    row = np.array([(i * 41 + 17) % 256 for i in range((n + 1) // 2)], np.uint8)
    x = np.array([((i * 29 % 53) - 26.0) / 27.0 for i in range(n)], np.float32)
    a = float(O.dot_i4(row, x))
    s = float(O.dot_i4(row, x, scalar=True))
    assert abs(a - s) <= 1e-4 * (1 + abs(s))
    exact = float(np.dot(nibbles(row, n).astype(np.float64), x.astype(np.float64)))
    assert abs(a - exact) <= 1e-5 * (1 + abs(exact))


@pytest.mark.parametrize("n", LENS)
def test_dot_i4_pair_rows(n):
    g = np.array([(i * 37 + 11) % 256 for i in range((n + 1) // 2)], np.uint8)
    u = np.array([(i * 53 + 23) % 256 for i in range((n + 1) // 2)], np.uint8)
    x = np.array([((i * 29 % 53) - 26.0) / 27.0 for i in range(n)], np.float32)
    for row in (g, u):
        exact = float(np.dot(nibbles(row, n).astype(np.float64), x.astype(np.float64)))
        got = float(O.dot_i4(row, x))
        assert abs(got - exact) <= 1e-5 * (1 + abs(exact))


def test_int4_expert_reference_case():
    H, I = 64, 32
    n = (H // 2) * I
    w = np.array([(i * 23 + 7) % 256 for i in range(3 * n)], np.uint8)
    s = np.array([0.003 * (1 + i % 11) for i in range(2 * I + H)], np.float32)
    x = np.array([((i * 11 % 29) - 14.0) / 15.0 for i in range(H)], np.float32)
    act, y = O.expert_forward(w, s, H, I, x)
    # float64 evaluation of the same nibbles
    q = nibbles(w, 3 * H * I).astype(np.float64)
    Wg = q[: I * H].reshape(I, H) * s[:I, None]
    Wu = q[I * H: 2 * I * H].reshape(I, H) * s[I:2 * I, None]
    Wd = q[2 * I * H:].reshape(H, I) * s[2 * I:, None]
    g, u = Wg @ x, Wu @ x
    a64 = g / (1 + np.exp(-g)) * u
    assert np.abs(act - a64).max() <= 1e-5 * (1 + np.abs(a64).max())
    y64 = Wd @ a64
    assert np.abs(y - y64).max() <= 1e-4 * (1 + np.abs(y64).max())
    _, y_scalar = O.expert_forward(w, s, H, I, x, scalar=True)
    assert np.abs(y - y_scalar).max() <= 1e-4 * (1 + np.abs(y).max())


def int4_layer(seed, H, I, E, K, norm):
    lw = O.synth_layer(seed, 0, H, I, E, K, norm)
    rng = np.random.default_rng(seed)
    packed = rng.integers(0, 256, size=(E, 3 * H * I // 2), dtype=np.uint8)
    return O.LayerWeights(H, I, E, K, norm, lw.router, packed, lw.scales, int4=True)


def test_int4_layer_schedules_agree():
    lw = int4_layer(91, 256, 128, 16, 4, True)
    h = O.synth_hidden(91, 9, 256)
    serial = O.layer_forward(lw, h)
    parallel = O.layer_forward(lw, h, nthreads=4)
    assert np.array_equal(serial.ids, parallel.ids)
    assert np.array_equal(serial.out.view(np.uint32), parallel.out.view(np.uint32))
