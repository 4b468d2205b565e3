"""ctypes view of the CPU oracle (oracle/libmoe_oracle.so).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, `__graft_entry__.smoke()` and
the CPU-baseline legs of bench.py, where it is the checker and the timed CPU
restatement of the reference engine's INT8 path.  The product package
(`doantotnghiepmoe_b200`) never imports this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libmoe_oracle.so")
_lib = None

OK, ERR_SHAPE, ERR_NONFINITE = 0, 1, 2


def build() -> str:
    """Compile the oracle in place with its Makefile (gcc, no CUDA)."""
    env = dict(os.environ)
    env.pop("CC", None)
    subprocess.run(["make", "-s", "-C", _HERE], check=True, env=env)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        i32, u32, u64, f32, sz = (ctypes.c_int, ctypes.c_uint32, ctypes.c_uint64,
                                  ctypes.c_float, ctypes.c_size_t)
        sig = {
            "oracle_dot_f32": (f32, [P, P, sz]),
            "oracle_dot_bf16": (f32, [P, P, sz]),
            "oracle_dot_seq": (f32, [P, P, sz]),
            "oracle_router_logits": (i32, [P, i32, i32, i32, P, P]),
            "oracle_softmax": (i32, [P, i32]),
            "oracle_rms_norm": (i32, [P, P, i32, f32, P]),
            "oracle_topk": (None, [P, i32, i32, i32, P, P]),
            "oracle_select_topk_then_softmax": (None, [P, i32, i32, P, P]),
            "oracle_dot_i8_avx2": (f32, [P, P, sz]),
            "oracle_dot_i8_scalar": (f32, [P, P, sz]),
            "oracle_dot_i4_avx2": (f32, [P, P, sz]),
            "oracle_dot_i4_scalar": (f32, [P, P, sz]),
            "oracle_expert_forward": (i32, [P, P, i32, i32, P, P, P, i32]),
            "oracle_expert_forward_q": (i32, [P, P, i32, i32, P, P, P, i32, i32]),
            "oracle_expf_table": (f32, [f32]),
            "oracle_expf_table_mismatches": (u64, [u32, u32, u32]),
            "oracle_expf_libm_range": (None, [u32, sz, P]),
            "oracle_layer_forward": (i32, [P, i32, P, P, P, P, P, P, P, P, P, i32, i32]),
            "oracle_stack_forward": (i32, [P, i32, i32, P, f32, P, P, i32, i32]),
            "oracle_synth_key": (u64, [u64, u32, u32, u32]),
            "oracle_synth_expert": (None, [u64, i32, i32, i32, i32, P, P]),
            "oracle_synth_normal": (None, [u64, u32, u32, sz, f32, P]),
            "oracle_gen_xorshift32_expert": (None, [u32, i32, i32, P, P]),
            "oracle_gen_xorshift64_case": (None, [u64, i32, i32, P, P, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


class _Layer(ctypes.Structure):
    _fields_ = [("H", ctypes.c_int), ("I", ctypes.c_int), ("E", ctypes.c_int),
                ("K", ctypes.c_int), ("norm_topk_prob", ctypes.c_int),
                ("router_bf16", ctypes.c_int), ("router", ctypes.c_void_p),
                ("experts", ctypes.c_void_p), ("scales", ctypes.c_void_p),
                ("norm_w", ctypes.c_void_p), ("int4", ctypes.c_int)]


@dataclass
class LayerWeights:
    """One MoE layer in the reference's merged layout (src/int8_expert.rs:90-97).

    experts: int8 [E, 3*I*H] = per expert [gate I*H | up I*H | down H*I]
    scales:  f32  [E, 2*I+H] = per expert [gate I | up I | down H]
    router:  f32 [E, H]  (or uint16 bf16 bits when router_bf16)
    """
    H: int
    I: int
    E: int
    K: int
    norm_topk_prob: bool
    router: np.ndarray
    experts: np.ndarray
    scales: np.ndarray
    router_bf16: bool = False
    norm_w: np.ndarray | None = None  # post-attention RMSNorm gain [H] (stacks); None = 1
    int4: bool = False  # experts are uint8 [E, 3*I*H/2] nibble pairs (src/int8_expert.rs:473)

    def c_struct(self) -> _Layer:
        for name in ("router", "experts", "scales"):
            a = getattr(self, name)
            assert a.flags["C_CONTIGUOUS"], name
        nw = None
        if self.norm_w is not None:
            assert self.norm_w.dtype == np.float32 and self.norm_w.flags["C_CONTIGUOUS"]
            nw = self.norm_w.ctypes.data
        return _Layer(self.H, self.I, self.E, self.K, int(self.norm_topk_prob),
                      int(self.router_bf16), self.router.ctypes.data,
                      self.experts.ctypes.data, self.scales.ctypes.data, nw, int(self.int4))


class OracleError(RuntimeError):
    pass


def _check(st: int, what: str):
    if st != OK:
        raise OracleError(f"{what}: oracle status {st}")


def dot_f32(a, b) -> np.float32:
    a = np.ascontiguousarray(a, np.float32); b = np.ascontiguousarray(b, np.float32)
    return np.float32(lib().oracle_dot_f32(_p(a), _p(b), a.size))


def dot_i8(q, x, scalar: bool = False) -> np.float32:
    q = np.ascontiguousarray(q, np.int8); x = np.ascontiguousarray(x, np.float32)
    fn = lib().oracle_dot_i8_scalar if scalar else lib().oracle_dot_i8_avx2
    return np.float32(fn(_p(q), _p(x), q.size))


def expf_libm_range(bits_lo: int, count: int) -> np.ndarray:
    out = np.empty(count, np.float32)
    lib().oracle_expf_libm_range(bits_lo, count, _p(out))
    return out


def softmax(v) -> np.ndarray:
    v = np.array(v, np.float32, copy=True)
    _check(lib().oracle_softmax(_p(v), v.size), "softmax")
    return v


def rms_norm(x, eps: float, w=None) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    w = None if w is None else np.ascontiguousarray(w, np.float32)
    _check(lib().oracle_rms_norm(_p(x), _p(w), x.size, eps, _p(out)), "rms_norm")
    return out


def topk(p, K: int, norm: bool):
    p = np.ascontiguousarray(p, np.float32)
    ids = np.empty(K, np.uint32); gates = np.empty(K, np.float32)
    lib().oracle_topk(_p(p), p.size, K, int(norm), _p(ids), _p(gates))
    return ids, gates


def select_topk_then_softmax(scores, K: int):
    s = np.ascontiguousarray(scores, np.float32)
    ids = np.empty(K, np.uint32); gates = np.empty(K, np.float32)
    lib().oracle_select_topk_then_softmax(_p(s), s.size, K, _p(ids), _p(gates))
    return ids, gates


def expert_forward(w, s, H: int, I: int, x, scalar: bool = False):
    """Int8Expert::forward_single_threaded.  Returns (act[I], y[H]).  A uint8
    `w` of 3*H*I/2 bytes is an INT4 expert."""
    int4 = np.asarray(w).dtype == np.uint8 and np.asarray(w).size * 2 == 3 * H * I
    w = np.ascontiguousarray(w, np.uint8 if int4 else np.int8)
    s = np.ascontiguousarray(s, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    assert w.size == 3 * H * I // (2 if int4 else 1) and s.size == 2 * I + H and x.size == H
    act = np.empty(I, np.float32); y = np.empty(H, np.float32)
    _check(lib().oracle_expert_forward_q(_p(w), _p(s), H, I, _p(x), _p(act), _p(y),
                                         int(scalar), int(int4)), "expert_forward")
    return act, y


def dot_i4(q, x, scalar: bool = False) -> np.float32:
    """INT4 row dot: q uint8 packed nibbles (element 2i low, 2i+1 high)."""
    q = np.ascontiguousarray(q, np.uint8); x = np.ascontiguousarray(x, np.float32)
    assert q.size == (x.size + 1) // 2
    fn = lib().oracle_dot_i4_scalar if scalar else lib().oracle_dot_i4_avx2
    return np.float32(fn(_p(q), _p(x), x.size))


@dataclass
class LayerResult:
    out: np.ndarray      # [T, H]
    ids: np.ndarray      # [T, K] uint32
    gates: np.ndarray    # [T, K] f32
    seg_off: np.ndarray  # [E+1] int32
    use_token: np.ndarray
    use_slot: np.ndarray
    use_gate: np.ndarray


def layer_forward(L: LayerWeights, h, resid=None, scalar: bool = False,
                  nthreads: int = 1, decode_schedule: bool = False) -> LayerResult:
    h = np.ascontiguousarray(h, np.float32).reshape(-1, L.H)
    T = h.shape[0]
    resid = None if resid is None else np.ascontiguousarray(resid, np.float32).reshape(T, L.H)
    out = np.empty((T, L.H), np.float32)
    ids = np.empty((T, L.K), np.uint32); gates = np.empty((T, L.K), np.float32)
    seg = np.empty(L.E + 1, np.int32)
    ut = np.empty(T * L.K, np.int32); us = np.empty(T * L.K, np.int32)
    ug = np.empty(T * L.K, np.float32)
    cs = L.c_struct()
    mode = int(scalar) | (2 if decode_schedule else 0)
    st = lib().oracle_layer_forward(ctypes.byref(cs), T, _p(h), _p(resid), _p(out), _p(ids),
                                    _p(gates), _p(seg), _p(ut), _p(us), _p(ug), mode,
                                    nthreads)
    _check(st, "layer_forward")
    return LayerResult(out, ids, gates, seg, ut, us, ug)


def stack_forward(layers: list[LayerWeights], x, eps: float = 1e-5, scalar: bool = False,
                  nthreads: int = 1):
    """x <- x + MoE(RMSNorm(x)) per layer.  Returns (x, ids[nl,T,K], gates[nl,T,K])."""
    H, K = layers[0].H, layers[0].K
    x = np.array(x, np.float32, copy=True).reshape(-1, H)
    T = x.shape[0]
    arr = (_Layer * len(layers))(*[l.c_struct() for l in layers])
    ids = np.empty((len(layers), T, K), np.uint32)
    gates = np.empty((len(layers), T, K), np.float32)
    st = lib().oracle_stack_forward(arr, len(layers), T, _p(x), eps, _p(ids), _p(gates),
                                    int(scalar), nthreads)
    _check(st, "stack_forward")
    return x, ids, gates


# ---- seeded synthetic inputs (bit-identical to the CUDA generator for the
# integer-derived tensors) ----
KIND_EXPERT_W, KIND_EXPERT_S, KIND_ROUTER, KIND_HIDDEN = 1, 2, 3, 4


def synth_expert(seed: int, layer: int, expert: int, H: int, I: int):
    w = np.empty(3 * H * I, np.int8); s = np.empty(2 * I + H, np.float32)
    lib().oracle_synth_expert(seed, layer, expert, H, I, _p(w), _p(s))
    return w, s


def synth_normal(seed: int, kind: int, layer: int, n: int, std: float) -> np.ndarray:
    out = np.empty(n, np.float32)
    lib().oracle_synth_normal(seed, kind, layer, n, std, _p(out))
    return out


def synth_layer(seed: int, layer: int, H: int, I: int, E: int, K: int, norm: bool,
                router_std: float = 0.02) -> LayerWeights:
    experts = np.empty((E, 3 * H * I), np.int8)
    scales = np.empty((E, 2 * I + H), np.float32)
    for e in range(E):
        experts[e], scales[e] = synth_expert(seed, layer, e, H, I)
    router = synth_normal(seed, KIND_ROUTER, layer, E * H, router_std).reshape(E, H)
    return LayerWeights(H, I, E, K, norm, router, experts, scales)


def synth_hidden(seed: int, T: int, H: int, stream: int = 0) -> np.ndarray:
    return synth_normal(seed, KIND_HIDDEN, stream, T * H, 1.0).reshape(T, H)
