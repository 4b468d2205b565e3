"""Input generators of the reference's own kernel tests, replayed through the
oracle library's C restatements (so they are fast at full size).

gpu_expert_weights / gpu_expert_input: src/gpu_expert.rs:517-530 and :549-551.
gate_up_case: src/int8_expert.rs:1188-1229 (GateUpBenchCase::new).
matvec_data: src/int8_expert.rs:1149-1158 (`data`).
"""
from __future__ import annotations

import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from oracle import oracle as O  # noqa: E402


def gpu_expert_weights(h: int, i: int, seed: int):
    w = np.empty(3 * h * i, np.int8)
    s = np.empty(2 * i + h, np.float32)
    O.lib().oracle_gen_xorshift32_expert(seed & 0xFFFFFFFF, h, i, w.ctypes.data, s.ctypes.data)
    return w, s


def gpu_expert_input(h: int) -> np.ndarray:
    c = np.arange(h)
    return ((((c * 37) % 101).astype(np.float32) - np.float32(50.0)) / np.float32(25.0)).astype(np.float32)


def gate_up_case(h: int, i: int, seed: int):
    w = np.empty(3 * h * i, np.int8)
    s = np.empty(2 * i + h, np.float32)
    x = np.empty(h, np.float32)
    O.lib().oracle_gen_xorshift64_case(seed, h, i, w.ctypes.data, s.ctypes.data, x.ctypes.data)
    return w, s, x


def matvec_data(rows: int, cols: int):
    idx = np.arange(rows * cols)
    weights = ((idx * 73 + 19) % 256).astype(np.uint8).view(np.int8)
    scales = np.array([np.float32(0.001) * np.float32(1 + r % 7) for r in range(rows)], np.float32)
    c = np.arange(cols)
    x = ((((c * 31) % 101).astype(np.float32) - np.float32(50.0)) / np.float32(51.0)).astype(np.float32)
    return weights, scales, x
