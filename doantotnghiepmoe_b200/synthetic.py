"""Seeded synthetic MoE-layer inputs for the benchmark workloads.

int8 expert weights U[-127, 127] and scales U[1e-4, 1e-3] are generated on
the device (moe_synth_expert); routers N(0, 0.02) and hidden states N(0, 1)
on the host (moe_synth_normal_host).  For the Zipf-routed prefill workload the
router gets a per-expert logit bias through one constant hidden feature:
hidden[:, H-1] = 1 and router[e, H-1] = b_e with b_e = 0.7 * ln(z_r / mean z),
z_r ~ r^-1.1 over a seeded permutation of the experts (rank r of expert e).
Exact Zipf(1.1) is not reachable at the head -- with top-8 routing no expert
can take more than 1/8 of the routes -- and 0.7 gives the closest shares.
"""
from __future__ import annotations

import numpy as np

from .layer import KIND_HIDDEN, KIND_ROUTER, synth_normal

ZIPF_S = 1.1
ZIPF_TAU = 0.7


def zipf_weights(num_experts: int, seed: int, s: float = ZIPF_S):
    """(weights by expert id, permutation rank -> expert id)."""
    perm = np.random.default_rng(seed).permutation(num_experts)
    z = np.arange(1, num_experts + 1, dtype=np.float64) ** -s
    z /= z.sum()
    w = np.empty(num_experts)
    w[perm] = z
    return w, perm


def router(seed: int, layer: int, E: int, H: int, zipf: bool = False) -> np.ndarray:
    r = synth_normal(seed, KIND_ROUTER, layer, E * H, 0.02).reshape(E, H)
    if zipf:
        w, _ = zipf_weights(E, seed)  # the same hot experts in every layer
        r[:, H - 1] = (ZIPF_TAU * np.log(w / w.mean())).astype(np.float32)
    return r


def hidden(seed: int, stream: int, T: int, H: int, zipf: bool = False) -> np.ndarray:
    h = synth_normal(seed, KIND_HIDDEN, stream, T * H, 1.0).reshape(T, H)
    if zipf:
        h[:, H - 1] = 1.0
    return h
