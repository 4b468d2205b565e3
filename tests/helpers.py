"""Shared test helpers: golden fixture loading and device upload of layers."""
from __future__ import annotations

import json
import os

import numpy as np

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
FIXTURES = ["olmoe_unnormalized-mha", "olmoe_normalized-gqa", "qwen3moe_gqa-headdim",
            "qwen3moe_many-experts", "qwen3moe_bf16-dense"]


def load_fixture(name: str):
    z = np.load(os.path.join(GOLDEN, f"fixture_{name}.npz"))
    meta = {k: int(z[k]) for k in ("H", "I", "E", "K", "norm", "router_bf16", "n_layers")}
    layers = []
    for li in range(meta["n_layers"]):
        lw = O.LayerWeights(meta["H"], meta["I"], meta["E"], meta["K"], bool(meta["norm"]),
                            np.ascontiguousarray(z[f"l{li}_router"]),
                            np.ascontiguousarray(z[f"l{li}_experts"]),
                            np.ascontiguousarray(z[f"l{li}_scales"]),
                            router_bf16=bool(meta["router_bf16"]))
        case = {k: z[f"l{li}_{k}"] for k in ("h", "out", "ids", "gates", "seg_off", "use_token",
                                             "use_slot", "hf_out")}
        layers.append((lw, case))
    return meta, layers


def unit_cases():
    with open(os.path.join(GOLDEN, "unit_cases.json")) as f:
        return json.load(f)


def rel_err(a, b) -> float:
    """max |a - b| / max |b|: the metric of src/gpu_expert.rs:566-575."""
    a = np.asarray(a, np.float64); b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-6))


def to_device(lw: "O.LayerWeights", device="cuda"):
    import torch
    experts = torch.from_numpy(np.ascontiguousarray(lw.experts)).to(device)  # uint8 = INT4
    scales = torch.from_numpy(np.ascontiguousarray(lw.scales)).to(device)
    if lw.router_bf16:
        router = torch.from_numpy(lw.router.view(np.int16).copy()).to(device)
    else:
        router = torch.from_numpy(np.ascontiguousarray(lw.router)).to(device)
    return experts, scales, router


def write_safetensors(path, tensors, metadata=None):
    """A shard in the safetensors layout: u64 header length, JSON header
    (padded with spaces to 8 bytes), then the payloads in the given order.
    tensors: [(name, dtype string, array)]."""
    import json
    import struct
    header, blobs, off = {}, [], 0
    for name, dt, arr in tensors:
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(np.shape(arr)), "data_offsets": [off, off + len(b)]}
        off += len(b)
        blobs.append(b)
    if metadata is not None:
        header["__metadata__"] = metadata
    hj = json.dumps(header).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)
