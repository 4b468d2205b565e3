"""Python mirror of the reference's GPU expert interface.

``GpuExpertKernels`` has the reference's method names and argument meaning
(src/gpu_expert.rs:250-495): ``init(hidden, intermediate, max_experts)``,
``forward(experts, input, outputs)``, ``forward_pairs(experts, inputs,
outputs)``.  Inputs/outputs are host float32 arrays; experts are device
weights borrowed for the call (``GpuExpertWeights``, src/gpu.rs:1552-1566).
Errors raise ``MoeError`` where the Rust code returns ``Err(String)``.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from ._lib import MOE_OK, MoeError, lib, ptr_array


@dataclass
class GpuExpertWeights:
    """Device pointers to one expert: 3*I*H int8 [gate|up|down] and 2*I+H f32."""
    d_weights: int
    d_scales: int
    weight_bytes: int
    scale_bytes: int

    @classmethod
    def from_tensors(cls, weights, scales) -> "GpuExpertWeights":
        """Borrow a CUDA int8 tensor and a CUDA float32 tensor (kept alive by the caller)."""
        return cls(weights.data_ptr(), scales.data_ptr(), weights.numel() * weights.element_size(),
                   scales.numel() * scales.element_size())


class GpuExpertKernels:
    def __init__(self, handle: int, hidden: int, intermediate: int, max_experts: int):
        self._h = handle
        self.hidden = hidden
        self.intermediate = intermediate
        self._max = max_experts

    @classmethod
    def init(cls, hidden: int, intermediate: int, max_experts: int, device: int = 0):
        out = ctypes.c_void_p()
        st = lib().moe_expert_kernels_init(device, hidden, intermediate, max_experts,
                                           ctypes.byref(out))
        if st != MOE_OK:
            raise MoeError(st, "expert kernel init failed")
        return cls(out.value, hidden, intermediate, max_experts)

    def max_experts(self) -> int:
        return int(lib().moe_expert_kernels_max_experts(self._h))

    def close(self):
        if self._h:
            lib().moe_expert_kernels_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _err(self, st: int):
        msg = lib().moe_expert_kernels_last_error(self._h)
        raise MoeError(st, msg.decode() if msg else "")

    def forward(self, experts, input, outputs):
        """Every expert on the same input (src/gpu_expert.rs:366)."""
        return self.forward_pairs(experts, [input], outputs)

    def forward_pairs(self, experts, inputs, outputs):
        """Pair j = (experts[j], inputs[j]); one shared input when len(inputs) == 1."""
        H = self.hidden
        n = len(experts)
        if len(outputs) != n:
            raise MoeError(1, "expert/output count mismatch")
        ins = [np.ascontiguousarray(x, np.float32) for x in inputs]
        if any(x.size != H for x in ins) or any(np.asarray(o).size != H for o in outputs):
            raise MoeError(1, "expert kernel dimension mismatch")
        outs = [np.empty(H, np.float32) for _ in range(n)]
        w = ptr_array([e.d_weights for e in experts])
        s = ptr_array([e.d_scales for e in experts])
        wb = (ctypes.c_size_t * max(1, n))(*[e.weight_bytes for e in experts])
        sb = (ctypes.c_size_t * max(1, n))(*[e.scale_bytes for e in experts])
        inp = ptr_array([x.ctypes.data for x in ins])
        outp = ptr_array([o.ctypes.data for o in outs])
        st = lib().moe_expert_forward_pairs(self._h, w, s, wb, sb, n, inp, len(ins), outp)
        if st != MOE_OK:
            self._err(st)
        for dst, src in zip(outputs, outs):
            dst[...] = src
