"""B200 (sm_100a) MoE-layer hot path for MoE-TierEngine.

The compute lives in libmoe_b200.so (hand-written CUDA for sm_100a behind the
C ABI of include/moe_b200.h).  This package is a thin ctypes mirror of the
reference's interfaces:

* ``GpuExpertKernels`` / ``GpuExpertWeights`` -- src/gpu_expert.rs, src/gpu.rs
* ``MoeLayerEngine`` -- the MoE block of OlmoeModel decode/prefill, on device.
"""
from ._lib import LIB_PATH, MoeDims, MoeError, lib  # noqa: F401
from .gpu_expert import GpuExpertKernels, GpuExpertWeights  # noqa: F401
from .layer import (Checkpoint, MoeConfig, MoeLayerEngine, host_empty,  # noqa: F401
                    synth_expert, synth_normal)
