"""Device MoE layer: router -> softmax -> top-k -> permutation -> INT8
SwiGLU experts -> slot-ordered combine, behind the C ABI's ``moe_handle``.

It replaces the MoE block of the reference's ``OlmoeModel::step_inner``
(src/olmoe.rs:2583-3158) and ``OlmoeModel::prefill`` (:3417-3714).  Tensors are
passed as CUDA tensors (torch provides device memory and streams only); every
computation happens in libmoe_b200.so.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from ._lib import (MOE_OK, MOE_ROUTER_BF16, MOE_ROUTER_F32, MoeDims, MoeError, lib,
                   ptr_array)


@dataclass
class MoeConfig:
    hidden: int
    intermediate: int
    num_experts: int
    top_k: int
    norm_topk_prob: bool
    max_tokens: int = 1
    num_layers: int = 1


def _ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        return None
    return getattr(stream, "cuda_stream", stream)


class MoeLayerEngine:
    def __init__(self, cfg: MoeConfig, device: int = 0):
        self.cfg = cfg
        self.device = device
        dims = MoeDims(cfg.hidden, cfg.intermediate, cfg.num_experts, cfg.top_k,
                       int(cfg.norm_topk_prob), cfg.max_tokens, cfg.num_layers)
        out = ctypes.c_void_p()
        st = lib().moe_create(device, ctypes.byref(dims), ctypes.byref(out))
        if st != MOE_OK:
            raise MoeError(st, "moe_create failed")
        self._h = out.value
        self._keep = {}

    def close(self):
        if getattr(self, "_h", None):
            lib().moe_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, st: int):
        if st != MOE_OK:
            msg = lib().moe_last_error(self._h)
            raise MoeError(st, msg.decode() if msg else "")

    # -- configuration ---------------------------------------------------
    def set_stream(self, stream):
        self._check(lib().moe_set_stream(self._h, _stream(stream)))

    def set_route_mode(self, mode: int):
        self._check(lib().moe_set_route_mode(self._h, mode))

    def set_path(self, path: int):
        self._check(lib().moe_set_path(self._h, path))

    def set_layer_packed(self, layer: int, experts, scales, router):
        """experts: CUDA int8 [E, 3*I*H] (or uint8 [E, 3*I*H/2]: INT4 nibble
        pairs); scales: CUDA f32 [E, 2I+H]; router: CUDA f32 [E, H] or
        int16/uint16-viewed bf16 bits [E, H]."""
        import torch
        dtype = MOE_ROUTER_F32 if router.dtype == torch.float32 else MOE_ROUTER_BF16
        quant = 1 if experts.dtype == torch.uint8 else 0
        self._keep[layer] = (experts, scales, router)
        self._check(lib().moe_set_layer_packed_q(self._h, layer, experts.data_ptr(),
                                                 scales.data_ptr(), router.data_ptr(), dtype,
                                                 quant))

    def set_layer(self, layer: int, expert_weights: list, expert_scales: list, router):
        """Per-expert device pointers (pool slots) -- the GpuExpertWeights borrow."""
        import torch
        dtype = MOE_ROUTER_F32 if router.dtype == torch.float32 else MOE_ROUTER_BF16
        self._keep[layer] = (expert_weights, expert_scales, router)
        w = ptr_array([t.data_ptr() for t in expert_weights])
        s = ptr_array([t.data_ptr() for t in expert_scales])
        self._check(lib().moe_set_layer(self._h, layer, w, s, router.data_ptr(), dtype))

    # -- compute -----------------------------------------------------------
    def route(self, layer: int, h, ids, gates, probs=None, stream=None):
        self._check(lib().moe_route(self._h, layer, h.data_ptr(), h.shape[0], ids.data_ptr(),
                                    gates.data_ptr(), _ptr(probs), _stream(stream)))

    def route_permute(self, layer: int, h, ids, gates, seg_off, route_token, route_slot,
                      stream=None):
        self._check(lib().moe_route_permute(self._h, layer, h.data_ptr(), h.shape[0],
                                            ids.data_ptr(), gates.data_ptr(),
                                            seg_off.data_ptr(), route_token.data_ptr(),
                                            route_slot.data_ptr(), _stream(stream)))

    def forward(self, layer: int, h, out, resid=None, ids=None, gates=None, stream=None):
        self._check(lib().moe_layer_forward(self._h, layer, h.data_ptr(), _ptr(resid),
                                            out.data_ptr(), h.shape[0], _ptr(ids), _ptr(gates),
                                            _stream(stream)))

    def stack_forward(self, first_layer: int, n_layers: int, x, eps: float = 1e-5, stream=None):
        self._check(lib().moe_stack_forward(self._h, first_layer, n_layers, x.data_ptr(),
                                            x.shape[0], eps, _stream(stream)))

    def forward_host(self, layer: int, h: np.ndarray, resid: np.ndarray | None = None,
                     out: np.ndarray | None = None, ids: np.ndarray | None = None,
                     gates: np.ndarray | None = None):
        """Host buffers in and out (the library copies them).  Buffers in pinned
        host memory are read and written by DMA directly; pageable ones are
        staged.  `out`, `ids` and `gates` may be passed to reuse buffers."""
        h = np.ascontiguousarray(h, np.float32)
        T = h.shape[0]
        K = self.cfg.top_k
        if out is None:
            out = np.empty_like(h)
        if ids is None:
            ids = np.empty((T, K), np.uint32)
        if gates is None:
            gates = np.empty((T, K), np.float32)
        for a, shape, dt in ((out, h.shape, np.float32), (ids, (T, K), np.uint32),
                             (gates, (T, K), np.float32)):
            if a.shape != shape or a.dtype != dt or not a.flags.c_contiguous:
                raise ValueError(f"output buffer must be C-contiguous {dt.__name__}{shape}")
        r = None if resid is None else np.ascontiguousarray(resid, np.float32)
        self._check(lib().moe_layer_forward_host(self._h, layer, h.ctypes.data,
                                                 None if r is None else r.ctypes.data,
                                                 out.ctypes.data, T, ids.ctypes.data,
                                                 gates.ctypes.data))
        return out, ids, gates

    def set_layer_norm(self, layer: int, norm_w=None):
        """Post-attention RMSNorm gain [H] (device tensor) used by stack_forward;
        None restores the unit gain."""
        self._check(lib().moe_set_layer_norm(self._h, layer, _ptr(norm_w)))

    def load_layer(self, ckpt: "Checkpoint", ckpt_layer: int, layer: int | None = None,
                   keep_bf16: bool = True):
        """moe_load_layer: checkpoint layer -> device copy owned by the engine."""
        self._check(lib().moe_load_layer(self._h, ckpt._c, ckpt_layer,
                                         ckpt_layer if layer is None else layer, int(keep_bf16)))

    def sync_status(self, stream=None):
        self._check(lib().moe_sync_status(self._h, _stream(stream)))

    def last_launch_count(self) -> int:
        return int(lib().moe_last_launch_count(self._h))

    def set_wait_limit(self, ns: int = 0):
        """Bound of the device-side waits (grid barriers, expert-parallel flag
        waits) in nanoseconds; 0 restores the defaults."""
        self._check(lib().moe_set_wait_limit(self._h, int(ns)))

    def debug_wait_flag(self, stream=None):
        """Failure-path probe: a bounded wait on a device flag that nothing
        sets; the next sync_status() raises MoeError(MOE_ERR_TIMEOUT)."""
        self._check(lib().moe_debug_wait_flag(self._h, _stream(stream)))

    # -- expert parallelism (one process per GPU) -------------------------
    def ep_init(self, rank: int, nranks: int, unique_id: bytes, owner):
        owner = np.ascontiguousarray(owner, np.int32)
        assert owner.size == self.cfg.num_experts
        uid = (ctypes.c_ubyte * 128).from_buffer_copy(unique_id)
        self._check(lib().moe_ep_init(self._h, rank, nranks, uid, owner.ctypes.data))

    def ep_set_layer(self, layer: int, experts_local, scales_local, router):
        """experts_local / scales_local: this rank's experts packed in ascending
        global id order; router: the full [E, H] router."""
        import torch
        dtype = MOE_ROUTER_F32 if router.dtype == torch.float32 else MOE_ROUTER_BF16
        self._keep[("ep", layer)] = (experts_local, scales_local, router)
        self._check(lib().moe_ep_set_layer(self._h, layer, _ptr(experts_local),
                                           _ptr(scales_local), router.data_ptr(), dtype))

    def ep_forward(self, layer: int, h, out, resid=None, stream=None):
        self._check(lib().moe_ep_layer_forward(self._h, layer, h.data_ptr(), _ptr(resid),
                                               out.data_ptr(), h.shape[0], _stream(stream)))

    def ep_finalize(self):
        self._check(lib().moe_ep_finalize(self._h))

    def ep_transport(self) -> str:
        """'p2p' (kernels write into peer memory), 'nccl' or 'none'."""
        return {1: "p2p", 0: "nccl"}.get(lib().moe_ep_transport(self._h), "none")

    def set_graphs(self, enable: bool):
        """Replay each call's launch sequence as a CUDA graph (default on)."""
        self._check(lib().moe_set_graphs(self._h, int(enable)))

    def profile(self, enable: bool):
        self._check(lib().moe_profile_enable(self._h, int(enable)))

    def profile_read(self) -> dict:
        """{kernel name: (launches, total ms)} since the previous read."""
        from ._lib import MoeKernelTime
        buf = (MoeKernelTime * 64)()
        n = ctypes.c_int()
        self._check(lib().moe_profile_read(self._h, buf, 64, ctypes.byref(n)))
        return {buf[i].name.decode(): (int(buf[i].launches), float(buf[i].total_ms))
                for i in range(min(n.value, 64))}


def synth_normal(seed: int, kind: int, layer: int, n: int, std: float) -> np.ndarray:
    out = np.empty(n, np.float32)
    st = lib().moe_synth_normal_host(seed, kind, layer, n, std, out.ctypes.data)
    if st != MOE_OK:
        raise MoeError(st, "moe_synth_normal_host failed")
    return out


KIND_ROUTER, KIND_HIDDEN = 3, 4


_DT = {0: ("U8", np.uint8), 1: ("I8", np.int8), 2: ("F16", np.float16),
       3: ("BF16", np.uint16), 4: ("F32", np.float32)}


class Checkpoint:
    """A directory of merged-INT8 safetensors shards (moe_ckpt_open); BF16
    payloads come back as their uint16 bit patterns."""

    def __init__(self, directory: str):
        c = ctypes.c_void_p()
        err = ctypes.create_string_buffer(512)
        st = lib().moe_ckpt_open(directory.encode(), ctypes.byref(c), err, len(err))
        if st != MOE_OK:
            raise MoeError(st, err.value.decode(errors="replace"))
        self._c = c.value

    def close(self):
        if getattr(self, "_c", None):
            lib().moe_ckpt_close(self._c)
            self._c = None

    def __del__(self):
        self.close()

    def __len__(self) -> int:
        return int(lib().moe_ckpt_num_tensors(self._c))

    def info(self, name: str):
        dt, nd = ctypes.c_int(), ctypes.c_int()
        shape = (ctypes.c_int64 * 8)()
        nbytes = ctypes.c_size_t()
        st = lib().moe_ckpt_tensor_info(self._c, name.encode(), ctypes.byref(dt), ctypes.byref(nd),
                                        shape, ctypes.byref(nbytes))
        if st != MOE_OK:
            raise MoeError(st, f"missing tensor: {name}")
        return _DT[dt.value][0], tuple(shape[i] for i in range(nd.value)), int(nbytes.value)

    def read(self, name: str) -> np.ndarray:
        dname, shape, nbytes = self.info(name)
        out = np.empty(shape, _DT[[k for k, v in _DT.items() if v[0] == dname][0]][1])
        st = lib().moe_ckpt_read(self._c, name.encode(), out.ctypes.data, nbytes)
        if st != MOE_OK:
            raise MoeError(st, f"read failed: {name}")
        return out


class _HostBlock:
    """Owner of one moe_host_alloc() block; freed when the last array view
    referring to it goes away."""

    def __init__(self, nbytes: int):
        p = ctypes.c_void_p()
        st = lib().moe_host_alloc(nbytes, ctypes.byref(p))
        if st != MOE_OK:
            raise MoeError(st, "moe_host_alloc failed")
        self.ptr = p.value

    def __del__(self):
        if getattr(self, "ptr", None):
            lib().moe_host_free(self.ptr)
            self.ptr = None


def host_empty(shape, dtype=np.float32) -> np.ndarray:
    """Pinned host array for MoeLayerEngine.forward_host (moe_host_alloc):
    allocate once and reuse across calls."""
    dtype = np.dtype(dtype)
    n = int(np.prod(shape)) * dtype.itemsize
    blk = _HostBlock(max(n, 1))
    raw = (ctypes.c_ubyte * max(n, 1)).from_address(blk.ptr)
    raw._moe_block = blk  # keeps the block alive while any view exists
    return np.frombuffer(raw, dtype=dtype, count=int(np.prod(shape))).reshape(shape)


def ep_unique_id() -> bytes:
    buf = (ctypes.c_ubyte * 128)()
    st = lib().moe_ep_unique_id(buf)
    if st != MOE_OK:
        raise MoeError(st, "moe_ep_unique_id failed (NCCL unavailable?)")
    return bytes(buf)


def synth_expert(seed: int, layer: int, expert: int, H: int, I: int, w, s, stream=None):
    st = lib().moe_synth_expert(seed, layer, expert, H, I, w.data_ptr(), s.data_ptr(),
                                _stream(stream))
    if st != MOE_OK:
        raise MoeError(st, "moe_synth_expert failed")
