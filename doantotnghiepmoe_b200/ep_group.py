"""Joining the expert-parallel group from the host, one process per GPU.

Every rank calls :func:`join` with its engine, the same expert placement and
a ``torch.distributed`` process group (any backend; the engine's own data
path never uses it).  Three steps, each a collective of that group:

1. Placement check.  The placement table (expert -> owner rank) must be the
   same on every rank: each rank contributes a digest of its table and all
   ranks compare.  A mismatch would route tokens to a rank that does not
   hold the expert, so it raises :class:`EpGroupError` on every rank.
2. Rank 0 creates the 128-byte NCCL unique id and broadcasts it.
3. ``engine.ep_init(rank, world, id, owner)``.

A rank that never arrives makes the others' next collective end with the
process group's own timeout error (give the group a short timeout), which is
re-raised as :class:`EpGroupError` naming the step; nothing waits forever.
The reference engine runs on one device (src/gpu.rs:457-460) and has no
counterpart; its circuit breaker (src/gpu.rs:534-550) plays the same role of
turning a failed device path into an error the caller sees.
"""
from __future__ import annotations

import hashlib

import numpy as np


class EpGroupError(RuntimeError):
    """The expert-parallel group could not be formed (a step failed or timed out)."""


def placement_digest(owner) -> bytes:
    """16-byte digest of an expert -> owner table (int32, little endian)."""
    a = np.ascontiguousarray(owner, dtype="<i4")
    return hashlib.blake2b(a.tobytes(), digest_size=16).digest()


def _unique_id() -> bytes:
    from .layer import ep_unique_id
    return ep_unique_id()


def join(engine, rank: int, world: int, owner, group=None, unique_id_fn=None) -> bytes:
    """Join the group; returns the NCCL unique id every rank used.

    ``engine`` needs an ``ep_init(rank, world, unique_id, owner)`` method
    (:class:`doantotnghiepmoe_b200.MoeLayerEngine`).  ``unique_id_fn``
    (rank 0 only) makes the id; the default asks the library for a fresh
    NCCL unique id."""
    import torch
    import torch.distributed as dist

    owner = np.ascontiguousarray(owner, np.int32)
    if owner.ndim != 1 or owner.size == 0 or owner.min() < 0 or owner.max() >= world:
        raise EpGroupError(f"rank {rank}: placement must map every expert to a rank in "
                           f"[0, {world})")
    # NCCL groups exchange device tensors, the others host tensors
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    # 1. the same placement on every rank
    mine = torch.tensor(list(placement_digest(owner)), dtype=torch.uint8, device=dev)
    digests = [torch.zeros(16, dtype=torch.uint8, device=dev) for _ in range(world)]
    try:
        dist.all_gather(digests, mine, group=group)
    except Exception as exc:  # a rank that never arrives: the group's timeout
        raise EpGroupError(f"rank {rank}: placement exchange failed: {exc}") from exc
    bad = [q for q in range(world) if not torch.equal(digests[q], mine)]
    if bad:
        raise EpGroupError(f"rank {rank}: expert placement differs on rank(s) {bad}")
    # 2. one NCCL unique id for the group
    uid = torch.zeros(128, dtype=torch.uint8, device=dev)
    if rank == 0:
        raw = (unique_id_fn or _unique_id)()
        if len(raw) != 128:
            raise EpGroupError("NCCL unique id must be 128 bytes")
        uid = torch.tensor(list(raw), dtype=torch.uint8, device=dev)
    try:
        dist.broadcast(uid, 0, group=group)
    except Exception as exc:
        raise EpGroupError(f"rank {rank}: unique id broadcast failed: {exc}") from exc
    uid_bytes = bytes(uid.cpu().tolist())
    # 3. the library's group (communicator, peer-memory regions)
    engine.ep_init(rank, world, uid_bytes, owner)
    return uid_bytes
