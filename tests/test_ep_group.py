"""Host-side failure detection of the expert-parallel group, on CPU with two
gloo ranks (no GPU): ep_group.join() forms the group when the ranks agree,
raises on every rank when their expert placements differ, and raises --
instead of waiting forever -- when a peer never arrives (the process
group's short timeout ends the collective)."""
import os
import socket
import tempfile

import numpy as np
import pytest

torch = pytest.importorskip("torch")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class FakeEngine:
    def __init__(self):
        self.calls = []

    def ep_init(self, rank, world, uid, owner):
        self.calls.append((rank, world, uid, np.asarray(owner).tolist()))


def _worker(rank, world, port, outdir, mode):
    import datetime

    import torch.distributed as dist

    from doantotnghiepmoe_b200 import ep_group

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=5))
    owner = np.array([0, 0, 1, 1, 0, 1], np.int32)
    if mode == "mismatch" and rank == 1:
        owner = np.array([0, 1, 0, 1, 0, 1], np.int32)
    if mode == "absent" and rank == 1:
        # this rank leaves before the group is formed (between steps: no
        # collective of its own is in flight)
        with open(os.path.join(outdir, "r1.txt"), "w") as f:
            f.write("left")
        os._exit(0)
    eng = FakeEngine()
    try:
        uid = ep_group.join(eng, rank, world, owner,
                            unique_id_fn=lambda: bytes(range(128)))
        res = "ok:" + uid.hex()
        assert eng.calls == [(rank, world, uid, owner.tolist())]
    except ep_group.EpGroupError as exc:
        res = "err:" + str(exc)
    with open(os.path.join(outdir, f"r{rank}.txt"), "w") as f:
        f.write(res)
    if mode != "absent":
        dist.destroy_process_group()


def _run(mode):
    import torch.multiprocessing as mp
    world = 2
    with tempfile.TemporaryDirectory() as d:
        ctx = mp.start_processes(_worker, args=(world, _free_port(), d, mode), nprocs=world,
                                 start_method="spawn", join=False)
        while not ctx.join(timeout=60):
            pass
        return [open(os.path.join(d, f"r{r}.txt")).read() for r in range(world)]


def test_join_forms_the_group():
    r0, r1 = _run("ok")
    assert r0 == r1 == "ok:" + bytes(range(128)).hex()


def test_join_rejects_differing_placements_on_every_rank():
    r0, r1 = _run("mismatch")
    assert r0.startswith("err:") and "placement differs" in r0
    assert r1.startswith("err:") and "placement differs" in r1


def test_join_raises_when_a_peer_never_arrives():
    r0, r1 = _run("absent")
    assert r1 == "left"
    assert r0.startswith("err:") and "placement exchange failed" in r0


def test_placement_digest_is_order_sensitive():
    from doantotnghiepmoe_b200.ep_group import placement_digest
    assert placement_digest([0, 1]) != placement_digest([1, 0])
    assert placement_digest(np.array([0, 1], np.int64)) == placement_digest([0, 1])
