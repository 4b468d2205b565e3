"""Failure paths on the GPU, made without faulting or hanging anything.

* One GPU: a bounded device wait on a flag that nothing sets runs out under a
  short wait limit; the handle reports MOE_ERR_TIMEOUT through its status
  word, and the same handle then computes a correct layer (the context stays
  usable, the status word is cleared by the read).
* Two GPUs (skipped with fewer): expert parallelism over peer memory where
  one rank skips a step between steps.  The other rank's flag waits run out
  under a short limit and its next status read is MOE_ERR_TIMEOUT; both ranks
  then leave the group cleanly.  NVLS is off and the library's kernels use
  plain peer stores and loads only.
"""
import os
import socket
import tempfile

import numpy as np
import pytest

from oracle import oracle as O
from tests import helpers

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import doantotnghiepmoe_b200 as M  # noqa: E402
from doantotnghiepmoe_b200 import _lib  # noqa: E402


def test_bounded_wait_runs_out_and_handle_recovers():
    H, I, E, K, T = 512, 256, 16, 4, 3
    lw = O.synth_layer(401, 0, H, I, E, K, True)
    eng = M.MoeLayerEngine(M.MoeConfig(H, I, E, K, True, T, 1))
    dev = helpers.to_device(lw)
    eng.set_layer_packed(0, *dev)
    eng.set_path(_lib.MOE_PATH_GEMV)
    eng.set_wait_limit(2_000_000)  # 2 ms
    eng.debug_wait_flag()
    with pytest.raises(M.MoeError) as ei:
        eng.sync_status()
    assert ei.value.status == _lib.MOE_ERR_TIMEOUT
    eng.sync_status()  # the read cleared it
    eng.set_wait_limit(0)
    h = O.synth_hidden(402, T, H)
    ref = O.layer_forward(lw, h)
    hd = torch.from_numpy(h).cuda()
    out = torch.empty_like(hd)
    eng.forward(0, hd, out)
    eng.sync_status()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), ref.out.view(np.uint32))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _skip_worker(rank, world, port, outdir):
    import datetime

    import torch.distributed as dist

    from doantotnghiepmoe_b200 import ep_group, placement

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    H, I, E, K, T = 512, 256, 16, 4, 32
    lw = O.synth_layer(411, 0, H, I, E, K, True)
    owner = placement.contiguous_owner(E, world)
    eng = M.MoeLayerEngine(M.MoeConfig(H, I, E, K, True, T, 1), device=rank)
    ep_group.join(eng, rank, world, owner)
    res = {"transport": eng.ep_transport()}
    loc = placement.local_experts(owner, rank)
    ex = torch.from_numpy(np.ascontiguousarray(lw.experts[loc])).cuda()
    sc = torch.from_numpy(np.ascontiguousarray(lw.scales[loc])).cuda()
    rt = torch.from_numpy(lw.router).cuda()
    eng.ep_set_layer(0, ex, sc, rt)
    eng.set_wait_limit(50_000_000)  # 50 ms
    hd = torch.from_numpy(O.synth_hidden(412 + rank, T, H)).cuda()
    out = torch.empty_like(hd)
    # step 1: both ranks
    eng.ep_forward(0, hd, out)
    eng.sync_status()
    res["step1"] = "ok"
    dist.barrier()
    # step 2: rank 1 skips it; rank 0's flag waits run out
    if rank == 0:
        eng.ep_forward(0, hd, out)
        try:
            eng.sync_status()
            res["step2"] = "ok"
        except M.MoeError as exc:
            res["step2"] = _lib.STATUS_NAMES.get(exc.status, str(exc.status))
    # nothing of rank 0 is in flight past here (it synchronised); both leave
    dist.barrier()
    eng.ep_finalize()
    dist.barrier()
    dist.destroy_process_group()
    with open(os.path.join(outdir, f"r{rank}.txt"), "w") as f:
        f.write(repr(res))


def test_peer_that_skips_a_step_times_out_the_other_rank():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_skip_worker, args=(world, _free_port(), d), nprocs=world,
                           start_method="spawn", join=True)
        r0 = eval(open(os.path.join(d, "r0.txt")).read())
        r1 = eval(open(os.path.join(d, "r1.txt")).read())
    if r0["transport"] != "p2p":
        pytest.skip(f"peer-memory transport unavailable ({r0['transport']})")
    assert r0["step1"] == r1["step1"] == "ok"
    assert r0["step2"] == "TIMEOUT"
