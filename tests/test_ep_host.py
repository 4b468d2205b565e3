"""Expert-parallel host logic on CPU, two gloo ranks (no GPU).

* Every rank derives the same expert placement from the same inputs.
* The dispatch position rule of the peer-memory transport (ep.cu
  ep_dest_bases / ep_recv_prep), restated in numpy and fed with counts that
  the ranks exchange through the process group: every owner's receive
  buffer must come out as its experts in ascending local order, each
  expert's routes ordered by source rank and then token, with no gaps or
  collisions -- the same order a single process would produce by a stable
  sort of all routes."""
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


def dest_positions(ids_local, owner, counts, me):
    """Owner rank and receive-buffer position of each local route (token-major
    ids [T, K] -> routes in expert-sorted order).  counts[q, e]: routes of rank
    q to expert e."""
    E = owner.size
    tot = counts.sum(axis=0)
    base = counts[:me].sum(axis=0).astype(np.int64)
    for e in range(E):
        same = (owner[:e] == owner[e])
        base[e] += tot[:e][same].sum()
    flat = ids_local.reshape(-1)
    order = np.argsort(flat, kind="stable")  # experts ascending, tokens ascending inside
    seg = np.concatenate([[0], np.cumsum(np.bincount(flat, minlength=E))])
    pos = np.empty(flat.size, np.int64)
    for r_sorted, r in enumerate(order):
        e = flat[r]
        pos[r] = base[e] + (r_sorted - seg[e])
    return owner[flat], pos


def _worker(rank, world, port, outdir):
    import datetime

    import torch.distributed as dist

    from doantotnghiepmoe_b200 import placement, synthetic

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    E, K, T = 16, 4, 37
    w, _ = synthetic.zipf_weights(E, seed=5)
    owner = placement.balanced_owner(np.minimum(w, 1.0 / K), world)
    mine = torch.from_numpy(owner.astype(np.int64))
    first = mine.clone()
    dist.broadcast(first, 0)
    assert torch.equal(mine, first)  # every rank derived the same table
    assert np.bincount(owner, minlength=world).tolist() == [E // world] * world
    rng = np.random.default_rng(100 + rank)
    ids = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int64)
    cnt = torch.from_numpy(np.bincount(ids.reshape(-1), minlength=E).astype(np.int64))
    gathered = [torch.zeros_like(cnt) for _ in range(world)]
    dist.all_gather(gathered, cnt)
    counts = torch.stack(gathered).numpy()
    dst, pos = dest_positions(ids, owner, counts, rank)
    np.savez(os.path.join(outdir, f"r{rank}.npz"), ids=ids, dst=dst, pos=pos, owner=owner)
    dist.barrier()
    dist.destroy_process_group()


def test_ep_host_logic_two_gloo_ranks():
    import torch.multiprocessing as mp
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(world, _free_port(), d), nprocs=world,
                           start_method="spawn", join=True)
        ranks = [np.load(os.path.join(d, f"r{r}.npz")) for r in range(world)]
        owner = ranks[0]["owner"]
        E = owner.size
        for p in range(world):
            # every route bound for p, with its expected sort key
            got = []
            for q, z in enumerate(ranks):
                flat = z["ids"].reshape(-1)
                K = z["ids"].shape[1]
                for r in np.flatnonzero(z["dst"] == p):
                    local = int(np.flatnonzero(np.flatnonzero(owner == p) == flat[r])[0])
                    got.append((int(z["pos"][r]), (local, q, r // K)))
            got.sort()
            positions = [g[0] for g in got]
            keys = [g[1] for g in got]
            assert positions == list(range(len(got)))  # dense, no collisions
            assert keys == sorted(keys)  # local expert, then source rank, then token
            assert len(got) == sum(int((owner[z["ids"]] == p).sum()) for z in ranks)
        assert E == 16
