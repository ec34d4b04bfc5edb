"""Host-side logic of the row-sharded linear, on CPU with two gloo ranks.

hexir_sharded_linear_f64 (and the VM's cuda:F-L dispatch) does, per rank:
broadcast w from rank 0, compute rows hexir_shard_rows(m, ranks, rank) of
a . w, send them to rank 0, which places them at their row offset.  Here the
same protocol runs with gloo in place of NCCL and the oracle in place of the
GPU kernel, and rank 0's assembled result must equal the whole product bit
for bit.  A second test drops a rank before the gather: the survivor's
collective must end with an error within the process-group timeout instead
of waiting for ever.
"""

import datetime
import os

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from tests.conftest import free_port, spawn_ranks


def _init(rank, world, port, timeout_s):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _sharded_rank(rank, world, port, m, n, k, result_path):
    import torch
    import hexir_b200 as hx
    from oracle import oracle
    _init(rank, world, port, 60)
    rng = np.random.default_rng(123)
    a_full = rng.uniform(-1, 1, (m, k))
    w = rng.uniform(-1, 1, (k, n)) if rank == 0 else np.zeros((k, n))
    wt = torch.from_numpy(w)
    dist.broadcast(wt, src=0)
    w = wt.numpy()
    begin, rows = hx.shard_rows(m, world, rank)
    mine = oracle.relu(oracle.matmul(a_full[begin:begin + rows], w))
    if rank == 0:
        c = np.empty((m, n))
        c[begin:begin + rows] = mine
        for peer in range(1, world):
            pb, pr = hx.shard_rows(m, world, peer)
            buf = torch.empty((pr, n), dtype=torch.float64)
            dist.recv(buf, src=peer)
            c[pb:pb + pr] = buf.numpy()
        want = oracle.relu(oracle.matmul(a_full, w))
        np.save(result_path, np.array([np.array_equal(c.view(np.uint64),
                                                      want.view(np.uint64))]))
    elif rows:
        dist.send(torch.from_numpy(np.ascontiguousarray(mine)), dst=0)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("m", [37, 64])
def test_two_rank_sharded_linear_matches_oracle(tmp_path, m):
    path = str(tmp_path / "ok.npy")
    spawn_ranks(_sharded_rank, 2, (m, 24, 40, path))
    assert bool(np.load(path)[0])


def _dropped_rank(rank, world, port, result_path):
    import torch
    _init(rank, world, port, 5)
    t = torch.zeros(4, dtype=torch.float64)
    dist.broadcast(t, src=0)
    if rank == 1:
        os._exit(0)  # leaves between steps, nothing in flight
    ok = False
    try:
        buf = torch.empty(4, dtype=torch.float64)
        dist.recv(buf, src=1)
    except Exception:  # the collective ends with an error
        ok = True
    np.save(result_path, np.array([ok]))
    os._exit(0)


def test_dropped_rank_surfaces_as_an_error(tmp_path):
    path = str(tmp_path / "ok.npy")
    ctx = mp.start_processes(_dropped_rank, args=(2, free_port(), path),
                             nprocs=2, join=False, start_method="spawn")
    for p in ctx.processes:
        p.join(timeout=120)
    assert bool(np.load(path)[0])
