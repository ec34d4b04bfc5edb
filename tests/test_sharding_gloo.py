"""The row-sharded linear's host-side plan, run on CPU ranks over gloo.

hexir_sharded_linear_f64 (comm.h) splits the job three ways, each by a rule
of this library's C ABI that every rank evaluates for itself:
  - rows of a and c over ranks: hexir_shard_rows;
  - the weight's broadcast from rank 0 in k pieces: hexir_shard_weight_pieces;
  - each rank's output rows back to rank 0 in pieces that shrink
    geometrically: hexir_shard_gather_pieces (the NCCL gather path).
Here gloo ranks follow that same plan with this library's CPU backend as
the compute: each piece of a rank's rows is a cpu-placed .hxb module
(linear + relu) run by hexir_execute, whose arithmetic is the reference's.
Rank 0 receives every peer's pieces in the order comm.cc posts them and
places them by the planners' offsets; the assembled result must equal the
oracle bit for bit.  A planner that left a gap, overlapped or lost rows
would leave NaN rows or wrong bits here.  A last test drops a rank before the
gather: the survivor's collective must end with an error within the
process-group timeout instead of waiting for ever.
"""

import datetime
import os

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

import hexir_b200 as hx
from tests.conftest import free_port, spawn_ranks


def _init(rank, world, port, timeout_s):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _cpu_linear_relu(a_rows, w):
    """relu(a_rows . w) by this library's CPU backend: a cpu-placed module
    run by hexir_execute (the product's host kernels, not the oracle)."""
    p = hx.Program()
    p.relu(p.linear(p.constant(a_rows), p.constant(w)))
    module = hx.Module(p.emit(""))
    dev = hx.Device("cpu")
    try:
        return hx.execute(module, dev, out_shape=(a_rows.shape[0], w.shape[1]))
    finally:
        module.close()
        dev.close()


def _sharded_rank(rank, world, port, m, n, k, result_path):
    import torch
    _init(rank, world, port, 120)
    rng = np.random.default_rng(123)
    a_full = rng.uniform(-1, 1, (m, k))
    w_src = rng.uniform(-1, 1, (k, n))
    # 1. The weight from rank 0, in the planned k pieces (rows of w).
    w = w_src.copy() if rank == 0 else np.full((k, n), np.nan)
    bounds = hx.shard_weight_pieces(k, world)
    for lo, hi in zip(bounds[:-1], bounds[1:]):
        piece = torch.from_numpy(np.ascontiguousarray(w[lo:hi]))
        dist.broadcast(piece, src=0)
        w[lo:hi] = piece.numpy()
    # 2. This rank's rows, piece by piece as they would be gathered.
    begin, rows = hx.shard_rows(m, world, rank)
    mine = hx.shard_gather_pieces(rows)
    if rank == 0:
        c = np.full((m, n), np.nan)
    for i in range(_max_pieces(m, world)):
        if i < len(mine):
            cb, cnt = mine[i]
            out = _cpu_linear_relu(a_full[begin + cb:begin + cb + cnt], w)
            if rank == 0:
                c[begin + cb:begin + cb + cnt] = out
        # 3. Piece i of every peer to rank 0 (comm.cc posts one group per
        #    piece index, peers in rank order).
        if rank == 0:
            for peer in range(1, world):
                pb, pr = hx.shard_rows(m, world, peer)
                pieces = hx.shard_gather_pieces(pr)
                if i >= len(pieces):
                    continue
                cb, cnt = pieces[i]
                buf = torch.empty((cnt, n), dtype=torch.float64)
                dist.recv(buf, src=peer)
                c[pb + cb:pb + cb + cnt] = buf.numpy()
        elif i < len(mine):
            dist.send(torch.from_numpy(np.ascontiguousarray(out)), dst=0)
    if rank == 0:
        from oracle import oracle
        want = oracle.relu(oracle.matmul(a_full, w_src))
        np.save(result_path, np.array([
            not np.isnan(c).any(),
            np.array_equal(c.view(np.uint64), want.view(np.uint64)),
            np.array_equal(w.view(np.uint64), w_src.view(np.uint64))]))
    dist.barrier()
    dist.destroy_process_group()


def _max_pieces(m, world):
    """Most gather pieces of any rank (the number of gather steps)."""
    return max(len(hx.shard_gather_pieces(hx.shard_rows(m, world, r)[1]))
               for r in range(world))


@pytest.mark.parametrize("world,m,n,k", [
    (2, 37, 24, 512),       # one weight piece, one gather piece per rank
    (2, 1000, 24, 2048),    # two weight pieces; 500 rows: one gather piece
    (2, 8192 + 5, 16, 8192),  # two weight pieces, five gather pieces
    (3, 3000, 8, 2048),     # three ranks, ragged split, two gather pieces
])
def test_sharded_plan_on_gloo_ranks_matches_oracle(tmp_path, world, m, n, k):
    path = str(tmp_path / "ok.npy")
    spawn_ranks(_sharded_rank, world, (m, n, k, path))
    no_gap, bit_exact, w_ok = (bool(x) for x in np.load(path))
    assert w_ok, "weight pieces did not rebuild the weight"
    assert no_gap, "gather pieces left rows unwritten"
    assert bit_exact


@pytest.mark.parametrize("rows", [0, 1, 127, 255, 256, 511, 512, 1000, 4096,
                                  4099, 8192, 8197, 32768, 100000])
def test_gather_pieces_tile_the_rows(rows):
    pieces = hx.shard_gather_pieces(rows)
    if rows == 0:
        assert pieces == []
        return
    assert 1 <= len(pieces) <= 5
    at = 0
    for i, (b, c) in enumerate(pieces):
        assert b == at and c > 0
        at += c
        if i + 1 < len(pieces):
            assert c % 128 == 0 and c >= 256
            # Each piece is at least the rest: later pieces shrink.
            assert c >= sum(x[1] for x in pieces[i + 1:]) - 128 * 2
    assert at == rows
    if len(pieces) > 1:
        assert pieces[-1][1] >= 256


@pytest.mark.parametrize("k,ranks", [(1, 2), (96, 2), (2047, 2), (2048, 2),
                                     (8192, 8), (8192, 1), (4096, 1)])
def test_weight_pieces_tile_k(k, ranks):
    b = hx.shard_weight_pieces(k, ranks)
    assert b[0] == 0 and b[-1] == k
    assert all(x < y for x, y in zip(b[:-1], b[1:]))
    if ranks == 1 or k < 2048:
        assert b == [0, k]
    else:
        # The first piece, the only exposed transfer, is a whole number of
        # the kernel's 32-wide k tiles.
        assert len(b) == 3 and b[1] % 32 == 0


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
