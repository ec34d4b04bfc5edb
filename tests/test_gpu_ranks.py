"""hexir_sharded_linear_f64 with one process per GPU (2 GPUs).

Each rank is a spawned process driving its own GPU; the NCCL unique id
travels over a gloo group on 127.0.0.1.  Rank 0 holds the whole output.
The same call runs twice: rows stored by every rank straight into rank 0's
output through a CUDA IPC mapping (the default where the set-up check
passes), and rows gathered with NCCL send/receive (HEXIR_SHARD_GATHER_NCCL).
Both must equal the oracle within the normwise tolerance.  With direct
stores every rank runs one launch over its rows, so each block of rows must
equal, bit for bit, the same launch on one GPU; and a second call into a
different output buffer must land there (the root sends its output's
location every call).  The NCCL path computes in pieces whose k-split may
differ, so it is held to the tolerance only.
"""

import ctypes as C
import datetime
import os

import numpy as np
import pytest

import hexir_b200 as hx
from hexir_b200 import _ffi
from tests.conftest import spawn_ranks

pytestmark = pytest.mark.gpu

TOL = 1e-12


def _rank(rank, world, port, m, n, k, result_path):
    import torch.distributed as dist
    from hexir_b200 import _ffi
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    lib = hx.lib()
    uid = C.create_string_buffer(128)
    if rank == 0:
        _ffi.check(lib.hexir_comm_unique_id(uid, 128), "unique id")
    obj = [uid.raw if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    uid = C.create_string_buffer(obj[0], 128)
    comm = C.c_void_p()
    _ffi.check(lib.hexir_comm_init_rank(uid, 128, world, rank, rank,
                                        C.byref(comm)), "comm init")
    comm = comm.value
    direct = lib.hexir_comm_direct_stores(comm)

    rng = hx.Rng(31)
    a = rng.uniform((m, k))
    w = rng.uniform((k, n))
    begin, rows = hx.shard_rows(m, world, rank)
    dev = hx.Device(f"cuda:{rank}")
    ba = dev.upload(a[begin:begin + rows] if rows else np.zeros(1))
    bw = dev.upload(w if rank == 0 else np.zeros_like(w))
    out_rows = m if rank == 0 else max(rows, 1)
    outs = [dev.buffer(out_rows * n * 8) for _ in range(2)]
    results = {}
    for name, buf, flags in [
            ("direct", outs[0], _ffi.MATMUL_RELU),
            ("nccl", outs[1], _ffi.MATMUL_RELU | _ffi.SHARD_GATHER_NCCL),
            ("direct_again", outs[1], _ffi.MATMUL_RELU)]:
        if rank == 0:
            buf.write(np.full((m, n), np.nan))
        dist.barrier()
        _ffi.check(lib.hexir_sharded_linear_f64(comm, ba.ptr, bw.ptr, buf.ptr,
                                                m, n, k, flags, dev.stream),
                   "sharded linear " + name)
        _ffi.check(lib.hexir_comm_synchronize(comm, dev.stream),
                   "comm synchronize " + name)
        if rank == 0:
            results[name] = buf.read((m, n))
    lib.hexir_comm_release(comm)
    if rank == 0:
        from oracle import oracle
        # Every rank's block as one launch on this GPU alone, planned as the
        # sharded path plans (no stream-K: a rank's rows may run in pieces).
        single = np.empty((m, n))
        for r in range(world):
            rb, rr = hx.shard_rows(m, world, r)
            if not rr:
                continue
            xa = dev.upload(a[rb:rb + rr])
            xc = dev.buffer(rr * n * 8)
            hx.cuda_matmul(0, xa.ptr, bw.ptr, xc.ptr, rr, n, k,
                           _ffi.MATMUL_RELU | _ffi.MATMUL_NO_STREAM_K,
                           dev.stream)
            hx.cuda_synchronize(0, dev.stream)
            single[rb:rb + rr] = xc.read((rr, n))
        bits = lambda x: x.view(np.uint64)
        # The oracle on rows spread over every rank's block.
        sample = np.unique(np.linspace(0, m - 1, min(m, 48)).astype(int))
        want = oracle.relu(oracle.matmul(a[sample], w))
        out = {"direct_flag": direct}
        for name, got in results.items():
            out["nan_" + name] = bool(np.isnan(got).any())
            out["err_" + name] = oracle.normwise_error(got[sample], want)
        out["direct_is_single"] = bool(np.array_equal(bits(results["direct"]),
                                                      bits(single)))
        out["direct_is_again"] = bool(np.array_equal(
            bits(results["direct"]), bits(results["direct_again"])))
        np.save(result_path, np.array([out], dtype=object))
    dist.barrier()
    dist.destroy_process_group()


def two_gpus():
    return hx.device_count() >= 2


@pytest.mark.skipif(not two_gpus(), reason="needs 2 GPUs")
@pytest.mark.parametrize("m,n,k", [
    (1000, 384, 512), (3, 130, 96), (2048, 1024, 1024),
    # k >= 2048: the weight is broadcast in k pieces and the peer computes
    # behind it, continuing its sums piece by piece (4096 rows x 2560: no k
    # split in the one-shot plan, so the pieces must match it bit for bit).
    (8192, 2560, 2048),
    # k >= 2048 but a one-shot plan that splits k: the peer waits for the
    # whole weight and runs that plan.
    (512, 256, 4096)])
def test_two_processes_sharded_linear(tmp_path, m, n, k):
    path = str(tmp_path / "out.npy")
    spawn_ranks(_rank, 2, (m, n, k, path))
    r = np.load(path, allow_pickle=True)[0]
    # Two processes on one host: the peers can map rank 0's memory.
    assert int(r["direct_flag"]) == 1
    for name in ["direct", "nccl", "direct_again"]:
        assert not r["nan_" + name], name
        assert r["err_" + name] <= TOL, name
    assert r["direct_is_single"]
    assert r["direct_is_again"]


def _failing_peer_rank(rank, world, port, m, n, k, flags, result_path):
    """Rank 1's first kernel launch fails (host-side fault injection, before
    the driver call); rank 0 must learn of it from hexir_comm_synchronize,
    and the next call, with no fault, must be right again."""
    import torch.distributed as dist
    from hexir_b200 import _ffi
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    lib = hx.lib()
    uid = C.create_string_buffer(128)
    if rank == 0:
        _ffi.check(lib.hexir_comm_unique_id(uid, 128), "unique id")
    obj = [uid.raw if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    uid = C.create_string_buffer(obj[0], 128)
    comm = C.c_void_p()
    _ffi.check(lib.hexir_comm_init_rank(uid, 128, world, rank, rank,
                                        C.byref(comm)), "comm init")
    comm = comm.value
    rng = hx.Rng(37)
    a = rng.uniform((m, k))
    w = rng.uniform((k, n))
    begin, rows = hx.shard_rows(m, world, rank)
    dev = hx.Device(f"cuda:{rank}")
    ba = dev.upload(a[begin:begin + rows])
    bw = dev.upload(w if rank == 0 else np.zeros_like(w))
    c = dev.buffer((m if rank == 0 else rows) * n * 8)
    out = {}
    for name, fault in (("faulted", rank == 1), ("clean", False)):
        if fault:
            hx.fault_configure("launch:1")
        dist.barrier()
        out["call_" + name] = lib.hexir_sharded_linear_f64(
            comm, ba.ptr, bw.ptr, c.ptr, m, n, k, flags, dev.stream)
        hx.fault_configure("")
        out["sync_" + name] = lib.hexir_comm_synchronize(comm, dev.stream)
        if rank == 0 and name == "clean":
            from oracle import oracle
            got = c.read((m, n))
            sample = np.unique(np.linspace(0, m - 1, 24).astype(int))
            out["err"] = oracle.normwise_error(
                got[sample], oracle.relu(oracle.matmul(a[sample], w)))
    lib.hexir_comm_release(comm)
    np.save(result_path.replace(".npy", f"_{rank}.npy"),
            np.array([out], dtype=object))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not two_gpus(), reason="needs 2 GPUs")
@pytest.mark.parametrize("gather", ["direct", "nccl"])
@pytest.mark.parametrize("k", [512, 2048])
def test_peer_failure_reaches_every_rank(tmp_path, gather, k):
    m, n = 1000, 256
    flags = _ffi.MATMUL_RELU | (_ffi.SHARD_GATHER_NCCL if gather == "nccl"
                                else 0)
    path = str(tmp_path / "out.npy")
    spawn_ranks(_failing_peer_rank, 2, (m, n, k, flags, path))
    r0 = np.load(path.replace(".npy", "_0.npy"), allow_pickle=True)[0]
    r1 = np.load(path.replace(".npy", "_1.npy"), allow_pickle=True)[0]
    # The failing rank's own call reports its launch failure ...
    assert r1["call_faulted"] == _ffi.ERROR_DEVICE
    # ... the root's call itself cannot know yet, but its synchronize does,
    # and so does the failing rank's.
    assert r0["call_faulted"] == _ffi.OK
    assert r0["sync_faulted"] == _ffi.ERROR_DEVICE
    assert r1["sync_faulted"] == _ffi.ERROR_DEVICE
    # The failure is cleared: the next call is whole and right.
    for r in (r0, r1):
        assert r["call_clean"] == _ffi.OK and r["sync_clean"] == _ffi.OK
    assert r0["err"] <= TOL


def _host_rank(rank, world, port, m, n, k, flags, result_path):
    """hexir_sharded_linear_host_f64: every rank hands in host rows of a
    (page-locked), the weight (root only, or every rank with
    SHARD_W_ON_ALL) and gets its rows of c back in host memory."""
    import torch.distributed as dist
    from hexir_b200 import _ffi
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    comm = _comm(rank, world, dist)
    lib = hx.lib()
    rng = hx.Rng(43)
    a = rng.uniform((m, k))
    w = rng.uniform((k, n))
    begin, rows = hx.shard_rows(m, world, rank)
    a_rows = np.ascontiguousarray(a[begin:begin + rows])
    c_rows = np.full((max(rows, 1), n), np.nan)
    for arr in (a_rows, c_rows):
        _ffi.check(lib.hexir_host_register(arr.ctypes.data, arr.nbytes),
                   "host register")
    w_arg = w.ctypes.data if (rank == 0 or flags & _ffi.SHARD_W_ON_ALL) else None
    dev = hx.Device(f"cuda:{rank}")
    statuses = []
    for _ in range(2):  # twice: the workspace kept in comm is reused
        c_rows[:] = np.nan
        statuses.append(lib.hexir_sharded_linear_host_f64(
            comm, a_rows.ctypes.data, w_arg, c_rows.ctypes.data, m, n, k,
            flags, dev.stream))
    for arr in (a_rows, c_rows):
        lib.hexir_host_unregister(arr.ctypes.data)
    lib.hexir_comm_release(comm)
    # Rank 0 assembles every rank's rows (gloo) and checks them.
    got = [None] * world
    dist.all_gather_object(got, (begin, rows, c_rows[:rows].copy(), statuses))
    if rank == 0:
        from oracle import oracle
        c = np.full((m, n), np.nan)
        all_ok = True
        for b, r, block, st in got:
            c[b:b + r] = block
            all_ok &= all(s == _ffi.OK for s in st)
        # One launch per rank's block on this GPU alone, without stream-K
        # (the rows run in chunks): the bits to match.
        single = np.empty((m, n))
        bw = dev.upload(w)
        for b, r, _, _ in got:
            if not r:
                continue
            xa = dev.upload(a[b:b + r])
            xc = dev.buffer(r * n * 8)
            hx.cuda_matmul(0, xa.ptr, bw.ptr, xc.ptr, r, n, k,
                           (flags & _ffi.MATMUL_RELU) | _ffi.MATMUL_NO_STREAM_K,
                           dev.stream)
            hx.cuda_synchronize(0, dev.stream)
            single[b:b + r] = xc.read((r, n))
        sample = np.unique(np.linspace(0, m - 1, min(m, 48)).astype(int))
        want = oracle.matmul(a[sample], w)
        if flags & _ffi.MATMUL_RELU:
            want = oracle.relu(want)
        np.save(result_path, np.array([{
            "ok": bool(all_ok), "nan": bool(np.isnan(c).any()),
            "bits": bool(np.array_equal(c.view(np.uint64), single.view(np.uint64))),
            "err": oracle.normwise_error(c[sample], want)}], dtype=object))
    dist.barrier()
    dist.destroy_process_group()


def _comm(rank, world, dist):
    from hexir_b200 import _ffi
    lib = hx.lib()
    uid = C.create_string_buffer(128)
    if rank == 0:
        _ffi.check(lib.hexir_comm_unique_id(uid, 128), "unique id")
    obj = [uid.raw if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    uid = C.create_string_buffer(obj[0], 128)
    comm = C.c_void_p()
    _ffi.check(lib.hexir_comm_init_rank(uid, 128, world, rank, rank,
                                        C.byref(comm)), "comm init")
    return comm.value


def _check_host_result(path):
    r = np.load(path, allow_pickle=True)[0]
    assert r["ok"]
    assert not r["nan"]
    assert r["bits"]
    assert r["err"] <= TOL


@pytest.mark.parametrize("m,n,k,flags", [
    (1000, 384, 512, _ffi.MATMUL_RELU),
    (2048 + 130, 256, 1024, 0),
    (3, 130, 96, _ffi.MATMUL_RELU),
    # k >= 2048 and an unsplit plan: the weight streams in k pieces and the
    # rows continue their sums piece by piece (bits of one launch).
    (8192 + 5, 1280, 2048, _ffi.MATMUL_RELU),
    # k >= 2048 but a plan that splits k: whole weight, then the plan.
    (300, 256, 4096, _ffi.MATMUL_RELU)])
def test_host_buffer_sharded_linear_one_rank(tmp_path, m, n, k, flags):
    """One rank (one GPU): the chunked upload / compute / download path."""
    path = str(tmp_path / "out.npy")
    spawn_ranks(_host_rank, 1, (m, n, k, flags, path))
    _check_host_result(path)


@pytest.mark.skipif(not two_gpus(), reason="needs 2 GPUs")
@pytest.mark.parametrize("m,n,k", [(1000, 384, 512), (4096 + 7, 1024, 2048),
                                   (3, 130, 96), (16384 + 6, 1280, 2048)])
@pytest.mark.parametrize("w_mode", [0, _ffi.SHARD_W_ON_ALL])
def test_host_buffer_sharded_linear_two_ranks(tmp_path, m, n, k, w_mode):
    path = str(tmp_path / "out.npy")
    spawn_ranks(_host_rank, 2, (m, n, k, _ffi.MATMUL_RELU | w_mode, path))
    _check_host_result(path)
