#!/usr/bin/env python3
"""Benchmark of the hexir hot path on B200: f64 hexir.linear + fused relu.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl hexir|reference]

Workload (per GPU): hexir.linear a[8192 x 8192] . w[8192 x 8192] f64 with
the relu fused in the epilogue, a and w uniform[-1, 1] from the writer's
seeded stream (seed 1, a then w).  At N GPUs the job is the row-sharded
linear a[8192N x 8192] . w: each GPU holds its 8192 rows of a, w is
broadcast from GPU 0 over NVLink (NCCL) and every GPU's kernel stores its
output tiles straight into GPU 0's output over NVLink (CUDA IPC mapping;
`--gather nccl` sends the rows with NCCL instead) every step (weak scaling;
N = 4 is the 32768 x 8192 x 8192 shape).

One JSON line on rank 0:
  value      GFLOP/s of the whole job, inputs resident in HBM, device time
             (CUDA events on the launching stream, max over ranks)
  e2e        the same through the public API with host buffers: a .hxb module
             run by hexir_execute_capture (constants copied host->device,
             result copied back) at N = 1; hexir_sharded_linear_host_f64 at
             N > 1 (each rank's rows of a up and of c down over its own host
             link, the weight in per-rank slices gathered over NVLink, the
             result rows in one shared host mapping)
  roofline   the GEMM kernel's FLOP rate against the FP64 tensor-core (DMMA)
             peak measured on this GPU by a register-only DMMA probe
  cpu_baseline  the reference's own CPU kernel (hexir_ref_matmul_f64, built
             from the reference sources into oracle/_ref) on a bounded row
             sample with all host threads (N = 1 only)
--impl reference times that CPU implementation alone, as the reference arm.

--suite prints one JSON line per configuration instead (1 GPU): the 256 x 256
parity graph's latency, the GEMM sweep 1024-8192, relu over 2^28, each
activation over 16384 x 16384 (softmax along the rows), the skinny linear
M = 1 / 16 / 128, the three-layer MLP chain, the fused linear -> add -> relu
and constants kept on the GPU.  --profile runs one kernel a few times: the
command line the committed ncu summaries capture.
"""

from __future__ import annotations

import argparse
import json
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = ("f64 hexir.linear GFLOP/s & % FP64 peak @8192³ (1/2/4/8 GPU); "
          "relu HBM GB/s")
M_PER_GPU = N_DIM = K_DIM = 8192
SEED = 1
PROFILE_SUMMARY = os.path.join(ROOT, "profiles", "linear_f64_tma_8192.json")


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["hexir", "reference"], default="hexir")
    p.add_argument("--m", type=int, default=M_PER_GPU,
                   help="rows of a per GPU (default 8192)")
    p.add_argument("--gather", choices=["auto", "nccl"], default="auto",
                   help="N > 1: how output rows reach GPU 0 (auto: kernel "
                        "stores through a CUDA IPC mapping where possible)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-relu", action="store_true")
    p.add_argument("--profile", choices=["relu", "skinny", "linear",
                                         "activation", "square"],
                   help="run only one kernel a few times (the small cases the "
                        "committed ncu summaries capture)")
    p.add_argument("--op", default="gelu",
                   help="--profile activation: which activation")
    p.add_argument("--cols", type=int, default=8192,
                   help="--profile activation: row length (2^log2n elements)")
    p.add_argument("--log2n", type=int, default=26,
                   help="--profile relu: 2^log2n elements")
    p.add_argument("--size", type=int, default=1024,
                   help="--profile square: size^3 linear + relu (seed 1), "
                        "the planner's plan")
    p.add_argument("--suite", action="store_true",
                   help="instead of the bench line, one JSON line per "
                        "configuration: GEMM sweep 1024-8192, relu 2^28, "
                        "the activations over 2^28, skinny linear "
                        "M=1/16/128, 3-layer MLP chain")
    return p.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return rank, world, local


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clock / throttle samples every 200 ms during the timed
    region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,"
             "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        if not shutil.which("nvidia-smi"):
            return
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.out = open(self.path, "w")
        self.proc = subprocess.Popen(
            ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
             "--format=csv,noheader,nounits", "-lms", "200"],
            stdout=self.out, stderr=subprocess.DEVNULL)
        time.sleep(0.3)

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.close()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                 "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax = float(parts[2])
                except ValueError:
                    continue
                for name, flag in zip(names, parts[5:9]):
                    if flag.lower() == "active":
                        reasons.add(name)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ helpers

def make_w(world: int, m_rows: int):
    import hexir_b200 as hx
    rng = hx.Rng(SEED)
    rng.skip(world * m_rows * K_DIM)
    return rng.uniform((K_DIM, N_DIM))


def a_rows_global(rows):
    """Rows `rows` (global indices) of the synthetic a."""
    import numpy as np
    import hexir_b200 as hx
    out = np.empty((len(rows), K_DIM))
    for i, g in enumerate(rows):
        rng = hx.Rng(SEED)
        rng.skip(int(g) * K_DIM)
        out[i] = rng.uniform(K_DIM)
    return out


def dmma_peak_tflops(ordinal: int) -> float:
    """FP64 DMMA throughput of this GPU: register-only probe, best of 5."""
    import torch
    import hexir_b200 as hx
    from hexir_b200 import _ffi
    import ctypes as C
    sms = hx.lib().hexir_cuda_sm_count(ordinal)
    blocks = sms * 4
    out = torch.empty(blocks * 256, dtype=torch.float64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    flops = C.c_double()
    best = 0.0
    iters = 4096
    for trial in range(6):
        start = torch.cuda.Event(enable_timing=True)
        stop = torch.cuda.Event(enable_timing=True)
        start.record()
        _ffi.check(hx.lib().hexir_cuda_dmma_probe(
            ordinal, out.data_ptr(), blocks, iters, stream, C.byref(flops)),
            "dmma probe")
        stop.record()
        torch.cuda.synchronize()
        if trial:
            best = max(best, flops.value / (start.elapsed_time(stop) * 1e-3) / 1e12)
    return best


def cublas_dgemm_tflops(a, w, steps: int = 3) -> float:
    """Vendor line: torch.matmul in f64 (cuBLAS DGEMM), kernel only."""
    import torch
    c = torch.matmul(a, w)
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        torch.matmul(a, w, out=c)
    stop.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop) / steps
    return 2.0 * a.shape[0] * a.shape[1] * w.shape[1] / (ms * 1e-3) / 1e12


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_reference_rate(rows: int, steps: int = 1, warmup: int = 0,
                       threads: int = 0):
    """GFLOP/s of the reference CPU kernel on `rows` rows of the workload
    (`threads` host threads, default all, each on its own row slice).
    Returns (gflops, threads, kind, sample description, step seconds)."""
    import numpy as np
    from oracle import oracle
    threads = threads or os.cpu_count() or 1
    kind = "reference" if oracle.have_reference() else "port"
    rng = np.random.default_rng(SEED)
    a = rng.uniform(-1, 1, (rows, K_DIM))
    w = rng.uniform(-1, 1, (K_DIM, N_DIM))
    c = np.empty((rows, N_DIM))

    def one_step():
        per = (rows + threads - 1) // threads
        jobs = []
        for t in range(threads):
            r0, r1 = t * per, min(rows, (t + 1) * per)
            if r0 >= r1:
                break
            if kind == "reference":
                fn = lambda r0=r0, r1=r1: oracle.ref_matmul_rows_into(a, w, c, r0, r1)
            else:
                fn = lambda r0=r0, r1=r1: c.__setitem__(
                    slice(r0, r1), oracle.matmul_rows(a, w, r0, r1))
            jobs.append(threading.Thread(target=fn))
        t0 = time.perf_counter()
        for j in jobs:
            j.start()
        for j in jobs:
            j.join()
        return time.perf_counter() - t0

    for _ in range(warmup):
        one_step()
    times = [one_step() for _ in range(steps)]
    flops = 2.0 * rows * N_DIM * K_DIM
    gflops = flops / statistics.median(times) / 1e9
    used = min(threads, rows)
    sample = (f"{rows} rows of the {M_PER_GPU}x{N_DIM}x{K_DIM} linear per step "
              f"(cost is linear in rows), hexir_ref_matmul_f64 on row slices, "
              f"{used} thread{'s' if used > 1 else ''} of {os.cpu_count()} "
              f"host cores ({cpu_model()})")
    return gflops, used, kind, sample, times


def reference_schedule_gpu(ordinal, a, w, peak, steps: int = 2) -> dict:
    """The reference's own GPU schedule for the linear (thread per output,
    serial k; hexir_cuda_baseline_reference_schedule_f64, a CUDA-C
    restatement, since the reference's compiler cannot be built here) on
    the same GPU and operands: a reported baseline."""
    import numpy as np
    import torch
    import hexir_b200 as hx
    from hexir_b200 import _ffi
    from oracle import oracle
    m, k = a.shape
    n = w.shape[1]
    c = torch.empty((m, n), dtype=torch.float64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    run = lambda: _ffi.check(hx.lib().hexir_cuda_baseline_reference_schedule_f64(
        ordinal, a.data_ptr(), w.data_ptr(), c.data_ptr(), m, n, k, stream),
        "reference schedule")
    ms = timed_ms(run, steps=steps, warmup=1)
    rows = np.linspace(0, m - 1, 3).astype(int)
    err = oracle.normwise_error(
        c[torch.from_numpy(rows).cuda()].cpu().numpy(),
        oracle.matmul(a[torch.from_numpy(rows).cuda()].cpu().numpy(),
                      w.cpu().numpy()))
    tf = 2.0 * m * n * k / (ms * 1e-3) / 1e12
    return {"value": round(tf * 1e3, 3), "unit": "GFLOP/s",
            "ms_per_launch": round(ms, 3), "frac_of_dmma_peak": round(tf / peak, 4),
            "kernel": "hexir_baseline_reference_schedule_f64",
            "kind": "CUDA-C restatement of the reference's generated schedule "
                    "(thread per output, grid (n/bs, m), serial k, FMA); the "
                    "reference compiler (MLIR, LLVM 24.0git) is not buildable "
                    "here",
            "normwise_err_sampled": err, "steps": steps}


# ------------------------------------------------------------------ arms

def workload_config(world: int, m_rows: int) -> dict:
    """The `config` of both arms' JSON lines for N = world GPUs."""
    m_total = m_rows * world
    return {"workload": f"hexir.linear+relu f64 row-sharded "
                        f"a[{m_total}x{K_DIM}] . w[{K_DIM}x{N_DIM}] "
                        f"({m_rows} rows per GPU)",
            "m": m_total, "n": N_DIM, "k": K_DIM,
            "parallelism": f"rows x{world}" + (
                ", w broadcast over NVLink (NCCL), output rows to GPU 0 over "
                "NVLink" if world > 1 else ""),
            "l2": "inputs larger than L2 (a+w = 1 GiB per GPU)"}


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    rows = max(2 * threads, 16)
    gflops, used, kind, sample, times = cpu_reference_rate(
        rows, steps=args.steps, warmup=args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gflops, 3),
        "unit": "GFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(statistics.median(times) * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f64", "data": "synthetic uniform[-1,1]",
        "config": {**workload_config(args.gpus, args.m),
                   "reference_sample_rows_per_step": rows},
        "cpu_baseline": {"value": round(gflops, 3), "unit": "GFLOP/s",
                         "cores": used, "kind": kind, "sample": sample},
        "e2e": {"value": round(gflops, 3), "unit": "GFLOP/s",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_hexir(args):
    import numpy as np
    import torch
    import hexir_b200 as hx
    from hexir_b200 import _ffi
    from oracle import oracle

    rank, world, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    ordinal = local
    m_rows = args.m
    m_total = m_rows * world

    pg = None
    comm = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        pg = dist
        import ctypes as C
        uid = C.create_string_buffer(128)
        if rank == 0:
            _ffi.check(hx.lib().hexir_comm_unique_id(uid, 128), "unique id")
        obj = [uid.raw if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        uid = C.create_string_buffer(obj[0], 128)
        h = C.c_void_p()
        _ffi.check(hx.lib().hexir_comm_init_rank(uid, 128, world, rank, ordinal,
                                                 C.byref(h)), "comm init")
        comm = h.value
        # One line per rank about its communicator (stderr).
        print(f"hexir comm: rank {hx.lib().hexir_comm_rank(comm)} of "
              f"{hx.lib().hexir_comm_size(comm)} on cuda:{ordinal}, direct "
              f"row stores {hx.lib().hexir_comm_direct_stores(comm)}, "
              f"NCCL {torch.cuda.nccl.version()}", file=sys.stderr, flush=True)
    shard_flags = _ffi.MATMUL_RELU | (_ffi.SHARD_GATHER_NCCL
                                      if args.gather == "nccl" else 0)
    direct = bool(comm) and args.gather != "nccl" and bool(
        hx.lib().hexir_comm_direct_stores(comm))

    # Inputs: this rank's rows of a; w on every rank (rank 0's is the source
    # of the broadcast; the others' buffers are overwritten every step).
    rng = hx.Rng(SEED)
    rng.skip(rank * m_rows * K_DIM)
    a_host = rng.uniform((m_rows, K_DIM))
    w_host = make_w(world, m_rows)
    a = torch.from_numpy(a_host).cuda()
    w = torch.from_numpy(w_host).cuda()
    c_rows = m_total if rank == 0 else m_rows
    c = torch.empty((c_rows, N_DIM), dtype=torch.float64, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream

    def step():
        if comm is None:
            hx.cuda_matmul(ordinal, a.data_ptr(), w.data_ptr(), c.data_ptr(),
                           m_rows, N_DIM, K_DIM, _ffi.MATMUL_RELU, stream)
        else:
            _ffi.check(hx.lib().hexir_sharded_linear_f64(
                comm, a.data_ptr(), w.data_ptr(), c.data_ptr(), m_total, N_DIM,
                K_DIM, shard_flags, stream), "sharded linear")

    def synchronize():
        hx.cuda_synchronize(ordinal, stream)
        if comm is not None:
            # Every rank: a failure on any rank's part of the step.
            _ffi.check(hx.lib().hexir_comm_synchronize(comm, stream),
                       "hexir_comm_synchronize")

    for _ in range(args.warmup):
        step()
    synchronize()
    torch.cuda.synchronize()
    if pg:
        pg.barrier()
    torch.cuda.synchronize()

    clocks = ClockSampler(ordinal)
    clocks.start()
    launches0 = hx.launch_count()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        step()
    stop.record()
    torch.cuda.synchronize()
    launches = hx.launch_count() - launches0
    clock_info = clocks.stop()
    synchronize()
    ms = start.elapsed_time(stop) / args.steps
    if pg:
        t = torch.tensor([ms], device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        ms = float(t.item())
        pg.barrier()

    # The timed step computes the right thing: one row of every 128-row
    # tile of every rank's block of the root's output (at a different
    # offset inside each tile), all columns, against the oracle.
    if rank == 0:
        tile_rows = np.array([t * 128 + (t * 37) % 128
                              for t in range((m_rows + 127) // 128)])
        tile_rows = tile_rows[tile_rows < m_rows]
        rows = np.concatenate([p * m_rows + tile_rows for p in range(world)])
        got = c[torch.from_numpy(rows).cuda()].cpu().numpy()
        want = oracle.relu(oracle.matmul(a_rows_global(rows), w_host))
        err = oracle.normwise_error(got, want)
        if not err <= 1e-12:
            raise SystemExit(f"bench output wrong: normwise error {err}")

    flops_total = 2.0 * m_total * N_DIM * K_DIM
    value = flops_total / (ms * 1e-3) / 1e9

    line = {"metric": METRIC, "value": round(value, 3), "unit": "GFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic: uniform[-1,1], SplitMix64 seed 1 (a then w)",
            "config": workload_config(world, m_rows),
            "checked": f"{len(rows) if rank == 0 else 0} rows (one per 128-row "
                       "tile, all columns) of the timed output against the "
                       "oracle, normwise <= 1e-12",
            "gpu_launches": launches,
            "clocks": clock_info}
    if world > 1:
        line["comm"] = {"nranks": hx.lib().hexir_comm_size(comm),
                        "direct_row_stores": bool(direct),
                        "nccl": ".".join(map(str, torch.cuda.nccl.version()))}
        line["rows_to_gpu0"] = ("kernel stores over NVLink into GPU 0's output "
                                "(CUDA IPC mapping)" if direct else
                                "NCCL send/receive in pieces behind the GEMM")

    if rank == 0:
        # Roofline of the dominant kernel (hexir_linear_f64_tma): one launch
        # per step at N = 1, so the step's device time is its duration.
        peak = dmma_peak_tflops(ordinal)
        gemm_ms = ms
        if world > 1:
            s0 = torch.cuda.Event(enable_timing=True)
            s1 = torch.cuda.Event(enable_timing=True)
            s0.record()
            for _ in range(3):
                hx.cuda_matmul(ordinal, a.data_ptr(), w.data_ptr(), c.data_ptr(),
                               m_rows, N_DIM, K_DIM, _ffi.MATMUL_RELU, stream)
            s1.record()
            torch.cuda.synchronize()
            gemm_ms = s0.elapsed_time(s1) / 3
        achieved = 2.0 * m_rows * N_DIM * K_DIM / (gemm_ms * 1e-3) / 1e12
        traffic = None
        if os.path.exists(PROFILE_SUMMARY):
            with open(PROFILE_SUMMARY) as f:
                traffic = json.load(f).get("dram_bytes_per_launch")
        line["roofline"] = {
            "bound": "tensor", "achieved": round(achieved, 3),
            "peak": round(peak, 3), "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4) if peak else None,
            "traffic": traffic,
            "peak_source": "FP64 DMMA register-only probe on this GPU "
                           "(hexir_dmma_peak_probe, best of 5)",
            "kernel": "hexir_linear_f64_tma"}
        line["vendor"] = {"cublas_dgemm_tflops": round(
            cublas_dgemm_tflops(a, w), 3)}

    if rank == 0 and world == 1 and not args.no_relu:
        line["relu"] = relu_stream(ordinal)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["reference_schedule_gpu"] = reference_schedule_gpu(
            ordinal, a, w, line["roofline"]["peak"])

    if not args.no_e2e:
        line["e2e"] = run_e2e(args, rank, world, ordinal, a_host, w_host, comm, pg,
                              shard_flags)

    # The CPU baseline is measured at N = 1 only (the other ranks would wait
    # on it at the closing barrier).
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        rows = max(2 * threads, 16)
        gflops, used, kind, sample, _ = cpu_reference_rate(rows, steps=1)
        line["cpu_baseline"] = {"value": round(gflops, 3), "unit": "GFLOP/s",
                                "cores": used, "kind": kind, "sample": sample}
        # The stock reference path is single-threaded by construction.
        g1, _, kind1, sample1, _ = cpu_reference_rate(4, steps=1, threads=1)
        line["cpu_baseline"]["single_thread"] = {
            "value": round(g1, 4), "unit": "GFLOP/s", "cores": 1,
            "kind": kind1, "sample": sample1,
            "note": "the reference's CPU path as it ships: one thread"}

    if comm:
        hx.lib().hexir_comm_release(comm)
    if pg:
        pg.barrier()
        pg.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def run_e2e(args, rank, world, ordinal, a_host, w_host, comm, pg, shard_flags):
    """Same metric through the public API with host buffers."""
    import numpy as np
    import torch
    import hexir_b200 as hx
    from hexir_b200 import _ffi

    m_rows = a_host.shape[0]
    m_total = m_rows * world
    steps = max(1, min(args.steps, 5))
    warm = max(1, min(args.warmup, 2))
    if world == 1:
        # A .hxb module run by the VM: CONST uploads of a and w from the
        # module's RODATA, the fused linear+relu, capture of the result into
        # pinned host memory.
        prog = hx.Program()
        prog.relu(prog.linear(prog.constant(a_host), prog.constant(w_host)))
        tmp = tempfile.mkdtemp()
        path = os.path.join(tmp, "linear_relu_8192.hxb")
        prog.emit_file(path, "hexir.linear=cuda,hexir.relu=cuda")
        del prog
        module = hx.Module(path)
        dev = hx.Device(f"cuda:{ordinal}")
        out = torch.empty((m_rows, N_DIM), dtype=torch.float64).pin_memory()
        out_np = out.numpy()
        import ctypes as C

        def once():
            _ffi.check(hx.lib().hexir_execute_capture(
                module.handle, dev.handle, b"main", out_np.ctypes.data,
                out_np.nbytes), "hexir_execute_capture")

        for _ in range(warm):
            once()
        t0 = time.perf_counter()
        for _ in range(steps):
            once()
        sec = (time.perf_counter() - t0) / steps
        module.close()
        dev.close()
        shutil.rmtree(tmp, ignore_errors=True)
        h2d = a_host.nbytes + w_host.nbytes
        d2h = m_rows * N_DIM * 8
    else:
        # Through hexir_sharded_linear_host_f64: every rank moves its own rows
        # of a up and of c down over its own host link, the weight is
        # uploaded in per-rank slices that meet over NVLink, and the rows
        # land in one shared host mapping, so rank 0's process holds the
        # whole result.  Inputs and result are page-locked once, outside
        # the timed region.
        import ctypes as C
        lib = hx.lib()
        begin, rows = hx.shard_rows(m_total, world, rank)
        c_bytes = m_total * N_DIM * 8
        obj = [None]
        if rank == 0:
            path = None
            st = os.statvfs("/dev/shm") if os.path.isdir("/dev/shm") else None
            if st and st.f_bavail * st.f_frsize > c_bytes + (1 << 30):
                path = f"/dev/shm/hexir_bench_{os.getpid()}.f64"
                np.memmap(path, dtype=np.float64, mode="w+",
                          shape=(m_total, N_DIM)).flush()
            obj = [path]
        pg.broadcast_object_list(obj, src=0)
        try:
            shared = obj[0]
            if shared:
                c_all = np.memmap(shared, dtype=np.float64, mode="r+",
                                  shape=(m_total, N_DIM))
                c_rows = c_all[begin:begin + rows]
            else:
                c_all = None
                c_rows = np.empty((rows, N_DIM))
            a_rows = np.ascontiguousarray(a_host)
            w_all = np.ascontiguousarray(w_host)
            registered = []
            for arr in (a_rows, w_all, c_rows):
                ptr = arr.ctypes.data
                _ffi.check(lib.hexir_host_register(ptr, arr.nbytes), "host register")
                registered.append(ptr)
            stream = torch.cuda.current_stream().cuda_stream
            flags = _ffi.MATMUL_RELU | _ffi.SHARD_W_ON_ALL

            def once():
                _ffi.check(lib.hexir_sharded_linear_host_f64(
                    comm, a_rows.ctypes.data, w_all.ctypes.data, c_rows.ctypes.data,
                    m_total, N_DIM, K_DIM, flags, stream),
                    "hexir_sharded_linear_host_f64")

            for _ in range(warm):
                once()
            pg.barrier()
            t0 = time.perf_counter()
            for _ in range(steps):
                once()
            sec = (time.perf_counter() - t0) / steps
            t = torch.tensor([sec], device="cuda")
            pg.all_reduce(t, op=pg.ReduceOp.MAX)
            sec = float(t.item())
            pg.barrier()
            checked = None
            if rank == 0 and c_all is not None:
                # Every rank's rows as they landed in the shared result.
                from oracle import oracle
                sample = np.concatenate([
                    hx.shard_rows(m_total, world, r)[0] + np.array([0, m_rows // 2,
                                                                    m_rows - 1])
                    for r in range(world)])
                want = oracle.relu(oracle.matmul(a_rows_global(sample), w_host))
                checked = oracle.normwise_error(np.asarray(c_all[sample]), want)
                if not checked <= 1e-12:
                    raise SystemExit(f"e2e result wrong: normwise error {checked}")
            for ptr in registered:
                lib.hexir_host_unregister(ptr)
            pg.barrier()
        finally:
            # The shared result file goes even if the leg failed.
            if rank == 0 and obj[0] and os.path.exists(obj[0]):
                os.unlink(obj[0])
        h2d = a_host.nbytes * world + w_host.nbytes
        d2h = m_total * N_DIM * 8
        path_desc = ("hexir_sharded_linear_host_f64: each rank's host rows "
                     "of a up and of c down over its own host link, w in "
                     "per-rank slices all-gathered over NVLink, result rows "
                     "in one shared host mapping" + (
                         "" if shared else " (per-rank host rows: /dev/shm "
                                           "too small for a shared one)"))
    value = 2.0 * m_total * N_DIM * K_DIM / sec / 1e9
    return {"value": round(value, 3), "unit": "GFLOP/s",
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "ms_per_step": round(sec * 1e3, 3),
            "path": ("hexir_execute_capture of a .hxb (linear=cuda, relu=cuda)"
                     if world == 1 else path_desc),
            "timing": "host wall clock around synchronous calls, max over ranks"}


def timed_ms(fn, steps: int, warmup: int = 3) -> float:
    """Average device time of fn() (launches on torch's current stream)."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        fn()
    stop.record()
    torch.cuda.synchronize()
    return start.elapsed_time(stop) / steps


MEASURED_PEAKS = os.path.join(ROOT, "MEASURED_PEAKS.json")
HBM_FALLBACK_GBS = 6650.0


def hbm_peak_gbs():
    """Measured copy bandwidth of this pool's B200s, else the fallback."""
    if os.path.exists(MEASURED_PEAKS):
        with open(MEASURED_PEAKS) as f:
            v = json.load(f).get("hbm_gbs")
        if v:
            return float(v), "MEASURED_PEAKS.json hbm_gbs"
    return HBM_FALLBACK_GBS, "fallback 6.65 TB/s"


def relu_stream(ordinal: int, log2n: int = 28) -> dict:
    """hexir.relu over 2^28 f64 ~ N(0,1) (seed 4): HBM GB/s, 16 B/element."""
    import torch
    import hexir_b200 as hx
    n = 1 << log2n
    x = torch.from_numpy(hx.Rng(4).normal(n)).cuda()
    y = torch.empty_like(x)
    stream = torch.cuda.current_stream().cuda_stream
    ms = timed_ms(lambda: hx.cuda_relu(ordinal, x.data_ptr(), y.data_ptr(), n,
                                       stream), steps=20)
    hx.cuda_synchronize(ordinal, stream)
    ok = bool(torch.equal(y, torch.where(x > 0, x, torch.zeros_like(x))))
    gbs = 16.0 * n / (ms * 1e-3) / 1e9
    peak, src = hbm_peak_gbs()
    return {"value": round(gbs, 1), "unit": "GB/s", "elements": n,
            "bytes_per_launch": 16 * n, "ms_per_launch": round(ms, 4),
            "frac": round(gbs / peak, 4), "peak_gbs": peak, "peak_source": src,
            "frac_of_8tbs_nominal": round(gbs / 8000.0, 4),
            "kernel": "hexir_relu_f64", "checked": ok}


def activation_stream(ordinal: int, op: str, rows: int = 16384,
                      cols: int = 16384) -> dict:
    """One activation over a rows x cols f64 tensor ~ N(0,1) (seed 4; 2^28
    elements, in + out 4 GiB, past L2 every launch): HBM GB/s at 16 B per
    element, sampled rows checked against the oracle."""
    import numpy as np
    import torch
    import hexir_b200 as hx
    from oracle import oracle
    n = rows * cols
    x = torch.from_numpy(hx.Rng(4).normal(n)).cuda()
    y = torch.empty_like(x)
    stream = torch.cuda.current_stream().cuda_stream
    ms = timed_ms(lambda: hx.cuda_activation(ordinal, op, x.data_ptr(),
                                             y.data_ptr(), rows, cols, stream),
                  steps=20)
    hx.cuda_synchronize(ordinal, stream)
    pick = [0, rows // 3, rows - 1]
    xs = x.view(rows, cols)[pick].cpu().numpy()
    ys = y.view(rows, cols)[pick].cpu().numpy()
    ulps = {"leaky_relu": 0, "gelu": 32, "softmax": cols + 16}.get(op, 16)
    want = oracle.activation(op, xs)
    ok = bool(np.array_equal(ys, want) if ulps == 0 else
              oracle.ulp_error_ok(ys, want, ulps).all())
    gbs = 16.0 * n / (ms * 1e-3) / 1e9
    peak, src = hbm_peak_gbs()
    return {"op": op, "value": round(gbs, 1), "unit": "GB/s", "rows": rows,
            "cols": cols, "bytes_per_launch": 16 * n,
            "ms_per_launch": round(ms, 4), "frac": round(gbs / peak, 4),
            "peak_gbs": peak, "peak_source": src,
            "checked_rows": len(pick), "within_tolerance_ulps": ulps,
            "checked": ok}


def run_suite(args):
    """One JSON line per configuration of the benchmark plan (1 GPU)."""
    import numpy as np
    import torch
    import hexir_b200 as hx
    from hexir_b200 import _ffi
    from oracle import oracle
    ordinal = 0
    torch.cuda.set_device(ordinal)
    stream = torch.cuda.current_stream().cuda_stream
    peak = dmma_peak_tflops(ordinal)
    hbm, hbm_src = hbm_peak_gbs()
    out = []

    # C1 parity graph: 256x256 linear -> relu (seed 0, a then w) through the
    # VM on the GPU and on the host cores (the reference's CPU arithmetic);
    # latency of one hexir_execute_capture, median of 20 after warm-up.
    r = hx.Rng(0)
    a_h, w_h = r.uniform((256, 256)), r.uniform((256, 256))
    prog = hx.Program()
    prog.relu(prog.linear(prog.constant(a_h), prog.constant(w_h)))
    want = oracle.relu(oracle.matmul(a_h, w_h))
    line = {"suite": "parity_graph_256"}
    for name, placement, spec in (("cuda", "hexir.linear=cuda,hexir.relu=cuda", "cuda"),
                                  ("cpu", "", "cpu")):
        module = hx.Module(prog.emit(placement))
        dev = hx.Device(spec)
        got = hx.execute(module, dev, out_shape=(256, 256))
        wall, kms = [], []
        for _ in range(20):
            t0 = time.perf_counter()
            hx.execute(module, dev, out_shape=(256, 256))
            wall.append((time.perf_counter() - t0) * 1e3)
            kms.append(hx.last_kernel_ms())
        line[name + "_execute_ms"] = round(statistics.median(wall), 4)
        if name == "cuda":
            line["cuda_kernel_ms"] = round(statistics.median(kms), 4)
            line["cuda_normwise_err"] = oracle.normwise_error(got, want)
        else:
            line["cpu_bit_exact"] = bool(np.array_equal(got.view(np.uint64),
                                                        want.view(np.uint64)))
        module.close()
        dev.close()
    out.append(line)

    # GEMM sweep, square, relu fused (uniform[-1,1], seed 1, a then w).
    for size in (1024, 2048, 4096, 8192):
        r = hx.Rng(1)
        a_h, w_h = r.uniform((size, size)), r.uniform((size, size))
        a, w = torch.from_numpy(a_h).cuda(), torch.from_numpy(w_h).cuda()
        c = torch.empty_like(a)
        steps = max(3, int(2e12 / (2.0 * size ** 3)))
        steps = min(steps, 200)
        ms = timed_ms(lambda: hx.cuda_matmul(ordinal, a.data_ptr(), w.data_ptr(),
                                             c.data_ptr(), size, size, size,
                                             _ffi.MATMUL_RELU, stream), steps)
        rows = np.linspace(0, size - 1, 4).astype(int)
        err = oracle.normwise_error(c.cpu().numpy()[rows],
                                    oracle.relu(oracle.matmul(a_h[rows], w_h)))
        tf = 2.0 * size ** 3 / (ms * 1e-3) / 1e12
        out.append({"suite": "gemm_sweep", "m": size, "n": size, "k": size,
                    "ms": round(ms, 4), "tflops": round(tf, 3),
                    "frac_dmma_peak": round(tf / peak, 4),
                    "cublas_tflops": round(cublas_dgemm_tflops(a, w), 3),
                    "max_normwise_err_sampled": err})
        del a, w, c

    # relu stream.
    out.append({"suite": "relu_2^28", **relu_stream(ordinal)})

    # The activations, each over 16384 x 16384 (softmax along the rows).
    for op in sorted(_ffi.ACTIVATIONS):
        out.append({"suite": "activation_2^28", **activation_stream(ordinal, op)})
        torch.cuda.empty_cache()

    # Skinny linear: weight-read bandwidth.
    r = hx.Rng(5)
    w_h = None
    for m in (1, 16, 128):
        r = hx.Rng(5)
        a_h = r.uniform((m, 8192))
        w_h = r.uniform((8192, 8192))
        a, w = torch.from_numpy(a_h).cuda(), torch.from_numpy(w_h).cuda()
        c = torch.empty((m, 8192), dtype=torch.float64, device="cuda")
        ms = timed_ms(lambda: hx.cuda_matmul(ordinal, a.data_ptr(), w.data_ptr(),
                                             c.data_ptr(), m, 8192, 8192, 0,
                                             stream), 50)
        err = oracle.normwise_error(c.cpu().numpy()[:4],
                                    oracle.matmul(a_h[:4], w_h))
        variant, split = hx.matmul_plan(m, 8192, 8192)
        wbytes = 8.0 * 8192 * 8192
        out.append({"suite": "skinny", "m": m, "n": 8192, "k": 8192,
                    "ms": round(ms, 4),
                    "weight_gbs": round(wbytes / (ms * 1e-3) / 1e9, 1),
                    "weight_frac_hbm": round(wbytes / (ms * 1e-3) / 1e9 / hbm, 4),
                    "total_gbs": round(8.0 * (m * 8192 * 2 + 8192 * 8192) /
                                       (ms * 1e-3) / 1e9, 1),
                    "tflops": round(2.0 * m * 8192 * 8192 / (ms * 1e-3) / 1e12, 3),
                    "plan": {"variant": variant, "split_k": split},
                    "cublas_tflops": round(cublas_dgemm_tflops(a, w, 20), 3),
                    "max_normwise_err": err})
        del a, w, c

    # 3-layer MLP through the VM: all-cuda and linear=cuda / relu=cpu.
    r = hx.Rng(2)
    x = r.normal((8192, 1024))
    w1 = r.normal((1024, 4096), std=1 / np.sqrt(1024))
    w2 = r.normal((4096, 4096), std=1 / np.sqrt(4096))
    w3 = r.normal((4096, 1024), std=1 / np.sqrt(4096))
    prog = hx.Program()
    h = prog.relu(prog.linear(prog.constant(x), prog.constant(w1)))
    h = prog.relu(prog.linear(h, prog.constant(w2)))
    prog.linear(h, prog.constant(w3))
    flops = 2.0 * 8192 * (1024 * 4096 + 4096 * 4096 + 4096 * 1024)
    dev = hx.Device("cuda")
    results = {}
    for name, placement in (("all_cuda", "hexir.linear=cuda,hexir.relu=cuda"),
                            ("mixed", "hexir.linear=cuda,hexir.relu=cpu")):
        module = hx.Module(prog.emit(placement))
        res = hx.execute(module, dev, out_shape=(8192, 1024))
        kms, wall = [], []
        for _ in range(3):
            t0 = time.perf_counter()
            hx.execute(module, dev, out_shape=(8192, 1024))
            wall.append((time.perf_counter() - t0) * 1e3)
            kms.append(hx.last_kernel_ms())
        results[name] = res
        line = {"suite": "mlp_chain", "placement": placement,
                # dispatch spans: kernels plus the uploads they wait on
                "dispatch_ms": round(statistics.median(kms), 3),
                "e2e_ms": round(statistics.median(wall), 3),
                "e2e_tflops": round(flops / (statistics.median(wall) * 1e-3)
                                    / 1e12, 3)}
        if name == "all_cuda":
            # With the constants kept on the GPU no dispatch waits on an
            # upload: the spans are the three GEMMs alone.
            module.keep_constants(True)
            hx.execute(module, dev, out_shape=(8192, 1024))
            kept = []
            for _ in range(3):
                hx.execute(module, dev, out_shape=(8192, 1024))
                kept.append(hx.last_kernel_ms())
            line["kernel_ms"] = round(statistics.median(kept), 3)
            line["kernel_tflops"] = round(flops / (statistics.median(kept) * 1e-3)
                                          / 1e12, 3)
        out.append(line)
        module.close()
    # linear -> add -> relu at 8192^3: one fused kernel against three.
    r = hx.Rng(3)
    a_h, w_h, b_h = (r.uniform((8192, 8192)) for _ in range(3))
    a, w, b = (torch.from_numpy(t).cuda() for t in (a_h, w_h, b_h))
    del a_h, w_h
    c1, c2 = torch.empty_like(a), torch.empty_like(a)
    n_el = 8192 * 8192
    fused_ms = timed_ms(lambda: hx.cuda_matmul_add(
        ordinal, a.data_ptr(), w.data_ptr(), b.data_ptr(), c1.data_ptr(), 8192,
        8192, 8192, _ffi.MATMUL_RELU, stream), 5)

    def three():
        hx.cuda_matmul(ordinal, a.data_ptr(), w.data_ptr(), c2.data_ptr(), 8192,
                       8192, 8192, 0, stream)
        hx.cuda_add(ordinal, c2.data_ptr(), b.data_ptr(), c2.data_ptr(), n_el,
                    stream)
        hx.cuda_relu(ordinal, c2.data_ptr(), c2.data_ptr(), n_el, stream)
    three_ms = timed_ms(three, 5)
    out.append({"suite": "linear_add_relu_8192", "fused_ms": round(fused_ms, 4),
                "three_kernels_ms": round(three_ms, 4),
                "fused_tflops": round(2.0 * 8192 ** 3 / (fused_ms * 1e-3) / 1e12, 3),
                "bit_identical": bool(torch.equal(c1.view(torch.int64),
                                                  c2.view(torch.int64)))})
    del a, w, b, c1, c2

    # The 8192^3 module executed repeatedly with its constants kept on the
    # GPU (hexir_module_keep_constants): a serving loop's per-call time.
    r = hx.Rng(1)
    a_h, w_h = r.uniform((8192, 8192)), r.uniform((8192, 8192))
    kept = hx.Program()
    kept.relu(kept.linear(kept.constant(a_h), kept.constant(w_h)))
    module = hx.Module(kept.emit("hexir.linear=cuda,hexir.relu=cuda"))
    del kept, a_h, w_h
    module.keep_constants(True)
    dev = hx.Device("cuda")
    res = torch.empty((8192, 8192), dtype=torch.float64).pin_memory().numpy()

    def once():
        _ffi.check(hx.lib().hexir_execute_capture(
            module.handle, dev.handle, b"main", res.ctypes.data, res.nbytes),
            "hexir_execute_capture")
    once()
    wall = []
    for _ in range(3):
        t0 = time.perf_counter()
        once()
        wall.append((time.perf_counter() - t0) * 1e3)
    out.append({"suite": "kept_constants_8192", "execute_ms": round(statistics.median(wall), 3),
                "tflops": round(2.0 * 8192 ** 3 / (statistics.median(wall) * 1e-3) / 1e12, 3),
                "kept_bytes": module.kept_bytes,
                "note": "hexir_execute_capture with a and w kept on the GPU; "
                        "the 512 MiB result still copied to pinned host memory"})
    module.close()
    dev.close()
    del res

    rows = np.linspace(0, 8191, 8).astype(int)
    want = oracle.matmul(oracle.relu(oracle.matmul(
        oracle.relu(oracle.matmul(x[rows], w1)), w2)), w3)
    out.append({"suite": "mlp_chain_check",
                "all_cuda_equals_mixed_bitwise": bool(np.array_equal(
                    results["all_cuda"].view(np.uint64),
                    results["mixed"].view(np.uint64))),
                "max_normwise_err_sampled": oracle.normwise_error(
                    results["all_cuda"][rows], want)})
    for o in out:
        o["dmma_peak_tflops"] = round(peak, 3)
        print(json.dumps(o), flush=True)
    return 0


def run_profile(args):
    """One kernel, 5 launches, nothing else: the command line ncu captures."""
    import torch
    import hexir_b200 as hx
    from hexir_b200 import _ffi
    torch.cuda.set_device(0)
    stream = torch.cuda.current_stream().cuda_stream
    if args.profile == "relu":
        n = 1 << args.log2n
        x = torch.from_numpy(hx.Rng(4).normal(n)).cuda()
        y = torch.empty_like(x)
        run = lambda: hx.cuda_relu(0, x.data_ptr(), y.data_ptr(), n, stream)
        what = f"relu 2^{args.log2n} f64"
    elif args.profile == "square":
        size = args.size
        r = hx.Rng(1)
        a = torch.from_numpy(r.uniform((size, size))).cuda()
        w = torch.from_numpy(r.uniform((size, size))).cuda()
        c = torch.empty_like(a)
        run = lambda: hx.cuda_matmul(0, a.data_ptr(), w.data_ptr(), c.data_ptr(),
                                     size, size, size, _ffi.MATMUL_RELU, stream)
        what = (f"linear+relu {size}^3 plan "
                f"{hx.matmul_plan(size, size, size, _ffi.MATMUL_RELU)}")
    elif args.profile == "activation":
        n = 1 << args.log2n
        rows = n // args.cols
        x = torch.from_numpy(hx.Rng(4).normal(n)).cuda()
        y = torch.empty_like(x)
        run = lambda: hx.cuda_activation(0, args.op, x.data_ptr(), y.data_ptr(),
                                         rows, args.cols, stream)
        what = f"{args.op} {rows}x{args.cols} f64"
    else:
        m = args.m
        r = hx.Rng(5 if args.profile == "skinny" else 1)
        a = torch.from_numpy(r.uniform((m, K_DIM))).cuda()
        w = torch.from_numpy(r.uniform((K_DIM, N_DIM))).cuda()
        c = torch.empty((m, N_DIM), dtype=torch.float64, device="cuda")
        flags = _ffi.MATMUL_RELU if args.profile == "linear" else 0
        run = lambda: hx.cuda_matmul(0, a.data_ptr(), w.data_ptr(), c.data_ptr(),
                                     m, N_DIM, K_DIM, flags, stream)
        what = f"linear {m}x{N_DIM}x{K_DIM} plan {hx.matmul_plan(m, N_DIM, K_DIM, flags)}"
    ms = timed_ms(run, steps=3, warmup=2)
    hx.cuda_synchronize(0, stream)
    print(json.dumps({"profile": what, "ms": round(ms, 4)}))
    return 0


def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference(args)
    if args.profile:
        return run_profile(args)
    if args.suite:
        return run_suite(args)
    return run_hexir(args)


if __name__ == "__main__":
    sys.exit(main())
