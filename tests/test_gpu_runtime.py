"""GPU runs through the reference-facing surface: hexir-run, the VM
(hexir_execute / hexir_execute_devices), the HAL, compared with the CPU path
(the reference's own differential test style, runtime/test/hxb-cpu-vs-gpu.mlir)
and with the oracle.

Bars: relu bit-exact against the CPU relu of the same m; linear normwise
max|c - c_ref| / max|c_ref| <= 1e-12.
"""

import json
import os
import shutil
import struct
import subprocess

import numpy as np
import pytest

import hexir_b200 as hx
from hexir_b200 import _ffi
from oracle import oracle
from tests.conftest import bin_path

pytestmark = pytest.mark.gpu

TOL = 1e-12
GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden",
                                     "golden.json")))
RUN = bin_path("hexir-run")


def bits(a):
    return np.ascontiguousarray(a).view(np.uint64)


def known_program(case):
    p = hx.Program()
    a = p.constant(np.array(case["a"]))
    b = p.constant(np.array(case["b"]))
    v = p.linear(a, b)
    for op in case["ops"][1:]:
        v = p.add(v, b) if op == "add_b" else p.relu(v)
    p.print(v)
    return p


@pytest.mark.parametrize("case", GOLDEN["known_answers"], ids=lambda c: c["name"])
@pytest.mark.parametrize("fuse", [True, False])
def test_hexir_run_cuda_matches_cpu_output(tmp_path, case, fuse):
    """CPU module vs all-cuda module, printed output diffed, as
    hxb-cpu-vs-gpu.mlir does; both equal the reference's printed answer."""
    p = known_program(case)
    cpu, gpu = tmp_path / "cpu.hxb", tmp_path / "gpu.hxb"
    p.emit_file(str(cpu))
    p.emit_file(str(gpu), "hexir.linear=cuda,hexir.add=cuda,hexir.relu=cuda",
                0 if fuse else _ffi.EMIT_NO_FUSE)
    out_cpu = subprocess.run([RUN, "--quiet", str(cpu)], capture_output=True,
                             text=True, check=True).stdout
    out_gpu = subprocess.run([RUN, "--quiet", "--device=cuda", str(gpu)],
                             capture_output=True, text=True, check=True).stdout
    assert out_gpu == out_cpu == case["stdout_quiet"]


def test_selftest_cuda():
    res = subprocess.run([RUN, "--selftest", "--device=cuda"],
                         capture_output=True, text=True, check=True)
    assert "device        : cuda" in res.stdout
    assert "hal roundtrip : ok" in res.stdout


def test_module_report_names_the_gpu(tmp_path):
    path = tmp_path / "m.hxb"
    known_program(GOLDEN["known_answers"][0]).emit_file(str(path),
                                                        "hexir.linear=cuda")
    out = subprocess.run([RUN, "--device=cuda", "--time", str(path)],
                         capture_output=True, text=True, check=True)
    assert "device        : cuda (NVIDIA" in out.stdout
    assert "launch" in out.stdout  # the LAUNCH section is listed
    assert "kernel time" in out.stderr


def parity_graph():
    r = hx.Rng(0)  # a then w, uniform[-1, 1], seed 0
    return r.uniform((256, 256)), r.uniform((256, 256))


def test_parity_graph_256():
    """The CPU-runnable reference graph recompiled for cuda: relu bit-exact
    against the CPU relu of the same m, linear within 1e-12."""
    a, w = parity_graph()
    dev = hx.Device("cuda")

    p = hx.Program()
    p.linear(p.constant(a), p.constant(w))
    m_gpu = hx.execute(hx.Module(p.emit("hexir.linear=cuda")), dev,
                       out_shape=(256, 256))
    assert oracle.normwise_error(m_gpu, oracle.matmul(a, w)) <= TOL

    p2 = hx.Program()
    p2.relu(p2.linear(p2.constant(a), p2.constant(w)))
    for flags in (_ffi.EMIT_NO_FUSE, 0):  # separate relu kernel, then fused
        r_gpu = hx.execute(hx.Module(p2.emit(
            "hexir.linear=cuda,hexir.relu=cuda", flags)), dev, out_shape=(256, 256))
        assert np.array_equal(bits(r_gpu), bits(oracle.relu(m_gpu)))
    # relu on the CPU of the GPU's m: placement-propagated transfer.
    r_mixed = hx.execute(hx.Module(p2.emit("hexir.linear=cuda,hexir.relu=cpu")),
                         dev, out_shape=(256, 256))
    assert np.array_equal(bits(r_mixed), bits(oracle.relu(m_gpu)))
    # And the whole graph on the CPU backend is the oracle, bit for bit.
    r_cpu = hx.execute(hx.Module(p2.emit()), hx.Device("cpu"), out_shape=(256, 256))
    assert np.array_equal(bits(r_cpu), bits(oracle.relu(oracle.matmul(a, w))))


def test_mlp_chain_all_cuda_and_mixed_placement():
    """x[8192x1024] -> W1[1024x4096] -> relu -> W2[4096x4096] -> relu ->
    W3[4096x1024], x ~ N(0,1), Wi ~ N(0, 1/fan_in), seed 2.  All-cuda and
    linear=cuda/relu=cpu must agree bit for bit (the relu is the same
    function on both sides); sampled rows against the oracle."""
    r = hx.Rng(2)
    x = r.normal((8192, 1024))
    w1 = r.normal((1024, 4096), std=1 / np.sqrt(1024))
    w2 = r.normal((4096, 4096), std=1 / np.sqrt(4096))
    w3 = r.normal((4096, 1024), std=1 / np.sqrt(4096))
    p = hx.Program()
    h = p.relu(p.linear(p.constant(x), p.constant(w1)))
    h = p.relu(p.linear(h, p.constant(w2)))
    p.linear(h, p.constant(w3))
    dev = hx.Device("cuda")
    all_cuda = hx.execute(hx.Module(p.emit("hexir.linear=cuda,hexir.relu=cuda")),
                          dev, out_shape=(8192, 1024))
    mixed = hx.execute(hx.Module(p.emit("hexir.linear=cuda,hexir.relu=cpu")),
                       dev, out_shape=(8192, 1024))
    assert np.array_equal(bits(all_cuda), bits(mixed))
    rows = np.linspace(0, 8191, 12).astype(int)
    want = oracle.matmul(oracle.relu(oracle.matmul(
        oracle.relu(oracle.matmul(x[rows], w1)), w2)), w3)
    assert oracle.normwise_error(all_cuda[rows], want) <= TOL


@pytest.mark.parametrize("m,n,k,capture_rows", [
    (4096, 2048, 2048, 4096),   # 64 MiB a uploads in chunks; 64 MiB result streams out
    (4096, 2048, 2048, 1000),   # partial capture: only the first 1000 rows
    (2048, 1024, 4096, 2048),   # a pipelined, result too small to stream
])
def test_pipelined_dispatch(m, n, k, capture_rows):
    """A large host-sourced linear runs as an upload / compute / download
    pipeline of row chunks; the captured rows equal the oracle's."""
    r = hx.Rng(7)
    a = r.uniform((m, k))
    w = r.uniform((k, n))
    p = hx.Program()
    p.relu(p.linear(p.constant(a), p.constant(w)))
    dev = hx.Device("cuda")
    module = hx.Module(p.emit("hexir.linear=cuda,hexir.relu=cuda"))
    first = hx.execute(module, dev, out_shape=(capture_rows, n))
    again = hx.execute(module, dev, out_shape=(capture_rows, n))  # pinned + pooled
    assert np.array_equal(bits(first), bits(again))
    rows = np.linspace(0, capture_rows - 1, 16).astype(int)
    want = oracle.relu(oracle.matmul(a[rows], w))
    assert oracle.normwise_error(first[rows], want) <= TOL


@pytest.mark.parametrize("m,n,k,capture_rows", [
    (4096, 4096, 2048, 4096),
    (4096, 4096, 4100, 3000),   # ragged last k tile, partial capture
])
def test_weight_streamed_pipeline_is_bit_identical(gpu, m, n, k, capture_rows):
    """With w still on the host and no k split in the one-shot plan, the VM
    runs k in pieces while w's rows (and a's columns) upload, then the second
    half of k per row chunk while rows download: every element sees the
    one-shot launch's operations in the same order, so the captured rows
    equal hexir_cuda_matmul_f64's bit for bit."""
    assert hx.matmul_plan(m, n, k, _ffi.MATMUL_RELU)[1] == 1
    r = hx.Rng(8)
    a = r.uniform((m, k))
    w = r.uniform((k, n))
    p = hx.Program()
    p.relu(p.linear(p.constant(a), p.constant(w)))
    module = hx.Module(p.emit("hexir.linear=cuda,hexir.relu=cuda"))
    dev = hx.Device("cuda")
    got = hx.execute(module, dev, out_shape=(capture_rows, n))
    ba, bw = gpu.upload(a), gpu.upload(w)
    bc = gpu.buffer(m * n * 8)
    hx.cuda_matmul(0, ba.ptr, bw.ptr, bc.ptr, m, n, k, _ffi.MATMUL_RELU,
                   gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    one_shot = bc.read((m, n))[:capture_rows]
    assert np.array_equal(bits(got), bits(one_shot))
    rows = np.linspace(0, capture_rows - 1, 8).astype(int)
    want = oracle.relu(oracle.matmul(a[rows], w))
    assert oracle.normwise_error(got[rows], want) <= TOL
    module.close()


def test_relu_stream_2_28_bit_exact():
    """relu on 2^28 f64 ~ N(0,1) seed 4 as tensor<16384x16384xf64>: bit-exact
    against the oracle's relu of the same bytes."""
    n = 1 << 28
    x = hx.Rng(4).normal(n)
    dev = hx.Device("cuda")
    bx, by = dev.upload(x), dev.buffer(n * 8)
    hx.cuda_relu(0, bx.ptr, by.ptr, n, dev.stream)
    hx.cuda_synchronize(0, dev.stream)
    del bx
    got = by.read(n)
    del by
    want = oracle.relu(x)
    del x
    assert np.array_equal(bits(got), bits(want))


def test_linear_8192_every_tile_against_oracle():
    """The headline shape, 8192^3 with relu (seed 1, a then w): one row of
    every 128-row tile, at a different offset inside each tile, against the
    oracle over all 8192 columns -- every output tile of the launch is
    sampled."""
    size = 8192
    r = hx.Rng(1)
    a, w = r.uniform((size, size)), r.uniform((size, size))
    dev = hx.Device("cuda")
    ba, bw, bc = dev.upload(a), dev.upload(w), dev.buffer(size * size * 8)
    hx.cuda_matmul(0, ba.ptr, bw.ptr, bc.ptr, size, size, size,
                   _ffi.MATMUL_RELU, dev.stream)
    hx.cuda_synchronize(0, dev.stream)
    del ba, bw
    got = bc.read((size, size))
    rows = np.array([t * 128 + (t * 37) % 128 for t in range(size // 128)])
    want = oracle.relu(oracle.matmul(a[rows], w))
    assert oracle.normwise_error(got[rows], want) <= TOL
    # and column-wise: the sampled rows' per-column maxima stay in bar too
    per_col = np.abs(got[rows] - want).max(axis=0) / np.abs(want).max()
    assert per_col.max() <= TOL


def test_launch_fault_reports_and_next_execute_is_exact():
    """HEXIR_FAULT's launch site on the GPU: the injected failure comes back
    as HEXIR_ERROR_DEVICE before the driver is called, and the next
    execute, with no fault, gives the same bits as one before it."""
    r = hx.Rng(9)
    a, w = r.uniform((256, 192)), r.uniform((192, 320))
    p = hx.Program()
    p.relu(p.linear(p.constant(a), p.constant(w)))
    module = hx.Module(p.emit("hexir.linear=cuda,hexir.relu=cuda"))
    dev = hx.Device("cuda")
    before = hx.execute(module, dev, out_shape=(256, 320))
    hx.fault_configure("launch:1")
    try:
        with pytest.raises(hx.HexirError) as err:
            hx.execute(module, dev, out_shape=(256, 320))
        assert err.value.status == _ffi.ERROR_DEVICE
        assert hx.fault_calls("launch") >= 1
    finally:
        hx.fault_configure("")
    after = hx.execute(module, dev, out_shape=(256, 320))
    assert np.array_equal(bits(after), bits(before))
    assert oracle.normwise_error(after, oracle.relu(oracle.matmul(a, w))) <= TOL
    module.close()
    dev.close()


@pytest.mark.parametrize("m", [1, 16, 128])
def test_skinny_linear(m):
    """a[m x 8192] . w[8192 x 8192], uniform weights seed 5."""
    r = hx.Rng(5)
    a = r.uniform((m, 8192))
    w = r.uniform((8192, 8192))
    dev = hx.Device("cuda")
    ba, bw, bc = dev.upload(a), dev.upload(w), dev.buffer(m * 8192 * 8)
    hx.cuda_matmul(0, ba.ptr, bw.ptr, bc.ptr, m, 8192, 8192, 0, dev.stream)
    hx.cuda_synchronize(0, dev.stream)
    rows = np.arange(m) if m <= 16 else np.linspace(0, m - 1, 8).astype(int)
    got = bc.read((m, 8192))[rows]
    assert oracle.normwise_error(got, oracle.matmul(a[rows], w)) <= TOL


def test_bounded_wait_reports_an_error_and_context_survives():
    dev = hx.Device("cuda")
    st = hx.lib().hexir_cuda_wait_probe(0, 2_000_000, dev.stream)  # 2 ms
    assert st == _ffi.OK
    st = hx.lib().hexir_cuda_synchronize(0, dev.stream)
    assert st == _ffi.ERROR_DEVICE
    assert "ran out of time" in hx.lib().hexir_cuda_last_error().decode()
    # The word is cleared and the context still runs kernels.
    a = np.eye(8)
    ba, bc = dev.upload(a), dev.buffer(64 * 8)
    hx.cuda_matmul(0, ba.ptr, ba.ptr, bc.ptr, 8, 8, 8, 0, dev.stream)
    hx.cuda_synchronize(0, dev.stream)
    assert np.array_equal(bc.read((8, 8)), a)


def test_reference_style_image_launches_by_entry_name(tmp_path):
    """The HAL plugin point for images that follow the reference convention
    (one bare device pointer per buffer, kernel named after the entry):
    hexir_device_launch loads the image and launches the named kernel."""
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("nvcc not available to build a test image")
    src = tmp_path / "k.cu"
    src.write_text('extern "C" __global__ void relu_1(const double *x, double *y)'
                   ' { unsigned i = blockIdx.x * blockDim.x + threadIdx.x;'
                   ' y[i] = x[i] > 0.0 ? x[i] : 0.0; }\n')
    cubin = tmp_path / "k.cubin"
    subprocess.run([nvcc, "-cubin", "-gencode", "arch=compute_100a,code=sm_100a",
                    "-o", str(cubin), str(src)], check=True)
    image = cubin.read_bytes()
    dev = hx.Device("cuda")
    x = np.linspace(-1, 1, 256)
    bx, by = dev.upload(x), dev.buffer(256 * 8)
    import ctypes as C
    args = (C.c_void_p * 2)(bx._h, by._h)
    buf = C.create_string_buffer(image, len(image))
    st = hx.lib().hexir_device_launch(dev.handle, buf, len(image), b"relu_1",
                                      2, 1, 128, 1, args, 2)
    assert st == _ffi.OK
    dev.wait()
    assert np.array_equal(bits(by.read(256)), bits(oracle.relu(x)))
    st = hx.lib().hexir_device_launch(dev.handle, buf, len(image), b"nosuch",
                                      1, 1, 1, 1, args, 2)
    assert st == _ffi.ERROR_NOT_FOUND


def two_gpus():
    return hx.device_count() >= 2


@pytest.mark.skipif(not two_gpus(), reason="needs 2 GPUs")
def test_row_sharded_linear_in_process(tmp_path):
    """linear + relu placed on cuda:0-1: rows split over two GPUs, weight
    broadcast and rows gathered with NCCL; equals the one-GPU result bit for
    bit (same kernels, same per-row arithmetic)."""
    r = hx.Rng(3)
    a = r.uniform((1000, 512))
    w = r.uniform((512, 384))
    p = hx.Program()
    p.relu(p.linear(p.constant(a), p.constant(w)))
    devs = [hx.Device("cuda:0"), hx.Device("cuda:1")]
    sharded = hx.execute(hx.Module(p.emit("hexir.linear=cuda:0-1,"
                                          "hexir.relu=cuda:0-1")),
                         devs, out_shape=(1000, 384))
    single = hx.execute(hx.Module(p.emit("hexir.linear=cuda,hexir.relu=cuda")),
                        devs[0], out_shape=(1000, 384))
    assert oracle.normwise_error(sharded, oracle.relu(oracle.matmul(a, w))) <= TOL
    # Shards of 500 rows use the same kernel plan as the single GPU's tiles.
    assert np.array_equal(bits(sharded), bits(single))


@pytest.mark.skipif(not two_gpus(), reason="needs 2 GPUs")
@pytest.mark.parametrize("m", [1, 3, 257, 1001])
def test_row_sharded_odd_rows_and_elementwise(m):
    """Row splits that do not divide evenly, and add / relu placed on a GPU
    range: each shard's rows, gathered on the first GPU, equal the oracle."""
    r = hx.Rng(11 + m)
    a = r.uniform((m, 96))
    w = r.uniform((96, 130))
    b = r.uniform((m, 130))
    p = hx.Program()
    lin = p.linear(p.constant(a), p.constant(w))
    p.relu(p.add(lin, p.constant(b)))
    devs = [hx.Device("cuda:0"), hx.Device("cuda:1")]
    out = hx.execute(hx.Module(p.emit("hexir.linear=cuda:0-1,hexir.add=cuda:0-1,"
                                      "hexir.relu=cuda:0-1")),
                     devs, out_shape=(m, 130))
    m_ref = oracle.matmul(a, w)
    want = oracle.relu(oracle.add(m_ref, b))
    assert oracle.normwise_error(out, want) <= TOL


@pytest.mark.skipif(not two_gpus(), reason="needs 2 GPUs")
def test_kernels_on_the_second_gpu():
    """A linear placed on cuda:1 runs there (kernel-level C ABI and VM)."""
    r = hx.Rng(12)
    a, w = r.uniform((200, 64)), r.uniform((64, 72))
    dev1 = hx.Device("cuda:1")
    ba, bw, bc = dev1.upload(a), dev1.upload(w), dev1.buffer(200 * 72 * 8)
    hx.cuda_matmul(1, ba.ptr, bw.ptr, bc.ptr, 200, 72, 64, 0, dev1.stream)
    hx.cuda_synchronize(1, dev1.stream)
    assert oracle.normwise_error(bc.read((200, 72)), oracle.matmul(a, w)) <= TOL
    p = hx.Program()
    p.linear(p.constant(a), p.constant(w))
    devs = [hx.Device("cuda:0"), dev1]
    out = hx.execute(hx.Module(p.emit("hexir.linear=cuda:1")), devs,
                     out_shape=(200, 72))
    assert oracle.normwise_error(out, oracle.matmul(a, w)) <= TOL


def test_hexir_bench_tool_verifies_and_times(tmp_path):
    """The extended reference benchmark tool on a cuda module: sampled
    verification, end-to-end and kernel time, cuBLAS line, JSON output."""
    r = hx.Rng(13)
    a, w = r.uniform((512, 512)), r.uniform((512, 512))
    p = hx.Program()
    p.relu(p.linear(p.constant(a), p.constant(w)))
    path = tmp_path / "m.hxb"
    p.emit_file(str(path), "hexir.linear=cuda,hexir.relu=cuda")
    res = subprocess.run([bin_path("hexir-bench"), str(path), "--iters=3",
                          "--json"], capture_output=True, text=True, check=True)
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["verify_ok"] is True and line["verify_max_rel_err"] < 1e-12
    assert line["kernel"] == "matmul_relu" and line["m"] == 512
    assert line["e2e_ms"] > 0 and line["kernel_ms"] > 0
    assert line["cublas_ms"] > 0
    # A fused linear -> add -> relu module is verified too (addend included).
    d = r.uniform((512, 512))
    p2 = hx.Program()
    p2.relu(p2.add(p2.linear(p2.constant(a), p2.constant(w)), p2.constant(d)))
    path2 = tmp_path / "fused.hxb"
    p2.emit_file(str(path2), "hexir.linear=cuda,hexir.add=cuda,hexir.relu=cuda")
    res = subprocess.run([bin_path("hexir-bench"), str(path2), "--iters=2",
                          "--json", "--no-baseline"], capture_output=True,
                         text=True, check=True)
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["verify_ok"] is True and line["verify_max_rel_err"] < 1e-12
    assert line["kernel"] == "matmul_add_relu"



def test_kept_constants_are_reused_and_bit_identical():
    """hexir_module_keep_constants: the first execute uploads a and w into
    memory kept with the module; later executes (also through another device
    object for the same GPU) reuse it and give the same bits."""
    r = hx.Rng(41)
    a = r.uniform((1000, 512))
    w = r.uniform((512, 384))
    p = hx.Program()
    p.relu(p.linear(p.constant(a), p.constant(w)))
    mod = hx.Module(p.emit("hexir.linear=cuda,hexir.relu=cuda"))
    dev = hx.Device("cuda")
    base = hx.execute(mod, dev, out_shape=(1000, 384))
    assert mod.kept_bytes == 0
    mod.keep_constants(True)
    first = hx.execute(mod, dev, out_shape=(1000, 384))
    assert mod.kept_bytes == a.nbytes + w.nbytes
    second = hx.execute(mod, dev, out_shape=(1000, 384))
    other = hx.Device("cuda:0")
    third = hx.execute(mod, other, out_shape=(1000, 384))
    assert mod.kept_bytes == a.nbytes + w.nbytes
    for out in (first, second, third):
        assert np.array_equal(bits(out), bits(base))
    assert oracle.normwise_error(base, oracle.relu(oracle.matmul(a, w))) <= TOL
    mod.keep_constants(False)
    assert mod.kept_bytes == 0
    assert np.array_equal(bits(hx.execute(mod, dev, out_shape=(1000, 384))),
                          bits(base))
    other.close()
    mod.close()


def _dispatch_into_constant_slot(blob: bytes) -> bytes:
    """The module with its first DISPATCH's destination replaced by the slot
    of its first operand (a CONST): the serializer never emits this, a
    hand-made module can."""
    sections = hx.read_sections(blob)
    poff, _ = sections[2]
    out = bytearray(blob)
    pc = 0
    while True:
        kind, argc = struct.unpack_from("<II", blob, poff + pc)
        if kind == 3:  # DISPATCH: index, argc, args...
            ops = struct.unpack_from(f"<{argc}Q", blob, poff + pc + 8)
            struct.pack_into("<Q", out, poff + pc + 8 + 8 * (argc - 1), ops[2])
            return bytes(out)
        assert kind != 0
        pc += 8 + 8 * argc


def test_dispatch_into_a_kept_constant_never_changes_it():
    """A dispatch whose destination is a CONST slot writes a private buffer:
    the kept copy, and so the next execute, still see the module's bytes."""
    r = hx.Rng(42)
    a = r.uniform((256, 256))
    w = r.uniform((256, 256))
    p = hx.Program()
    p.linear(p.constant(a), p.constant(w))
    blob = _dispatch_into_constant_slot(p.emit("hexir.linear=cuda"))
    mod = hx.Module(blob)
    mod.keep_constants(True)
    dev = hx.Device("cuda")
    want = oracle.matmul(a, w)
    outs = [hx.execute(mod, dev, out_shape=(256, 256)) for _ in range(3)]
    for out in outs:
        assert oracle.normwise_error(out, want) <= TOL
        assert np.array_equal(bits(out), bits(outs[0]))
    assert mod.kept_bytes == a.nbytes + w.nbytes
    mod.close()


def test_fused_linear_add_relu_module_matches_unfused():
    """The reference's roundtrip graph shape (linear -> add -> relu) placed
    on cuda: one fused executable, bit-identical to the three unfused
    kernels and within the bar of the oracle."""
    r = hx.Rng(19)
    a, w, b = r.uniform((700, 512)), r.uniform((512, 384)), r.uniform((700, 384))
    p = hx.Program()
    p.relu(p.add(p.linear(p.constant(a), p.constant(w)), p.constant(b)))
    placement = "hexir.linear=cuda,hexir.add=cuda,hexir.relu=cuda"
    fused_blob = p.emit(placement)
    assert [e.kind for e in hx.read_executables(fused_blob)] == [6]
    dev = hx.Device("cuda")
    fused = hx.execute(hx.Module(fused_blob), dev, out_shape=(700, 384))
    plain = hx.execute(hx.Module(p.emit(placement, _ffi.EMIT_NO_FUSE)), dev,
                       out_shape=(700, 384))
    assert np.array_equal(bits(fused), bits(plain))
    want = oracle.relu(oracle.add(oracle.matmul(a, w), b))
    assert oracle.normwise_error(fused, want) <= TOL


@pytest.mark.skipif(not two_gpus(), reason="needs 2 GPUs")
def test_row_sharded_fused_linear_add_relu():
    """linear -> add -> relu on cuda:0-1: the fused kernel per shard with the
    addend's rows split like a's; equals the one-GPU fused module."""
    r = hx.Rng(23)
    a, w, b = r.uniform((1001, 256)), r.uniform((256, 132)), r.uniform((1001, 132))
    p = hx.Program()
    p.relu(p.add(p.linear(p.constant(a), p.constant(w)), p.constant(b)))
    devs = [hx.Device("cuda:0"), hx.Device("cuda:1")]
    sharded = hx.execute(hx.Module(p.emit("hexir.linear=cuda:0-1,hexir.add=cuda:0-1,"
                                          "hexir.relu=cuda:0-1")),
                         devs, out_shape=(1001, 132))
    want = oracle.relu(oracle.add(oracle.matmul(a, w), b))
    assert oracle.normwise_error(sharded, want) <= TOL


def test_kept_constants_with_fused_add_and_second_use():
    """Kept constants feeding a fused linear -> add -> relu and a second,
    unfused use of the same constant: three executes, the same bits."""
    r = hx.Rng(47)
    a, w, b = r.uniform((300, 256)), r.uniform((256, 200)), r.uniform((300, 200))
    p = hx.Program()
    bc = p.constant(b)
    s = p.relu(p.add(p.linear(p.constant(a), p.constant(w)), bc))
    p.print(p.add(s, bc))
    mod = hx.Module(p.emit("hexir.linear=cuda,hexir.add=cuda,hexir.relu=cuda"))
    assert [e.kind for e in hx.read_executables(p.emit(
        "hexir.linear=cuda,hexir.add=cuda,hexir.relu=cuda"))] == [6, 2]
    dev = hx.Device("cuda")
    plain = hx.execute(mod, dev, out_shape=(300, 200))
    mod.keep_constants(True)
    outs = [hx.execute(mod, dev, out_shape=(300, 200)) for _ in range(3)]
    for out in outs:
        assert np.array_equal(bits(out), bits(plain))
    assert mod.kept_bytes == a.nbytes + w.nbytes + b.nbytes
    want = oracle.add(oracle.relu(oracle.add(oracle.matmul(a, w), b)), b)
    assert oracle.normwise_error(plain, want) <= TOL
    mod.close()


@pytest.mark.skipif(not two_gpus(), reason="needs 2 GPUs")
def test_kept_constants_with_row_sharding():
    """A row-sharded linear on cuda:0-1 with its constants kept: the weight's
    kept copy on GPU 0 is broadcast every execute (the rows of a still go
    to each GPU from the module); repeated executes equal the first bit for
    bit."""
    r = hx.Rng(53)
    a, w = r.uniform((777, 320)), r.uniform((320, 256))
    p = hx.Program()
    p.relu(p.linear(p.constant(a), p.constant(w)))
    mod = hx.Module(p.emit("hexir.linear=cuda:0-1,hexir.relu=cuda:0-1"))
    devs = [hx.Device("cuda:0"), hx.Device("cuda:1")]
    first = hx.execute(mod, devs, out_shape=(777, 256))
    mod.keep_constants(True)
    for _ in range(3):
        again = hx.execute(mod, devs, out_shape=(777, 256))
        assert np.array_equal(bits(again), bits(first))
    assert mod.kept_bytes == w.nbytes
    assert oracle.normwise_error(first, oracle.relu(oracle.matmul(a, w))) <= TOL
    mod.close()


def test_hexir_run_repeat_with_kept_constants_on_cuda(tmp_path):
    """hexir-run --device=cuda --repeat=3 --keep-constants: the printed
    result once, equal to the cpu run's digits; medians on stderr."""
    case = GOLDEN["known_answers"][1]
    p = known_program(case)
    path = tmp_path / "m.hxb"
    p.emit_file(str(path), "hexir.linear=cuda,hexir.add=cuda,hexir.relu=cuda")
    res = subprocess.run([RUN, "--device=cuda", "--quiet", "--repeat=3",
                          "--time", "--keep-constants", str(path)],
                         capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    assert res.stdout == case["stdout_quiet"]
    assert "kernel time   :" in res.stderr and "median" in res.stderr


@pytest.mark.skipif(not two_gpus(), reason="needs 2 GPUs")
def test_nccl_fault_in_sharded_dispatch_reports_and_recovers():
    """HEXIR_FAULT's NCCL site: a row-sharded dispatch whose weight
    broadcast is made to fail returns HEXIR_ERROR_DEVICE with no rank left
    waiting, and the next execute is whole."""
    r = hx.Rng(10)
    a, w = r.uniform((600, 256)), r.uniform((256, 384))
    p = hx.Program()
    p.relu(p.linear(p.constant(a), p.constant(w)))
    module = hx.Module(p.emit("hexir.linear=cuda:0-1,hexir.relu=cuda:0-1"))
    devs = [hx.Device("cuda:0"), hx.Device("cuda:1")]
    before = hx.execute(module, devs, out_shape=(600, 384))
    hx.fault_configure("nccl:1")
    try:
        with pytest.raises(hx.HexirError) as err:
            hx.execute(module, devs, out_shape=(600, 384))
        assert err.value.status == _ffi.ERROR_DEVICE
    finally:
        hx.fault_configure("")
    after = hx.execute(module, devs, out_shape=(600, 384))
    assert np.array_equal(bits(after), bits(before))
    module.close()
    for d in devs:
        d.close()
