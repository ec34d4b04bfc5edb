"""hexir-run and the VM on the CPU backend: the reference's runtime tests
(runtime/test/*.test, *.mlir) re-expressed against this runtime, plus the
bounds checks on everything a module file can say."""

import json
import os
import struct
import subprocess

import numpy as np
import pytest

import hexir_b200 as hx
from hexir_b200 import _ffi
from oracle import oracle
from tests.conftest import bin_path

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden",
                                     "golden.json")))
RUN = bin_path("hexir-run")
MK = bin_path("hexir-mkhxb")


def run(*args, check=False):
    return subprocess.run([RUN, *args], capture_output=True, text=True,
                          check=check)


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
def test_known_answers_print_like_the_reference(tmp_path, case):
    path = tmp_path / "m.hxb"
    known_program(case).emit_file(str(path))
    res = run("--quiet", str(path), check=True)
    assert res.stdout == case["stdout_quiet"]


def test_builtin_module_report(tmp_path):
    # fixture-cpu.test:14-31: report lines and results.
    path = tmp_path / "builtin.hxb"
    subprocess.run([MK, "-o", str(path)], check=True)
    out = run(str(path), check=True).stdout
    assert "version       : 3" in out
    assert "sections      : 4" in out
    for kind in ["symbols", "program", "rodata", "executables"]:
        assert kind in out
    assert "device        : cpu" in out
    assert out.endswith(GOLDEN["reference_fixture"]["stdout_quiet"])


def test_selftest_cpu():
    res = run("--selftest", check=True)
    assert "device        : cpu" in res.stdout
    assert "hal roundtrip : ok" in res.stdout


def test_not_a_module_is_refused(tmp_path):
    bad = tmp_path / "bad.hxb"
    bad.write_text("func.func @main() { return }\n")
    res = run(str(bad))
    assert res.returncode == 1
    assert "invalid module" in res.stderr


def test_missing_entry_is_reported(tmp_path):
    path = tmp_path / "m.hxb"
    known_program(GOLDEN["known_answers"][0]).emit_file(str(path))
    res = run(str(path), "--entry=nosuchfunc")
    assert res.returncode == 1 and "not found" in res.stderr


def test_usage_errors_exit_2():
    assert run().returncode == 2
    assert run("--device=tpu", "x.hxb").returncode == 2
    assert run("--bogus").returncode == 2


@pytest.mark.parametrize("flags", [0, _ffi.EMIT_NO_IMAGE])
def test_cuda_module_refused_on_cpu(tmp_path, flags):
    # hxb-cuda.mlir:25-30 / hxb-errors.mlir:29-31: no host fallback.
    path = tmp_path / "m.hxb"
    known_program(GOLDEN["known_answers"][0]).emit_file(
        str(path), "hexir.linear=cuda", flags)
    res = run("--quiet", str(path))
    assert res.returncode == 1
    assert "placed on cuda but the active device is cpu" in res.stderr


def test_mkhxb_text_program_and_unlowered_op(tmp_path):
    src = tmp_path / "p.mlir"
    src.write_text("""func.func @main() {
  %a = hexir.constant dense<[[3.0, -1.0], [2.0, 2.0]]> : tensor<2x2xf64>
  %b = hexir.constant dense<[[1.0, 5.0], [5.0, -2.0]]> : tensor<2x2xf64>
  %m = hexir.linear %a, %b : tensor<2x2xf64>
  %r = hexir.relu %m : tensor<2x2xf64>
  hexir.print %r : tensor<2x2xf64>
  return
}
""")
    out = tmp_path / "p.hxb"
    subprocess.run([MK, "-emit=hxb", "-o", str(out), str(src)], check=True)
    assert run("--quiet", str(out), check=True).stdout == \
        "0.000000 17.000000 \n12.000000 6.000000 \n"
    bad = tmp_path / "bad.mlir"
    bad.write_text(src.read_text().replace("hexir.relu", "hexir.sigmoid"))
    res = subprocess.run([MK, "-o", str(tmp_path / "x.hxb"), str(bad)],
                         capture_output=True, text=True)
    assert res.returncode == 1
    assert "cannot serialize this op into a host program" in res.stderr
    res = subprocess.run([MK, "-placement=hexir.linear=tpu", "-o",
                          str(tmp_path / "y.hxb"), str(src)],
                         capture_output=True, text=True)
    assert res.returncode == 1 and "is not a device" in res.stderr


def test_parity_graph_256_on_cpu_matches_oracle():
    # The CPU-runnable reference graph: linear then relu on 256x256 f64,
    # a then w uniform[-1,1] from seed 0.
    r = hx.Rng(0)
    a, w = r.uniform((256, 256)), r.uniform((256, 256))
    p = hx.Program()
    p.relu(p.linear(p.constant(a), p.constant(w)))
    out = hx.execute(hx.Module(p.emit()), hx.Device("cpu"), out_shape=(256, 256))
    want = oracle.relu(oracle.matmul(a, w))
    assert np.array_equal(out.view(np.uint64), want.view(np.uint64))
    vec = [v for v in GOLDEN["matmul_vectors"] if v["m"] == 256][0]
    import hashlib
    assert hashlib.sha256(out.tobytes()).hexdigest() == vec["relu_sha256"]


def test_mlp_chain_on_cpu_matches_oracle():
    r = hx.Rng(2)
    x = r.normal((64, 32))
    w1 = r.normal((32, 48), std=1 / np.sqrt(32))
    w2 = r.normal((48, 48), std=1 / np.sqrt(48))
    w3 = r.normal((48, 16), std=1 / np.sqrt(48))
    p = hx.Program()
    h = p.relu(p.linear(p.constant(x), p.constant(w1)))
    h = p.relu(p.linear(h, p.constant(w2)))
    p.linear(h, p.constant(w3))
    out = hx.execute(hx.Module(p.emit()), hx.Device("cpu"), out_shape=(64, 16))
    want = oracle.matmul(oracle.relu(oracle.matmul(
        oracle.relu(oracle.matmul(x, w1)), w2)), w3)
    assert np.array_equal(out.view(np.uint64), want.view(np.uint64))


def activation_input(rows=37, cols=53, seed=21):
    """Normal values at scale 4 plus the special ones: signed zeros,
    infinities, NaN, huge magnitudes and the exp overflow edges."""
    x = np.random.default_rng(seed).normal(0, 4, (rows, cols))
    specials = [0.0, -0.0, np.inf, -np.inf, np.nan, 1e300, -1e300, 709.8,
                -709.8, 745.2, -745.2, 5e-324, -5e-324, 40.0, -40.0]
    x[0, :len(specials)] = specials
    return x


@pytest.mark.parametrize("op", sorted(_ffi.ACTIVATIONS))
def test_activations_on_cpu_match_oracle_bit_for_bit(op):
    """cpu-placed activations run the host backend: the oracle's formulas
    with the same C library, so the bits agree (softmax rows included, a
    row of specials among them)."""
    x = activation_input()
    p = hx.Program()
    p.activation(op, p.constant(x))
    out = hx.execute(hx.Module(p.emit(flags=_ffi.EMIT_ACTIVATIONS)),
                     hx.Device("cpu"), out_shape=x.shape)
    want = oracle.activation(op, x)
    assert np.array_equal(out.view(np.uint64), want.view(np.uint64))


def test_activation_chain_through_hexir_run(tmp_path):
    """linear -> gelu -> softmax written by hexir-mkhxb --activations and
    printed by hexir-run on the CPU; without the flag the writer refuses."""
    src = tmp_path / "act.mlir"
    src.write_text("""func.func @main() {
  %a = hexir.constant dense<[[3.0, -1.0], [2.0, 2.0]]> : tensor<2x2xf64>
  %b = hexir.constant dense<[[1.0, 5.0], [5.0, -2.0]]> : tensor<2x2xf64>
  %m = hexir.linear %a, %b : tensor<2x2xf64>
  %g = hexir.gelu %m : tensor<2x2xf64>
  %s = hexir.softmax %g : tensor<2x2xf64>
  hexir.print %s : tensor<2x2xf64>
  return
}
""")
    out = tmp_path / "act.hxb"
    res = subprocess.run([MK, "-o", str(out), str(src)], capture_output=True,
                         text=True)
    assert res.returncode == 1
    assert "cannot serialize this op into a host program" in res.stderr
    subprocess.run([MK, "--activations", "-o", str(out), str(src)], check=True)
    m = oracle.matmul(np.array([[3.0, -1.0], [2.0, 2.0]]),
                      np.array([[1.0, 5.0], [5.0, -2.0]]))
    want = oracle.activation("softmax", oracle.activation("gelu", m))
    text = "".join("".join(f"{v:f} " for v in row) + "\n" for row in want)
    assert run("--quiet", str(out), check=True).stdout == text
    exes = hx.read_executables(out.read_bytes())
    assert [(e.name, e.kind) for e in exes] == [
        ("linear_0", 1), ("gelu_1", 12), ("softmax_2", 11)]


def test_execute_devices_with_no_gpu_runs_cpu_programs():
    p = known_program(GOLDEN["known_answers"][1])
    out = hx.execute(hx.Module(p.emit()), [], out_shape=(2, 2))
    assert np.array_equal(out, [[9.0, 22.0], [17.0, 16.0]])


# ---- everything in a module file is checked before use -------------------

def valid_module():
    p = known_program(GOLDEN["known_answers"][1])
    return bytearray(p.emit())


def run_blob(blob, tmp_path):
    path = tmp_path / "fuzz.hxb"
    path.write_bytes(bytes(blob))
    return run("--quiet", str(path))


def patch_u64(blob, offset, value):
    struct.pack_into("<Q", blob, offset, value)


def program_offset(blob):
    return hx.read_sections(bytes(blob))[2][0]


def test_truncated_module_is_invalid(tmp_path):
    blob = valid_module()
    for cut in [0, 10, 24, 100, len(blob) - 8]:
        res = run_blob(blob[:cut], tmp_path)
        assert res.returncode == 1
        assert "invalid module" in res.stderr or "io error" in res.stderr


def test_bad_section_bounds_are_invalid(tmp_path):
    blob = valid_module()
    struct.pack_into("<Q", blob, 24 + 8, len(blob) + 100)  # symbols offset
    res = run_blob(blob, tmp_path)
    assert res.returncode == 1 and "invalid module" in res.stderr


@pytest.mark.parametrize("field,value", [
    ("const_slot", 300), ("const_offset", 1 << 40), ("const_bytes", 1 << 40),
    ("dispatch_index", 99), ("dispatch_argc", 9), ("dispatch_slot", 255),
    # ALLOC sizes that would wrap a byte count or exceed any memory
    ("alloc_bytes", (1 << 64) - 1), ("alloc_bytes", (1 << 40) + 8)])
def test_bad_operands_are_invalid(tmp_path, field, value):
    blob = valid_module()
    base = program_offset(blob)
    # Program: CONST(0) CONST(1) ALLOC(2) DISPATCH(linear) ...
    const0 = base + 8
    alloc = base + 2 * (8 + 24)
    dispatch = alloc + 8 + 16
    where = {"const_slot": const0, "const_offset": const0 + 8,
             "const_bytes": const0 + 16, "dispatch_index": dispatch + 8,
             "dispatch_argc": dispatch + 16, "dispatch_slot": dispatch + 24,
             "alloc_bytes": alloc + 16}[field]
    patch_u64(blob, where, value)
    res = run_blob(blob, tmp_path)
    assert res.returncode == 1
    assert "invalid module" in res.stderr


def test_extent_larger_than_buffers_is_invalid(tmp_path):
    blob = valid_module()
    off, _ = hx.read_sections(bytes(blob))[4]
    # executable 0 is the 2x2 matmul: claim m = 1000.
    struct.pack_into("<I", blob, off + 8 + 32 + 8, 1000)
    res = run_blob(blob, tmp_path)
    assert res.returncode == 1 and "invalid module" in res.stderr


def test_random_byte_flips_never_crash(tmp_path):
    rng = np.random.default_rng(0)
    base = valid_module()
    for _ in range(150):
        blob = bytearray(base)
        for pos in rng.integers(0, len(blob), size=3):
            blob[pos] = int(rng.integers(0, 256))
        res = run_blob(blob, tmp_path)
        assert res.returncode in (0, 1), res.stderr  # never a signal


def test_keep_constants_on_a_cpu_run_keeps_nothing():
    """hexir_module_keep_constants only concerns GPU copies: a CPU execute is
    unchanged and keeps no bytes; the call checks its argument."""
    p = known_program(GOLDEN["known_answers"][1])
    mod = hx.Module(p.emit())
    mod.keep_constants(True)
    for _ in range(2):
        out = hx.execute(mod, hx.Device("cpu"), out_shape=(2, 2))
        assert np.array_equal(out, [[9.0, 22.0], [17.0, 16.0]])
    assert mod.kept_bytes == 0
    mod.keep_constants(False)
    assert hx.lib().hexir_module_keep_constants(None, 1) == _ffi.ERROR_INVALID_ARGUMENT


def _as_host_module(blob: bytes) -> bytes:
    """The module with every executable moved to the host (device 0, no
    image): the form a hand-made module takes to run a fused kind on a CPU."""
    off, _ = hx.read_sections(blob)[4]
    count, _ = struct.unpack_from("<II", blob, off)
    out = bytearray(blob)
    for i in range(count):
        e = off + 8 + 80 * i
        struct.pack_into("<I", out, e + 36, 0)           # device
        struct.pack_into("<II", out, e + 56, 0, 0)       # image offset, size
    return bytes(out)


@pytest.mark.parametrize("relu", [False, True])
def test_fused_matmul_add_kinds_run_on_the_host(relu):
    """Kinds 5 and 6 on the host: the reference's matmul, add and relu in
    sequence, bit for bit."""
    r = hx.Rng(17)
    a, w, b = r.uniform((24, 40)), r.uniform((40, 16)), r.uniform((24, 16))
    p = hx.Program()
    s = p.add(p.linear(p.constant(a), p.constant(w)), p.constant(b))
    p.print(p.relu(s) if relu else s)
    blob = p.emit("hexir.linear=cuda,hexir.add=cuda,hexir.relu=cuda")
    assert [e.kind for e in hx.read_executables(blob)] == [6 if relu else 5]
    out = hx.execute(hx.Module(_as_host_module(blob)), hx.Device("cpu"),
                     out_shape=(24, 16))
    want = oracle.add(oracle.matmul(a, w), b)
    if relu:
        want = oracle.relu(want)
    assert np.array_equal(out.view(np.uint64), want.view(np.uint64))


def test_hexir_run_repeat_prints_once(tmp_path):
    """hexir-run --repeat=N runs the entry N times, PRINT output from the
    first run only; --time then reports medians; N < 1 is a usage error."""
    p = known_program(GOLDEN["known_answers"][0])
    path = tmp_path / "m.hxb"
    p.emit_file(str(path))
    res = subprocess.run([bin_path("hexir-run"), "--quiet", "--repeat=4",
                          "--time", "--keep-constants", str(path)],
                         capture_output=True, text=True)
    assert res.returncode == 0
    assert res.stdout == GOLDEN["known_answers"][0]["stdout_quiet"]
    assert "runs          : 4" in res.stderr and "median" in res.stderr
    bad = subprocess.run([bin_path("hexir-run"), "--repeat=0", str(path)],
                         capture_output=True, text=True)
    assert bad.returncode == 2


def test_unaligned_section_is_invalid(tmp_path):
    """Sections sit on 8-byte boundaries; a table moved off one is refused."""
    blob = bytearray(valid_module())
    # first section entry: kind u32, flags u32, offset u64 at 24 + 8
    off = struct.unpack_from("<Q", blob, 24 + 8)[0]
    struct.pack_into("<Q", blob, 24 + 8, off + 4)
    res = run_blob(blob, tmp_path)
    assert res.returncode == 1 and "invalid module" in res.stderr


def test_misaligned_const_runs_on_the_host(tmp_path):
    """A CONST at an offset that is not a multiple of 8 (never written by the
    serializer) still computes the reference's answer on the host: the
    kernels read an aligned copy."""
    a = np.array([[3.0, 1.0], [2.0, 2.0]])
    b = np.array([[1.0, 5.0], [5.0, 2.0]])
    # 40 bytes holding b's 32 bytes at byte offset 4.
    raw = np.frombuffer(bytes(4) + b.tobytes() + bytes(4), dtype=np.float64)
    p = hx.Program()
    p.relu(p.constant(raw.reshape(1, 5)))    # keeps the 40 bytes in RODATA
    p.linear(p.constant(a), p.constant(b))   # the captured dispatch
    blob = bytearray(p.emit())
    poff, _ = hx.read_sections(bytes(blob))[2]
    pc, consts = 0, []
    for kind, ops in hx.read_program(bytes(blob)):
        if kind == 2:
            consts.append((pc, ops))
        pc += 8 + 8 * len(ops)
    (_, raw_ops), _, (b_pc, b_ops) = consts
    assert raw_ops[2] == 40 and b_ops[2] == 32
    struct.pack_into("<Q", blob, poff + b_pc + 16, raw_ops[1] + 4)
    out = hx.execute(hx.Module(bytes(blob)), hx.Device("cpu"), out_shape=(2, 2))
    assert np.array_equal(out, [[8.0, 17.0], [12.0, 14.0]])


def test_hexir_bench_verifies_cpu_modules(tmp_path):
    """hexir-bench --device=cpu checks the captured result: a relu over an
    unfused linear (the cpu form) against the reference arithmetic."""
    r = hx.Rng(5)
    a, w = r.uniform((64, 48)), r.uniform((48, 40))
    p = hx.Program()
    p.relu(p.linear(p.constant(a), p.constant(w)))
    path = tmp_path / "m.hxb"
    p.emit_file(str(path))
    res = subprocess.run([bin_path("hexir-bench"), "--device=cpu", "--iters=2",
                          "--no-baseline", "--json", str(path)],
                         capture_output=True, text=True, check=True)
    line = json.loads(res.stdout.strip().splitlines()[-1])
    assert line["verify_ok"] is True and line["verify_max_rel_err"] == 0


def test_one_module_executes_concurrently_from_many_threads():
    """One loaded module, executed at once from 8 threads (ctypes releases
    the GIL for the call), each on its own CPU device and on one shared
    device: every result has the oracle's bits."""
    import threading
    r = hx.Rng(41)
    a, w = r.uniform((96, 64)), r.uniform((64, 48))
    p = hx.Program()
    p.activation("softmax", p.relu(p.linear(p.constant(a), p.constant(w))))
    module = hx.Module(p.emit(flags=_ffi.EMIT_ACTIVATIONS))
    want = oracle.activation("softmax", oracle.relu(oracle.matmul(a, w)))
    shared = hx.Device("cpu")
    bad = []

    def worker(own):
        dev = hx.Device("cpu") if own else shared
        for _ in range(25):
            out = hx.execute(module, dev, out_shape=want.shape)
            if not np.array_equal(out.view(np.uint64), want.view(np.uint64)):
                bad.append(own)

    threads = [threading.Thread(target=worker, args=(i % 2 == 0,))
               for i in range(8)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not bad


def test_cuda_placed_activation_is_refused_on_cpu(tmp_path):
    """A cuda-placed activation on a CPU device gets the reference's
    misplacement message, like a cuda-placed linear."""
    p = hx.Program()
    p.print(p.activation("tanh", p.constant(np.ones((2, 2)))))
    path = tmp_path / "t.hxb"
    p.emit_file(str(path), "hexir.tanh=cuda", _ffi.EMIT_ACTIVATIONS)
    res = run("--quiet", str(path))
    assert res.returncode != 0
    assert "placed on cuda but the active device is cpu" in res.stderr
