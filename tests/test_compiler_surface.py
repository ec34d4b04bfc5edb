"""The compiler-side surface (hexir_b200/compiler), on CPU.

The reference compiler needs MLIR from LLVM 24.0git, so its part of the
integration (B200Serializer.cpp and the patch to the reference tree) cannot
be compiled here.  What carries the logic is standard C++ and is compiled
and run here with g++:
  - DeviceSpec.cpp, the placement grammar the patched -placement flag,
    target registry and lowerings use: it must accept and reject exactly
    what the runtime's writer accepts, and spell specs canonically;
  - B200ModuleWriter.cpp, which turns the host program the serializer reads
    off the kernel-level IR into module bytes through libhexir_b200's writer:
    for the same program and placement the bytes must equal the Python
    writer's, the section order and kernel kinds must be those of
    include/hexir_runtime/module.h and program.h, and each cuda:F-L
    placement must reach the LAUNCH section.
Where the reference tree is present the patch must apply to it cleanly.
"""

import os
import re
import shutil
import subprocess

import numpy as np
import pytest

import hexir_b200 as hx
from hexir_b200 import _ffi
from oracle import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
COMPILER = os.path.join(ROOT, "hexir_b200", "compiler")
PATCH = os.path.join(COMPILER, "patches",
                     "0001-b200-placement-and-serializer.patch")

DRIVER = r'''
#include "hexir_b200/compiler/Serialization/B200ModuleWriter.h"
#include "hexir_b200/compiler/Target/DeviceSpec.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <string>

using namespace hexir_b200;

// spec: one device spec per stdin line -> parse result, kind, canonical.
// write <out> <flags> <linear> <add> <relu>: the program of
//   relu(linear(a, w) + bias), printed, plus an unused constant, with each
//   op kind on the given device.
int main(int argc, char **argv) {
  if (argc >= 2 && !std::strcmp(argv[1], "spec")) {
    std::string line;
    while (std::getline(std::cin, line)) {
      DeviceSpec d;
      const bool ok = parseDeviceSpec(line, &d);
      std::printf("%s\t%d\t%s\t%s\t%d\t%u\t%u\n", line.c_str(), ok,
                  std::string(deviceKind(line)).c_str(),
                  canonicalDeviceSpec(line).c_str(), isCudaSpec(line),
                  ok ? d.first : 0u, ok ? d.count : 0u);
    }
    return 0;
  }
  if (argc != 7 || std::strcmp(argv[1], "write"))
    return 2;
  std::vector<HostOp> ops;
  auto push = [&](HostOp op) { ops.push_back(op); return (int32_t)ops.size() - 1; };
  HostOp f; f.kind = HostOpKind::BeginFunction; f.name = "main"; push(f);
  HostOp a; a.kind = HostOpKind::Constant; a.rows = 2; a.cols = 3;
  a.data = {3.0, 1.0, -2.0, 2.0, 2.0, 0.5};
  const int32_t ia = push(a);
  HostOp unused; unused.kind = HostOpKind::Splat; unused.rows = 4;
  unused.cols = 4; unused.splat = 9.0; push(unused);
  HostOp w; w.kind = HostOpKind::Constant; w.rows = 3; w.cols = 2;
  w.data = {1.0, 5.0, 5.0, 2.0, -1.0, 4.0};
  const int32_t iw = push(w);
  HostOp bias; bias.kind = HostOpKind::Splat; bias.rows = 2; bias.cols = 2;
  bias.splat = -7.5;
  const int32_t ib = push(bias);
  HostOp lin; lin.kind = HostOpKind::Linear; lin.operands = {ia, iw};
  lin.device = argv[4];
  const int32_t il = push(lin);
  HostOp add; add.kind = HostOpKind::Add; add.operands = {il, ib};
  add.device = argv[5];
  const int32_t id = push(add);
  HostOp relu; relu.kind = HostOpKind::Relu; relu.operands = {id};
  relu.device = argv[6];
  const int32_t ir = push(relu);
  HostOp pr; pr.kind = HostOpKind::Print; pr.operands = {ir}; push(pr);
  std::string bytes, error;
  if (!writeModule(ops, (uint32_t)std::strtoul(argv[3], nullptr, 0), &bytes,
                   &error)) {
    std::fprintf(stderr, "%s\n", error.c_str());
    return 1;
  }
  FILE *out = std::fopen(argv[2], "wb");
  std::fwrite(bytes.data(), 1, bytes.size(), out);
  std::fclose(out);
  return 0;
}
'''


@pytest.fixture(scope="module")
def driver(tmp_path_factory):
    if not shutil.which("g++"):
        pytest.skip("g++ is not installed")
    d = tmp_path_factory.mktemp("compiler")
    src = d / "driver.cpp"
    src.write_text(DRIVER)
    exe = d / "driver"
    lib_dir = os.path.dirname(_ffi.LIB_PATH)
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror",
           f"-I{ROOT}", f"-I{ROOT}/include", str(src),
           os.path.join(COMPILER, "Target", "DeviceSpec.cpp"),
           os.path.join(COMPILER, "Serialization", "B200ModuleWriter.cpp"),
           f"-L{lib_dir}", "-lhexir_b200", f"-Wl,-rpath,{lib_dir}",
           "-o", str(exe)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    return str(exe)


SPECS = {
    # text: (accepted, kind, canonical, first, count)
    "cpu": (1, "cpu", "cpu", 0, 1),
    "cuda": (1, "cuda", "cuda", 0, 1),
    "gpu": (1, "cuda", "cuda", 0, 1),
    "cuda:0": (1, "cuda", "cuda:0", 0, 1),
    "cuda:7": (1, "cuda", "cuda:7", 7, 1),
    "gpu:3": (1, "cuda", "cuda:3", 3, 1),
    "cuda:007": (1, "cuda", "cuda:7", 7, 1),
    "cuda:0-7": (1, "cuda", "cuda:0-7", 0, 8),
    "gpu:2-5": (1, "cuda", "cuda:2-5", 2, 4),
    "cuda:4-4": (1, "cuda", "cuda:4", 4, 1),
    "cuda:9999": (1, "cuda", "cuda:9999", 9999, 1),
    "cuda:10000": (0, "", "", 0, 0),
    "cuda:5-3": (0, "", "", 0, 0),
    "cuda:": (0, "", "", 0, 0),
    "cuda:-1": (0, "", "", 0, 0),
    "cuda:1-": (0, "", "", 0, 0),
    "cuda:a": (0, "", "", 0, 0),
    "cuda:1-2-3": (0, "", "", 0, 0),
    "CUDA": (0, "", "", 0, 0),
    "tpu": (0, "", "", 0, 0),
    "cpu:0": (0, "", "", 0, 0),
    " cuda": (0, "", "", 0, 0),
}


def test_device_spec_grammar(driver):
    res = subprocess.run([driver, "spec"], input="\n".join(SPECS) + "\n",
                         capture_output=True, text=True, check=True)
    rows = [line.split("\t") for line in res.stdout.splitlines()]
    assert len(rows) == len(SPECS)
    for text, ok, kind, canon, is_cuda, first, count in rows:
        want = SPECS[text]
        assert (int(ok), kind, canon) == want[:3], text
        assert int(is_cuda) == (kind == "cuda"), text
        if want[0]:
            assert (int(first), int(count)) == want[3:], text


def test_device_spec_grammar_is_the_writers(driver):
    """Every spec DeviceSpec accepts the runtime's writer accepts as a
    placement, and every one it rejects the writer rejects."""
    p = hx.Program()
    p.print(p.linear(p.constant(np.ones((2, 2))), p.constant(np.ones((2, 2)))))
    for text, want in SPECS.items():
        if text.strip() != text:
            continue  # the writer's list splitting is not the grammar's
        try:
            p.emit(f"hexir.linear={text}", _ffi.EMIT_NO_IMAGE)
            accepted = 1
        except ValueError:
            accepted = 0
        assert accepted == want[0], text


def python_module(placement, flags):
    """The same program through the Python face of the writer."""
    p = hx.Program()
    a = p.constant(np.array([[3.0, 1.0, -2.0], [2.0, 2.0, 0.5]]))
    p.splat(9.0, 4, 4)
    w = p.constant(np.array([[1.0, 5.0], [5.0, 2.0], [-1.0, 4.0]]))
    b = p.splat(-7.5, 2, 2)
    p.print(p.relu(p.add(p.linear(a, w), b)))
    return p.emit(placement, flags)


def run_write(driver, tmp_path, devices, flags=0):
    out = tmp_path / "m.hxb"
    res = subprocess.run([driver, "write", str(out), str(flags), *devices],
                         capture_output=True, text=True)
    return res, (out.read_bytes() if res.returncode == 0 else None)


@pytest.mark.parametrize("devices,placement", [
    (("cpu", "cpu", "cpu"), ""),
    (("cuda", "cuda", "cuda"), "hexir.linear=cuda,hexir.add=cuda,hexir.relu=cuda"),
    (("gpu:1", "cpu", "cuda:1"), "hexir.linear=cuda:1,hexir.relu=cuda:1"),
    (("cuda:0-3", "cuda:0-3", "cuda:0-3"),
     "hexir.linear=cuda:0-3,hexir.add=cuda:0-3,hexir.relu=cuda:0-3"),
    (("cuda", "cpu", "cpu"), "hexir.linear=cuda"),
])
@pytest.mark.parametrize("flags", [0, _ffi.EMIT_NO_FUSE])
def test_compiler_writes_the_writers_bytes(driver, tmp_path, devices,
                                           placement, flags):
    res, blob = run_write(driver, tmp_path, devices, flags)
    assert res.returncode == 0, res.stderr
    assert blob == python_module(placement, flags)


def header_enum(path, prefix):
    text = open(os.path.join(ROOT, "include", "hexir_runtime", path)).read()
    return {m.group(1): int(m.group(2)) for m in
            re.finditer(rf"\b({prefix}\w+)\s*=\s*(\d+)", text)}


def test_compiler_modules_follow_the_headers(driver, tmp_path):
    """Section order and kinds, fused kernel kinds and LAUNCH entries of a
    module the compiler side writes, read back with the format's own
    numbers from include/hexir_runtime."""
    sec = header_enum("module.h", "HEXIR_SECTION_")
    kinds = header_enum("program.h", "HEXIR_KERNEL_")
    # cpu: the reference's four sections, in its order, no LAUNCH.
    _, blob = run_write(driver, tmp_path, ("cpu", "cpu", "cpu"))
    order = list(hx.read_sections(blob))
    assert order == [sec["HEXIR_SECTION_SYMBOLS"], sec["HEXIR_SECTION_PROGRAM"],
                     sec["HEXIR_SECTION_RODATA"],
                     sec["HEXIR_SECTION_EXECUTABLES"]]
    assert [e.kind for e in hx.read_executables(blob)] == [
        kinds["HEXIR_KERNEL_MATMUL"], kinds["HEXIR_KERNEL_ADD"],
        kinds["HEXIR_KERNEL_RELU"]]
    # all on GPUs 2..3: linear + add + relu fuse into one kind-6 executable
    # that carries the range in its LAUNCH entry.
    _, blob = run_write(driver, tmp_path, ("cuda:2-3",) * 3)
    assert list(hx.read_sections(blob)) == order + [sec["HEXIR_SECTION_LAUNCH"]]
    exes = hx.read_executables(blob)
    assert [e.kind for e in exes] == [kinds["HEXIR_KERNEL_MATMUL_ADD_RELU"]]
    launch = hx.read_launch(blob)
    assert len(launch) == 1
    assert (launch[0].device_first, launch[0].device_count) == (2, 2)
    # linear + relu on one GPU, the add between them on the host: no fusion
    # across devices.
    _, blob = run_write(driver, tmp_path, ("cuda:1", "cpu", "cuda:1"))
    assert [e.kind for e in hx.read_executables(blob)] == [
        kinds["HEXIR_KERNEL_MATMUL"], kinds["HEXIR_KERNEL_ADD"],
        kinds["HEXIR_KERNEL_RELU"]]


def test_compiler_module_runs_on_the_host(driver, tmp_path):
    """The compiler-side module of a cpu placement runs in this runtime and
    prints the reference's arithmetic."""
    _, blob = run_write(driver, tmp_path, ("cpu", "cpu", "cpu"))
    a = np.array([[3.0, 1.0, -2.0], [2.0, 2.0, 0.5]])
    w = np.array([[1.0, 5.0], [5.0, 2.0], [-1.0, 4.0]])
    want = oracle.relu(oracle.add(oracle.matmul(a, w), np.full((2, 2), -7.5)))
    module = hx.Module(blob)
    dev = hx.Device("cpu")
    got = hx.execute(module, dev, out_shape=(2, 2))
    assert np.array_equal(got.view(np.uint64), want.view(np.uint64))
    module.close()
    dev.close()


def test_compiler_refuses_one_kind_on_two_devices(driver, tmp_path):
    res, _ = run_write(driver, tmp_path, ("cuda:0", "cuda:0", "cuda:1"))
    assert res.returncode == 0  # different kinds may differ
    res, _ = run_write(driver, tmp_path, ("cuda:0", "bogus", "cpu"))
    assert res.returncode == 1 and "not a device" in res.stderr


def test_patch_names_only_what_the_compiler_sources_declare():
    """Every hexir_b200:: name the patch calls is declared in the
    compiler-side headers, and every header it includes exists."""
    text = open(PATCH).read()
    added = "\n".join(l[1:] for l in text.splitlines()
                      if l.startswith("+") and not l.startswith("+++"))
    headers = open(os.path.join(COMPILER, "Target", "DeviceSpec.h")).read() + \
        open(os.path.join(COMPILER, "Serialization", "B200Serializer.h")).read()
    for name in set(re.findall(r"hexir_b200::(\w+)", added)):
        assert re.search(rf"\b{name}\(", headers), name
    for inc in set(re.findall(r'#include "(hexir_b200/[^"]+)"', added)):
        assert os.path.exists(os.path.join(ROOT, inc)), inc
    for src in re.findall(r"\$\{HEXIR_B200_COMPILER\}/(\S+\.cpp)", added):
        assert os.path.exists(os.path.join(COMPILER, src)), src


def test_patch_applies_to_the_reference_tree(tmp_path):
    root = oracle.reference_root()
    if not root or not shutil.which("patch"):
        pytest.skip("the reference tree (or patch) is not present here")
    for d in ("tools", "compiler"):
        shutil.copytree(os.path.join(root, d), tmp_path / d)
    res = subprocess.run(["patch", "-p1", "--dry-run", "-i", PATCH],
                         cwd=tmp_path, capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr
