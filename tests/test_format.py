"""The .hxb writer against the reference format.

The reference serializer (compiler/Serialization/ModuleSerializer.cpp) cannot
be built here, but its output for the built-in program is checked into the
reference as runtime/test/fixtures/mlp-cpu.hxb; the writer must reproduce it
byte for byte (size and sha256 recorded in tests/golden/golden.json).  The
rest pins the layout rules the serializer follows.
"""

import hashlib
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


def test_builtin_program_is_byte_identical_to_reference_fixture(tmp_path):
    out = tmp_path / "builtin.hxb"
    subprocess.run([bin_path("hexir-mkhxb"), "-emit=hxb", "-o", str(out)],
                   check=True)
    blob = out.read_bytes()
    ref = GOLDEN["reference_fixture"]
    assert len(blob) == ref["size"]
    assert hashlib.sha256(blob).hexdigest() == ref["sha256"]


def two_by_two(p):
    a = p.constant(np.array([[3.0, 1.0], [2.0, 2.0]]))
    b = p.constant(np.array([[1.0, 5.0], [5.0, 2.0]]))
    return a, b


def test_sections_are_aligned_and_in_reference_order():
    p = hx.Program()
    a, b = two_by_two(p)
    p.print(p.relu(p.add(p.linear(a, b), b)))
    for placement in ["", "hexir.linear=cuda,hexir.add=cuda,hexir.relu=cuda"]:
        blob = p.emit(placement)
        magic, version, flags, count, _ = struct.unpack_from("<8sIIII", blob)
        assert magic == b"HEXIRMOD" and version == 3 and flags == 0
        kinds = []
        for i in range(count):
            kind, sflags, off, size = struct.unpack_from("<IIQQ", blob, 24 + 24 * i)
            assert off % 8 == 0 and off + size <= len(blob)
            kinds.append(kind)
        assert kinds[:4] == [1, 2, 3, 4]
        assert kinds[4:] == ([5] if placement else [])


def test_executable_names_kinds_and_fusion():
    p = hx.Program()
    a, b = two_by_two(p)
    m = p.linear(a, b)
    r = p.relu(m)
    s = p.add(r, b)
    p.print(p.relu(s))
    cpu = hx.read_executables(p.emit())
    assert [(e.name, e.kind, e.device) for e in cpu] == [
        ("linear_0", 1, 0), ("relu_1", 3, 0), ("add_2", 2, 0), ("relu_3", 3, 0)]
    gpu = hx.read_executables(p.emit("hexir.linear=cuda,hexir.relu=cuda,"
                                     "hexir.add=cuda"))
    # linear -> relu folds into one matmul_relu executable named after the
    # linear; later kernels keep their walk-order numbers.
    assert [(e.name, e.kind, e.device) for e in gpu] == [
        ("linear_0", 4, 1), ("add_2", 2, 1), ("relu_3", 3, 1)]
    # One shared image for every cuda entry.
    assert len({(e.image_offset, e.image_size) for e in gpu}) == 1
    assert gpu[0].image_size == len(hx.kernel_image())
    nofuse = hx.read_executables(p.emit("hexir.linear=cuda,hexir.relu=cuda,"
                                        "hexir.add=cuda", _ffi.EMIT_NO_FUSE))
    assert [e.name for e in nofuse] == ["linear_0", "relu_1", "add_2", "relu_3"]
    # Different devices never fuse.
    mixed = hx.read_executables(p.emit("hexir.linear=cuda,hexir.relu=cpu"))
    assert [(e.name, e.device) for e in mixed][:2] == [("linear_0", 1),
                                                       ("relu_1", 0)]


def test_linear_with_second_user_is_not_fused():
    p = hx.Program()
    a, b = two_by_two(p)
    m = p.linear(a, b)
    p.print(p.relu(m))
    p.print(m)
    exes = hx.read_executables(p.emit("hexir.linear=cuda,hexir.relu=cuda"))
    assert [e.kind for e in exes] == [1, 3]


def test_program_commands_follow_serializer():
    p = hx.Program()
    p.constant(np.ones((1, 2)))  # unused: dropped
    a, b = two_by_two(p)
    m = p.linear(a, b)
    p.print(m)
    cmds = hx.read_program(p.emit())
    assert cmds == [(2, (0, 0, 32)), (2, (1, 32, 32)), (1, (2, 32)),
                    (3, (0, 3, 0, 1, 2)), (4, (2, 2, 2)), (0, ())]


def test_splat_is_expanded():
    p = hx.Program()
    s = p.splat(2.0, 3, 4)
    p.print(s)
    blob = p.emit()
    off, size = hx.read_sections(blob)[3]
    assert size == 3 * 4 * 8
    assert np.array_equal(np.frombuffer(blob[off:off + size]), np.full(12, 2.0))


def test_launch_section_records_devices():
    p = hx.Program()
    a, b = two_by_two(p)
    p.print(p.relu(p.linear(a, b)))
    blob = p.emit("hexir.linear=cuda:2-5,hexir.relu=cuda:2-5")
    off, size = hx.read_sections(blob)[5]
    count, _ = struct.unpack_from("<II", blob, off)
    assert count == 1
    abi, flags, first, n = struct.unpack_from("<4I", blob, off + 8)
    assert (abi, flags, first, n) == (1, 1, 2, 4)
    assert hx.read_launch(blob)[0].device_count == 4
    # cpu entries get an empty launch record; all-cpu modules no section.
    mixed = p.emit("hexir.linear=cuda:1,hexir.relu=cpu", _ffi.EMIT_NO_FUSE)
    recs = hx.read_launch(mixed)
    assert [(r.abi, r.device_first) for r in recs] == [(1, 1), (0, 0)]
    assert hx.read_launch(p.emit()) == []


@pytest.mark.parametrize("bad,msg", [
    ("hexir.linear", "is not of the form <op-name>=<device>"),
    ("hexir.linear=tpu", "'tpu' is not a device; expected cpu, cuda or gpu"),
    ("hexir.softmax=cuda", "'hexir.softmax' is not a placeable op"),
    ("hexir.linear=cuda:3-1", "is not a device"),
])
def test_placement_errors_use_reference_wording(bad, msg):
    p = hx.Program()
    a, b = two_by_two(p)
    p.linear(a, b)
    with pytest.raises(ValueError, match=msg.replace("(", r"\(").replace(")", r"\)")):
        p.emit(bad)


def test_gpu_alias_and_ordinals_parse():
    p = hx.Program()
    a, b = two_by_two(p)
    p.linear(a, b)
    for dev in ["gpu", "cuda", "cuda:0", "cuda:7", "gpu:1-2"]:
        assert hx.read_executables(p.emit(f"hexir.linear={dev}"))[0].device == 1


TEXT = """
// comment
func.func @main() {
  %a = hexir.constant dense<[[3.0, 1.0], [2.0, 2.0]]> : tensor<2x2xf64>
  %b = hexir.constant dense<[[1.0, 5.0], [5.0, 2.0]]> : tensor<2x2xf64>
  %m = hexir.linear %a, %b : tensor<2x2xf64>
  %s = hexir.add %m, %b : tensor<2x2xf64>
  %r = hexir.relu %s : tensor<2x2xf64>
  hexir.print %r : tensor<2x2xf64>
  return
}
"""


def test_text_program_matches_builder():
    p = hx.Program()
    a, b = two_by_two(p)
    p.print(p.relu(p.add(p.linear(a, b), b)))
    assert hx.parse(TEXT).emit() == p.emit()


def test_text_functional_type_and_splat():
    text = """func.func @main() {
      %x = hexir.constant dense<1.000000e+00> : tensor<3x4xf64>
      %w = hexir.constant dense<2.0> : tensor<4x5xf64>
      %m = hexir.linear %x, %w : (tensor<3x4xf64>, tensor<4x5xf64>) -> tensor<3x5xf64>
      return
    }"""
    exe = hx.read_executables(hx.parse(text).emit())[0]
    assert (exe.m, exe.n, exe.k) == (3, 5, 4)


def test_text_unlowered_op_is_refused_like_the_reference():
    """The reference serializer refuses hexir.sigmoid (runtime/test/
    hxb-errors.mlir:6-10); so does the writer unless activations are asked
    for."""
    text = """func.func @main() {
      %a = hexir.constant dense<[[3.0, 1.0], [2.0, 2.0]]> : tensor<2x2xf64>
      %s = hexir.sigmoid %a : tensor<2x2xf64>
      hexir.print %s : tensor<2x2xf64>
      return
    }"""
    prog = hx.parse(text)
    with pytest.raises(ValueError, match="cannot serialize this op into a host program"):
        prog.emit()
    with pytest.raises(ValueError, match="'hexir.sigmoid' is not a placeable op"):
        prog.emit("hexir.sigmoid=cuda", _ffi.EMIT_NO_FUSE)
    exe = hx.read_executables(prog.emit(flags=_ffi.EMIT_ACTIVATIONS))
    assert [(e.name, e.kind, e.m, e.n, e.k) for e in exe] == [("sigmoid_0", 9, 2, 2, 0)]
    # Ops the dialect does not declare stay refused at parse time.
    with pytest.raises(ValueError, match="cannot serialize this op into a host program"):
        hx.parse(text.replace("hexir.sigmoid", "hexir.softplus"))


@pytest.mark.parametrize("op,kind", sorted(_ffi.ACTIVATIONS.items()))
def test_activation_executables(op, kind):
    """Each activation: parsed from text and built through the API, named
    <op>_<n> in walk order, placeable on cpu or cuda, never fused into the
    linear that feeds it."""
    text = f"""func.func @main() {{
      %x = hexir.constant dense<1.5> : tensor<3x4xf64>
      %w = hexir.constant dense<0.5> : tensor<4x5xf64>
      %m = hexir.linear %x, %w : (tensor<3x4xf64>, tensor<4x5xf64>) -> tensor<3x5xf64>
      %a = hexir.{op} %m : tensor<3x5xf64>
      hexir.print %a : tensor<3x5xf64>
      return
    }}"""
    for placement, device in (("", 0), (f"hexir.linear=cuda,hexir.{op}=cuda", 1)):
        blob = hx.parse(text).emit(placement, _ffi.EMIT_ACTIVATIONS)
        exes = hx.read_executables(blob)
        assert [(e.name, e.kind, e.device) for e in exes] == [
            ("linear_0", 1, device), (f"{op}_1", kind, device)]
        assert (exes[1].m, exes[1].n, exes[1].k) == (3, 5, 0)
        assert [c[0] for c in hx.read_program(blob)].count(3) == 2
    p = hx.Program()
    x = p.constant(np.ones((2, 3)))
    y = p.activation(op, x)
    p.print(y)
    exes = hx.read_executables(p.emit(f"hexir.{op}=cuda:0-1", _ffi.EMIT_ACTIVATIONS))
    assert [(e.name, e.kind, e.device) for e in exes] == [(f"{op}_0", kind, 1)]
    launch = hx.read_launch(p.emit(f"hexir.{op}=cuda:0-1", _ffi.EMIT_ACTIVATIONS))
    assert (launch[0].device_first, launch[0].device_count) == (0, 2)


def test_activation_api_errors():
    p = hx.Program()
    x = p.constant(np.ones((2, 3)))
    with pytest.raises(Exception, match="not an activation"):
        p.activation("softplus", x)
    with pytest.raises(Exception, match="unknown operand"):
        p.activation("gelu", 99)
    assert p.activation("hexir.gelu", x) >= 0


def test_shape_mismatch_is_refused():
    p = hx.Program()
    a = p.constant(np.ones((2, 3)))
    with pytest.raises(ValueError, match="linear"):
        p.linear(a, p.constant(np.ones((2, 3))))


def test_multiple_functions_share_slots_and_rodata():
    p = hx.Program()
    p.function("first")
    a, b = two_by_two(p)
    p.print(p.linear(a, b))
    p.function("second")
    c = p.constant(np.eye(2))
    p.print(p.relu(c))
    blob = p.emit()
    assert hx.read_program(blob, "first")[2] == (1, (2, 32))
    # Slot numbers continue across functions, as the serializer's counter.
    assert hx.read_program(blob, "second")[0][1][0] == 3
    assert [e.name for e in hx.read_executables(blob)] == ["linear_0", "relu_1"]


def test_rng_stream_is_stable():
    r = hx.Rng(0)
    first = r.uniform(4)
    again = hx.Rng(0).uniform(8)
    assert np.array_equal(first, again[:4])
    assert np.all((again >= -1) & (again < 1))
    # a then w continue one stream.
    r2 = hx.Rng(0)
    r2.uniform(4)
    assert np.array_equal(r2.uniform(4), again[4:])
    r3 = hx.Rng(0)
    r3.skip(5)
    assert np.array_equal(r3.uniform(3), again[5:])
    n = hx.Rng(5).normal(20000)
    assert abs(n.mean()) < 0.05 and abs(n.std() - 1) < 0.05


def test_reference_runtime_runs_our_cpu_modules(tmp_path):
    """Drop-in check: modules from this writer run on the reference runtime
    and print what the reference's own tests expect."""
    if not oracle.have_reference():
        pytest.skip("reference runtime not built here")
    for case in GOLDEN["known_answers"]:
        p = hx.Program()
        a = p.constant(np.array(case["a"]))
        b = p.constant(np.array(case["b"]))
        v = p.linear(a, b)
        for op in case["ops"][1:]:
            v = p.add(v, b) if op == "add_b" else p.relu(v)
        p.print(v)
        path = tmp_path / (case["name"] + ".hxb")
        p.emit_file(str(path))
        res = subprocess.run([oracle.REF_RUN, "--quiet", str(path)],
                             capture_output=True, text=True, check=True)
        assert res.stdout == case["stdout_quiet"]


@pytest.mark.parametrize("op", sorted(_ffi.ACTIVATIONS))
def test_reference_runtime_refuses_activation_kinds(tmp_path, op):
    """Kinds 7-14 are additive: the reference runtime, which has no kernel
    for them, refuses such a module ("unimplemented") instead of running
    something else, while this runtime prints the oracle's values."""
    if not oracle.have_reference():
        pytest.skip("reference runtime not built here")
    x = np.array([[1.0, -2.0], [0.5, 3.0]])
    p = hx.Program()
    p.print(p.activation(op, p.constant(x)))
    path = tmp_path / f"{op}.hxb"
    p.emit_file(str(path), "", _ffi.EMIT_ACTIVATIONS)
    res = subprocess.run([oracle.REF_RUN, "--quiet", str(path)],
                         capture_output=True, text=True)
    assert res.returncode != 0 and "unimplemented" in res.stderr
    ours = subprocess.run([bin_path("hexir-run"), "--quiet", str(path)],
                          capture_output=True, text=True, check=True)
    want = oracle.activation(op, x)
    assert ours.stdout == "".join("".join(f"{v:f} " for v in row) + "\n"
                                  for row in want)


def test_linear_add_relu_fuses_at_the_add():
    """linear -> add -> relu on one GPU spec: one matmul_add_relu executable
    named after the linear (kind 6), dispatched where the add stands with
    operands a, w, addend, destination; the relu is folded."""
    p = hx.Program()
    a, b = two_by_two(p)
    p.print(p.relu(p.add(p.linear(a, b), b)))
    blob = p.emit("hexir.linear=cuda,hexir.add=cuda,hexir.relu=cuda")
    exes = hx.read_executables(blob)
    assert [(e.name, e.kind, e.device, e.m, e.n, e.k) for e in exes] == [
        ("linear_0", 6, 1, 2, 2, 2)]
    assert hx.read_program(blob) == [
        (2, (0, 0, 32)), (2, (1, 32, 32)), (1, (2, 32)),
        (3, (0, 4, 0, 1, 1, 2)), (4, (2, 2, 2)), (0, ())]
    # The linear as the add's second operand fuses the same way.
    p2 = hx.Program()
    a, b = two_by_two(p2)
    p2.print(p2.relu(p2.add(b, p2.linear(a, b))))
    assert [e.kind for e in hx.read_executables(
        p2.emit("hexir.linear=cuda,hexir.add=cuda,hexir.relu=cuda"))] == [6]
    nofuse = hx.read_executables(p.emit(
        "hexir.linear=cuda,hexir.add=cuda,hexir.relu=cuda", _ffi.EMIT_NO_FUSE))
    assert [(e.name, e.kind) for e in nofuse] == [
        ("linear_0", 1), ("add_1", 2), ("relu_2", 3)]


def test_linear_add_fusion_rules():
    p = hx.Program()
    a, b = two_by_two(p)
    s = p.add(p.linear(a, b), b)
    p.print(s)
    p.print(p.relu(s))  # the add has a second user: the relu stays
    exes = hx.read_executables(p.emit("hexir.linear=cuda,hexir.add=cuda,"
                                      "hexir.relu=cuda"))
    assert [(e.name, e.kind) for e in exes] == [("linear_0", 5), ("relu_2", 3)]
    # Different devices never fuse; a linear with two users never fuses.
    mixed = hx.read_executables(p.emit("hexir.linear=cuda,hexir.add=cpu"))
    assert [(e.name, e.kind, e.device) for e in mixed][:2] == [
        ("linear_0", 1, 1), ("add_1", 2, 0)]
    p3 = hx.Program()
    a, b = two_by_two(p3)
    m = p3.linear(a, b)
    p3.print(p3.add(m, m))
    assert [e.kind for e in hx.read_executables(
        p3.emit("hexir.linear=cuda,hexir.add=cuda"))] == [1, 2]


def test_fused_add_waits_for_an_addend_computed_after_the_linear():
    """The addend is a relu computed after the linear: the fused dispatch
    stands where the add does, after the relu that defines its addend."""
    p = hx.Program()
    a, b = two_by_two(p)
    lin = p.linear(a, b)
    x = p.relu(p.constant(np.array([[-1.0, 2.0], [3.0, -4.0]])))
    p.print(p.add(lin, x))
    blob = p.emit("hexir.linear=cuda,hexir.add=cuda,hexir.relu=cuda")
    exes = hx.read_executables(blob)
    assert [(e.name, e.kind) for e in exes] == [("relu_1", 3), ("linear_0", 5)]
    cmds = hx.read_program(blob)
    dispatches = [ops for kind, ops in cmds if kind == 3]
    assert dispatches[0][0] == 0 and dispatches[1][0] == 1  # relu, then fused
    assert dispatches[1][1] == 4 and dispatches[1][4] == dispatches[0][3]


def test_dump_tool_decodes_fused_kinds_and_launch(tmp_path):
    """python -m hexir_b200.dump: sections, fused kinds, the LAUNCH range and
    the command list of each entry; a non-module exits 1."""
    import sys
    p = hx.Program()
    a, b = two_by_two(p)
    p.print(p.relu(p.add(p.linear(a, b), b)))
    path = tmp_path / "m.hxb"
    p.emit_file(str(path), "hexir.linear=cuda:0-1,hexir.add=cuda:0-1,"
                           "hexir.relu=cuda:0-1")
    res = subprocess.run([sys.executable, "-m", "hexir_b200.dump", str(path)],
                         capture_output=True, text=True, check=True,
                         cwd=os.path.dirname(os.path.dirname(__file__)))
    assert "section LAUNCH" in res.stdout
    assert "linear_0" in res.stdout and "matmul_add_relu" in res.stdout
    assert "cuda:0-1" in res.stdout
    assert "DISPATCH linear_0 (0 1 1) -> slot 2" in res.stdout
    bad = tmp_path / "bad.hxb"
    bad.write_bytes(b"not a module at all, not even close")
    res = subprocess.run([sys.executable, "-m", "hexir_b200.dump", str(bad)],
                         capture_output=True, text=True,
                         cwd=os.path.dirname(os.path.dirname(__file__)))
    assert res.returncode == 1 and "not a version 3 hexir module" in res.stderr


def test_dump_tool_names_the_activation_kinds(tmp_path):
    import sys
    p = hx.Program()
    a, _ = two_by_two(p)
    v = a
    for op in sorted(_ffi.ACTIVATIONS):
        v = p.activation(op, v)
    p.print(v)
    path = tmp_path / "act.hxb"
    p.emit_file(str(path), "hexir.gelu=cuda", _ffi.EMIT_ACTIVATIONS)
    res = subprocess.run([sys.executable, "-m", "hexir_b200.dump", str(path)],
                         capture_output=True, text=True, check=True,
                         cwd=os.path.dirname(os.path.dirname(__file__)))
    for i, op in enumerate(sorted(_ffi.ACTIVATIONS)):
        assert f"{op}_{i}" in res.stdout
    assert "kind " not in res.stdout  # every kind has a name


def test_linear_relu_fusion_next_to_an_activation():
    """linear -> relu -> gelu on one GPU: linear and relu fuse (kind 4, the
    relu's number taken but folded), the gelu stays its own executable and
    reads the fused result."""
    p = hx.Program()
    a, b = two_by_two(p)
    p.print(p.activation("gelu", p.relu(p.linear(a, b))))
    blob = p.emit("hexir.linear=cuda,hexir.relu=cuda,hexir.gelu=cuda",
                  _ffi.EMIT_ACTIVATIONS)
    exes = hx.read_executables(blob)
    assert [(e.name, e.kind) for e in exes] == [("linear_0", 4), ("gelu_2", 12)]
    dispatches = [ops for kind, ops in hx.read_program(blob) if kind == 3]
    # gelu reads the slot the fused kernel writes.
    assert dispatches[1][2] == dispatches[0][-1]
