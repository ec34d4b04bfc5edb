"""Host-side fault injection (include/hexir_b200/fault.h): each error path
the runtime has for a failed allocation, reached without a GPU fault.

Rules are process-wide, so every test here restores "no rules" when it ends.
The GPU-side sites (kernel launches, the in-process NCCL steps) are counted
the same way; these tests exercise the host ones on the CPU device.
"""

import os
import subprocess

import numpy as np
import pytest

import hexir_b200 as hx
from hexir_b200 import _ffi
from oracle import oracle
from tests.conftest import bin_path


@pytest.fixture(autouse=True)
def no_rules_after():
    yield
    hx.fault_configure("")


@pytest.mark.parametrize("spec", ["alloc", "alloc:", "alloc:0", "alloc:x",
                                  "disk:1", "alloc:1,", "alloc:-1", ":1",
                                  "alloc:1++", "launch:99999999999999999999"])
def test_malformed_rules_are_refused_and_leave_the_old_ones(spec):
    hx.fault_configure("alloc:7")
    with pytest.raises(_ffi.HexirError) as err:
        hx.fault_configure(spec)
    assert err.value.status == _ffi.ERROR_INVALID_ARGUMENT
    dev = hx.Device("cpu")
    for _ in range(3):
        dev.buffer(8).close()
    assert hx.fault_calls("alloc") == 3


def test_nth_allocation_fails_once():
    dev = hx.Device("cpu")
    hx.fault_configure("alloc:2")
    dev.buffer(64).close()
    with pytest.raises(_ffi.HexirError) as err:
        dev.buffer(64)
    assert err.value.status == _ffi.ERROR_OUT_OF_MEMORY
    dev.buffer(64).close()
    assert hx.fault_calls("alloc") == 3
    assert hx.fault_calls("launch") == 0 and hx.fault_calls("disk") == 0


def test_onward_rule_and_several_rules():
    dev = hx.Device("cpu")
    hx.fault_configure("alloc:2,alloc:5+")
    outcome = []
    for _ in range(7):
        try:
            dev.buffer(8).close()
            outcome.append(True)
        except _ffi.HexirError:
            outcome.append(False)
    assert outcome == [True, False, True, True, False, False, False]
    hx.fault_configure("")
    assert hx.fault_calls("alloc") == 0
    dev.buffer(8).close()


def chain_module():
    r = hx.Rng(31)
    a, w1, w2 = r.uniform((40, 24)), r.uniform((24, 16)), r.uniform((16, 16))
    p = hx.Program()
    h = p.relu(p.linear(p.constant(a), p.constant(w1)))
    p.add(p.linear(h, p.constant(w2)), h)
    want = oracle.add(oracle.matmul(oracle.relu(oracle.matmul(a, w1)), w2),
                      oracle.relu(oracle.matmul(a, w1)))
    return hx.Module(p.emit()), want


def test_every_allocation_of_an_execute_fails_cleanly():
    """Fail each allocation one execute makes, one at a time: the execute
    reports out of memory, and the module and device then run correctly."""
    module, want = chain_module()
    dev = hx.Device("cpu")
    hx.fault_configure("alloc:1000000000")
    out = hx.execute(module, dev, out_shape=want.shape)
    count = hx.fault_calls("alloc")
    assert count >= 3  # the destinations of linear, relu, linear, add
    assert np.array_equal(out, want)
    for n in range(1, count + 1):
        hx.fault_configure(f"alloc:{n}")
        with pytest.raises(_ffi.HexirError) as err:
            hx.execute(module, dev, out_shape=want.shape)
        assert err.value.status == _ffi.ERROR_OUT_OF_MEMORY, n
        hx.fault_configure("")
        again = hx.execute(module, dev, out_shape=want.shape)
        assert np.array_equal(again.view(np.uint64), want.view(np.uint64)), n


def test_launch_rules_do_not_touch_the_cpu_path():
    module, want = chain_module()
    hx.fault_configure("launch:1+,nccl:1+")
    out = hx.execute(module, hx.Device("cpu"), out_shape=want.shape)
    assert np.array_equal(out, want)
    assert hx.fault_calls("launch") == 0 and hx.fault_calls("nccl") == 0


def test_environment_rules_reach_hexir_run(tmp_path):
    module_path = tmp_path / "m.hxb"
    p = hx.Program()
    p.print(p.relu(p.linear(p.constant(np.array([[3.0, -1.0], [2.0, 2.0]])),
                            p.constant(np.array([[1.0, 5.0], [5.0, -2.0]])))))
    p.emit_file(str(module_path))
    run = bin_path("hexir-run")
    env = dict(os.environ, HEXIR_FAULT="alloc:1")
    res = subprocess.run([run, "--quiet", str(module_path)], env=env,
                         capture_output=True, text=True)
    assert res.returncode != 0 and "out of memory" in res.stderr
    env["HEXIR_FAULT"] = "alloc:1000"
    res = subprocess.run([run, "--quiet", str(module_path)], env=env,
                         capture_output=True, text=True, check=True)
    assert res.stdout == "0.000000 17.000000 \n12.000000 6.000000 \n"
    env["HEXIR_FAULT"] = "alloc:zero"
    res = subprocess.run([run, "--quiet", str(module_path)], env=env,
                         capture_output=True, text=True, check=True)
    assert "ignoring malformed HEXIR_FAULT" in res.stderr
    assert res.stdout == "0.000000 17.000000 \n12.000000 6.000000 \n"


def test_trace_prints_one_line_per_dispatch(tmp_path):
    """HEXIR_TRACE=1: one stderr line per DISPATCH with its name, kind,
    extents and device; results unchanged; off by default."""
    module_path = tmp_path / "t.hxb"
    p = hx.Program()
    x = p.constant(np.array([[3.0, -1.0], [2.0, 2.0]]))
    w = p.constant(np.array([[1.0, 5.0], [5.0, -2.0]]))
    p.print(p.add(p.relu(p.linear(x, w)), x))
    p.emit_file(str(module_path))
    run = bin_path("hexir-run")
    res = subprocess.run([run, "--quiet", str(module_path)],
                         env=dict(os.environ, HEXIR_TRACE="1"),
                         capture_output=True, text=True, check=True)
    lines = [ln for ln in res.stderr.splitlines() if ln.startswith("hexir: dispatch")]
    assert lines == ["hexir: dispatch linear_0 matmul 2x2x2 on cpu",
                     "hexir: dispatch relu_1 relu 2x2x0 on cpu",
                     "hexir: dispatch add_2 add 2x2x0 on cpu"]
    assert res.stdout == "3.000000 16.000000 \n14.000000 8.000000 \n"
    quiet = subprocess.run([run, "--quiet", str(module_path)],
                           env=dict(os.environ, HEXIR_TRACE="0"),
                           capture_output=True, text=True, check=True)
    assert "dispatch" not in quiet.stderr
