"""Random programs through the writer and the VM on the CPU device, against
the same graph evaluated by the oracle.

Each seed builds a small graph of linear / add / relu / activation ops over
random shapes, reusing earlier values (so slots are read several times and
live across dispatches), writes it, runs it with hexir_execute_capture and
compares the captured result (the last dispatch's) bit for bit with the
oracle.  The host backend keeps the reference's arithmetic, so nothing but
exact equality passes.
"""

import random

import numpy as np
import pytest

import hexir_b200 as hx
from hexir_b200 import _ffi
from oracle import oracle

OPS = ["linear", "add", "relu", "activation"]


def ty(shape):
    return f"tensor<{shape[0]}x{shape[1]}xf64>"


def build(seed, text=None, ops=OPS):
    """(program, expected result, its program value); with `text` a list,
    the same graph is also rendered there as hexir text, one statement per
    entry."""
    rnd = random.Random(seed)
    rng = np.random.default_rng(seed)
    p = hx.Program()
    values = []  # (program value, numpy value)
    names = {}
    lines = text if text is not None else []

    def emit_line(value, line):
        names[value] = f"%v{value}"
        lines.append(f"%v{value} = {line}")

    def constant(r, c):
        a = rng.uniform(-2, 2, (r, c))
        values.append((p.constant(a), a))
        rows = ", ".join("[" + ", ".join(repr(float(e)) for e in row) + "]"
                         for row in a)
        emit_line(values[-1][0], f"hexir.constant dense<[{rows}]> : {ty(a.shape)}")
        return values[-1]

    for _ in range(rnd.randint(1, 3)):
        constant(rnd.randint(1, 9), rnd.randint(1, 9))
    last = None
    for _ in range(rnd.randint(1, 8)):
        op = rnd.choice(ops)
        v, x = rnd.choice(values)
        if op == "linear":
            k = x.shape[1]
            ws = [(wv, w) for wv, w in values if w.shape[0] == k]
            wv, w = rnd.choice(ws) if ws and rnd.random() < 0.5 else \
                constant(k, rnd.randint(1, 9))
            out = (p.linear(v, wv), oracle.matmul(x, w))
            emit_line(out[0], f"hexir.linear {names[v]}, {names[wv]} : "
                              f"({ty(x.shape)}, {ty(w.shape)}) -> {ty(out[1].shape)}")
        elif op == "add":
            same = [(ov, o) for ov, o in values if o.shape == x.shape]
            ov, o = rnd.choice(same)
            out = (p.add(v, ov), oracle.add(x, o))
            emit_line(out[0], f"hexir.add {names[v]}, {names[ov]} : {ty(x.shape)}")
        elif op == "relu":
            out = (p.relu(v), oracle.relu(x))
            emit_line(out[0], f"hexir.relu {names[v]} : {ty(x.shape)}")
        else:
            name = rnd.choice(sorted(_ffi.ACTIVATIONS))
            out = (p.activation(name, v), oracle.activation(name, x))
            emit_line(out[0], f"hexir.{name} {names[v]} : {ty(x.shape)}")
        values.append(out)
        last = out
    if last is None:  # every graph ends in at least one dispatch
        v, x = values[0]
        last = (p.relu(v), oracle.relu(x))
        emit_line(last[0], f"hexir.relu {names[v]} : {ty(x.shape)}")
    return p, last[1], last[0]


@pytest.mark.parametrize("seed", range(120))
def test_random_program_matches_oracle(seed):
    p, want, _ = build(seed)
    out = hx.execute(hx.Module(p.emit(flags=_ffi.EMIT_ACTIVATIONS)),
                     hx.Device("cpu"), out_shape=want.shape)
    assert np.array_equal(out.view(np.uint64), want.view(np.uint64))


@pytest.mark.parametrize("seed", range(0, 120, 3))
def test_random_program_text_writes_the_same_module(seed):
    """The same graph written as hexir text and parsed gives a module
    byte-identical to the one built through the API (placements and the
    fusion rules included)."""
    lines = []
    p, _, _ = build(seed, lines)
    text = "func.func @main() {\n  " + "\n  ".join(lines) + "\n  return\n}\n"
    q = hx.parse(text)
    for placement in ("", "hexir.linear=cuda,hexir.relu=cuda,hexir.add=cuda"):
        flags = _ffi.EMIT_ACTIVATIONS | _ffi.EMIT_NO_IMAGE
        assert q.emit(placement, flags) == p.emit(placement, flags)


@pytest.mark.parametrize("seed", range(40))
def test_reference_runtime_prints_random_programs_like_this_one(tmp_path, seed):
    """Graphs of the reference's own ops (linear, add, relu) with a PRINT:
    the reference runtime, built from its sources, and this runtime print
    the same text for the same module."""
    import subprocess
    from tests.conftest import bin_path
    if not oracle.have_reference():
        pytest.skip("reference runtime not built here")
    p, _, v = build(seed, ops=["linear", "add", "relu"])
    p.print(v)
    path = tmp_path / "r.hxb"
    p.emit_file(str(path))
    ref = subprocess.run([oracle.REF_RUN, "--quiet", str(path)],
                         capture_output=True, text=True, check=True)
    ours = subprocess.run([bin_path("hexir-run"), "--quiet", str(path)],
                          capture_output=True, text=True, check=True)
    assert ours.stdout == ref.stdout and ref.stdout
