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


def build(seed):
    rnd = random.Random(seed)
    rng = np.random.default_rng(seed)
    p = hx.Program()
    values = []  # (program value, numpy value)

    def constant(r, c):
        a = rng.uniform(-2, 2, (r, c))
        values.append((p.constant(a), a))
        return values[-1]

    for _ in range(rnd.randint(1, 3)):
        constant(rnd.randint(1, 9), rnd.randint(1, 9))
    last = None
    for _ in range(rnd.randint(1, 8)):
        op = rnd.choice(OPS)
        v, x = rnd.choice(values)
        if op == "linear":
            k = x.shape[1]
            ws = [(wv, w) for wv, w in values if w.shape[0] == k]
            wv, w = rnd.choice(ws) if ws and rnd.random() < 0.5 else \
                constant(k, rnd.randint(1, 9))
            out = (p.linear(v, wv), oracle.matmul(x, w))
        elif op == "add":
            same = [(ov, o) for ov, o in values if o.shape == x.shape]
            ov, o = rnd.choice(same)
            out = (p.add(v, ov), oracle.add(x, o))
        elif op == "relu":
            out = (p.relu(v), oracle.relu(x))
        else:
            name = rnd.choice(sorted(_ffi.ACTIVATIONS))
            out = (p.activation(name, v), oracle.activation(name, x))
        values.append(out)
        last = out
    if last is None:  # every graph ends in at least one dispatch
        v, x = values[0]
        last = (p.relu(v), oracle.relu(x))
    return p, last[1]


@pytest.mark.parametrize("seed", range(120))
def test_random_program_matches_oracle(seed):
    p, want = build(seed)
    out = hx.execute(hx.Module(p.emit(flags=_ffi.EMIT_ACTIVATIONS)),
                     hx.Device("cpu"), out_shape=want.shape)
    assert np.array_equal(out.view(np.uint64), want.view(np.uint64))
