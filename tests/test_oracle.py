"""The oracle is pinned before it is trusted.

oracle/hexir_oracle.c restates runtime/src/kernels/reference_kernels.c.  It is
checked here against
  - tests/golden/golden.json: outputs of the reference's own hexir_ref_*_f64
    kernels (built from the reference sources) on seeded inputs, as sha256 of
    the output bytes, and the relu of IEEE special values;
  - the reference library itself (oracle/_ref/libhexir_ref.so) when it is
    present, on further random and special inputs.
"""

import hashlib
import json
import os

import numpy as np
import pytest

import hexir_b200 as hx
from oracle import oracle

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden",
                                     "golden.json")))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.mark.parametrize("vec", GOLDEN["matmul_vectors"],
                         ids=lambda v: f"{v['m']}x{v['n']}x{v['k']}")
def test_oracle_matches_reference_vectors(vec):
    rng = hx.Rng(vec["seed"])
    a = rng.uniform((vec["m"], vec["k"]))
    b = rng.uniform((vec["k"], vec["n"]))
    c = oracle.matmul(a, b)
    assert sha(c) == vec["matmul_sha256"]
    assert sha(oracle.relu(c)) == vec["relu_sha256"]
    assert sha(oracle.add(c, c[::-1].copy())) == vec["add_reversed_rows_sha256"]
    for i, j, v in vec["samples"]:
        assert c[i, j] == v


def test_oracle_relu_specials_match_reference():
    spec = GOLDEN["relu_specials"]
    x = np.array([float.fromhex(h) if h not in ("inf", "-inf", "nan")
                  else float(h) for h in spec["input_hex"]])
    got = oracle.relu(x).view(np.uint64)
    assert [int(v) for v in got] == spec["output_bits"]
    # NaN and -0.0 both become +0.0 (bit pattern 0).
    assert got[1] == 0 and got[6] == 0


@pytest.mark.parametrize("threads", [1, 2, 3, 8])
def test_oracle_threads_do_not_change_bits(threads):
    rng = np.random.default_rng(3)
    a = rng.standard_normal((61, 77))
    b = rng.standard_normal((77, 45))
    one = oracle.matmul(a, b, threads=1)
    assert np.array_equal(oracle.matmul(a, b, threads=threads).view(np.uint64),
                          one.view(np.uint64))


def test_oracle_rows_slice_matches_full():
    rng = np.random.default_rng(4)
    a = rng.uniform(-1, 1, (40, 33))
    b = rng.uniform(-1, 1, (33, 21))
    full = oracle.matmul(a, b)
    assert np.array_equal(oracle.matmul_rows(a, b, 7, 19), full[7:19])


needs_ref = pytest.mark.skipif(not oracle.have_reference(),
                               reason="reference library not built here")


@needs_ref
@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (3, 4, 5), (33, 17, 65),
                                   (128, 96, 200)])
def test_oracle_bit_identical_to_reference_library(m, n, k):
    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal((m, k)) * 10
    b = rng.standard_normal((k, n))
    if m * k > 4:
        a.flat[:4] = [np.inf, -0.0, 1e-310, np.nan]
    want = oracle.ref_matmul(a, b)
    got = oracle.matmul(a, b)
    assert np.array_equal(got.view(np.uint64), want.view(np.uint64))


@needs_ref
def test_oracle_elementwise_bit_identical_to_reference_library():
    rng = np.random.default_rng(9)
    x = rng.standard_normal(10007)
    x[:8] = [0.0, -0.0, np.nan, -np.nan, np.inf, -np.inf, 5e-324, -5e-324]
    y = rng.standard_normal(10007)
    assert np.array_equal(oracle.relu(x).view(np.uint64),
                          oracle.ref_relu(x).view(np.uint64))
    assert np.array_equal(oracle.add(x, y).view(np.uint64),
                          oracle.ref_add(x, y).view(np.uint64))


def test_normwise_error_definition():
    want = np.array([[1.0, -4.0], [2.0, 0.0]])
    got = want + np.array([[0.0, 4e-12], [0.0, 0.0]])
    assert oracle.normwise_error(got, want) == pytest.approx(1e-12)
    assert oracle.normwise_error(np.zeros(3), np.zeros(3)) == 0.0


# ---- activations: the oracle against the op descriptions ------------------
#
# No reference kernel, test or golden value exists for the activations
# (HexirOps.td:189-308 declares them without a lowering), so the oracle is
# checked against the descriptions themselves, evaluated independently with
# numpy / scipy where the literal formula is well conditioned.

def _activation_inputs():
    rng = np.random.default_rng(11)
    x = np.concatenate([np.linspace(-8, 8, 401), rng.normal(0, 3, 599)])
    return x.reshape(10, 100)


def test_oracle_activations_follow_the_op_descriptions():
    import scipy.special as sp
    x = _activation_inputs()
    lit = {
        "leaky_relu": np.maximum(x, 0.01 * x),
        "elu": np.where(x > 0, x, 1.0 * (np.exp(x) - 1)),
        "sigmoid": 1 / (1 + np.exp(-x)),
        "tanh": np.tanh(x),
        "softmax": sp.softmax(x, axis=1),
        "gelu": x * 0.5 * (1 + sp.erf(x / np.sqrt(2))),
        "swish": x * sp.expit(x),
        "mish": x * np.tanh(np.log1p(np.exp(x))),
    }
    for op, want in lit.items():
        got = oracle.activation(op, x)
        if op == "leaky_relu":
            assert np.array_equal(got, want)
            continue
        # The literal forms lose relative accuracy where they cancel
        # (exp(x) - 1 near 0, 1 + erf for x < 0): compare those against the
        # result's scale instead.
        scale = np.maximum(np.abs(want), 1.0 if op in ("elu", "gelu") else 0)
        err = np.abs(got - want) / np.where(scale > 0, scale, 1)
        assert err.max() < 1e-13, op


def test_oracle_activation_stable_forms_keep_relative_accuracy():
    """Where the literal forms cancel, the oracle's rewritten forms stay
    accurate: gelu's left tail against x/2 erfc(-x/sqrt 2) evaluated with
    scipy's erfc, and mish at large |x|."""
    import scipy.special as sp
    x = np.linspace(-30, -5, 251).reshape(1, -1)
    # The same rounded argument: erfc's condition number 2 z^2 would turn a
    # last-place difference in z into ~1e-13 at x = -30.
    want = 0.5 * x * sp.erfc(-x * 0.70710678118654752440)
    got = oracle.activation("gelu", x)
    assert np.all(np.abs(got - want) <= 1e-13 * np.abs(want))
    assert oracle.activation("mish", np.array([[800.0]]))[0, 0] == 800.0
    assert oracle.activation("sigmoid", np.array([[-800.0, 800.0]])).tolist() == [[0.0, 1.0]]


def test_oracle_softmax_rows_sum_to_one_and_specials():
    x = _activation_inputs()
    y = oracle.activation("softmax", x)
    assert np.all(np.abs(y.sum(axis=1) - 1) < 1e-14)
    # A NaN, +inf, or an all -inf row turns that row to NaN; other rows keep
    # their values.
    z = x.copy()
    z[1, 5] = np.nan
    z[2, 7] = np.inf
    z[3, :] = -np.inf
    w = oracle.activation("softmax", z)
    assert np.all(np.isnan(w[1:4]))
    assert np.array_equal(w[0], y[0]) and np.array_equal(w[4:], y[4:])


def test_oracle_activations_within_a_few_ulp_of_exact():
    """Against 200-bit values from mpmath of the op descriptions themselves:
    every elementwise activation of the oracle is within 4 ulp, except gelu,
    and softmax within (cols + 4) ulp (its row sum is a left-to-right f64
    sum).  gelu evaluates erfc at the rounded argument z = fl(-x * (1/sqrt 2)),
    whose error of up to 2 ulp erfc's condition number 2 z^2 multiplies: the
    bound there is 4 + 4 z^2 ulp (about 3e-13 relative at the underflow edge,
    x = -37), as in the GPU kernel, which rounds the same argument.  Results
    below 2^-1000 are compared absolutely."""
    mpmath = pytest.importorskip("mpmath")
    mpmath.mp.prec = 200
    rng = np.random.default_rng(17)
    x = np.concatenate([rng.normal(0, 4, 300), rng.uniform(-40, 40, 200),
                        np.ldexp(rng.uniform(1, 2, 100),
                                 rng.integers(-60, 9, 100)) *
                        rng.choice([-1, 1], 100)]).reshape(6, 100)
    mp = mpmath.mpf
    exact = {
        "leaky_relu": lambda v: v if v > 0 else mp("0.01") * v,
        "elu": lambda v: v if v > 0 else mpmath.expm1(v),
        "sigmoid": lambda v: 1 / (1 + mpmath.exp(-v)),
        "tanh": mpmath.tanh,
        # 1 + erf(z) = erfc(-z) exactly; mpmath's erfc keeps the left tail
        # that 1 + erf would cancel even at 200 bits.
        "gelu": lambda v: v / 2 * mpmath.erfc(-v / mpmath.sqrt(2)),
        "swish": lambda v: v / (1 + mpmath.exp(-v)),
        "mish": lambda v: v * mpmath.tanh(mpmath.log1p(mpmath.exp(v))),
    }
    for op, f in exact.items():
        got = oracle.activation(op, x)
        want = np.array([[float(f(mp(float(v)))) for v in row] for row in x])
        tiny = np.abs(want) < 2.0 ** -1000
        ulp = np.abs(got - want) / np.spacing(np.abs(want))
        bound = 4 + 4 * (x / np.sqrt(2)) ** 2 if op == "gelu" else 4
        assert np.all(np.where(tiny, np.abs(got - want) <= 2.0 ** -1000,
                               ulp <= bound)), (op, ulp[~tiny].max())
    got = oracle.activation("softmax", x)
    for r, row in enumerate(x):
        es = [mpmath.exp(mp(float(v))) for v in row]
        total = mpmath.fsum(es)
        want = np.array([float(e / total) for e in es])
        ulp = np.abs(got[r] - want) / np.spacing(np.abs(want))
        assert ulp.max() <= x.shape[1] + 4, ulp.max()
