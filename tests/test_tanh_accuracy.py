"""The accuracy of the GPU tanh's arithmetic, and of the exp / expm1 core it
shares with elu and mish, on the host.

tests/tanh_accuracy.c restates the kernel's evaluation (Cody-Waite
reduction, Taylor polynomial of expm1, one Newton-Raphson step on a
reciprocal estimate and a Markstein quotient correction) with C's fma()
for the GPU's fused multiply-add, and compares it with the C library's
64-bit-mantissa tanhl on 10^6 inputs: normal, uniform to +-25, near zero,
tiny down to subnormals, and around the first reduction boundary.  The GPU
test (test_gpu_activations.py::test_tanh_is_within_4_ulp) checks the kernel
itself against the oracle.
"""

import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.fixture(scope="module")
def program(tmp_path_factory):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    exe = str(tmp_path_factory.mktemp("tanh") / "tanh_accuracy")
    subprocess.run([cc, "-O2", "-std=c11", "-ffp-contract=off", "-o", exe,
                    os.path.join(HERE, "tanh_accuracy.c"), "-lm"], check=True)
    return exe


@pytest.mark.parametrize("seed_bits", [20, 23, 52])
def test_tanh_arithmetic_is_within_3_ulp(program, seed_bits):
    """Within 2.6 ulp of tanhl and 3 ulp of the double tanh, with the special
    values (signed zeros, saturation, infinities, NaN) as tanh has them, for
    any reciprocal estimate of 20 bits or more."""
    out = subprocess.run([program, str(seed_bits), "200000"], check=True,
                         capture_output=True, text=True).stdout.split()
    worst, worst_libm, bad = float(out[0]), float(out[1]), int(out[2])
    assert worst <= 2.6, worst
    assert worst_libm <= 3.0, worst_libm
    assert bad == 0


def test_exp_core_is_within_1_2_ulp(program):
    """exp_neg (mish's e^-|x|, scaled in two halves of k so that subnormal
    results round once) within 1 ulp of expl over [-750, 0], underflow and
    the subnormal range included; expm1_neg (elu below zero, clamped at -40)
    within 1.2 ulp of expm1l."""
    out = subprocess.run([program, "exp", "200000"], check=True,
                         capture_output=True, text=True).stdout.split()
    worst_exp, worst_expm1 = float(out[0]), float(out[1])
    assert worst_exp <= 1.0, worst_exp
    assert worst_expm1 <= 1.2, worst_expm1


def test_gelu_arithmetic_is_within_4_ulp(program):
    """The table-driven gelu (a degree-9 polynomial per interval for
    erfc(u) e^{u^2} / 2, times e^{-u^2} from the exp core) within 4 ulp of
    the formula as written evaluated in long double, 5 ulp of its double
    evaluation with the C library's erfc (the oracle's), and with the
    oracle's special values (signed zeros, saturation, infinities, NaN)."""
    out = subprocess.run([program, "gelu", "200000"], check=True,
                         capture_output=True, text=True).stdout.split()
    worst, worst_libm, bad = float(out[0]), float(out[1]), int(out[2])
    assert worst <= 4.0, worst
    assert worst_libm <= 5.0, worst_libm
    assert bad == 0


def test_gelu_table_is_its_generators_output(tmp_path):
    """gelu_table.inc is exactly what gelu_table_gen.c writes."""
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    kernels = os.path.join(HERE, "..", "hexir_b200", "csrc", "kernels")
    exe = str(tmp_path / "gelu_table_gen")
    subprocess.run([cc, "-O2", "-o", exe,
                    os.path.join(kernels, "gelu_table_gen.c"), "-lm"], check=True)
    out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    with open(os.path.join(kernels, "gelu_table.inc")) as f:
        assert f.read() == out
