"""The activation kernels (kernel kinds 7-14) on a B200 against the oracle.

No reference kernel exists for these ops (HexirOps.td:189-308 declares them
without a lowering), so parity is with the oracle's restatement of the op
descriptions, which the host backend reproduces bit for bit.  The GPU calls
CUDA's exp / expm1 / log1p / tanh / erfc where the oracle calls the C
library's, so results agree to a few units in the last place, not bit for
bit.  Tolerances, per element (oracle.ulp_error_ok):

  leaky_relu            bit-exact (a compare and one multiply)
  elu, sigmoid, tanh,   16 ulp of the oracle's value (2^-1000 absolute floor
  swish, mish           for results that underflow)
  gelu                  8 ulp (its table-driven erfc is within 5 of the
                        oracle's C-library form on the host)
  softmax               (cols + 16) ulp: the row sum is taken in a different
                        order (a tree over the row instead of left to right)

NaN where the oracle has NaN, the same infinity where it has one.
"""

import numpy as np
import pytest

import hexir_b200 as hx
from hexir_b200 import _ffi
from oracle import oracle

pytestmark = pytest.mark.gpu

ULPS = {"leaky_relu": 0, "elu": 16, "sigmoid": 16, "tanh": 16, "gelu": 8,
        "swish": 16, "mish": 16}
ELEMENTWISE = sorted(ULPS)


def specials_input(rows, cols, seed=0, scale=4.0):
    x = np.random.default_rng(seed).normal(0, scale, (rows, cols))
    specials = [0.0, -0.0, np.inf, -np.inf, np.nan, 1e300, -1e300, 709.8,
                -709.8, 745.2, -745.2, 5e-324, -5e-324, 40.0, -40.0, 1e-8,
                -1e-8, 20.0, -20.0]
    flat = x.reshape(-1)
    flat[:min(len(specials), flat.size)] = specials[:flat.size]
    return x


def run_gpu(gpu, op, x, shift=0):
    """op(x) through hexir_cuda_activation_f64; `shift` bytes moves both
    pointers off their 16-byte alignment."""
    rows, cols = x.shape
    n = x.size
    bx = gpu.buffer(n * 8 + 16)
    by = gpu.buffer(n * 8 + 16)
    raw = np.zeros(n + 2)
    raw[shift // 8:shift // 8 + n] = x.reshape(-1)
    bx.write(raw)
    hx.cuda_activation(0, op, bx.ptr + shift, by.ptr + shift, rows, cols,
                       gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    out = by.read(n + 2)
    return out[shift // 8:shift // 8 + n].reshape(rows, cols)


def assert_close(op, got, want):
    ulps = ULPS.get(op, want.shape[1] + 16)
    if ulps == 0:
        assert np.array_equal(got.view(np.uint64), want.view(np.uint64)), op
        return
    ok = oracle.ulp_error_ok(got, want, ulps)
    if not ok.all():
        bad = np.argwhere(~ok)[0]
        raise AssertionError(f"{op}: {bad} got {got[tuple(bad)]!r} "
                             f"want {want[tuple(bad)]!r}")


@pytest.mark.parametrize("op", ELEMENTWISE)
@pytest.mark.parametrize("rows,cols,shift", [
    (1, 1, 0), (1, 3, 8), (37, 53, 0), (37, 53, 8), (1000, 1025, 0),
    (3, (1 << 20) + 7, 0)])
def test_elementwise_activation_matches_oracle(gpu, op, rows, cols, shift):
    x = specials_input(rows, cols, seed=rows + cols)
    assert_close(op, run_gpu(gpu, op, x, shift), oracle.activation(op, x))


@pytest.mark.parametrize("op", ELEMENTWISE)
def test_elementwise_activation_over_the_whole_range(gpu, op):
    """Every binade from 2^-1074 to 2^1023, both signs, a few mantissas
    each."""
    rng = np.random.default_rng(3)
    exps = np.repeat(np.arange(-1074, 1024), 8)
    mant = rng.uniform(1, 2, exps.size)
    x = np.ldexp(mant, exps)
    x = np.concatenate([x, -x]).reshape(2 * 2098, 8)
    assert_close(op, run_gpu(gpu, op, x), oracle.activation(op, x))


@pytest.mark.parametrize("rows,cols", [
    (1, 1), (5, 2), (300, 31), (300, 33), (64, 1000), (64, 1024), (64, 1025),
    (64, 1026), (1000, 2048), (1200, 1026), (700, 2050), (450, 3000),
    (700, 4096), (40, 4097), (17, 8192), (700, 8192), (9, 8193),
    (9, 16384), (300, 12000), (5, 16385), (3, 40000),
    (400, 8194), (400, 12000), (200, 16386), (200, 20000),
    # clusters of 4-8 CTAs per row (28674-65536 even columns), with more
    # rows than resident clusters so every cluster walks several rows
    (300, 24578), (300, 28674), (160, 32768), (100, 32770), (100, 40000), (60, 49152),
    (50, 57000), (40, 65536)])
def test_softmax_matches_oracle(gpu, rows, cols):
    """Every launch shape at and around its column limit: warp per row; the
    persistent bulk-prefetch blocks for even rows, short-row (<= 2048, <=
    4096 columns) and long (more rows than blocks, so each block walks
    several); rows of 28674-65536 even columns split over thread-block
    clusters of 4-8 CTAs; the 256- and 512-thread blocks for odd rows; the
    three-pass block for the rest."""
    x = np.random.default_rng(rows * cols).normal(0, 3, (rows, cols))
    got = run_gpu(gpu, "softmax", x)
    want = oracle.activation("softmax", x)
    assert_close("softmax", got, want)
    assert np.all(np.abs(got.sum(axis=1) - 1) <= (cols + 16) * 2.0 ** -52)


@pytest.mark.parametrize("cols", [7, 1024, 5000, 16384, 20000, 40000, 65536])
def test_softmax_special_rows(gpu, cols):
    """A NaN or +inf anywhere in a row, or a row of -inf, makes that row NaN
    (x - max is NaN), like the oracle; -inf elsewhere gives exact zeros; a
    huge spread underflows to zero without NaN; other rows are unaffected."""
    x = np.random.default_rng(cols).normal(0, 3, (6, cols))
    x[1, cols // 2] = np.nan
    x[2, cols - 1] = np.inf
    x[3, :] = -np.inf
    x[4, ::2] = -np.inf
    x[5, 0] = 1e300
    got = run_gpu(gpu, "softmax", x)
    want = oracle.activation("softmax", x)
    assert_close("softmax", got, want)
    assert np.all(np.isnan(got[1:4]))
    assert np.all(got[4, ::2] == 0.0) and got[5, 0] == 1.0


@pytest.mark.parametrize("op", sorted(_ffi.ACTIVATIONS))
def test_activation_in_place_and_deterministic(gpu, op):
    rows, cols = (64, 3000) if op == "softmax" else (64, 3001)
    x = specials_input(rows, cols, seed=9)
    once = run_gpu(gpu, op, x)
    assert np.array_equal(once.view(np.uint64), run_gpu(gpu, op, x).view(np.uint64))
    buf = gpu.upload(x)
    hx.cuda_activation(0, op, buf.ptr, buf.ptr, rows, cols, gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    inplace = buf.read((rows, cols))
    assert np.array_equal(inplace.view(np.uint64), once.view(np.uint64))


def test_activation_argument_errors(gpu):
    buf = gpu.buffer(64)
    with pytest.raises(_ffi.HexirError) as err:
        hx.cuda_activation(0, 3, buf.ptr, buf.ptr, 2, 4, gpu.stream)
    assert err.value.status == _ffi.ERROR_INVALID_ARGUMENT
    with pytest.raises(_ffi.HexirError) as err:
        hx.cuda_activation(0, "gelu", 0, buf.ptr, 2, 4, gpu.stream)
    assert err.value.status == _ffi.ERROR_INVALID_ARGUMENT
    with pytest.raises(_ffi.HexirError) as err:
        hx.cuda_activation(0, "gelu", buf.ptr, buf.ptr, 1 << 40, 1 << 30,
                           gpu.stream)
    assert err.value.status == _ffi.ERROR_INVALID_ARGUMENT
    # Empty tensors launch nothing.
    before = hx.launch_count()
    hx.cuda_activation(0, "softmax", 0, 0, 0, 5, gpu.stream)
    hx.cuda_activation(0, "mish", 0, 0, 7, 0, gpu.stream)
    assert hx.launch_count() == before


@pytest.mark.parametrize("op", ["gelu", "softmax", "mish"])
def test_activation_after_linear_in_a_module(gpu, op):
    """linear -> op written with EMIT_ACTIVATIONS: all-cuda against the
    host backend's all-cpu run of the same program."""
    r = hx.Rng(7)
    a, w = r.uniform((300, 200)), r.uniform((200, 260))
    p = hx.Program()
    p.activation(op, p.linear(p.constant(a), p.constant(w)))
    flags = _ffi.EMIT_ACTIVATIONS
    cpu = hx.execute(hx.Module(p.emit("", flags)), hx.Device("cpu"),
                     out_shape=(300, 260))
    cuda = hx.execute(hx.Module(p.emit(f"hexir.linear=cuda,hexir.{op}=cuda",
                                       flags)), gpu, out_shape=(300, 260))
    # The linear differs from the reference order by f64 rounding
    # (<= 1e-12 normwise); the activation carries that through.
    assert oracle.normwise_error(cuda, cpu) <= 1e-12
    # Activation alone, on the GPU's own linear output, meets the kernel bar.
    p2 = hx.Program()
    p2.linear(p2.constant(a), p2.constant(w))
    lin = hx.execute(hx.Module(p2.emit("hexir.linear=cuda")), gpu,
                     out_shape=(300, 260))
    assert_close(op, cuda, oracle.activation(op, lin))


def test_activation_full_size_rows_sampled(gpu):
    """softmax and gelu over a 16384 x 16384 tensor (2 GiB): sampled rows
    against the oracle, every row summing to one."""
    rows = cols = 16384
    x = np.random.default_rng(4).normal(0, 1, (rows, cols))
    bx = gpu.upload(x)
    by = gpu.buffer(x.nbytes)
    for op in ("softmax", "gelu"):
        hx.cuda_activation(0, op, bx.ptr, by.ptr, rows, cols, gpu.stream)
        hx.cuda_synchronize(0, gpu.stream)
        got = by.read((rows, cols))
        pick = [0, 1, 4095, 8191, 12345, rows - 1]
        assert_close(op, got[pick], oracle.activation(op, x[pick]))
        if op == "softmax":
            assert np.all(np.abs(got.sum(axis=1) - 1) <= (cols + 16) * 2.0 ** -52)


def test_sharded_activation_across_gpus(gpu):
    """A row-sharded softmax on cuda:0-1 equals the single-GPU result bit for
    bit (rows are independent; each GPU runs the same kernel on its rows)."""
    if hx.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    x = np.random.default_rng(5).normal(0, 2, (1000, 700))
    p = hx.Program()
    p.activation("softmax", p.constant(x))
    flags = _ffi.EMIT_ACTIVATIONS
    one = hx.execute(hx.Module(p.emit("hexir.softmax=cuda", flags)), gpu,
                     out_shape=x.shape)
    devs = [hx.Device("cuda:0"), hx.Device("cuda:1")]
    try:
        two = hx.execute(hx.Module(p.emit("hexir.softmax=cuda:0-1", flags)),
                         devs, out_shape=x.shape)
    finally:
        for d in devs:
            d.close()
    assert np.array_equal(one.view(np.uint64), two.view(np.uint64))
    assert_close("softmax", one, oracle.activation("softmax", x))


@pytest.mark.parametrize("rows,cols", [(40, 2048), (9, 16384)])
def test_softmax_misaligned_rows_take_the_register_blocks(gpu, rows, cols):
    """x 8 bytes off its 16-byte alignment: the bulk copy cannot start there,
    so the per-row register blocks run; same results within the bar."""
    x = np.random.default_rng(cols).normal(0, 3, (rows, cols))
    aligned = run_gpu(gpu, "softmax", x)
    shifted = run_gpu(gpu, "softmax", x, shift=8)
    want = oracle.activation("softmax", x)
    assert_close("softmax", aligned, want)
    assert_close("softmax", shifted, want)


def test_tanh_is_within_4_ulp(gpu):
    """tanh is evaluated as -u / (2 + u) with u = expm1(-2|x|) computed in
    the kernel (Cody-Waite reduction, Taylor polynomial, Newton-Raphson
    quotient), |x| capped at 20: within 4 ulp of the oracle's C-library tanh
    over a dense grid through the cap, tiny magnitudes (where the relative
    accuracy of expm1 is what keeps it), and the sign of zero."""
    grid = np.linspace(-25.0, 25.0, 1 << 18)
    tiny = np.geomspace(1e-300, 1e-2, 4096)
    x = np.concatenate([grid, tiny, -tiny, [0.0, -0.0, 20.0, -20.0,
                                            np.nextafter(20.0, 21.0)]])
    x = x.reshape(1, -1)
    got = run_gpu(gpu, "tanh", x)
    want = oracle.activation("tanh", x)
    assert oracle.ulp_error_ok(got, want, 4, floor=0.0).all()
    assert np.signbit(got[0, -4]) and not np.signbit(got[0, -5])
    assert got[0, -1] == 1.0
