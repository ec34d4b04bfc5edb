"""GPU parity of the kernel-level C ABI (include/hexir_b200/kernels.h) against
the CPU oracle (oracle/hexir_oracle.c, a restatement of
runtime/src/kernels/reference_kernels.c).

Bars:
  relu, add          bit-exact (compared as uint64 bit patterns)
  matmul             normwise  max|c - c_ref| / max|c_ref| <= 1e-12
  fused relu         bit-exact against relu of the unfused kernel's output
"""

import numpy as np
import pytest

import hexir_b200 as hx
from hexir_b200 import _ffi
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-12  # normwise relative error bar for f64 linear


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float64).view(np.uint64)


def run_matmul(dev, a, b, flags=0, offset_bytes=0):
    m, k = a.shape
    n = b.shape[1]
    pad = offset_bytes
    ba = dev.buffer(a.nbytes + pad + 8)
    bb = dev.buffer(b.nbytes + pad + 8)
    bc = dev.buffer(m * n * 8 + pad + 8)
    if pad:
        # Write through a host staging array so the data starts at +pad.
        for buf, arr in ((ba, a), (bb, b)):
            stage = np.zeros((arr.nbytes + pad + 8) // 8, dtype=np.float64)
            stage[pad // 8: pad // 8 + arr.size] = arr.ravel()
            buf.write(stage)
    else:
        ba.write(a)
        bb.write(b)
    hx.cuda_matmul(0, ba.ptr + pad, bb.ptr + pad, bc.ptr + pad, m, n, k, flags,
                   dev.stream)
    hx.cuda_synchronize(0, dev.stream)
    out = bc.read((m * n * 8 + pad + 8) // 8)
    return out[pad // 8: pad // 8 + m * n].reshape(m, n)


SHAPES = [
    (1, 1, 1), (2, 2, 2), (3, 5, 7), (37, 53, 29), (64, 64, 64),
    (128, 128, 128), (129, 257, 67), (130, 258, 64), (256, 256, 256),
    (300, 200, 1000), (16, 2048, 2048), (1, 1024, 4096), (513, 130, 96),
    (17, 130, 96), (40, 200, 3000), (5, 6, 8), (2, 4098, 512),
]


@pytest.mark.parametrize("m", [1, 7, 16, 17, 33, 64, 65])
@pytest.mark.parametrize("flags", [0, _ffi.MATMUL_SPLIT_K(3),
                                   _ffi.MATMUL_RELU | _ffi.MATMUL_SPLIT_K(1)])
def test_row_tile_variants(gpu, m, flags):
    """16-, 64- and 128-row TMA tiles chosen by m, each against the oracle."""
    n, k = 264, 1024
    rng = np.random.default_rng(1000 + m)
    a = rng.uniform(-1, 1, (m, k))
    b = rng.uniform(-1, 1, (k, n))
    variant, split = hx.matmul_plan(m, n, k, flags)
    assert variant == (3 if m <= 16 else 4 if m <= 64 else 1)
    want = oracle.matmul(a, b)
    if flags & _ffi.MATMUL_RELU:
        want = oracle.relu(want)
    assert oracle.normwise_error(run_matmul(gpu, a, b, flags), want) <= TOL


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_matmul_matches_oracle(gpu, m, n, k):
    rng = np.random.default_rng(m * 1000003 + n * 1009 + k)
    a = rng.uniform(-1, 1, (m, k))
    b = rng.uniform(-1, 1, (k, n))
    want = oracle.matmul(a, b)
    got = run_matmul(gpu, a, b)
    assert oracle.normwise_error(got, want) <= TOL


@pytest.mark.parametrize("variant", ["tma", "guarded"])
@pytest.mark.parametrize("split", [0, 1, 3])
def test_matmul_variants_and_split(gpu, variant, split):
    m, n, k = 200, 136, 520
    rng = np.random.default_rng(7 + split)
    a = rng.uniform(-1, 1, (m, k))
    b = rng.uniform(-1, 1, (k, n))
    flags = _ffi.MATMUL_FORCE_TMA if variant == "tma" else _ffi.MATMUL_FORCE_GUARDED
    flags |= _ffi.MATMUL_SPLIT_K(split)
    want = oracle.matmul(a, b)
    got = run_matmul(gpu, a, b, flags)
    assert oracle.normwise_error(got, want) <= TOL
    # The plan reports the kernel that the flags select.
    v, s = hx.matmul_plan(m, n, k, flags)
    assert v == (1 if variant == "tma" else 2)  # m = 200: 128-row tiles
    if split:
        assert s == split


def test_plan_picks_tma_for_aligned_even_shapes(gpu):
    assert hx.matmul_plan(8192, 8192, 8192)[0] == 1
    assert hx.matmul_plan(64, 64, 63)[0] == 2      # odd k: row stride not 16 B
    assert hx.matmul_plan(64, 63, 64)[0] == 2      # odd n
    assert hx.matmul_plan(16, 8192, 8192)[1] > 1   # too few tiles: split k
    assert hx.matmul_plan(16, 8192, 8192)[0] == 3  # 16-row tiles
    assert hx.matmul_plan(48, 8192, 8192)[0] == 4  # 64-row tiles


def test_misaligned_pointers_use_guarded_kernel(gpu):
    rng = np.random.default_rng(11)
    a = rng.uniform(-1, 1, (70, 48))
    b = rng.uniform(-1, 1, (48, 90))
    got = run_matmul(gpu, a, b, offset_bytes=8)
    assert oracle.normwise_error(got, oracle.matmul(a, b)) <= TOL


@pytest.mark.parametrize("variant", [_ffi.MATMUL_FORCE_TMA,
                                     _ffi.MATMUL_FORCE_GUARDED,
                                     _ffi.MATMUL_SPLIT_K(4)])
def test_fused_relu_is_relu_of_unfused(gpu, variant):
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, (190, 256))
    b = rng.uniform(-1, 1, (256, 144))
    plain = run_matmul(gpu, a, b, variant)
    fused = run_matmul(gpu, a, b, variant | _ffi.MATMUL_RELU)
    assert np.array_equal(bits(fused), bits(oracle.relu(plain)))
    assert oracle.normwise_error(fused, oracle.relu(oracle.matmul(a, b))) <= TOL


def test_matmul_k_zero_gives_zeros(gpu):
    m, n = 5, 6
    bc = gpu.buffer(m * n * 8)
    bc.write(np.full((m, n), 7.0))
    ba, bb = gpu.buffer(8), gpu.buffer(8)
    hx.cuda_matmul(0, ba.ptr, bb.ptr, bc.ptr, m, n, 0, 0, gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    assert np.array_equal(bc.read((m, n)), np.zeros((m, n)))


def test_matmul_exact_integers(gpu):
    # [[3,1],[2,2]] . [[1,5],[5,2]] = [[8,17],[12,14]]
    # (runtime/test/hxb-cuda.mlir:19-30, known answer).
    a = np.array([[3.0, 1.0], [2.0, 2.0]])
    b = np.array([[1.0, 5.0], [5.0, 2.0]])
    assert np.array_equal(run_matmul(gpu, a, b), [[8.0, 17.0], [12.0, 14.0]])


SPECIALS = np.array([0.0, -0.0, 1.0, -1.0, np.inf, -np.inf, np.nan, -np.nan,
                     5e-324, -5e-324, 2.2250738585072014e-308, 1e308, -1e308,
                     np.float64(np.frombuffer(b"\x01\x00\x00\x00\x00\x00\xf8\x7f",
                                              dtype=np.float64)[0])])


@pytest.mark.parametrize("n", [0, 1, 2, 3, 15, 1024, 1025, 100003])
@pytest.mark.parametrize("offset", [0, 8])
def test_relu_bit_exact(gpu, n, offset):
    rng = np.random.default_rng(n + offset)
    x = rng.standard_normal(n)
    if n >= SPECIALS.size:
        x[:SPECIALS.size] = SPECIALS
    bx = gpu.buffer(x.nbytes + 16)
    by = gpu.buffer(x.nbytes + 16)
    stage = np.zeros(n + 2)
    stage[offset // 8: offset // 8 + n] = x
    bx.write(stage)
    hx.cuda_relu(0, bx.ptr + offset, by.ptr + offset, n, gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    got = by.read(n + 2)[offset // 8: offset // 8 + n]
    assert np.array_equal(bits(got), bits(oracle.relu(x)))


@pytest.mark.parametrize("n", [1, 7, 4096, 99991])
def test_add_bit_exact(gpu, n):
    rng = np.random.default_rng(n)
    a = rng.standard_normal(n) * 1e3
    b = rng.standard_normal(n)
    if n >= 8:
        a[:6] = [np.inf, -np.inf, 1e308, -0.0, 5e-324, 0.0]
        b[:6] = [1.0, 2.0, 1e308, -0.0, 5e-324, -0.0]
    ba, bb, bc = gpu.upload(a), gpu.upload(b), gpu.buffer(a.nbytes)
    hx.cuda_add(0, ba.ptr, bb.ptr, bc.ptr, n, gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    assert np.array_equal(bits(bc.read(n)), bits(oracle.add(a, b)))


def test_add_nan_inputs_give_nan(gpu):
    # NaN payloads are not part of the contract (the GPU returns a canonical
    # NaN); NaN-ness is.
    a = np.array([np.nan, 1.0, np.inf, np.nan])
    b = np.array([1.0, np.nan, -np.inf, np.nan])
    ba, bb, bc = gpu.upload(a), gpu.upload(b), gpu.buffer(a.nbytes)
    hx.cuda_add(0, ba.ptr, bb.ptr, bc.ptr, 4, gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    assert np.isnan(bc.read(4)).all()


def test_large_gemm_sampled_rows(gpu):
    """4096^3 through the TMA pipeline; 24 spread rows checked against the
    oracle (cost is linear in rows), plus a size-independent identity:
    sum over rows of c equals (column sums of a) . b."""
    m = n = k = 4096
    r = hx.Rng(1)
    a = r.uniform((m, k))
    b = r.uniform((k, n))
    got = run_matmul(gpu, a, b)
    rows = np.linspace(0, m - 1, 24).astype(int)
    want = oracle.matmul(a[rows], b)
    assert oracle.normwise_error(got[rows], want) <= TOL
    colsum = oracle.matmul(a.sum(axis=0, keepdims=True), b)[0]
    assert oracle.normwise_error(got.sum(axis=0), colsum) <= 1e-10


def test_launch_counter_counts(gpu):
    before = hx.launch_count()
    run_matmul(gpu, np.ones((4, 4)), np.ones((4, 4)))
    assert hx.launch_count() > before


@pytest.mark.parametrize("m,n,k,cuts,force", [
    (1000, 384, 1024, [256, 512, 768], 0),
    (1000, 384, 1000, [256, 512, 768], 0),         # ragged last piece
    (40, 264, 2048, [1024], 0),                    # 64-row tile
    (9, 264, 512, [128, 384], 0),                  # 16-row tile
    (77, 131, 301, [64, 160], _ffi.MATMUL_FORCE_GUARDED),
])
def test_matmul_over_k_pieces_is_bit_identical(gpu, m, n, k, cuts, force):
    """hexir_cuda_matmul_acc_f64 over consecutive k ranges (a + k0 with
    lda = K, b + k0 * n, each piece continuing from c, relu on the last) gives
    the bits of one unsplit launch over all of k."""
    rng = np.random.default_rng(m + 7 * k)
    a = rng.uniform(-1, 1, (m, k))
    b = rng.uniform(-1, 1, (k, n))
    whole = run_matmul(gpu, a, b, _ffi.MATMUL_RELU | _ffi.MATMUL_SPLIT_K(1) |
                       force)
    ba, bb = gpu.upload(a), gpu.upload(b)
    bc = gpu.buffer(m * n * 8)
    bounds = [0] + cuts + [k]
    for i in range(len(bounds) - 1):
        k0, k1 = bounds[i], bounds[i + 1]
        last = i == len(bounds) - 2
        hx.cuda_matmul_acc(0, ba.ptr + 8 * k0, k, bb.ptr + 8 * k0 * n,
                           bc.ptr if i else 0, bc.ptr, m, n, k1 - k0,
                           (_ffi.MATMUL_RELU if last else 0) | force, gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    got = bc.read((m, n))
    assert np.array_equal(bits(got), bits(whole))
    assert oracle.normwise_error(got, oracle.relu(oracle.matmul(a, b))) <= TOL


def test_matmul_acc_separate_input_and_errors(gpu):
    """c_in distinct from c; an empty k copies (or relus) c_in; lda < k and a
    requested k split are refused."""
    rng = np.random.default_rng(5)
    m, n, k = 70, 96, 64
    a = rng.uniform(-1, 1, (m, k))
    b = rng.uniform(-1, 1, (k, n))
    c0 = rng.uniform(-1, 1, (m, n))
    ba, bb, bi = gpu.upload(a), gpu.upload(b), gpu.upload(c0)
    bc = gpu.buffer(m * n * 8)
    hx.cuda_matmul_acc(0, ba.ptr, k, bb.ptr, bi.ptr, bc.ptr, m, n, k, 0,
                       gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    want = oracle.add(c0, oracle.matmul(a, b))
    assert oracle.normwise_error(bc.read((m, n)), want) <= TOL
    assert np.array_equal(bits(bi.read((m, n))), bits(c0))  # input untouched
    hx.cuda_matmul_acc(0, ba.ptr, k, bb.ptr, bi.ptr, bc.ptr, m, n, 0,
                       _ffi.MATMUL_RELU, gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    assert np.array_equal(bits(bc.read((m, n))), bits(oracle.relu(c0)))
    lib = hx.lib()
    assert lib.hexir_cuda_matmul_acc_f64(0, ba.ptr, k - 2, bb.ptr, None, bc.ptr,
                                         m, n, k, 0, None) == \
        _ffi.ERROR_INVALID_ARGUMENT
    assert lib.hexir_cuda_matmul_acc_f64(0, ba.ptr, k, bb.ptr, bi.ptr, bc.ptr,
                                         m, n, k, _ffi.MATMUL_SPLIT_K(2),
                                         None) == _ffi.ERROR_INVALID_ARGUMENT


@pytest.mark.parametrize("m,n,k,flags", [
    (256, 256, 256, 0),
    (300, 200, 1000, _ffi.MATMUL_RELU),                 # 128-row tile
    (40, 264, 2048, _ffi.MATMUL_RELU),                  # 64-row tile
    (9, 130, 512, 0),                                   # 16-row tile, n % 4 != 0
    (1024, 1024, 1024, _ffi.MATMUL_RELU),               # split k
    (77, 131, 301, _ffi.MATMUL_RELU | _ffi.MATMUL_FORCE_GUARDED),
    (64, 64, 0, _ffi.MATMUL_RELU),                      # empty sum
])
def test_fused_matmul_add_is_matmul_then_add(gpu, m, n, k, flags):
    """hexir_cuda_matmul_add_f64 = hexir_cuda_matmul_f64, then
    hexir_cuda_add_f64 (then the relu), bit for bit under the same plan."""
    rng = np.random.default_rng(m * 31 + n + k)
    a = rng.uniform(-1, 1, (m, k))
    b = rng.uniform(-1, 1, (k, n))
    d = rng.uniform(-1, 1, (m, n))
    ba, bb, bd = gpu.upload(a if k else np.zeros(1)), \
        gpu.upload(b if k else np.zeros(1)), gpu.upload(d)
    fused, prod, two = (gpu.buffer(m * n * 8) for _ in range(3))
    hx.cuda_matmul_add(0, ba.ptr, bb.ptr, bd.ptr, fused.ptr, m, n, k, flags,
                       gpu.stream)
    hx.cuda_matmul(0, ba.ptr, bb.ptr, prod.ptr, m, n, k,
                   flags & ~_ffi.MATMUL_RELU, gpu.stream)
    hx.cuda_add(0, prod.ptr, bd.ptr, two.ptr, m * n, gpu.stream)
    if flags & _ffi.MATMUL_RELU:
        hx.cuda_relu(0, two.ptr, two.ptr, m * n, gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    got, want2 = fused.read((m, n)), two.read((m, n))
    assert np.array_equal(bits(got), bits(want2))
    want = oracle.add(oracle.matmul(a, b) if k else np.zeros((m, n)), d)
    if flags & _ffi.MATMUL_RELU:
        want = oracle.relu(want)
    assert oracle.normwise_error(got, want) <= TOL


@pytest.mark.parametrize("m,n,k,flags,add", [
    (2048, 2048, 2048, 0, False),
    (2048, 1024, 4096, _ffi.MATMUL_RELU, False),
    (500, 2560, 2048, _ffi.MATMUL_RELU, True),     # ragged row tiles, fused add
    (640, 2048, 1024, 0, True),
    (128, 8192, 8192, _ffi.MATMUL_RELU, False),    # one row of tiles, long k
    (100, 8192, 2048, 0, False),                   # a partial row tile
    (300, 2050, 1536, _ffi.MATMUL_RELU, True),     # n % 4 != 0: scalar fix-up
    (1024, 1024, 1024, _ffi.MATMUL_RELU, False),
    # 304 tiles: the first wave data-parallel, then every CTA's stream-K
    # run (a data-parallel tile and a run in one CTA).
    (2432, 2048, 1024, _ffi.MATMUL_RELU, True),
    (4736, 512, 512, 0, False),                    # exactly one wave of tiles
])
def test_stream_k_schedule(gpu, m, n, k, flags, add):
    """The stream-K schedule: a persistent launch plus fix-up, within the bar
    of the oracle (rows sampled for the large shapes), deterministic run to
    run, and within the bar of the data-parallel / split-K schedule."""
    flags |= _ffi.MATMUL_FORCE_STREAM_K
    assert hx.matmul_plan(m, n, k, flags)[0] == 5
    assert hx.matmul_plan(m, n, k, flags | _ffi.MATMUL_NO_STREAM_K)[0] == 1
    rng = np.random.default_rng(m + n + k)
    a = rng.uniform(-1, 1, (m, k))
    b = rng.uniform(-1, 1, (k, n))
    d = rng.uniform(-1, 1, (m, n)) if add else None
    ba, bb = gpu.upload(a), gpu.upload(b)
    bd = gpu.upload(d) if add else None
    outs = []
    for extra in (0, 0, _ffi.MATMUL_NO_STREAM_K):  # twice, then without
        bc = gpu.buffer(m * n * 8)
        if add:
            hx.cuda_matmul_add(0, ba.ptr, bb.ptr, bd.ptr, bc.ptr, m, n, k,
                               flags | extra, gpu.stream)
        else:
            hx.cuda_matmul(0, ba.ptr, bb.ptr, bc.ptr, m, n, k, flags | extra,
                           gpu.stream)
        hx.cuda_synchronize(0, gpu.stream)
        outs.append(bc.read((m, n)))
    assert np.array_equal(bits(outs[0]), bits(outs[1]))
    rows = np.unique(np.linspace(0, m - 1, 40).astype(int))
    want = oracle.matmul(a[rows], b)
    if add:
        want = oracle.add(want, d[rows])
    if flags & _ffi.MATMUL_RELU:
        want = oracle.relu(want)
    assert oracle.normwise_error(outs[0][rows], want) <= TOL
    assert oracle.normwise_error(outs[0], outs[2]) <= TOL


@pytest.mark.parametrize("m,n,k", [(5, 7, 9), (37, 96, 64), (128, 130, 40),
                                   (256, 256, 256), (3, 1024, 300), (1, 1, 1)])
def test_reference_schedule_baseline_matches_oracle(gpu, m, n, k):
    """The measurement baseline restating the reference's generated GPU
    schedule (thread per output, serial k, FMA-contracted) computes the
    same product: within the linear's normwise bar (its contraction differs
    from the CPU's separate multiply and add in the last bits)."""
    rng = hx.Rng(71)
    a, b = rng.uniform((m, k)), rng.uniform((k, n))
    ba, bb, bc = gpu.upload(a), gpu.upload(b), gpu.buffer(m * n * 8)
    _ffi.check(hx.lib().hexir_cuda_baseline_reference_schedule_f64(
        0, ba.ptr, bb.ptr, bc.ptr, m, n, k, gpu.stream), "baseline")
    hx.cuda_synchronize(0, gpu.stream)
    got = bc.read((m, n))
    assert oracle.normwise_error(got, oracle.matmul(a, b)) <= TOL


def test_reference_schedule_baseline_refuses_what_the_reference_cannot_launch(gpu):
    st = hx.lib().hexir_cuda_baseline_reference_schedule_f64(
        0, 0, 0, 0, 65536, 8, 8, gpu.stream)
    assert st == _ffi.ERROR_INVALID_ARGUMENT
