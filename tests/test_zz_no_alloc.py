"""hexir_cuda_matmul_f64_noalloc, the matmul entry point that allocates no
device memory (include/hexir_b200/kernels.h).

It serves callers that cannot allocate: an application whose device memory
belongs to its own pool, a service that cannot absorb the synchronisation a
cudaFree brings, a caller that budgets every byte at start-up.  Its split-K
partial sums live in a fixed array that ships with the library's device code.

Checked here through the C ABI, against the regular entry point
(hexir_cuda_matmul_f64, which may allocate its workspace) within the
normwise 1e-12 bar of the other matmul tests, on two calls in a row with
different shapes so the second call runs over what the first left in the
shared array.  This file is collected last (test_zz_*) so that a failure
here stops a `pytest -x` run only after every other test has run.
"""

import numpy as np
import pytest

import hexir_b200 as hx
from hexir_b200 import _ffi
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-12  # the normwise bar of every f64 linear test


def noalloc(a, b, c, m, n, k, flags, stream):
    return hx.lib().hexir_cuda_matmul_f64_noalloc(0, a, b, c, m, n, k, flags,
                                                  stream or None)


def test_noalloc_matches_allocating_entry_point_on_two_calls():
    dev = hx.Device("cuda")
    cases = [  # (m, n, k, flags, seed): both shapes split k over the scratch
        (64, 256, 4096, 0, 21),
        (40, 200, 3000, _ffi.MATMUL_RELU, 22),
    ]
    for m, n, k, flags, seed in cases:
        variant, split = hx.matmul_plan(m, n, k,
                                        flags | _ffi.MATMUL_FORCE_GUARDED)
        assert variant == 2 and split > 1  # the scratch is in use
        assert split * m * n * 8 <= _SCRATCH_BYTES
        rng = hx.Rng(seed)
        a_host = rng.uniform((m, k))
        b_host = rng.uniform((k, n))
        a, b = dev.upload(a_host), dev.upload(b_host)
        c_alloc, c_free = dev.buffer(m * n * 8), dev.buffer(m * n * 8)
        hx.cuda_matmul(0, a.ptr, b.ptr, c_alloc.ptr, m, n, k, flags, dev.stream)
        st = noalloc(a.ptr, b.ptr, c_free.ptr, m, n, k, flags, dev.stream)
        assert st == _ffi.OK, hx.lib().hexir_cuda_last_error().decode()
        hx.cuda_synchronize(0, dev.stream)
        want = c_alloc.read((m, n))
        got = c_free.read((m, n))
        assert oracle.normwise_error(got, want) <= TOL
        # And both against the CPU oracle.
        ref = oracle.matmul(a_host, b_host)
        if flags & _ffi.MATMUL_RELU:
            ref = oracle.relu(ref)
        assert oracle.normwise_error(got, ref) <= TOL


def test_noalloc_rejects_shapes_beyond_the_scratch():
    dev = hx.Device("cuda")
    m, n, k = 1024, 1024, 64
    a, b, c = dev.buffer(m * k * 8), dev.buffer(k * n * 8), dev.buffer(m * n * 8)
    # k split 4 ways: 4 * 1024 * 1024 * 8 bytes of partial sums > 16 MiB.
    st = noalloc(a.ptr, b.ptr, c.ptr, m, n, k, _ffi.MATMUL_SPLIT_K(4),
                 dev.stream)
    assert st == _ffi.ERROR_INVALID_ARGUMENT
    assert "scratch" in hx.lib().hexir_cuda_last_error().decode()


_SCRATCH_BYTES = 16 << 20  # HEXIR_NOALLOC_SCRATCH_BYTES
