"""Guard bands around every output: the kernels write exactly their output.

Each output buffer is surrounded by 4096 canary doubles on both sides
(a signalling-NaN bit pattern no kernel produces); after the launch the
canaries must be intact and every output element written.  Shapes are
ragged on purpose (partial row and column tiles, odd k and n, m below and
above every tile height), across the 128/64/16-row TMA kernels, the guarded
kernel, split-K, stream-K, the fused addend, continued sums, relu and add,
and a misaligned output pointer.
"""

import numpy as np
import pytest

import hexir_b200 as hx
from hexir_b200 import _ffi

pytestmark = pytest.mark.gpu

GUARD = 4096
CANARY = np.uint64(0x7FF4DEADBEEF1234)


def guarded(dev, count, shift=0):
    """A buffer holding `count` doubles between two canary bands; `shift`
    bytes moves the output off its natural alignment."""
    total = count + 2 * GUARD + 1
    buf = dev.buffer(total * 8)
    buf.write(np.full(total, CANARY, dtype=np.uint64))
    return buf, buf.ptr + GUARD * 8 + shift


def check(buf, count, shift=0):
    raw = bytes(buf.read((count + 2 * GUARD + 1) * 8, dtype=np.uint8))
    head = np.frombuffer(raw[:GUARD * 8 + shift], dtype=np.uint8)
    body = raw[GUARD * 8 + shift:GUARD * 8 + shift + count * 8]
    tail = np.frombuffer(raw[GUARD * 8 + shift + count * 8:], dtype=np.uint8)
    canary = np.full(len(raw) // 8, CANARY, dtype=np.uint64).tobytes()
    assert head.tobytes() == canary[:len(head)], "write before the output"
    assert tail.tobytes() == canary[len(raw) - len(tail):], "write after the output"
    vals = np.frombuffer(body, dtype=np.uint64)
    assert not np.any(vals == CANARY), "output element left unwritten"


SHAPES = [(1, 9, 7), (5, 130, 96), (17, 264, 100), (65, 131, 301),
          (129, 258, 64), (300, 200, 1000), (777, 384, 512)]


@pytest.mark.parametrize("m,n,k", SHAPES)
@pytest.mark.parametrize("flags", [
    0, _ffi.MATMUL_RELU, _ffi.MATMUL_FORCE_GUARDED, _ffi.MATMUL_SPLIT_K(3),
    _ffi.MATMUL_FORCE_STREAM_K | _ffi.MATMUL_RELU])
def test_matmul_writes_only_its_output(gpu, m, n, k, flags):
    rng = np.random.default_rng(m + n + k)
    a, b = gpu.upload(rng.uniform(-1, 1, (m, k))), gpu.upload(rng.uniform(-1, 1, (k, n)))
    buf, c = guarded(gpu, m * n)
    hx.cuda_matmul(0, a.ptr, b.ptr, c, m, n, k, flags, gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    check(buf, m * n)


@pytest.mark.parametrize("m,n,k", SHAPES[1:])
def test_fused_add_and_continued_sums_write_only_their_output(gpu, m, n, k):
    rng = np.random.default_rng(7 * m + n)
    a, b = gpu.upload(rng.uniform(-1, 1, (m, k))), gpu.upload(rng.uniform(-1, 1, (k, n)))
    d = gpu.upload(rng.uniform(-1, 1, (m, n)))
    buf, c = guarded(gpu, m * n)
    hx.cuda_matmul_add(0, a.ptr, b.ptr, d.ptr, c, m, n, k, _ffi.MATMUL_RELU,
                       gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    check(buf, m * n)
    # Two k pieces, the second continuing the first from the guarded output.
    buf2, c2 = guarded(gpu, m * n)
    half = (k // 2) // 32 * 32
    hx.cuda_matmul_acc(0, a.ptr, k, b.ptr, 0, c2, m, n, half, 0, gpu.stream)
    hx.cuda_matmul_acc(0, a.ptr + 8 * half, k, b.ptr + 8 * half * n, c2, c2, m,
                       n, k - half, _ffi.MATMUL_RELU, gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    check(buf2, m * n)


@pytest.mark.parametrize("m,n,k", [(500, 2560, 2048), (300, 2050, 1536)])
def test_stream_k_writes_only_its_output(gpu, m, n, k):
    """The stream-K launch and its fix-up (partial tiles in the workspace,
    split tiles summed into c) on ragged shapes: a partial row tile, and a
    partial column tile with n % 4 != 0 (the fix-up's scalar stores)."""
    flags = _ffi.MATMUL_FORCE_STREAM_K | _ffi.MATMUL_RELU
    assert hx.matmul_plan(m, n, k, flags)[0] == 5
    rng = np.random.default_rng(5)
    a, b = gpu.upload(rng.uniform(-1, 1, (m, k))), gpu.upload(rng.uniform(-1, 1, (k, n)))
    buf, c = guarded(gpu, m * n)
    hx.cuda_matmul(0, a.ptr, b.ptr, c, m, n, k, flags, gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    check(buf, m * n)


def test_misaligned_output_uses_the_guarded_kernel_safely(gpu):
    m, n, k = 70, 90, 48
    rng = np.random.default_rng(3)
    a, b = gpu.upload(rng.uniform(-1, 1, (m, k))), gpu.upload(rng.uniform(-1, 1, (k, n)))
    buf, c = guarded(gpu, m * n, shift=8)
    hx.cuda_matmul(0, a.ptr, b.ptr, c, m, n, k, _ffi.MATMUL_RELU, gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    check(buf, m * n, shift=8)


@pytest.mark.parametrize("count", [1, 2, 3, 1023, 1025, (1 << 20) + 7])
def test_elementwise_write_only_their_output(gpu, count):
    rng = np.random.default_rng(count)
    x, y = gpu.upload(rng.normal(size=count)), gpu.upload(rng.normal(size=count))
    buf, out = guarded(gpu, count)
    hx.cuda_relu(0, x.ptr, out, count, gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    check(buf, count)
    buf2, out2 = guarded(gpu, count, shift=8)
    hx.cuda_add(0, x.ptr, y.ptr, out2, count, gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    check(buf2, count, shift=8)


@pytest.mark.parametrize("op", sorted(_ffi.ACTIVATIONS))
@pytest.mark.parametrize("rows,cols,shift", [
    (1, 1, 0), (3, 7, 8), (33, 1025, 0), (9, 8193, 8), (5, 16385, 0),
    (2, 40001, 8), (333, 2050, 0), (151, 16384, 0), (5, 4096, 8)])
def test_activations_write_only_their_output(gpu, op, rows, cols, shift):
    """Each activation kernel (and every softmax launch shape) on ragged
    rows and columns, aligned and 8 bytes off."""
    x = gpu.upload(np.random.default_rng(rows + cols).normal(size=rows * cols + 1))
    buf, out = guarded(gpu, rows * cols, shift=shift)
    hx.cuda_activation(0, op, x.ptr + shift, out, rows, cols, gpu.stream)
    hx.cuda_synchronize(0, gpu.stream)
    check(buf, rows * cols, shift=shift)
