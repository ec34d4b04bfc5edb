"""The matmul planner (hexir_cuda_matmul_plan) on the CPU: which kernel and
k split a call would get.  Without a GPU the planner assumes B200's 148 SMs,
so these are the decisions a B200 sees.

  variant 1  TMA, 128-row tiles      3  TMA, 16-row tiles (m <= 16)
  variant 2  guarded (any shape)     4  TMA, 64-row tiles (16 < m <= 64)
  variant 5  128-row tiles as a stream-K launch (where the wave model would
             split k for 128-row tiles, or on request)
"""

import pytest

import hexir_b200 as hx
from hexir_b200 import _ffi


@pytest.mark.parametrize("m,variant", [(1, 3), (16, 3), (17, 4), (64, 4),
                                       (65, 1), (8192, 1)])
def test_tile_height_follows_the_row_count(m, variant):
    assert hx.matmul_plan(m, 8192, 8192, _ffi.MATMUL_NO_STREAM_K)[0] == variant
    # 65 rows: one row of 128-row tiles, run as stream-K unless ruled out.
    want = 5 if m == 65 else variant
    assert hx.matmul_plan(m, 8192, 8192)[0] == want


@pytest.mark.parametrize("shape,split", [
    ((8192, 8192, 8192), 1), ((4096, 4096, 4096), 1), ((2048, 2048, 2048), 4),
    ((1024, 1024, 1024), 2), ((1, 8192, 8192), 9), ((16, 8192, 8192), 9),
    ((64, 8192, 8192), 9)])
def test_k_split_model_choices(shape, split):
    """The fitted wave model: no split where the tiles fill the GPU, a split
    for the skinny and small shapes (stream-K ruled out, which takes the
    128-row shapes the model splits)."""
    assert hx.matmul_plan(*shape, _ffi.MATMUL_NO_STREAM_K)[1] == split


@pytest.mark.parametrize("shape,plan", [
    ((2048, 2048, 2048), (5, 148)), ((1024, 1024, 1024), (5, 148)),
    ((512, 8192, 8192), (5, 148)), ((8192, 1024, 4096), (5, 148)),
    ((8192, 8192, 8192), (1, 1)), ((4096, 4096, 4096), (1, 1)),
    ((1536, 1536, 1536), (1, 1)),
    ((16, 8192, 8192), (3, 9)), ((64, 8192, 8192), (4, 9)),
    ((1000, 384, 512), (1, 4))])   # a split but < 4 k-tiles per CTA
def test_stream_k_where_the_model_splits_k(shape, plan):
    """The 128-row tiles run as stream-K where the wave model would split k;
    the 16- and 64-row tiles keep their split, and so do shapes too small
    to give every CTA a run of 4 k-tiles."""
    assert hx.matmul_plan(*shape, _ffi.MATMUL_RELU) == plan
    assert hx.matmul_plan(*shape, _ffi.MATMUL_RELU | _ffi.MATMUL_SPLIT_K(2))[0] != 5


@pytest.mark.parametrize("m,n,k", [(8192, 8191, 8192), (8192, 8192, 8191),
                                   (37, 53, 29)])
def test_odd_extents_take_the_guarded_kernel(m, n, k):
    assert hx.matmul_plan(m, n, k)[0] == 2


@pytest.mark.parametrize("which", ["a", "b", "c"])
def test_a_pointer_off_16_bytes_takes_the_guarded_kernel(which):
    ptrs = {"a": 4096, "b": 4096, "c": 4096}
    assert hx.matmul_plan(8192, 8192, 8192, 0, 0, **ptrs)[0] == 1
    ptrs[which] = 4096 + 8
    assert hx.matmul_plan(8192, 8192, 8192, 0, 0, **ptrs)[0] == 2


def test_flags_force_a_kernel_or_a_split():
    assert hx.matmul_plan(8192, 8192, 8192, _ffi.MATMUL_FORCE_GUARDED)[0] == 2
    assert hx.matmul_plan(8192, 8192, 8192, _ffi.MATMUL_SPLIT_K(3)) == (1, 3)
    # Stream-K on request even where the model keeps k whole: one CTA per
    # SM, never with a k split or against NO_STREAM_K.
    assert hx.matmul_plan(8192, 8192, 8192, _ffi.MATMUL_FORCE_STREAM_K) == (5, 148)
    assert hx.matmul_plan(8192, 8192, 8192, _ffi.MATMUL_FORCE_STREAM_K |
                          _ffi.MATMUL_SPLIT_K(2))[0] == 1
    assert hx.matmul_plan(8192, 8192, 8192, _ffi.MATMUL_FORCE_STREAM_K |
                          _ffi.MATMUL_NO_STREAM_K)[0] == 1
    # The relu changes no decision.
    assert hx.matmul_plan(2048, 2048, 2048, _ffi.MATMUL_RELU) == \
        hx.matmul_plan(2048, 2048, 2048)
