"""ctypes face of the CPU oracle.  TEST INFRASTRUCTURE ONLY.

Importable by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
leg; nothing in hexir_b200/ imports it.  Two libraries:
  - _build/liboracle.so   the C restatement in hexir_oracle.c
  - _ref/libhexir_ref.so  the reference runtime itself, compiled from its own
                          sources by `make ref` (present when it was built in
                          a container that has the reference tree)
"""

from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libhexir_ref.so")
REF_RUN = os.path.join(HERE, "_ref", "hexir-run")

_oracle = None
_ref = None
_dp = C.POINTER(C.c_double)


def build() -> None:
    subprocess.run(["make", "-C", HERE], check=True, capture_output=True)
    subprocess.run(["make", "-C", HERE, "ref"], check=True, capture_output=True)


def _load_oracle():
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_SO):
            build()
        lib = C.CDLL(ORACLE_SO)
        lib.oracle_matmul_f64.argtypes = [_dp, _dp, _dp, C.c_uint32, C.c_uint32,
                                          C.c_uint32, C.c_int]
        lib.oracle_matmul_rows_f64.argtypes = [_dp, _dp, _dp, C.c_uint32,
                                               C.c_uint32, C.c_uint32,
                                               C.c_uint32]
        lib.oracle_add_f64.argtypes = [_dp, _dp, _dp, C.c_size_t]
        lib.oracle_relu_f64.argtypes = [_dp, _dp, C.c_size_t]
        for f in ("oracle_matmul_f64", "oracle_matmul_rows_f64",
                  "oracle_add_f64", "oracle_relu_f64"):
            getattr(lib, f).restype = None
        lib.oracle_activation_f64.argtypes = [C.c_uint32, _dp, _dp, C.c_uint64,
                                              C.c_uint64]
        lib.oracle_activation_f64.restype = C.c_int
        _oracle = lib
    return _oracle


def have_reference() -> bool:
    return os.path.exists(REF_SO)


REF_ROOT_RECORD = os.path.join(HERE, "_ref", "REFERENCE_ROOT")


def reference_root():
    """The reference checkout's root, or None where it is absent: the
    environment variable HEXIR_REFERENCE, else the checkout `make ref` last
    compiled _ref from (recorded in _ref/REFERENCE_ROOT)."""
    root = os.environ.get("HEXIR_REFERENCE")
    if not root and os.path.exists(REF_ROOT_RECORD):
        with open(REF_ROOT_RECORD) as f:
            root = f.read().strip()
    return root if root and os.path.isdir(root) else None


def _load_ref():
    global _ref
    if _ref is None:
        lib = C.CDLL(REF_SO, mode=C.RTLD_LOCAL)
        lib.hexir_ref_matmul_f64.argtypes = [_dp, _dp, _dp, C.c_uint32,
                                             C.c_uint32, C.c_uint32]
        lib.hexir_ref_add_f64.argtypes = [_dp, _dp, _dp, C.c_size_t]
        lib.hexir_ref_relu_f64.argtypes = [_dp, _dp, C.c_size_t]
        for f in ("hexir_ref_matmul_f64", "hexir_ref_add_f64",
                  "hexir_ref_relu_f64"):
            getattr(lib, f).restype = None
        _ref = lib
    return _ref


def _p(a: np.ndarray):
    return a.ctypes.data_as(_dp)


def _f64(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float64)


def matmul(a, b, threads: int = 0) -> np.ndarray:
    """c = a . b with the reference's per-element summation order."""
    a, b = _f64(a), _f64(b)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2
    c = np.empty((m, n), dtype=np.float64)
    _load_oracle().oracle_matmul_f64(_p(a), _p(b), _p(c), m, n, k,
                                     threads or (os.cpu_count() or 1))
    return c


def matmul_rows(a, b, row_begin: int, row_end: int) -> np.ndarray:
    """Rows [row_begin, row_end) of a . b, single thread."""
    a, b = _f64(a), _f64(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.zeros((m, n), dtype=np.float64)
    _load_oracle().oracle_matmul_rows_f64(_p(a), _p(b), _p(c), row_begin,
                                          row_end, n, k)
    return c[row_begin:row_end]


def relu(x) -> np.ndarray:
    x = _f64(x)
    y = np.empty_like(x)
    _load_oracle().oracle_relu_f64(_p(x), _p(y), x.size)
    return y


def add(a, b) -> np.ndarray:
    a, b = _f64(a), _f64(b)
    c = np.empty_like(a)
    _load_oracle().oracle_add_f64(_p(a), _p(b), _p(c), a.size)
    return c


ACTIVATION_KINDS = {"leaky_relu": 7, "elu": 8, "sigmoid": 9, "tanh": 10,
                    "softmax": 11, "gelu": 12, "swish": 13, "mish": 14}


def activation(op: str, x) -> np.ndarray:
    """op(x) for a rank-2 x (softmax along each row), by the op descriptions
    of HexirOps.td:189-308 as restated in hexir_oracle.c."""
    x = _f64(x)
    assert x.ndim == 2
    y = np.empty_like(x)
    rc = _load_oracle().oracle_activation_f64(ACTIVATION_KINDS[op], _p(x), _p(y),
                                              x.shape[0], x.shape[1])
    assert rc == 0
    return y


def ulp_error_ok(got, want, ulps: float, floor: float = 2.0 ** -1000) -> np.ndarray:
    """Elementwise: |got - want| <= ulps * 2^-52 * |want| + floor, NaN exactly
    where want is NaN, equal infinities where want is infinite."""
    got, want = np.asarray(got), np.asarray(want)
    nan = np.isnan(want)
    inf = np.isinf(want)
    with np.errstate(invalid="ignore", over="ignore"):
        close = np.abs(got - want) <= ulps * 2.0 ** -52 * np.abs(want) + floor
    return np.where(nan, np.isnan(got), np.where(inf, got == want, close))


def ref_matmul(a, b) -> np.ndarray:
    """The reference's own hexir_ref_matmul_f64 (needs _ref)."""
    a, b = _f64(a), _f64(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.empty((m, n), dtype=np.float64)
    _load_ref().hexir_ref_matmul_f64(_p(a), _p(b), _p(c), m, n, k)
    return c


def ref_matmul_rows_into(a, b, c, row_begin: int, row_end: int) -> None:
    """hexir_ref_matmul_f64 on a row slice, written into c (threads call
    this concurrently; ctypes releases the GIL during the call)."""
    m, k = a.shape
    n = b.shape[1]
    rows = row_end - row_begin
    a_ptr = C.cast(a.ctypes.data + row_begin * k * 8, _dp)
    c_ptr = C.cast(c.ctypes.data + row_begin * n * 8, _dp)
    _load_ref().hexir_ref_matmul_f64(a_ptr, _p(b), c_ptr, rows, n, k)


def ref_relu(x) -> np.ndarray:
    x = _f64(x)
    y = np.empty_like(x)
    _load_ref().hexir_ref_relu_f64(_p(x), _p(y), x.size)
    return y


def ref_add(a, b) -> np.ndarray:
    a, b = _f64(a), _f64(b)
    c = np.empty_like(a)
    _load_ref().hexir_ref_add_f64(_p(a), _p(b), _p(c), a.size)
    return c


def normwise_error(got, want) -> float:
    """max |got - want| / max |want| (0 when both are all zero)."""
    got, want = np.asarray(got), np.asarray(want)
    scale = float(np.max(np.abs(want))) if want.size else 0.0
    diff = float(np.max(np.abs(got - want))) if want.size else 0.0
    if scale == 0.0:
        return diff
    return diff / scale
