"""Python face of the hexir runtime and writer (thin wrappers over the C ABI).

Mirrors the reference's user-facing pieces for this path:
  Program  -- a hexir program (constant / linear / add / relu / print) and
              its serialization with a -placement= string, as `hexir
              -emit=hxb -placement=...` does (tools/hexir/hexir.cpp)
  Module   -- a loaded .hxb (runtime/include/hexir_runtime/module.h)
  Device   -- a HAL device, "cpu", "cuda" or "cuda:N" (hal.h)
  execute  -- run an entry point and capture the last dispatch's result
              (vm.h hexir_execute_capture / hexir_execute_devices)
and the kernel-level GPU calls that replace the reference CPU kernels
(include/hexir_b200/kernels.h).
"""

from __future__ import annotations

import ctypes as C
import struct
import weakref
from dataclasses import dataclass
from typing import Iterable, List, Optional, Sequence

import numpy as np

from . import _ffi
from ._ffi import check, lib


# ---------------------------------------------------------------- program


class Program:
    """A hexir program built op by op; values are small integers."""

    def __init__(self, _handle: Optional[int] = None):
        self._h = _handle if _handle is not None else lib().hexir_program_create()
        if not self._h:
            raise MemoryError("hexir_program_create")

    def __del__(self):
        h = getattr(self, "_h", None)
        handle = _ffi.loaded()
        if h and handle is not None:
            handle.hexir_program_release(h)
        self._h = None

    def _value(self, v: int, what: str) -> int:
        if v < 0:
            raise ValueError(f"{what}: "
                             f"{lib().hexir_program_last_error(self._h).decode()}")
        return v

    def function(self, name: str) -> None:
        check(lib().hexir_program_begin_function(self._h, name.encode()),
              "begin_function")

    def constant(self, data) -> int:
        a = np.ascontiguousarray(data, dtype=np.float64)
        if a.ndim != 2:
            raise ValueError("constants are rank-2 f64 tensors")
        ptr = a.ctypes.data_as(C.POINTER(C.c_double))
        return self._value(lib().hexir_program_constant(
            self._h, ptr, a.shape[0], a.shape[1]), "constant")

    def splat(self, value: float, rows: int, cols: int) -> int:
        return self._value(lib().hexir_program_splat(self._h, value, rows, cols),
                           "splat")

    def linear(self, x: int, w: int) -> int:
        return self._value(lib().hexir_program_linear(self._h, x, w), "linear")

    def add(self, a: int, b: int) -> int:
        return self._value(lib().hexir_program_add(self._h, a, b), "add")

    def relu(self, x: int) -> int:
        return self._value(lib().hexir_program_relu(self._h, x), "relu")

    def activation(self, op: str, x: int) -> int:
        """One of the dialect's declared activations (leaky_relu, elu,
        sigmoid, tanh, softmax, gelu, swish, mish); emit() serializes it only
        with flags including EMIT_ACTIVATIONS."""
        return self._value(
            lib().hexir_program_activation(self._h, op.encode(), x), op)

    def print(self, x: int) -> None:
        check(lib().hexir_program_print(self._h, x), "print")

    def emit(self, placement: str = "", flags: int = 0) -> bytes:
        data, size = C.c_void_p(), C.c_size_t()
        st = lib().hexir_program_emit_memory(self._h, placement.encode(), flags,
                                             C.byref(data), C.byref(size))
        if st != _ffi.OK:
            raise ValueError(lib().hexir_program_last_error(self._h).decode())
        try:
            return C.string_at(data.value, size.value)
        finally:
            lib().hexir_free(data)

    def emit_file(self, path: str, placement: str = "", flags: int = 0) -> None:
        st = lib().hexir_program_emit_file(self._h, placement.encode(), flags,
                                           str(path).encode())
        if st != _ffi.OK:
            raise ValueError(lib().hexir_program_last_error(self._h).decode())


def parse(text: str) -> Program:
    """Parse the textual subset (func.func / hexir.* ops) into a Program."""
    out = C.c_void_p()
    err = C.create_string_buffer(512)
    st = lib().hexir_program_parse(text.encode(), C.byref(out), err, len(err))
    if st != _ffi.OK:
        raise ValueError(err.value.decode())
    return Program(out.value)


# ---------------------------------------------------------------- rng


class Rng:
    """The writer's seeded SplitMix64 stream (hxb_writer.h)."""

    def __init__(self, seed: int):
        self._r = _ffi.Rng()
        lib().hexir_rng_seed(C.byref(self._r), seed)

    def uniform(self, shape, lo: float = -1.0, hi: float = 1.0) -> np.ndarray:
        out = np.empty(shape, dtype=np.float64)
        lib().hexir_rng_uniform(C.byref(self._r),
                                out.ctypes.data_as(C.POINTER(C.c_double)),
                                out.size, lo, hi)
        return out

    def skip(self, draws: int) -> None:
        """Advance the stream by `draws` draws without producing them (the
        SplitMix64 state moves by a constant per draw)."""
        self._r.state = (self._r.state + draws * 0x9E3779B97F4A7C15) % (1 << 64)

    def normal(self, shape, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
        out = np.empty(shape, dtype=np.float64)
        lib().hexir_rng_normal(C.byref(self._r),
                               out.ctypes.data_as(C.POINTER(C.c_double)),
                               out.size, mean, std)
        return out


# ---------------------------------------------------------------- module

HEADER = struct.Struct("<8sIIII")
SECTION = struct.Struct("<IIQQ")
SYMBOL = struct.Struct("<32sII")
EXEC_ENTRY = struct.Struct("<32s12I")
LAUNCH_ENTRY = struct.Struct("<8I")


@dataclass
class Executable:
    name: str
    kind: int
    device: int
    m: int
    n: int
    k: int
    elem_size: int
    image_offset: int
    image_size: int
    grid: tuple
    block: tuple


def read_executables(blob: bytes) -> List[Executable]:
    """Executable table of a .hxb held in memory (a second reader of the
    format, independent of the C loader)."""
    sections = read_sections(blob)
    off, size = sections[4]
    count, _ = struct.unpack_from("<II", blob, off)
    out = []
    for i in range(count):
        f = EXEC_ENTRY.unpack_from(blob, off + 8 + i * EXEC_ENTRY.size)
        out.append(Executable(f[0].rstrip(b"\0").decode(), *f[1:9],
                              (f[9], f[10]), (f[11], f[12])))
    return out


def read_sections(blob: bytes) -> dict:
    magic, version, _flags, count, _ = HEADER.unpack_from(blob, 0)
    if magic != b"HEXIRMOD" or version != 3:
        raise ValueError("not a version 3 hexir module")
    out = {}
    for i in range(count):
        kind, _f, off, size = SECTION.unpack_from(blob, HEADER.size + i * SECTION.size)
        out.setdefault(kind, (off, size))
    return out


@dataclass
class LaunchEntry:
    abi: int
    flags: int
    device_first: int
    device_count: int


def read_launch(blob: bytes) -> List[LaunchEntry]:
    """The LAUNCH section (kind 5), one entry per executable; [] if absent."""
    sections = read_sections(blob)
    if 5 not in sections:
        return []
    off, _size = sections[5]
    count, _ = struct.unpack_from("<II", blob, off)
    return [LaunchEntry(*LAUNCH_ENTRY.unpack_from(blob, off + 8 + 32 * i)[:4])
            for i in range(count)]


def read_program(blob: bytes, entry: str = "main") -> List[tuple]:
    """Commands of an entry point as (kind, operands) tuples."""
    sections = read_sections(blob)
    soff, ssize = sections[1]
    poff, psize = sections[2]
    pc = None
    for i in range(ssize // SYMBOL.size):
        name, off, _ = SYMBOL.unpack_from(blob, soff + i * SYMBOL.size)
        if name.rstrip(b"\0").decode() == entry:
            pc = off
    if pc is None:
        raise KeyError(entry)
    cmds = []
    while True:
        kind, argc = struct.unpack_from("<II", blob, poff + pc)
        ops = struct.unpack_from(f"<{argc}Q", blob, poff + pc + 8)
        pc += 8 + 8 * argc
        cmds.append((kind, ops))
        if kind == 0:
            return cmds


class Module:
    """A loaded .hxb module."""

    def __init__(self, source):
        h = C.c_void_p()
        if isinstance(source, (bytes, bytearray)):
            buf = C.create_string_buffer(bytes(source), len(source))
            st = lib().hexir_module_load_memory(buf, len(source), C.byref(h))
        else:
            st = lib().hexir_module_load_file(str(source).encode(), C.byref(h))
        check(st, "hexir_module_load")
        self._h = h.value

    @property
    def handle(self) -> int:
        return self._h

    def close(self) -> None:
        handle = _ffi.loaded()
        if getattr(self, "_h", None) and handle is not None:
            handle.hexir_module_release(self._h)
        self._h = None

    __del__ = close

    def version(self) -> int:
        return lib().hexir_module_version(self._h)

    def keep_constants(self, enable: bool = True) -> None:
        """Keep CONST uploads on the GPUs between executes
        (hexir_module_keep_constants); False frees them."""
        check(lib().hexir_module_keep_constants(self._h, int(enable)),
              "hexir_module_keep_constants")

    @property
    def kept_bytes(self) -> int:
        return lib().hexir_module_kept_bytes(self._h)

    def sections(self) -> List[tuple]:
        out = []
        for i in range(lib().hexir_module_section_count(self._h)):
            p = lib().hexir_module_section_at(self._h, i)
            kind, _f, off, size = SECTION.unpack(C.string_at(p, SECTION.size))
            out.append((lib().hexir_section_kind_string(kind).decode(), off, size))
        return out


# ---------------------------------------------------------------- devices


class Device:
    """A HAL device: "cpu", "cuda" (GPU 0) or "cuda:N"."""

    def __init__(self, spec: str = "cpu"):
        h = C.c_void_p()
        if spec == "cpu":
            st = lib().hexir_device_create(_ffi.DEVICE_CPU, C.byref(h))
        elif spec in ("cuda", "gpu"):
            st = lib().hexir_device_create(_ffi.DEVICE_CUDA, C.byref(h))
        elif spec.startswith("cuda:"):
            st = lib().hexir_device_create_cuda(int(spec[5:]), C.byref(h))
        else:
            raise ValueError(f"unknown device {spec!r}")
        check(st, f"hexir_device_create({spec})")
        self._h = h.value
        self.spec = spec
        # Buffers still alive when the device closes are released first (a
        # buffer must not outlive its device in the C ABI).
        self._buffers = weakref.WeakSet()

    @property
    def handle(self) -> int:
        return self._h

    @property
    def name(self) -> str:
        return lib().hexir_device_name(self._h).decode()

    @property
    def ordinal(self) -> int:
        return lib().hexir_device_ordinal(self._h)

    @property
    def stream(self) -> int:
        return lib().hexir_device_stream(self._h) or 0

    def wait(self) -> None:
        check(lib().hexir_device_wait(self._h), "hexir_device_wait")

    def close(self) -> None:
        handle = _ffi.loaded()
        if getattr(self, "_h", None) and handle is not None:
            for b in list(getattr(self, "_buffers", ())):
                b.close()
            handle.hexir_device_release(self._h)
        self._h = None

    __del__ = close

    def buffer(self, nbytes: int) -> "Buffer":
        return Buffer(self, nbytes)

    def upload(self, array: np.ndarray) -> "Buffer":
        a = np.ascontiguousarray(array)
        b = Buffer(self, a.nbytes)
        b.write(a)
        return b


class Buffer:
    """A HAL buffer (DEVICE_LOCAL)."""

    def __init__(self, device: Device, nbytes: int):
        h = C.c_void_p()
        check(lib().hexir_buffer_allocate(device.handle, nbytes,
                                          _ffi.MEMORY_DEVICE_LOCAL, C.byref(h)),
              "hexir_buffer_allocate")
        self._h = h.value
        self.device = device
        self.nbytes = nbytes
        device._buffers.add(self)

    @property
    def ptr(self) -> int:
        return lib().hexir_buffer_device_pointer(self._h) or 0

    def write(self, array: np.ndarray) -> None:
        a = np.ascontiguousarray(array)
        check(lib().hexir_buffer_write(self._h, a.ctypes.data, a.nbytes),
              "hexir_buffer_write")

    def read(self, shape, dtype=np.float64) -> np.ndarray:
        out = np.empty(shape, dtype=dtype)
        check(lib().hexir_buffer_read(self._h, out.ctypes.data, out.nbytes),
              "hexir_buffer_read")
        return out

    def close(self) -> None:
        handle = _ffi.loaded()
        if getattr(self, "_h", None) and handle is not None:
            handle.hexir_buffer_release(self._h)
        self._h = None

    __del__ = close


def device_count() -> int:
    n = C.c_int()
    check(lib().hexir_device_count(_ffi.DEVICE_CUDA, C.byref(n)), "device_count")
    return n.value


def execute(module: Module, devices, entry: str = "main",
            out_shape: Optional[Sequence[int]] = None) -> Optional[np.ndarray]:
    """Run `entry`; return the last dispatch's result as f64 `out_shape`.

    `devices` is one Device (hexir_execute_capture) or a list of CUDA devices
    serving cuda:0..N-1 (hexir_execute_devices)."""
    out = np.empty(out_shape, dtype=np.float64) if out_shape is not None else None
    ptr = out.ctypes.data if out is not None else None
    nbytes = out.nbytes if out is not None else 0
    if isinstance(devices, Device):
        st = lib().hexir_execute_capture(module.handle, devices.handle,
                                         entry.encode(), ptr, nbytes)
    else:
        arr = (C.c_void_p * len(devices))(*[d.handle for d in devices])
        st = lib().hexir_execute_devices(module.handle, arr, len(devices),
                                         entry.encode(), ptr, nbytes)
    check(st, f"execute({entry})")
    return out


def last_kernel_ms() -> float:
    return lib().hexir_last_execute_kernel_ms()


# ---------------------------------------------------------------- kernels


def cuda_matmul(ordinal: int, a: int, b: int, c: int, m: int, n: int, k: int,
                flags: int = 0, stream: int = 0) -> None:
    """c = a . b on device pointers (hexir_cuda_matmul_f64)."""
    check(lib().hexir_cuda_matmul_f64(ordinal, a, b, c, m, n, k, flags,
                                      stream or None), "hexir_cuda_matmul_f64")


def cuda_matmul_acc(ordinal: int, a: int, lda: int, b: int, c_in: int, c: int,
                    m: int, n: int, k: int, flags: int = 0,
                    stream: int = 0) -> None:
    """c = epilogue(c_in + a . b) with a's row stride lda
    (hexir_cuda_matmul_acc_f64); c_in 0 starts the sums at zero."""
    check(lib().hexir_cuda_matmul_acc_f64(ordinal, a, lda, b, c_in or None, c,
                                          m, n, k, flags, stream or None),
          "hexir_cuda_matmul_acc_f64")


def cuda_matmul_add(ordinal: int, a: int, b: int, addend: int, c: int, m: int,
                    n: int, k: int, flags: int = 0, stream: int = 0) -> None:
    """c = epilogue(a . b + addend) (hexir_cuda_matmul_add_f64)."""
    check(lib().hexir_cuda_matmul_add_f64(ordinal, a, b, addend, c, m, n, k,
                                          flags, stream or None),
          "hexir_cuda_matmul_add_f64")


def cuda_relu(ordinal: int, x: int, y: int, n: int, stream: int = 0) -> None:
    check(lib().hexir_cuda_relu_f64(ordinal, x, y, n, stream or None),
          "hexir_cuda_relu_f64")


def cuda_add(ordinal: int, a: int, b: int, c: int, n: int,
             stream: int = 0) -> None:
    check(lib().hexir_cuda_add_f64(ordinal, a, b, c, n, stream or None),
          "hexir_cuda_add_f64")


def cuda_activation(ordinal: int, op, x: int, y: int, rows: int, cols: int,
                    stream: int = 0) -> None:
    """y = op(x) over a [rows x cols] f64 tensor (hexir_cuda_activation_f64);
    op is a name of _ffi.ACTIVATIONS or its code."""
    code = _ffi.ACTIVATIONS[op] if isinstance(op, str) else int(op)
    check(lib().hexir_cuda_activation_f64(ordinal, code, x, y, rows, cols,
                                          stream or None),
          "hexir_cuda_activation_f64")


def cuda_synchronize(ordinal: int, stream: int = 0) -> None:
    check(lib().hexir_cuda_synchronize(ordinal, stream or None),
          "hexir_cuda_synchronize")


def matmul_plan(m: int, n: int, k: int, flags: int = 0, ordinal: int = 0,
                a: int = 0, b: int = 0, c: int = 0) -> tuple:
    """(variant, split_k): 1 = TMA 128-row tiles, 2 = guarded kernel,
    3 = TMA 16-row tiles, 4 = TMA 64-row tiles, 5 = 128-row tiles as a
    stream-K launch (split_k: CTAs sharing the k units)."""
    v, s = C.c_int(), C.c_uint32()
    lib().hexir_cuda_matmul_plan(ordinal, a, b, c, m, n, k, flags, C.byref(v),
                                 C.byref(s))
    return v.value, s.value


def fault_configure(spec: str = "") -> None:
    """Host-side fault injection rules (hexir_fault_configure): e.g.
    "alloc:3", "launch:1+", "alloc:2,nccl:1"; "" turns injection off."""
    check(lib().hexir_fault_configure(spec.encode()), "hexir_fault_configure")


def fault_calls(site: str) -> int:
    """Calls counted at "alloc", "launch" or "nccl" since the rules were set."""
    return lib().hexir_fault_calls(site.encode())


def launch_count() -> int:
    return lib().hexir_cuda_launch_count()


def shard_rows(rows: int, shards: int, index: int) -> tuple:
    b, c = C.c_uint64(), C.c_uint64()
    check(lib().hexir_shard_rows(rows, shards, index, C.byref(b), C.byref(c)),
          "hexir_shard_rows")
    return b.value, c.value


def shard_gather_pieces(rows: int) -> List[tuple]:
    """[(begin, count), ...]: the pieces a rank's `rows` output rows are
    gathered to the root in (hexir_shard_gather_pieces)."""
    out = []
    i = 0
    while True:
        b, c, n = C.c_uint64(), C.c_uint64(), C.c_uint32()
        check(lib().hexir_shard_gather_pieces(rows, i, C.byref(b), C.byref(c),
                                              C.byref(n)),
              "hexir_shard_gather_pieces")
        if i >= n.value:
            return out
        out.append((b.value, c.value))
        i += 1


def shard_weight_pieces(k: int, ranks: int) -> List[int]:
    """[0, ..., k]: the k bounds the weight is broadcast in
    (hexir_shard_weight_pieces)."""
    bounds = (C.c_uint32 * 3)()
    n = C.c_uint32()
    check(lib().hexir_shard_weight_pieces(k, ranks, bounds, C.byref(n)),
          "hexir_shard_weight_pieces")
    return [bounds[i] for i in range(n.value + 1)]


def kernel_image() -> bytes:
    p, n = C.c_void_p(), C.c_size_t()
    check(lib().hexir_cuda_kernel_image(C.byref(p), C.byref(n)),
          "hexir_cuda_kernel_image")
    return C.string_at(p.value, n.value)
