"""ctypes bindings of libhexir_b200.so, the C ABI declared in include/.

Every foreign function gets explicit argtypes/restype here, so a wrong call
fails in Python instead of corrupting the stack.  The library is built
in-tree (hexir_b200/lib) by ``hexir_b200.build.build()``; there is no other
implementation to fall back to, so a missing library raises.
"""

from __future__ import annotations

import ctypes as C
import os

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "lib", "libhexir_b200.so")
CUBIN_PATH = os.path.join(PKG_DIR, "lib", "hexir_kernels.cubin")
BIN_DIR = os.path.join(PKG_DIR, "bin")

# hexir_status_t (include/hexir_runtime/status.h)
OK = 0
ERROR_INVALID_ARGUMENT = 1
ERROR_NOT_FOUND = 2
ERROR_OUT_OF_MEMORY = 3
ERROR_UNIMPLEMENTED = 4
ERROR_INVALID_MODULE = 5
ERROR_IO = 6
ERROR_DEVICE = 7

DEVICE_CPU = 0
DEVICE_CUDA = 1
MEMORY_DEVICE_LOCAL = 1

# include/hexir_b200/kernels.h
MATMUL_RELU = 0x1
MATMUL_FORCE_TMA = 0x100
MATMUL_FORCE_GUARDED = 0x200
MATMUL_REMOTE_OUTPUT = 0x400
MATMUL_NO_STREAM_K = 0x800
MATMUL_FORCE_STREAM_K = 0x2000
SHARD_GATHER_NCCL = 0x1000
SHARD_W_ON_ALL = 0x4000

# Activation codes = kernel kinds 7-14 (include/hexir_runtime/program.h).
ACTIVATIONS = {"leaky_relu": 7, "elu": 8, "sigmoid": 9, "tanh": 10,
               "softmax": 11, "gelu": 12, "swish": 13, "mish": 14}


def MATMUL_SPLIT_K(s: int) -> int:
    return (s & 0xFF) << 16


# include/hexir_b200/hxb_writer.h
EMIT_NO_FUSE = 0x1
EMIT_NO_IMAGE = 0x2
EMIT_ACTIVATIONS = 0x4


class Rng(C.Structure):
    _fields_ = [("state", C.c_uint64)]


_vp, _sz, _u32, _u64, _i32, _int = (C.c_void_p, C.c_size_t, C.c_uint32,
                                    C.c_uint64, C.c_int32, C.c_int)
_dp = C.POINTER(C.c_double)

# (name, restype, argtypes)
_SIGNATURES = [
    # status.h
    ("hexir_status_string", C.c_char_p, [_int]),
    # hal.h
    ("hexir_device_create", _int, [_int, C.POINTER(_vp)]),
    ("hexir_device_create_cuda", _int, [_int, C.POINTER(_vp)]),
    ("hexir_device_release", None, [_vp]),
    ("hexir_device_name", C.c_char_p, [_vp]),
    ("hexir_device_kind", _int, [_vp]),
    ("hexir_device_ordinal", _int, [_vp]),
    ("hexir_device_count", _int, [_int, C.POINTER(_int)]),
    ("hexir_device_stream", _vp, [_vp]),
    ("hexir_device_wait", _int, [_vp]),
    ("hexir_buffer_allocate", _int, [_vp, _sz, _int, C.POINTER(_vp)]),
    ("hexir_buffer_release", None, [_vp]),
    ("hexir_buffer_size", _sz, [_vp]),
    ("hexir_buffer_memory_kind", _int, [_vp]),
    ("hexir_buffer_host_pointer", _vp, [_vp]),
    ("hexir_buffer_device_pointer", _vp, [_vp]),
    ("hexir_buffer_write", _int, [_vp, _vp, _sz]),
    ("hexir_buffer_read", _int, [_vp, _vp, _sz]),
    ("hexir_device_launch", _int, [_vp, _vp, _sz, C.c_char_p, C.c_uint,
                                   C.c_uint, C.c_uint, C.c_uint,
                                   C.POINTER(_vp), C.c_uint]),
    # module.h
    ("hexir_module_load_file", _int, [C.c_char_p, C.POINTER(_vp)]),
    ("hexir_module_load_memory", _int, [_vp, _u64, C.POINTER(_vp)]),
    ("hexir_module_release", None, [_vp]),
    ("hexir_module_version", _u32, [_vp]),
    ("hexir_module_section_count", _u32, [_vp]),
    ("hexir_module_section_at", _vp, [_vp, _u32]),
    ("hexir_module_section", _int, [_vp, _int, C.POINTER(_vp),
                                    C.POINTER(_u64)]),
    ("hexir_section_kind_string", C.c_char_p, [_u32]),
    # program.h
    ("hexir_kernel_kind_string", C.c_char_p, [_u32]),
    # vm.h
    ("hexir_execute", _int, [_vp, _vp, C.c_char_p]),
    ("hexir_execute_capture", _int, [_vp, _vp, C.c_char_p, _vp, _sz]),
    ("hexir_execute_devices", _int, [_vp, C.POINTER(_vp), C.c_uint,
                                     C.c_char_p, _vp, _sz]),
    ("hexir_last_execute_kernel_ms", C.c_double, []),
    ("hexir_module_keep_constants", _int, [_vp, _int]),
    ("hexir_module_kept_bytes", _sz, [_vp]),
    # hexir_b200/kernels.h
    ("hexir_cuda_matmul_f64", _int, [_int, _vp, _vp, _vp, _u32, _u32, _u32,
                                     _u32, _vp]),
    ("hexir_cuda_matmul_acc_f64", _int, [_int, _vp, _u32, _vp, _vp, _vp, _u32,
                                         _u32, _u32, _u32, _vp]),
    ("hexir_cuda_matmul_add_f64", _int, [_int, _vp, _vp, _vp, _vp, _u32, _u32,
                                         _u32, _u32, _vp]),
    ("hexir_cuda_add_f64", _int, [_int, _vp, _vp, _vp, _sz, _vp]),
    ("hexir_cuda_relu_f64", _int, [_int, _vp, _vp, _sz, _vp]),
    ("hexir_cuda_activation_f64", _int, [_int, _u32, _vp, _vp, _u64, _u32, _vp]),
    ("hexir_cuda_matmul_f64_noalloc", _int, [_int, _vp, _vp, _vp, _u32, _u32,
                                             _u32, _u32, _vp]),
    ("hexir_cuda_synchronize", _int, [_int, _vp]),
    ("hexir_cuda_matmul_plan", _int, [_int, _vp, _vp, _vp, _u32, _u32, _u32,
                                      _u32, C.POINTER(_int),
                                      C.POINTER(_u32)]),
    ("hexir_cuda_baseline_reference_schedule_f64", _int,
     [_int, _vp, _vp, _vp, _u32, _u32, _u32, _vp]),
    ("hexir_cuda_dmma_probe", _int, [_int, _vp, _u32, _u32, _vp,
                                     C.POINTER(C.c_double)]),
    ("hexir_cuda_wait_probe", _int, [_int, _u64, _vp]),
    ("hexir_cuda_launch_count", _u64, []),
    ("hexir_cuda_sm_count", _int, [_int]),
    ("hexir_cuda_kernel_image", _int, [C.POINTER(_vp), C.POINTER(_sz)]),
    ("hexir_cuda_last_error", C.c_char_p, []),
    # hexir_b200/comm.h
    ("hexir_shard_rows", _int, [_u64, _u32, _u32, C.POINTER(_u64),
                                C.POINTER(_u64)]),
    ("hexir_comm_unique_id", _int, [_vp, _sz]),
    ("hexir_comm_init_rank", _int, [_vp, _sz, _int, _int, _int,
                                    C.POINTER(_vp)]),
    ("hexir_comm_release", None, [_vp]),
    ("hexir_comm_rank", _int, [_vp]),
    ("hexir_comm_size", _int, [_vp]),
    ("hexir_comm_direct_stores", _int, [_vp]),
    ("hexir_comm_synchronize", _int, [_vp, _vp]),
    ("hexir_sharded_linear_host_f64", _int, [_vp, _vp, _vp, _vp, _u32, _u32,
                                             _u32, _u32, _vp]),
    ("hexir_host_register", _int, [_vp, _sz]),
    ("hexir_host_unregister", _int, [_vp]),
    ("hexir_shard_gather_pieces", _int, [_u64, _u32, C.POINTER(_u64),
                                         C.POINTER(_u64), C.POINTER(_u32)]),
    ("hexir_shard_weight_pieces", _int, [_u32, _u32, C.POINTER(_u32),
                                         C.POINTER(_u32)]),
    # fault.h
    ("hexir_fault_configure", _int, [C.c_char_p]),
    ("hexir_fault_calls", _u64, [C.c_char_p]),
    ("hexir_sharded_linear_f64", _int, [_vp, _vp, _vp, _vp, _u32, _u32, _u32,
                                        _u32, _vp]),
    # hexir_b200/hxb_writer.h
    ("hexir_program_create", _vp, []),
    ("hexir_program_release", None, [_vp]),
    ("hexir_program_begin_function", _int, [_vp, C.c_char_p]),
    ("hexir_program_constant", _i32, [_vp, _dp, _u32, _u32]),
    ("hexir_program_splat", _i32, [_vp, C.c_double, _u32, _u32]),
    ("hexir_program_linear", _i32, [_vp, _i32, _i32]),
    ("hexir_program_add", _i32, [_vp, _i32, _i32]),
    ("hexir_program_relu", _i32, [_vp, _i32]),
    ("hexir_program_activation", _i32, [_vp, C.c_char_p, _i32]),
    ("hexir_program_print", _int, [_vp, _i32]),
    ("hexir_program_emit_file", _int, [_vp, C.c_char_p, _u32, C.c_char_p]),
    ("hexir_program_emit_memory", _int, [_vp, C.c_char_p, _u32,
                                         C.POINTER(_vp), C.POINTER(_sz)]),
    ("hexir_free", None, [_vp]),
    ("hexir_program_parse", _int, [C.c_char_p, C.POINTER(_vp), C.c_char_p,
                                   _sz]),
    ("hexir_program_last_error", C.c_char_p, [_vp]),
    ("hexir_rng_seed", None, [C.POINTER(Rng), _u64]),
    ("hexir_rng_uniform", None, [C.POINTER(Rng), _dp, _sz, C.c_double,
                                 C.c_double]),
    ("hexir_rng_normal", None, [C.POINTER(Rng), _dp, _sz, C.c_double,
                                C.c_double]),
]

EXPORTED = [name for name, _, _ in _SIGNATURES]

_LIB = None


class HexirError(RuntimeError):
    """A call into the runtime returned a non-OK hexir_status_t."""

    def __init__(self, status: int, what: str, detail: str = ""):
        self.status = status
        msg = f"{what}: {status_string(status)}"
        if detail:
            msg += f" ({detail})"
        super().__init__(msg)


def loaded():
    """The library if it has been loaded, else None; never loads it.  For
    finalizers: at interpreter shutdown module globals may already be gone,
    and the process's exit frees what they would release."""
    return _LIB


def lib() -> C.CDLL:
    """The loaded library; raises if it has not been built."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with "
                "`python -c 'import hexir_b200.build as b; b.build()'`")
        handle = C.CDLL(LIB_PATH, mode=C.RTLD_LOCAL)
        for name, restype, argtypes in _SIGNATURES:
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _LIB = handle
    return _LIB


def status_string(status: int) -> str:
    return lib().hexir_status_string(status).decode()


def check(status: int, what: str) -> None:
    if status != OK:
        detail = lib().hexir_cuda_last_error().decode()
        raise HexirError(status, what, detail)
