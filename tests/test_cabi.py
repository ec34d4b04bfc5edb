"""The C-ABI library loads on a CPU-only machine and exports every function
the headers in include/ declare.  No compute calls: without a GPU the CUDA
entry points must refuse (no CPU fallback), which is checked through device
creation only."""

import ctypes as C
import os
import re

import pytest

import hexir_b200 as hx
from hexir_b200 import _ffi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, "include")

DECL = re.compile(r"^\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_ ]*[\s\*]+"
                  r"(hexir_[a-z0-9_]+)\s*\(", re.M)


def declared_functions():
    names = set()
    for dirpath, _, files in os.walk(INCLUDE):
        for f in files:
            if f.endswith(".h"):
                text = open(os.path.join(dirpath, f)).read()
                text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
                text = re.sub(r"#define[^\n]*(\\\n[^\n]*)*", "", text)
                names.update(DECL.findall(text))
    return names


def exported_symbols():
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", _ffi.LIB_PATH],
                         capture_output=True, text=True, check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if line.strip()}


def test_headers_declare_the_expected_surface():
    names = declared_functions()
    # Reference HAL / module / VM entry points (runtime/include/hexir_runtime).
    for name in ["hexir_device_create", "hexir_device_release",
                 "hexir_device_name", "hexir_device_kind", "hexir_device_wait",
                 "hexir_buffer_allocate", "hexir_buffer_release",
                 "hexir_buffer_size", "hexir_buffer_memory_kind",
                 "hexir_buffer_host_pointer", "hexir_buffer_device_pointer",
                 "hexir_buffer_write", "hexir_buffer_read",
                 "hexir_device_launch", "hexir_module_load_file",
                 "hexir_module_release", "hexir_module_version",
                 "hexir_module_section_count", "hexir_module_section_at",
                 "hexir_module_section", "hexir_section_kind_string",
                 "hexir_execute", "hexir_execute_capture",
                 "hexir_status_string", "hexir_kernel_kind_string"]:
        assert name in names, name
    assert len(names) > 60


def test_library_exports_every_declared_function():
    missing = declared_functions() - exported_symbols()
    assert not missing, sorted(missing)


def test_library_exports_nothing_but_its_c_abi():
    """The C++ and CUDA runtimes linked statically into the library stay
    private (no operator new, __cxa_* or cuda* symbols leak into a program
    that links it)."""
    foreign = {s for s in exported_symbols() if not s.startswith("hexir_")}
    assert not foreign, sorted(foreign)[:20]


def test_python_bindings_cover_every_declared_function():
    missing = declared_functions() - set(_ffi.EXPORTED)
    assert not missing, sorted(missing)
    lib = hx.lib()
    for name in _ffi.EXPORTED:
        assert getattr(lib, name) is not None


def test_status_strings_match_reference():
    want = ["ok", "invalid argument", "not found", "out of memory",
            "unimplemented", "invalid module", "io error", "device error"]
    assert [_ffi.status_string(i) for i in range(8)] == want
    assert _ffi.status_string(99) == "unknown"


def test_kernel_image_is_an_elf_cubin():
    img = hx.kernel_image()
    assert img[:4] == b"\x7fELF" and len(img) > 10000


def test_shard_rows_is_balanced_and_covering():
    for rows in [0, 1, 7, 8, 9, 8192, 32768, 32769]:
        for shards in [1, 2, 3, 4, 8]:
            seen, sizes = 0, []
            for i in range(shards):
                b, c = hx.shard_rows(rows, shards, i)
                assert b == seen
                seen += c
                sizes.append(c)
            assert seen == rows
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(_ffi.HexirError):
        hx.shard_rows(10, 0, 0)


def cuda_available():
    return hx.device_count() > 0


@pytest.mark.skipif(cuda_available(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback_without_a_gpu():
    with pytest.raises(_ffi.HexirError) as err:
        hx.Device("cuda")
    assert err.value.status == _ffi.ERROR_DEVICE
    with pytest.raises(_ffi.HexirError):
        hx.Device("cuda:3")
    # Kernel-level calls refuse too: no host fallback behind them.
    lib = hx.lib()
    assert lib.hexir_cuda_matmul_f64(0, None, None, None, 4, 4, 4, 0, None) == \
        _ffi.ERROR_DEVICE
    assert lib.hexir_cuda_relu_f64(0, None, None, 16, None) == _ffi.ERROR_DEVICE
    assert lib.hexir_cuda_matmul_add_f64(0, None, None, None, None, 4, 4, 4, 0,
                                         None) == _ffi.ERROR_DEVICE
    for code in _ffi.ACTIVATIONS.values():
        assert lib.hexir_cuda_activation_f64(0, code, None, None, 4, 4,
                                             None) == _ffi.ERROR_DEVICE


def test_comm_arguments_are_checked_without_a_gpu():
    """The multi-process entry points check their arguments before touching
    NCCL or a GPU, and never crash on bad ones."""
    import ctypes as C
    lib = hx.lib()
    assert lib.hexir_sharded_linear_f64(None, None, None, None, 8, 8, 8, 0,
                                        None) == _ffi.ERROR_INVALID_ARGUMENT
    small = C.create_string_buffer(16)
    assert lib.hexir_comm_unique_id(small, 16) == _ffi.ERROR_INVALID_ARGUMENT
    out = C.c_void_p()
    uid = C.create_string_buffer(128)
    assert lib.hexir_comm_init_rank(uid, 128, 2, 5, 0, C.byref(out)) == \
        _ffi.ERROR_INVALID_ARGUMENT                     # rank >= nranks
    assert lib.hexir_comm_init_rank(None, 128, 2, 0, 0, C.byref(out)) == \
        _ffi.ERROR_INVALID_ARGUMENT
    assert lib.hexir_comm_rank(None) == -1 and lib.hexir_comm_size(None) == 0
    assert lib.hexir_comm_direct_stores(None) == 0
    lib.hexir_comm_release(None)  # a no-op


def test_sharded_entry_points_check_arguments_without_a_gpu():
    """The multi-GPU entry points refuse what they are not given before
    they touch a device or a collective."""
    lib = hx.lib()
    assert lib.hexir_comm_synchronize(None, None) == _ffi.ERROR_INVALID_ARGUMENT
    assert lib.hexir_sharded_linear_host_f64(
        None, None, None, None, 8, 8, 8, 0, None) == _ffi.ERROR_INVALID_ARGUMENT
    assert lib.hexir_sharded_linear_f64(
        None, None, None, None, 8, 8, 8, 0, None) == _ffi.ERROR_INVALID_ARGUMENT
    assert lib.hexir_host_register(None, 64) == _ffi.ERROR_INVALID_ARGUMENT
    assert lib.hexir_host_unregister(None) == _ffi.ERROR_INVALID_ARGUMENT
    b, c, n = C.c_uint64(), C.c_uint64(), C.c_uint32()
    assert lib.hexir_shard_gather_pieces(10, 0, None, C.byref(c), None) == \
        _ffi.ERROR_INVALID_ARGUMENT
    bounds = (C.c_uint32 * 3)()
    assert lib.hexir_shard_weight_pieces(64, 0, bounds, C.byref(n)) == \
        _ffi.ERROR_INVALID_ARGUMENT
    assert lib.hexir_shard_weight_pieces(64, 2, None, C.byref(n)) == \
        _ffi.ERROR_INVALID_ARGUMENT
