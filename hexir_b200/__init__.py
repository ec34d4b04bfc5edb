"""hexir_b200 -- a B200-native (sm_100a) runtime for Hexir's GPU hot path.

The f64 hexir.linear (FP64 tensor-core DMMA GEMM, TMA-fed, relu fused in the
epilogue) and the elementwise hexir.relu / hexir.add (plus, on request, the
dialect's declared activations leaky_relu ... mish), behind the reference's
surface: the .hxb module format, the HAL / module / VM C ABI
(include/hexir_runtime), the hexir-run tool, and the -placement= syntax
(extended with cuda:N and row-sharded cuda:F-L).  See include/ for the C ABI;
this package is a thin Python face over it.
"""

from ._ffi import HexirError, lib  # noqa: F401
from .api import (Buffer, Device, Module, Program, Rng, cuda_activation,  # noqa: F401
                  cuda_add, cuda_matmul, cuda_matmul_acc, cuda_matmul_add, cuda_relu,
                  cuda_synchronize, device_count, fault_calls,
                  fault_configure,
                  execute, kernel_image, last_kernel_ms, launch_count,
                  matmul_plan, parse, read_executables, read_launch,
                  read_program,
                  read_sections, shard_gather_pieces, shard_rows,
                  shard_weight_pieces)
