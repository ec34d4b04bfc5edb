"""Test configuration.

Markers:
  gpu  -- needs an sm_100 GPU; run with `pytest -m gpu` on a B200.  Every
          other test runs on a CPU-only machine.

The session fixture builds the in-tree library and the oracle once if they
are missing (the same `make` that __graft_entry__.build() runs).
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


@pytest.fixture(scope="session", autouse=True)
def built():
    from hexir_b200 import _ffi
    from hexir_b200.build import build
    from oracle import oracle
    if not os.path.exists(_ffi.LIB_PATH):
        build()
    if not os.path.exists(oracle.ORACLE_SO):
        oracle.build()
    return True


@pytest.fixture(scope="session")
def gpu():
    """CUDA device 0 through the HAL; the test fails (not skips) without one,
    because gpu-marked tests only run where a GPU is expected."""
    import hexir_b200 as hx
    dev = hx.Device("cuda")
    yield dev
    dev.close()


def bin_path(name: str) -> str:
    return os.path.join(ROOT, "hexir_b200", "bin", name)


def free_port() -> int:
    """A TCP port on 127.0.0.1 that was free a moment ago."""
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def spawn_ranks(fn, nprocs: int, args: tuple, attempts: int = 3) -> None:
    """torch.multiprocessing spawn of `nprocs` ranks of fn(rank, nprocs, port,
    *args), joined.  The rendezvous port is picked free but can be taken
    before rank 0 binds it; that (EADDRINUSE) is retried with a new port."""
    import torch.multiprocessing as mp
    for attempt in range(attempts):
        try:
            mp.start_processes(fn, args=(nprocs, free_port()) + tuple(args),
                               nprocs=nprocs, join=True, start_method="spawn")
            return
        except mp.ProcessRaisedException as err:
            if "EADDRINUSE" not in str(err) or attempt + 1 == attempts:
                raise
