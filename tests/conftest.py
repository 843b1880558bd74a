"""Shared test setup: markers, import paths, the oracle and the CUDA package.

`-m "not gpu"` runs the oracle pins, host logic and C-ABI load checks on any
machine; `-m gpu` runs the parity tests proper, which call the CUDA library
through its C-ABI and check it against the CPU oracle.
"""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def O():
    """The oracle module (oracle/oracle.py), built on first use."""
    import oracle as _o
    if not os.path.exists(_o.ORACLE_SO):
        _o.build()
    return _o


@pytest.fixture(scope="session")
def orc(O):
    return O.oracle()


@pytest.fixture(scope="session")
def ref(O):
    """The reference's own host code, or skip where it was never built."""
    r = O.reference()
    if r is None:
        pytest.skip("oracle/_ref/libqgemm_ref.so not built (reference tree absent)")
    return r


@pytest.fixture(scope="session")
def qg():
    """The CUDA package (imports fail loudly if the library is missing)."""
    return importlib.import_module("qgemm-mx_b200")


@pytest.fixture(autouse=True)
def _no_bounded_wait_gave_up(request):
    """After every GPU test: no bounded device wait of a GEMM kernel gave up
    during it (its outputs would be wrong even where a sampled check passed).
    Tests that make a wait run out on purpose use other flags (tp, probe)."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    mod = sys.modules.get("qgemm-mx_b200")
    if mod is None:
        return
    import ctypes as C
    import torch
    if not torch.cuda.is_available():
        return
    torch.cuda.synchronize()
    f = C.c_int32(0)
    if mod.lib().qgemm_umma_status(C.byref(f)) != mod.OK:
        msg = mod.lib().qgemm_last_error_message().decode()
        mod.clear_faults()
        pytest.fail(f"a bounded device wait gave up: {msg}", pytrace=False)


@pytest.fixture(scope="session")
def cuda(qg):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
