import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "npu-embeddings-xdna1_b200"
for p in (str(PKG), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)

# PyTorch (device buffers, streams and gloo ranks in the tests) loads its own
# NCCL with libtorch; it is imported first so that libnebw's communicator
# calls use that copy (the dynamic loader shares one libnccl.so.2 per process)
try:
    import torch  # noqa: F401
except ImportError:
    pass

# the reference tree (read-only; present only where the reference is checked
# out): $NEBW_REFERENCE, else a checkout beside this repository
REFERENCE = Path(os.environ.get("NEBW_REFERENCE", str(REPO.parent / "reference")))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a) and libnebw.so")


def has_reference() -> bool:
    return (REFERENCE / "tools" / "lib" / "npue.py").exists()


@pytest.fixture(scope="session")
def port_oracle():
    from oracle.oracle import PortOracle

    return PortOracle()


@pytest.fixture(scope="session")
def ref_oracle():
    from oracle.oracle import REF_LIB, RefOracle

    if not REF_LIB.exists():
        pytest.skip("the reference's host path is not built here (oracle/_ref)")
    return RefOracle()


@pytest.fixture(scope="session")
def device():
    import nebw

    dev = nebw.Device(0, torch_stream=True)
    yield dev
    dev.close()


def parity(got, want):
    """(min per-row cosine, max abs diff) between two [rows, H] arrays."""
    import numpy as np

    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    cos = (got * want).sum(1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(want, axis=1))
    return float(cos.min()), float(np.abs(got - want).max())
