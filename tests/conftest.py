"""Shared pytest setup: the `gpu` marker, the repo root on sys.path, built artefacts.

`-m "not gpu"` runs the CPU suite (oracle vs golden vectors / known answers,
host logic, library load + exports). `-m gpu` runs parity of the CUDA kernels
through the C ABI against the CPU oracle on a B200.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def reference_dir():
    """The reference source tree for the tests that build against it: $CLOVE_REF_DIR,
    else a `reference` directory beside this repository; None when absent (as on the
    GPU hosts)."""
    d = os.environ.get("CLOVE_REF_DIR") or os.path.join(ROOT, "..", "reference")
    d = os.path.abspath(d)
    return d if os.path.isdir(os.path.join(d, "src", "kernels")) else None


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def clove_lib():
    """The product library, built if missing (nvcc cross-compiles without a GPU)."""
    from clove_compute_b200 import build as b
    if not os.path.exists(b.LIB):
        b.build()
    import clove_compute_b200 as cc
    return cc


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, _ = torch.cuda.get_device_capability()
    assert major == 10, "GPU tests need an sm_100 (B200) device"
    return torch.device("cuda:0")
