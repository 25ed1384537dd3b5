import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100) and libbybycuda.so")


def _have_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _have_gpu():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


PARITY_LOG = []


@pytest.fixture(scope="session")
def parity_log():
    """Tests append (what, worst per-element error, bound) here; the terminal summary prints
    every entry, so a green run still shows the measured worst cases."""
    return PARITY_LOG


def pytest_terminal_summary(terminalreporter):
    if PARITY_LOG:
        terminalreporter.write_sep("-", "measured parity (worst |got - want| / max(1, |want|) per element)")
        for what, worst, bound in PARITY_LOG:
            terminalreporter.write_line(f"{what}: {worst:.3e} (bound {bound:.0e})")


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    d = os.path.join(ROOT, "tests", "golden")
    return {name: dict(np.load(os.path.join(d, f"{name}.npz")))
            for name in ("ref_tile_cases", "ref_gate", "ref_q4b32")}
