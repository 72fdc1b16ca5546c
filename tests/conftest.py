"""Shared test setup: import paths, the ``gpu`` marker, and helpers for parity checks."""

import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "tensorquay-engine_b200"
GOLDEN = ROOT / "tests" / "golden"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


def pytest_collection_modifyitems(config, items):
    # A GPU test fails (never skips) when no GPU is present: the reference's rule
    # (docs/ARCHITECTURE.md:55). Selection is by marker only.
    pass


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"sm_100 required, found sm_{major}{minor}"
    return torch.device("cuda", 0)


# Tolerances for bf16 inputs with f32 accumulation (out: max-abs and relative L2; lse: abs).
OUT_MAX_ABS = 2e-2
OUT_REL_L2 = 1e-2
LSE_ABS = 1e-3


def assert_parity(out, lse, ref_out, ref_lse, *, label="", lse_abs=LSE_ABS,
                  out_abs=None, out_rel=None):
    """Compare a kernel result (float64 arrays) with the oracle: north-star tolerances, unless a
    caller whose inputs differ from the oracle's by a stated amount passes wider ones."""
    out_abs = OUT_MAX_ABS if out_abs is None else out_abs
    out_rel = OUT_REL_L2 if out_rel is None else out_rel
    out = np.asarray(out, dtype=np.float64)
    lse = np.asarray(lse, dtype=np.float64)
    assert out.shape == ref_out.shape and lse.shape == ref_lse.shape, label
    assert np.isfinite(out).all(), f"{label}: non-finite output"
    ninf = np.isneginf(ref_lse)
    np.testing.assert_array_equal(np.isneginf(lse), ninf, err_msg=f"{label}: -inf lse pattern")
    if (~ninf).any():
        err = np.abs(lse[~ninf] - ref_lse[~ninf]).max()
        assert err <= lse_abs, f"{label}: lse max abs err {err:.3e}"
    assert (out[ninf] == 0).all(), f"{label}: empty rows must be exact zeros"
    diff = np.abs(out - ref_out).max() if out.size else 0.0
    assert diff <= out_abs, f"{label}: out max abs err {diff:.3e}"
    denom = np.linalg.norm(ref_out)
    if denom > 0:
        rel = np.linalg.norm(out - ref_out) / denom
        assert rel <= out_rel, f"{label}: out rel L2 {rel:.3e}"
