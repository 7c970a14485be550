"""Shared test setup: import paths, the `gpu` marker, tolerance helpers."""
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
for p in (REPO, REPO / "rust-fp4-blackwell_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long-running")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def rel_floor(got, ref, floor=1e-3):
    """The reference's gate metric: |got - ref| / max(|ref|, floor) per element
    (examples/fp4_gemv/src/main.rs:165-166, llama_rmsnorm/src/main.rs:98)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return np.abs(got - ref) / np.maximum(np.abs(ref), floor)


def rel_rms(got, ref):
    """Per-element relative error with the output's RMS as the floor:
    |got - ref| / max(|ref|, rms(ref)).  Used for fp32-accumulated dot products,
    where a pure per-element relative error is undefined at cancellation."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    rms = np.sqrt(np.mean(ref * ref)) if ref.size else 1.0
    return np.abs(got - ref) / np.maximum(np.abs(ref), max(rms, 1e-30))
