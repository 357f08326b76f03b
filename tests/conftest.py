"""Shared fixtures.  GPU tests are marked ``gpu``; everything else runs on CPU."""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "faster-cosyvoice_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def golden_fingerprints() -> dict:
    return json.loads((GOLDEN / "weights_fingerprint.json").read_text())


def make_model(seed: int, depth: int):
    """B200DiT with the reference's random initialisation for ``seed`` (CPU, fp32)."""
    import torch
    from fcv_b200.model import B200DiT

    torch.manual_seed(seed)
    return B200DiT(depth=depth).eval()


def numpy_params(model) -> dict:
    return {k: v.detach().float().cpu().numpy() for k, v in model.state_dict().items()}


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="session")
def golden():
    return load_golden


def ensure_built():
    """Build the CUDA library in-tree if it is missing or stale (nvcc cross-compiles)."""
    from fcv_b200 import build

    build.build()
    return build.LIB


def cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False
