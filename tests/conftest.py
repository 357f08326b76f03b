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


def make_flow(dit_seed: int, depth: int):
    """B200Flow with the reference's random initialisation: the DiT from
    ``dit_seed``, then the CFM reseed and the front-end modules (CPU, fp32)."""
    import torch
    from fcv_b200.flow import B200Flow

    torch.manual_seed(dit_seed)
    return B200Flow(depth=depth).eval()


def flow_case(z: dict, mode: str) -> dict:
    """Per-request inputs of one mode of ``flow_frontend.npz``."""
    tl = [int(v) for v in z[f"{mode}_token_lengths"]]
    tok = z[f"{mode}_tokens"]
    cu = np.concatenate([[0], np.cumsum(tl)])
    pcu = z[f"{mode}_prompt_cu"]
    ocu = z[f"{mode}_out_cu"]
    mcu = z[f"{mode}_mu_cu"]
    R = len(tl)
    return {
        "tokens": [tok[cu[i]:cu[i + 1]] for i in range(R)],
        "prompts": [z[f"{mode}_prompt"][pcu[i]:pcu[i + 1]] for i in range(R)],
        "spk": z[f"{mode}_spk"],
        "spk_proj": z[f"{mode}_spk_proj"],
        "mu": [z[f"{mode}_mu"][mcu[i]:mcu[i + 1]] for i in range(R)],
        "out": [z[f"{mode}_out"][ocu[i]:ocu[i + 1]] for i in range(R)],
        "finalize": [bool(v) for v in z[f"{mode}_finalize"]] if f"{mode}_finalize" in z else None,
    }


def numpy_params(model) -> dict:
    return {k: v.detach().float().cpu().numpy() for k, v in model.state_dict().items()}


def hift_inputs():
    """Seeded HiFT test weights (reference state-dict format), the folded numpy
    weights for the oracle, the noise table and the golden case."""
    if str(GOLDEN) not in sys.path:
        sys.path.insert(0, str(GOLDEN))
    import hift_weights as HW

    z = load_golden("hift_case")
    sd = HW.hift_state(0)
    return sd, HW.folded(sd), HW.hift_noise(int(z["noise_rows"]), 1), z


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
