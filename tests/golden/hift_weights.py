"""Seeded HiFT test weights in the reference's state-dict format -- TEST INFRASTRUCTURE.

The reference's ``CausalHiFTGenerator`` is random-initialised by torch's global
generator and keeps its source-noise table outside the state dict, so the
golden case and the tests instead draw every parameter from numpy's
``default_rng(seed)`` here: ``make_golden.py hift`` loads them into the
reference module (``load_state_dict(strict=True)`` checks every key and shape)
and the tests load the same values into the B200 vocoder and the oracle.

Scales keep the activations of the 22-layer-deep decode of order one: each
weight-normed filter gets a norm g in [0.5, 1.0]; the f0 classifier is scaled so
that the predicted f0 spans unvoiced (<= 10) and voiced frames.
"""

from __future__ import annotations

import numpy as np
import torch

CH = (256, 128, 64)
UP_RATES, UP_KERNELS = (8, 5, 3), (16, 11, 7)
SRC_DOWN = ((30, 15), (6, 3), (1, 1))
SRC_RB_K, RB_K = (7, 7, 11), (3, 7, 11)


def conv_shapes() -> dict:
    """(C_out, C_in, k) and whether weight norm applies, per convolution path."""
    s = {"conv_pre": ((512, 80, 5), True), "conv_post": ((18, 64, 7), True)}
    for i in range(3):
        s[f"ups.{i}"] = ((CH[i], 512 if i == 0 else CH[i - 1], UP_KERNELS[i]), True)
        s[f"source_downs.{i}"] = ((CH[i], 18, SRC_DOWN[i][0]), False)
        for st in range(3):
            for c in (1, 2):
                s[f"source_resblocks.{i}.convs{c}.{st}"] = ((CH[i], CH[i], SRC_RB_K[i]), True)
    for n in range(9):
        for st in range(3):
            for c in (1, 2):
                s[f"resblocks.{n}.convs{c}.{st}"] = ((CH[n // 3], CH[n // 3], RB_K[n % 3]), True)
    s["f0_predictor.condnet.0"] = ((512, 80, 4), True)
    for i in (2, 4, 6, 8):
        s[f"f0_predictor.condnet.{i}"] = ((512, 512, 3), True)
    return s


def hift_state(seed: int = 0) -> dict:
    """State dict (float32 CPU tensors) with parametrization keys
    (``<conv>.parametrizations.weight.original0/1``)."""
    rng = np.random.default_rng(seed)
    f = np.float32
    sd = {}
    for name, ((co, ci, k), wn) in sorted(conv_shapes().items()):
        v = rng.standard_normal((co, ci, k))
        if wn:
            sd[f"{name}.parametrizations.weight.original0"] = rng.uniform(0.5, 1.0, (co, 1, 1)).astype(f)
            sd[f"{name}.parametrizations.weight.original1"] = v.astype(f)
        else:
            sd[f"{name}.weight"] = (v / np.sqrt(ci * k)).astype(f)
        sd[f"{name}.bias"] = (0.05 * rng.standard_normal(co)).astype(f)
    for prefix, count in (("source_resblocks", 3), ("resblocks", 9)):
        for n in range(count):
            c = CH[n] if prefix == "source_resblocks" else CH[n // 3]
            for st in range(3):
                for act in ("activations1", "activations2"):
                    sd[f"{prefix}.{n}.{act}.{st}.alpha"] = rng.uniform(0.5, 1.5, c).astype(f)
    sd["f0_predictor.classifier.weight"] = (4.0 * rng.standard_normal((1, 512))).astype(f)
    sd["f0_predictor.classifier.bias"] = np.array([10.0], f)
    sd["m_source.l_linear.weight"] = (0.5 * rng.standard_normal((1, 9))).astype(f)
    sd["m_source.l_linear.bias"] = np.array([0.05], f)
    return {k: torch.from_numpy(v) for k, v in sd.items()}


def hift_noise(rows: int, seed: int = 1) -> torch.Tensor:
    """(rows, 9) uniform [0, 1) source-noise table (stands in for ``sine_waves``)."""
    return torch.from_numpy(np.random.default_rng(seed).random((rows, 9)).astype(np.float32))


def folded(sd: dict) -> dict:
    """Numpy weights for the oracle: ``<conv>.weight`` with weight norm folded by
    ``torch._weight_norm`` (float64 for the f0 predictor, as its module runs)."""
    out = {}
    for k, v in sd.items():
        if k.endswith(".parametrizations.weight.original0"):
            name = k[: -len(".parametrizations.weight.original0")]
            dt = torch.float64 if name.startswith("f0_predictor") else torch.float32
            g, vv = v.to(dt), sd[f"{name}.parametrizations.weight.original1"].to(dt)
            out[f"{name}.weight"] = torch._weight_norm(vv, g, 0).numpy()
        elif not k.endswith(".original1"):
            out[k] = v.numpy()
    return out


def fingerprint(sd: dict) -> str:
    import hashlib

    h = hashlib.sha256()
    for k in sorted(sd):
        h.update(k.encode())
        h.update(sd[k].numpy().tobytes())
    return h.hexdigest()
