"""CFG-doubled batched Euler solver on the B200 estimator.

Mirror of ``solve_euler_batched`` (reference ``faster_cosyvoice/token2wav/flashinfer_flow.py:16-74``):
cosine schedule in the input dtype, the ``[cond; uncond]`` stack with mu,
speaker embedding and condition zeroed in the second half, ``x.repeat(2)``,
``d = (1 + r) d_c - r d_u`` and ``x += dt d``.

Differences that only remove work: the packed layout is computed once per
call (the mask is the same for all steps), the CFG combine, the Euler update
and the next step's repeated input are one fused kernel (``fcv_cfg_euler``),
and the sample is carried in float32 between steps.
"""

from __future__ import annotations

import math

import torch

from . import _lib
from ._lib import call
from .model import B200DiT, _dtype_code, _stream


def cosine_schedule(num_timesteps: int, dtype: torch.dtype) -> list[float]:
    """``1 - cos(linspace(0, 1, n+1) * pi/2)`` computed in ``dtype`` on the host
    (``flashinfer_flow.py:34-41``)."""
    span = torch.linspace(0, 1, num_timesteps + 1, dtype=dtype)
    span = 1 - torch.cos(span * 0.5 * torch.pi)
    return span


@torch.inference_mode()
def solve_euler_batched(decoder, noise: torch.Tensor, mu: torch.Tensor, mask: torch.Tensor,
                        speaker_embeddings: torch.Tensor, condition: torch.Tensor,
                        num_timesteps: int = 10, streaming: bool = False) -> torch.Tensor:
    """Run the classifier-free-guidance Euler solver for a padded batch.

    ``decoder.estimator`` must be a finalized :class:`B200DiT`;
    ``decoder.inference_cfg_rate`` is the guidance rate (0.7 for CosyVoice3).
    Returns the sample in ``speaker_embeddings.dtype`` with shape of ``noise``.
    """
    est: B200DiT = decoder.estimator
    if not isinstance(est, B200DiT):
        raise TypeError("decoder.estimator must be a B200DiT")
    rate = float(decoder.inference_cfg_rate)
    dev = est.proj_out.weight.device
    dt_w = est.weight_dtype
    sdtype = speaker_embeddings.dtype
    with torch.cuda.device(dev):
        R, C, T = noise.shape[0], noise.shape[1], noise.shape[2]
        mu = mu.to(dev)
        span = cosine_schedule(num_timesteps, sdtype)
        t = span[0]
        step = span[1] - span[0]

        mask_in = mask.to(dev).repeat(2, 1, 1)
        layout = est.layout_from_mask(mask_in, streaming)
        mu_in = torch.cat([mu, torch.zeros_like(mu)], 0).to(dt_w).contiguous()
        spk_in = torch.cat([speaker_embeddings.to(dev), torch.zeros_like(speaker_embeddings.to(dev))], 0)
        spk_in = spk_in.to(dt_w).contiguous()
        cond = condition.to(dev)
        cond_in = torch.cat([cond, torch.zeros_like(cond)], 0).to(dt_w).contiguous()

        # a private fp32 copy: the update is in place and must not touch the caller's noise
        x = noise.to(device=dev, dtype=sdtype).to(torch.float32, copy=True).contiguous()
        x_in = x.repeat(2, 1, 1).to(dt_w).contiguous()
        d = torch.empty(2 * R, C, T, dtype=torch.float32, device=dev)  # flow field kept in fp32
        t_in = torch.empty(2 * R, dtype=dt_w, device=dev)
        stream = _stream(dev)
        for k in range(1, num_timesteps + 1):
            t_in.fill_(float(t))
            est.forward_layout(layout, x_in, mu_in, t_in, spk_in, cond_in, out=d)
            nxt = x_in.data_ptr() if k < num_timesteps else None
            call("fcv_cfg_euler", x.data_ptr(), d.data_ptr(), _lib.DTYPE_F32, R, T, float(step), rate, nxt,
                 _dtype_code(dt_w), stream)
            t = t + step
            if k < num_timesteps:
                step = span[k + 1] - t
        return x.to(sdtype)
