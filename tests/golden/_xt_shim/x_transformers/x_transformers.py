"""Test-only restatement of the two rotary helpers the reference DiT imports
from ``x_transformers.x_transformers`` (``dit.py:17``, ``modules.py:20``).

Semantics follow the reference's own restatements of the same maths:
``flashinfer_dit.py:262-273`` (tables, "x_transformers semantics"),
``flashinfer_dit.py:586-594`` (complex multiply on interleaved pairs) and
``flashinfer_kernels.py:167-192``: rotary dim = dim_head (64), base 10000,
positions 0..L-1, interleaved pairs (2j, 2j+1), no xpos scaling.
Used only to import the reference in this container for fixture generation.
"""
import torch
from torch import nn


class RotaryEmbedding(nn.Module):
    def __init__(self, dim, use_xpos=False, scale_base=512, interpolation_factor=1.0,
                 base=10000, base_rescale_factor=1.0):
        super().__init__()
        base = base * base_rescale_factor ** (dim / (dim - 2))
        inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2).float() / dim))
        self.register_buffer("inv_freq", inv_freq)
        self.interpolation_factor = interpolation_factor

    def forward_from_seq_len(self, seq_len):
        t = torch.arange(seq_len, device=self.inv_freq.device)
        return self.forward(t)

    def forward(self, t):
        if t.ndim == 1:
            t = t[None, :]
        freqs = torch.einsum("bi,j->bij", t.type_as(self.inv_freq), self.inv_freq)
        freqs = freqs / self.interpolation_factor
        freqs = torch.stack((freqs, freqs), dim=-1).flatten(-2)
        return freqs, 1.0


def _rotate_half(x):
    x = x.unflatten(-1, (-1, 2))
    x1, x2 = x.unbind(dim=-1)
    return torch.stack((-x2, x1), dim=-1).flatten(-2)


def apply_rotary_pos_emb(t, freqs, scale=1):
    rot_dim, seq_len, orig_dtype = freqs.shape[-1], t.shape[-2], t.dtype
    freqs = freqs[:, -seq_len:, :]
    if t.ndim == 4 and freqs.ndim == 3:
        freqs = freqs[:, None]
    t_rot, t_pass = t[..., :rot_dim], t[..., rot_dim:]
    t_rot = t_rot * freqs.cos() * scale + _rotate_half(t_rot) * freqs.sin() * scale
    return torch.cat((t_rot, t_pass), dim=-1).type(orig_dtype)
