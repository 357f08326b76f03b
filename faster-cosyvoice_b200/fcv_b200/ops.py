"""Torch-facing wrappers of the C-ABI operators.

Names and argument meaning follow the reference's kernel wrappers
(``faster_cosyvoice/token2wav/flashinfer_kernels.py:327-438``) and its
attention runner (``flashinfer_attention.py``), so a caller of those can switch
to these.  Each wrapper only validates, allocates the output with torch and
passes device pointers plus the current stream to ``libfcv_b200.so``.
"""

from __future__ import annotations

import ctypes
from typing import Sequence

import torch

from . import _lib
from ._lib import call


def _dt(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return _lib.DTYPE_BF16
    if t.dtype == torch.float32:
        return _lib.DTYPE_F32
    raise TypeError(f"unsupported dtype {t.dtype}")


def _s(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _check_rows(*ts):
    for t in ts:
        if t.device.type != "cuda":
            raise ValueError("tensors must live on a CUDA device")


def mask_lengths(mask: torch.Tensor) -> torch.Tensor:
    """int32 document lengths from a (B, 1, T) right-padded 0/1 mask."""
    B, _, T = mask.shape
    m = mask.contiguous()
    out = torch.empty(B, dtype=torch.int32, device=mask.device)
    call("fcv_mask_lengths", m.data_ptr(), _dt(m), B, T, out.data_ptr(), _s(m))
    return out


def pack_layout(lengths: torch.Tensor, padded_length: int, num_rows: int):
    """Device pack layout from int32 device lengths: (gather int64, document_ids,
    positions, cu_seqlens, gap_rows); ``num_rows`` = sum(lengths)."""
    B = lengths.numel()
    dev = lengths.device
    gather = torch.empty(max(num_rows, 1), dtype=torch.int64, device=dev)
    doc = torch.empty(max(num_rows, 1), dtype=torch.int32, device=dev)
    pos = torch.empty(max(num_rows, 1), dtype=torch.int32, device=dev)
    cu = torch.empty(B + 1, dtype=torch.int32, device=dev)
    gap = torch.empty(num_rows + 30 * (B + 1), dtype=torch.int32, device=dev)
    call("fcv_pack_layout", lengths.data_ptr(), B, int(padded_length), int(num_rows), gather.data_ptr(),
         doc.data_ptr(), pos.data_ptr(), cu.data_ptr(), gap.data_ptr(), _s(lengths))
    return gather[:num_rows], doc[:num_rows], pos[:num_rows], cu, gap


def attention_tiles(lengths: Sequence[int], chunk: int, device) -> tuple[torch.Tensor, int]:
    """Work-list entries (doc, q0) of up to 384 query rows (three 128-row query
    tiles sharing K/V), most expensive first (host-built work list)."""
    lengths = [int(x) for x in lengths]
    cap = max(1, sum((L + 127) // 128 for L in lengths))
    buf = (ctypes.c_int32 * (2 * cap))()
    lens = (ctypes.c_int32 * max(1, len(lengths)))(*lengths)
    n = call("fcv_attn_tiles", ctypes.addressof(lens), len(lengths), int(chunk), ctypes.addressof(buf), cap)
    return torch.tensor(list(buf)[:2 * max(n, 1)], dtype=torch.int32).to(device), n


def layer_norm_modulate_packed(hidden: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor,
                               document_ids: torch.Tensor, modulation_stride: int,
                               out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """``LN(h) * scale[doc] + shift[doc]`` (``flashinfer_kernels.py:327-348``).
    ``shift``/``scale`` are float32 rows ``modulation_stride`` elements apart."""
    _check_rows(hidden, shift, scale, document_ids)
    N = hidden.shape[0]
    out = torch.empty(N, 1024, dtype=out_dtype or hidden.dtype, device=hidden.device)
    call("fcv_ln_modulate", hidden.data_ptr(), _dt(hidden), shift.data_ptr(), scale.data_ptr(),
         document_ids.data_ptr(), int(modulation_stride), N, out.data_ptr(), _dt(out), _s(hidden))
    return out


def gate_residual_layer_norm_modulate_packed(hidden, gate, residual, shift, scale, document_ids,
                                             modulation_stride: int):
    """``h += gate[doc] * r ; norm = LN(h) * scale[doc] + shift[doc]``
    (``flashinfer_kernels.py:351-378``).  Returns (hidden_out, norm)."""
    _check_rows(hidden, gate, residual, shift, scale, document_ids)
    N = hidden.shape[0]
    h_out = torch.empty_like(hidden)
    norm = torch.empty_like(hidden)
    call("fcv_gate_res_ln_modulate", hidden.data_ptr(), gate.data_ptr(), residual.data_ptr(),
         shift.data_ptr(), scale.data_ptr(), document_ids.data_ptr(), int(modulation_stride), N,
         h_out.data_ptr(), norm.data_ptr(), _dt(hidden), _s(hidden))
    return h_out, norm


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None, *,
           epilogue: int = _lib.EPI_BIAS, out: torch.Tensor | None = None, aux: torch.Tensor | None = None,
           gate: torch.Tensor | None = None, gate_stride: int = 0, rope_cos: torch.Tensor | None = None,
           rope_sin: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ weight.T + bias`` with a fused epilogue (``F.linear`` call sites
    ``flashinfer_dit.py:490, 500, 512, 535``).  bf16 runs on tcgen05 tensor
    cores, fp32 on CUDA cores.  ``bias``, ``gate`` and RoPE tables are fp32.

    * ``EPI_BIAS_ROPE_QKV``: ``aux`` = int32 positions; partial RoPE on Q/K head 0.
    * ``EPI_BIAS_GATE_RES``: ``out`` is the fp32 residual, updated in place as
      ``out += gate[aux[row]] * (x W^T + b)``; ``aux`` = int32 document ids.
    * ``EPI_BIAS_F32``: fp32 output.
    """
    _check_rows(x, weight)
    M, K = x.shape
    Nout = weight.shape[0]
    if weight.shape[1] != K or weight.dtype != x.dtype:
        raise ValueError("weight must be (Nout, K) with the dtype of x")
    if out is None:
        odt = torch.float32 if epilogue in (_lib.EPI_BIAS_F32, _lib.EPI_BIAS_GATE_RES) else x.dtype
        out = torch.empty(M, Nout, dtype=odt, device=x.device)
    call("fcv_gemm", x.data_ptr(), weight.data_ptr(), None if bias is None else bias.data_ptr(), M, Nout, K,
         _dt(x), int(epilogue), out.data_ptr(), None if aux is None else aux.data_ptr(),
         None if gate is None else gate.data_ptr(), int(gate_stride),
         None if rope_cos is None else rope_cos.data_ptr(), None if rope_sin is None else rope_sin.data_ptr(),
         _s(x))
    return out


def ragged_attention(qkv: torch.Tensor, cu_seqlens: torch.Tensor, tiles: torch.Tensor, n_tiles: int,
                     chunk: int = 0, max_len: int = 0, sched: torch.Tensor | None = None,
                     sched_ctas: int = 0) -> torch.Tensor:
    """Packed ragged attention over (N, 3072) [Q|K|V] rows (replaces
    ``RaggedAttentionRunner.wrapper.run``, ``flashinfer_dit.py:501``); chunk > 0
    applies the chunk-causal streaming mask (``flashinfer_attention.py:16-33``).
    ``sched``/``sched_ctas``: the balanced item schedule of a prepared layout
    (``PackedLayout.attn_sched``/``attn_ctas``); results do not depend on it."""
    _check_rows(qkv, cu_seqlens, tiles)
    N = qkv.shape[0]
    out = torch.empty(N, 1024, dtype=qkv.dtype, device=qkv.device)
    call("fcv_attention", qkv.data_ptr(), _dt(qkv), cu_seqlens.data_ptr(), cu_seqlens.numel() - 1, N,
         int(max_len), int(chunk), tiles.data_ptr(), int(n_tiles), None if sched is None else sched.data_ptr(),
         int(sched_ctas), out.data_ptr(), _s(qkv))
    return out


def unpack_output(packed: torch.Tensor, cu_seqlens: torch.Tensor, padded_length: int) -> torch.Tensor:
    """(N, 80) packed rows -> zero-padded (B, 80, T) (``flashinfer_dit.py:536-543``)."""
    B = cu_seqlens.numel() - 1
    out = torch.empty(B, 80, padded_length, dtype=packed.dtype, device=packed.device)
    call("fcv_unpack_output", packed.contiguous().data_ptr(), _dt(packed), cu_seqlens.data_ptr(), B,
         int(padded_length), packed.shape[0], out.data_ptr(), _s(packed))
    return out


def cfg_euler_(x: torch.Tensor, d: torch.Tensor, dt: float, cfg_rate: float,
               x_next: torch.Tensor | None = None) -> torch.Tensor:
    """In place ``x += dt * ((1+r) d[:R] - r d[R:])`` on float32 x (``flashinfer_flow.py:66-70``)."""
    R, _, T = x.shape
    call("fcv_cfg_euler", x.data_ptr(), d.data_ptr(), _dt(d), R, T, float(dt), float(cfg_rate),
         None if x_next is None else x_next.data_ptr(),
         _lib.DTYPE_BF16 if x_next is None else _dt(x_next), _s(x))
    return x


def device_error(device=None) -> int:
    """Read and clear the library's device error word (0 = none)."""
    code = ctypes.c_int(0)
    dev = torch.device(device or "cuda")
    call("fcv_device_error", ctypes.byref(code), torch.cuda.current_stream(dev).cuda_stream)
    return code.value
