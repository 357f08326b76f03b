"""``B200DiT``: the packed DiT estimator with the reference module interface.

Drop-in for ``FlashInferDiT`` (reference ``faster_cosyvoice/token2wav/flashinfer_dit.py:98-362``):

* the module tree, and therefore the state dict, equals the reference
  CosyVoice3 ``DiT`` (``cosyvoice/flow/DiT/dit.py:104-143``) -- keys such as
  ``transformer_blocks.{i}.attn.to_q.weight`` -- and parameters are created in
  the same order, so ``torch.manual_seed(s)`` followed by construction yields
  the same random initialisation as the reference constructor;
* ``finalize_weights()`` derives the fused inference weights once
  (``flashinfer_dit.py:228-313``; a second call raises ``RuntimeError``);
* ``forward(x, mask, mu, t, spks=None, cond=None, streaming=False)`` returns
  ``(B, 80, T)`` (``flashinfer_dit.py:315-362``; ``ValueError`` without spks/cond).

All GPU work runs in ``libfcv_b200.so`` through its C ABI; this module only
owns tensors (weights, layouts, workspace) and passes device pointers.
"""

from __future__ import annotations

import ctypes
from collections import OrderedDict
from dataclasses import dataclass
from typing import Sequence

import torch
import torch.nn as nn

from . import _lib
from ._lib import DitBatch, DitWeights, call, lib

DIM = 1024
HEADS = 16
DIM_HEAD = 64
MEL = 80
CONV_K = 31
CONV_GROUPS = 16
ROPE_DIM = 64
ROPE_TABLE_LEN = 16384  # positions covered by the RoPE tables (the reference stops at 4096)
MAX_LAYOUT_CACHE = 64   # flashinfer_dit.py:62


# ---------------------------------------------------------------------------
# Module tree (same names, shapes and creation order as the reference DiT)
# ---------------------------------------------------------------------------

class _TimeEmbedding(nn.Module):
    def __init__(self, dim: int, freq_dim: int = 256):
        super().__init__()
        self.time_mlp = nn.Sequential(nn.Linear(freq_dim, dim), nn.SiLU(), nn.Linear(dim, dim))


class _CausalConvPos(nn.Module):
    def __init__(self, dim: int, kernel_size: int = CONV_K, groups: int = CONV_GROUPS):
        super().__init__()
        self.conv1 = nn.Sequential(nn.Conv1d(dim, dim, kernel_size, groups=groups, padding=0), nn.Mish())
        self.conv2 = nn.Sequential(nn.Conv1d(dim, dim, kernel_size, groups=groups, padding=0), nn.Mish())


class _InputEmbedding(nn.Module):
    def __init__(self, mel_dim: int, mu_dim: int, out_dim: int, spk_dim: int):
        super().__init__()
        self.proj = nn.Linear(mel_dim * 2 + mu_dim + spk_dim, out_dim)
        self.conv_pos_embed = _CausalConvPos(out_dim)


class _Rotary(nn.Module):
    def __init__(self, dim: int):
        super().__init__()
        self.register_buffer("inv_freq", 1.0 / (10000 ** (torch.arange(0, dim, 2).float() / dim)))


class _AdaLNZero(nn.Module):
    def __init__(self, dim: int, chunks: int):
        super().__init__()
        self.linear = nn.Linear(dim, dim * chunks)


class _Attention(nn.Module):
    def __init__(self, dim: int, heads: int, dim_head: int, dropout: float):
        super().__init__()
        inner = heads * dim_head
        self.to_q = nn.Linear(dim, inner)
        self.to_k = nn.Linear(dim, inner)
        self.to_v = nn.Linear(dim, inner)
        self.to_out = nn.ModuleList([nn.Linear(inner, dim), nn.Dropout(dropout)])


class _FeedForward(nn.Module):
    def __init__(self, dim: int, mult: int, dropout: float):
        super().__init__()
        inner = dim * mult
        self.ff = nn.Sequential(nn.Sequential(nn.Linear(dim, inner), nn.GELU(approximate="tanh")),
                                nn.Dropout(dropout), nn.Linear(inner, dim))


class _Block(nn.Module):
    def __init__(self, dim: int, heads: int, dim_head: int, ff_mult: int, dropout: float):
        super().__init__()
        self.attn_norm = _AdaLNZero(dim, 6)
        self.attn = _Attention(dim, heads, dim_head, dropout)
        self.ff = _FeedForward(dim, ff_mult, dropout)


# ---------------------------------------------------------------------------
# Packed layout ("plan") of one batch composition
# ---------------------------------------------------------------------------

@dataclass
class PackedLayout:
    """Device index arrays of one batch composition (``flashinfer_dit.py:75-82``
    plus the attention work list that replaces the FlashInfer plan)."""

    lengths: tuple
    padded_length: int
    chunk: int
    N: int
    max_len: int
    lengths_dev: torch.Tensor
    cu_seqlens: torch.Tensor
    gather_indices: torch.Tensor
    document_ids: torch.Tensor
    positions: torch.Tensor
    gap_rows: torch.Tensor
    attn_tiles: torch.Tensor
    n_attn_tiles: int
    attn_sched: torch.Tensor | None = None  # per-CTA items (fcv_attn_schedule)
    attn_ctas: int = 0


@dataclass
class PrefixState:
    """Cached-prefix arguments of one estimator call (streaming prefix reuse,
    see ``fcv_dit_batch``): absolute positions of the new rows, each document's
    prefix length and first cache row, this ODE step's K/V cache
    (depth x layer_rows x 2048) and the convolutions' left context in and out
    ((B, 2, 30, 1024) each; ctx_row0 = local row where the next call starts)."""

    positions: torch.Tensor
    doc_pos0: torch.Tensor
    doc_kv_base: torch.Tensor
    kv_cache: torch.Tensor
    layer_rows: int
    conv_ctx: torch.Tensor
    conv_ctx_out: torch.Tensor | None = None
    ctx_row0: torch.Tensor | None = None
    max_pos: int = 0


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _dtype_code(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return _lib.DTYPE_BF16
    if dtype == torch.float32:
        return _lib.DTYPE_F32
    raise ValueError(f"unsupported estimator dtype {dtype}; use torch.bfloat16 or torch.float32")


class B200DiT(nn.Module):
    """State-dict-compatible packed DiT estimator running on ``libfcv_b200``."""

    def __init__(self, dim: int = DIM, depth: int = 22, heads: int = HEADS, dim_head: int = DIM_HEAD,
                 ff_mult: int = 2, mel_dim: int = MEL, mu_dim: int = MEL, spk_dim: int = MEL,
                 out_channels: int = MEL, static_chunk_size: int = 50, dropout: float = 0.1,
                 use_cuda_graph: bool = False, graph_buckets: Sequence[int] | None = None):
        super().__init__()
        if (dim, heads, dim_head, ff_mult, mel_dim, mu_dim, spk_dim) != (DIM, HEADS, DIM_HEAD, 2, MEL, MEL, MEL):
            raise ValueError("the kernels implement the CosyVoice3 geometry "
                             "(dim 1024, 16x64 heads, ff_mult 2, mel/mu/spk 80)")
        self._chunk_size = static_chunk_size
        self.static_chunk_size = static_chunk_size
        self.dim = dim
        self.depth = depth
        self.heads = heads
        self.dim_head = dim_head
        self.out_channels = out_channels
        # creation order of dit.py:124-141
        self.time_embed = _TimeEmbedding(dim)
        self.input_embed = _InputEmbedding(mel_dim, mu_dim, dim, spk_dim)
        self.rotary_embed = _Rotary(dim_head)
        self.transformer_blocks = nn.ModuleList(
            [_Block(dim, heads, dim_head, ff_mult, dropout) for _ in range(depth)])
        self.norm_out = _AdaLNZero(dim, 2)
        self.proj_out = nn.Linear(dim, mel_dim)

        self.use_cuda_graph = use_cuda_graph
        # row capacities of the bucketed graphs (None: one graph per exact layout)
        self.graph_buckets = tuple(sorted({int(b) for b in graph_buckets})) if graph_buckets else None
        self._bucket_graphs: OrderedDict = OrderedDict()
        self.bucket_captures = 0
        # balanced (LPT) attention schedule per batch composition; False deals items round robin
        self.use_attn_schedule = True
        # AdaLN modulation rows per timestep value (the ODE schedule's t values repeat on every call)
        self._mod_cache: dict = {}
        self._mod_ws: torch.Tensor | None = None
        self._stage: OrderedDict = OrderedDict()  # device buffers for host inputs
        self._copy_stream: torch.cuda.Stream | None = None
        self._finalized = False
        self._derived: dict[str, torch.Tensor] = {}
        self._graphs: OrderedDict = OrderedDict()
        self._weights: DitWeights | None = None
        self._layouts: OrderedDict = OrderedDict()
        self._workspace: torch.Tensor | None = None
        self.plan_calls = 0

    # ------------------------------------------------------------------ weights
    @property
    def weight_dtype(self) -> torch.dtype:
        return self.proj_out.weight.dtype

    @torch.no_grad()
    def finalize_weights(self) -> None:
        """Derive the fused inference weights (``flashinfer_dit.py:228-313``).

        Matrices keep the module dtype (bf16 or fp32); biases and RoPE tables
        are fp32.  ``1 + scale`` is folded into the AdaLN scale biases in fp32.
        """
        if self._finalized:
            raise RuntimeError("B200DiT weights have already been finalized")
        dev = self.proj_out.weight.device
        if dev.type != "cuda":
            raise RuntimeError("B200DiT.finalize_weights() needs the module on a CUDA device")
        dt = self.weight_dtype
        _dtype_code(dt)
        self._finalized = True

        def mat(t):
            return t.detach().to(device=dev, dtype=dt).contiguous()

        def vec(t):
            return t.detach().to(device=dev, dtype=torch.float32).contiguous()

        blocks = self.transformer_blocks
        d = {}
        d["time_w1"] = mat(self.time_embed.time_mlp[0].weight)
        d["time_b1"] = vec(self.time_embed.time_mlp[0].bias)
        d["time_w2"] = mat(self.time_embed.time_mlp[2].weight)
        d["time_b2"] = vec(self.time_embed.time_mlp[2].bias)
        d["ada_w"] = mat(torch.cat([b.attn_norm.linear.weight for b in blocks] + [self.norm_out.linear.weight], 0))
        ada_b = torch.cat([vec(b.attn_norm.linear.bias) for b in blocks] + [vec(self.norm_out.linear.bias)], 0)
        for i in range(self.depth):  # chunk order shift, scale, gate, shift, scale, gate (modules.py:241)
            ada_b[i * 6 * DIM + 1 * DIM:i * 6 * DIM + 2 * DIM] += 1.0
            ada_b[i * 6 * DIM + 4 * DIM:i * 6 * DIM + 5 * DIM] += 1.0
        ada_b[self.depth * 6 * DIM:self.depth * 6 * DIM + DIM] += 1.0  # final (scale, shift)
        d["ada_b"] = ada_b.contiguous()
        d["in_w"] = mat(self.input_embed.proj.weight)
        d["in_b"] = vec(self.input_embed.proj.bias)
        for name, conv in (("conv1", self.input_embed.conv_pos_embed.conv1[0]),
                           ("conv2", self.input_embed.conv_pos_embed.conv2[0])):
            w = conv.weight  # (1024 out, 64 in per group, 31 taps) -> [g*64+co, tap*64+ci]
            d[f"{name}_w"] = mat(w.permute(0, 2, 1).reshape(DIM, CONV_K * (DIM // CONV_GROUPS)))
            d[f"{name}_b"] = vec(conv.bias)
        d["qkv_w"] = mat(torch.stack([torch.cat([b.attn.to_q.weight, b.attn.to_k.weight, b.attn.to_v.weight], 0)
                                      for b in blocks]))
        d["qkv_b"] = torch.stack([torch.cat([vec(b.attn.to_q.bias), vec(b.attn.to_k.bias), vec(b.attn.to_v.bias)])
                                  for b in blocks]).contiguous()
        d["o_w"] = mat(torch.stack([b.attn.to_out[0].weight for b in blocks]))
        d["o_b"] = torch.stack([vec(b.attn.to_out[0].bias) for b in blocks]).contiguous()
        d["ff1_w"] = mat(torch.stack([b.ff.ff[0][0].weight for b in blocks]))
        d["ff1_b"] = torch.stack([vec(b.ff.ff[0][0].bias) for b in blocks]).contiguous()
        d["ff2_w"] = mat(torch.stack([b.ff.ff[2].weight for b in blocks]))
        d["ff2_b"] = torch.stack([vec(b.ff.ff[2].bias) for b in blocks]).contiguous()
        d["out_w"] = mat(self.proj_out.weight)
        d["out_b"] = vec(self.proj_out.bias)
        # partial-RoPE tables, fp32 (flashinfer_dit.py:262-273)
        inv = (1.0 / (10000 ** (torch.arange(0, ROPE_DIM, 2, dtype=torch.float32) / ROPE_DIM)))
        theta = torch.arange(ROPE_TABLE_LEN, dtype=torch.float32)[:, None] * inv[None, :]
        d["rope_cos"] = theta.cos().to(dev).contiguous()
        d["rope_sin"] = theta.sin().to(dev).contiguous()
        self._derived = d
        w = DitWeights()
        w.depth = self.depth
        w.dtype = _dtype_code(dt)
        for k, v in d.items():
            setattr(w, k, v.data_ptr())
        w.rope_max_len = ROPE_TABLE_LEN
        self._weights = w

    def weights_struct(self) -> DitWeights:
        if self._weights is None:
            raise RuntimeError("call finalize_weights() first")
        return self._weights

    def shared_modulations(self, t: float) -> torch.Tensor:
        """The AdaLN modulation row (depth * 6144 + 2048 floats) of timestep ``t``
        rounded to the weight dtype, computed once per value and kept: the ODE
        solver's documents share t and its ten schedule values repeat on every
        call, so the time embedding and the 281 MB modulation GEMM run once per
        value instead of once per estimator call."""
        dev, dt = self.proj_out.weight.device, self.weight_dtype
        tv = torch.tensor([float(t)], dtype=dt)
        key = float(tv.float().item())
        row = self._mod_cache.get(key)
        if row is None:
            need = int(lib().fcv_dit_workspace_bytes(0, 1, self.depth, _dtype_code(dt)))
            if self._mod_ws is None or self._mod_ws.numel() < need:
                self._mod_ws = torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
            row = torch.empty(self.depth * 6144 + 2048, dtype=torch.float32, device=dev)
            t_dev = tv.to(dev)
            call("fcv_dit_modulations", ctypes.byref(self.weights_struct()), t_dev.data_ptr(), row.data_ptr(),
                 self._mod_ws.data_ptr(), self._mod_ws.numel(), _stream(dev))
            self._mod_cache[key] = row
        return row

    # ------------------------------------------------------------------ layout
    def prepare_layout(self, lengths: Sequence[int], padded_length: int, streaming: bool,
                       device: torch.device | None = None, lengths_dev: torch.Tensor | None = None) -> PackedLayout:
        """Packed layout + attention work list for a batch composition, cached
        in a FIFO of 64 entries (``flashinfer_dit.py:364-405`` and the plan
        pool of ``:192-226``)."""
        device = device or self.proj_out.weight.device
        lengths = tuple(int(x) for x in lengths)
        chunk = self._chunk_size if streaming else 0
        key = (lengths, int(padded_length), chunk)
        lay = self._layouts.get(key)
        if lay is not None:
            return lay
        self.plan_calls += 1
        B = len(lengths)
        if B < 1:
            raise ValueError("empty batch")
        if any(L < 0 or L > padded_length for L in lengths):
            raise ValueError("document lengths must lie in [0, T]")
        N = sum(lengths)
        stream = _stream(device)
        if lengths_dev is None:
            lengths_dev = torch.tensor(lengths, dtype=torch.int32).to(device, non_blocking=True)
        cu = torch.empty(B + 1, dtype=torch.int32, device=device)
        gather = torch.empty(max(N, 1), dtype=torch.int64, device=device)
        doc_ids = torch.empty(max(N, 1), dtype=torch.int32, device=device)
        positions = torch.empty(max(N, 1), dtype=torch.int32, device=device)
        gap_rows = torch.empty(N + 30 * (B + 1), dtype=torch.int32, device=device)
        call("fcv_pack_layout", lengths_dev.data_ptr(), B, int(padded_length), N, gather.data_ptr(),
             doc_ids.data_ptr(), positions.data_ptr(), cu.data_ptr(), gap_rows.data_ptr(), stream)
        cap = sum((L + 127) // 128 for L in lengths)
        ctas = int(lib().fcv_attn_ctas(cap))
        # one host block, one upload: work list (2 * cap) then the balanced schedule
        host = (ctypes.c_int32 * (2 * max(cap, 1) + ctas + 1 + 16 * cap))()
        lens_host = (ctypes.c_int32 * B)(*lengths)
        n_tiles = call("fcv_attn_tiles", ctypes.addressof(lens_host), B, chunk, ctypes.addressof(host), cap)
        ctas = int(call("fcv_attn_ctas", n_tiles))
        s_off = 2 * max(n_tiles, 1)
        n_sched = call("fcv_attn_schedule", ctypes.addressof(lens_host), B, chunk, ctypes.addressof(host), n_tiles,
                       ctas, ctypes.addressof(host) + 4 * s_off, len(host) - s_off)
        block = torch.frombuffer(host, dtype=torch.int32)[:s_off + n_sched].clone().to(device)
        tiles, sched = block[:s_off], block[s_off:]
        lay = PackedLayout(lengths, int(padded_length), chunk, N, max(lengths) if lengths else 0, lengths_dev,
                           cu, gather[:N], doc_ids[:N], positions[:N], gap_rows, tiles, n_tiles, sched, ctas)
        if len(self._layouts) >= MAX_LAYOUT_CACHE:
            self._layouts.popitem(last=False)
        self._layouts[key] = lay
        return lay

    def layout_from_mask(self, mask: torch.Tensor, streaming: bool) -> PackedLayout:
        """Document lengths from the (B, 1, T) mask (``flashinfer_dit.py:460``),
        counted on the device and read back once, like the reference's
        ``.tolist()`` (``:370``)."""
        B, _, T = mask.shape
        m = mask.to(self.weight_dtype).contiguous()
        lengths_dev = torch.empty(B, dtype=torch.int32, device=mask.device)
        call("fcv_mask_lengths", m.data_ptr(), _dtype_code(m.dtype), B, T, lengths_dev.data_ptr(),
             _stream(mask.device))
        lengths = lengths_dev.cpu().tolist()
        return self.prepare_layout(lengths, T, streaming, mask.device, lengths_dev)

    # ------------------------------------------------------------------ forward
    def _workspace_for(self, N: int, B: int, device: torch.device) -> torch.Tensor:
        need = int(lib().fcv_dit_workspace_bytes(N, B, self.depth, _dtype_code(self.weight_dtype)))
        if self._workspace is None or self._workspace.numel() < need or self._workspace.device != device:
            self._graphs.clear()  # captured graphs reference the old workspace
            self._workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=device)
        return self._workspace

    def batch_struct(self, layout: PackedLayout, x, mu, t, spks, cond, out, packed: bool = False,
                     prefix: PrefixState | None = None, shared_mods: torch.Tensor | None = None) -> DitBatch:
        """C-ABI batch descriptor.  ``packed``: x, mu, cond and out are (N, 80)
        rows in document order instead of (B, 80, T)."""
        b = DitBatch()
        b.B = len(layout.lengths)
        b.T = layout.padded_length
        b.N = layout.N
        b.max_len = layout.max_len
        b.chunk = layout.chunk
        b.x, b.mu, b.cond, b.spks, b.t = (_ptr(x), _ptr(mu), _ptr(cond), _ptr(spks), _ptr(t))
        b.cu_seqlens = layout.cu_seqlens.data_ptr()
        b.doc_ids = layout.document_ids.data_ptr() if layout.N else layout.cu_seqlens.data_ptr()
        b.positions = layout.positions.data_ptr() if layout.N else layout.cu_seqlens.data_ptr()
        b.gap_rows = layout.gap_rows.data_ptr()
        b.attn_tiles = layout.attn_tiles.data_ptr()
        b.n_attn_tiles = layout.n_attn_tiles
        if layout.attn_sched is not None and self.use_attn_schedule:
            b.attn_sched = layout.attn_sched.data_ptr()
            b.attn_sched_ctas = layout.attn_ctas
        if shared_mods is not None:
            b.shared_mods = shared_mods.data_ptr()
        if prefix is not None:
            if not packed:
                raise ValueError("a cached prefix runs on packed rows")
            b.positions = prefix.positions.data_ptr() if layout.N else b.positions
            b.max_len = max(b.max_len, prefix.max_pos)
            b.doc_pos0 = prefix.doc_pos0.data_ptr()
            b.doc_kv_base = prefix.doc_kv_base.data_ptr()
            b.kv_cache = prefix.kv_cache.data_ptr()
            b.kv_layer_rows = prefix.layer_rows
            b.conv_ctx = prefix.conv_ctx.data_ptr()
            if prefix.conv_ctx_out is not None:
                b.conv_ctx_out = prefix.conv_ctx_out.data_ptr()
                b.ctx_row0 = prefix.ctx_row0.data_ptr()
        b.out = out.data_ptr()
        b.packed = 1 if packed else 0
        if out.dtype == torch.float32:
            b.out_f32 = 1
        elif out.dtype == self.weight_dtype:
            b.out_f32 = 0
        else:
            raise ValueError(f"output must be float32 or {self.weight_dtype}")
        return b

    def _launch(self, layout: PackedLayout, x, mu, t, spks, cond, out: torch.Tensor, packed: bool = False,
                prefix: PrefixState | None = None, shared_mods: torch.Tensor | None = None) -> None:
        ws = self._workspace_for(layout.N, len(layout.lengths), x.device)
        bs = self.batch_struct(layout, x, mu, t, spks, cond, out, packed, prefix, shared_mods)
        call("fcv_dit_forward", ctypes.byref(self.weights_struct()), ctypes.byref(bs), ws.data_ptr(),
             ws.numel(), _stream(x.device))

    def forward_layout(self, layout: PackedLayout, x, mu, t, spks, cond, out: torch.Tensor | None = None,
                       graph: bool = False, packed: bool = False, prefix: PrefixState | None = None,
                       shared_mods: torch.Tensor | None = None):
        """One estimator call on a prepared layout.  Inputs must already be
        contiguous tensors of the weight dtype on the module's device; ``out``
        may be float32 (the solver keeps the flow field unrounded).

        With ``graph=True`` the call is captured once into a CUDA graph per
        (layout, buffer addresses) and replayed afterwards; without ``out`` the
        result is then a view of the graph's static output buffer, valid until
        the next replay of that graph (the reference's graph path,
        ``flashinfer_dit.py:806-826``, returns such views too).

        ``packed=True``: x, mu, cond are (N, 80) rows in document order and the
        result is (N, 80) rows (the device-packed flow, no padded layout).
        ``prefix``: the documents continue cached prefixes (streaming prefix
        reuse, eager only).  ``shared_mods``: every document shares this
        modulation row (:meth:`shared_modulations`), ``t`` is then unused."""
        if not graph or prefix is not None or shared_mods is not None:
            if out is None:
                out = self._new_out(layout, x.device, packed)
            self._launch(layout, x, mu, t, spks, cond, out, packed, prefix, shared_mods)
            return out
        entry = self.capture_graph(layout, x, mu, t, spks, cond, out, packed=packed)
        entry[0].replay()
        return entry[1]

    def _new_out(self, layout: PackedLayout, device: torch.device, packed: bool) -> torch.Tensor:
        if packed:
            return torch.empty(max(layout.N, 1), MEL, dtype=self.weight_dtype, device=device)[:layout.N]
        return torch.empty(len(layout.lengths), MEL, layout.padded_length, dtype=self.weight_dtype, device=device)

    def capture_graph(self, layout: PackedLayout, x, mu, t, spks, cond, out: torch.Tensor | None = None,
                      warmup: bool = True, packed: bool = False):
        """CUDA graph of one estimator call for this layout and these buffers
        (cached, FIFO of 16).  Returns ``(graph, output buffer, layout)``.  With
        ``warmup=False`` the caller guarantees an eager call already ran."""
        B = len(layout.lengths)
        self._workspace_for(layout.N, B, x.device)  # settle the workspace before capturing
        key = (id(layout), x.data_ptr(), mu.data_ptr(), t.data_ptr(), spks.data_ptr(), cond.data_ptr(),
               None if out is None else (out.data_ptr(), out.dtype), packed)
        entry = self._graphs.get(key)
        if entry is None:
            static_out = out if out is not None else self._new_out(layout, x.device, packed)
            if warmup:
                self._launch(layout, x, mu, t, spks, cond, static_out, packed)  # first launches outside the capture
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self._launch(layout, x, mu, t, spks, cond, static_out, packed)
            if len(self._graphs) >= 16:
                self._graphs.popitem(last=False)
            entry = (g, static_out, layout)  # the layout is kept alive with its graph
            self._graphs[key] = entry
        return entry

    def forward(self, x: torch.Tensor, mask: torch.Tensor, mu: torch.Tensor, t: torch.Tensor,
                spks: torch.Tensor | None = None, cond: torch.Tensor | None = None,
                streaming: bool = False) -> torch.Tensor:
        """Estimate the flow field (``FlashInferDiT.forward``, ``flashinfer_dit.py:315-362``)."""
        if spks is None or cond is None:
            raise ValueError("spks and cond are required")
        if not self._finalized:
            raise RuntimeError("call finalize_weights() before forward()")
        dt = self.weight_dtype
        dev = self.proj_out.weight.device
        with torch.cuda.device(dev):
            B, C, T = x.shape
            if C != MEL or mu.shape != x.shape or cond.shape != x.shape or spks.shape != (B, MEL):
                raise ValueError("expected x, mu, cond of shape (B, 80, T) and spks of shape (B, 80)")
            if t.ndim == 0:
                t = t.repeat(B)
            t = t.reshape(B)
            staged = None
            if x.device.type == "cpu":
                # host inputs: uploaded on a copy stream into one of two persistent device buffer
                # sets (stable addresses for graph replay), so the next call's upload overlaps this
                # call's compute; asynchronous when the host memory is pinned, and the caller keeps
                # the host tensors unchanged until the upload has run
                staged = self._staging(B, T, dt, dev)
                cs = self._copy_stream_for(dev)
                cs.wait_event(staged["free"])  # the compute that last read this set is done
                with torch.cuda.stream(cs):
                    for name, src in (("x", x), ("mu", mu), ("cond", cond), ("spks", spks), ("t", t)):
                        staged[name].copy_(src, non_blocking=src.is_pinned())
                    staged["ready"].record(cs)
                torch.cuda.current_stream(dev).wait_event(staged["ready"])
                x, mu, cond, spks, t = staged["x"], staged["mu"], staged["cond"], staged["spks"], staged["t"]
            else:
                x = x.to(device=dev, dtype=dt).contiguous()
                mu = mu.to(device=dev, dtype=dt).contiguous()
                cond = cond.to(device=dev, dtype=dt).contiguous()
                spks = spks.to(device=dev, dtype=dt).contiguous()
                t = t.to(device=dev, dtype=dt).contiguous()
            if mask.device.type == "cpu":
                # lengths counted on the host (entries > 0.5, exact): no device round trip per call
                lengths = (mask.reshape(B, -1)[:, :T] > 0.5).sum(-1).tolist()
                y = None
                if self.use_cuda_graph and self.graph_buckets:
                    y = self.forward_bucketed(lengths, x, mu, t, spks, cond, streaming)
                if y is None:
                    layout = self.prepare_layout(lengths, T, streaming, dev)
                    y = self.forward_layout(layout, x, mu, t, spks, cond,
                                            graph=self.use_cuda_graph and not self.graph_buckets)
                if staged is not None:
                    staged["free"].record(torch.cuda.current_stream(dev))
                return y
            if staged is not None:  # device mask: every use of the staged set is enqueued below
                m = mask.to(device=dev, dtype=dt).contiguous()
                layout = self.layout_from_mask(m, streaming)
                y = self.forward_layout(layout, x, mu, t, spks, cond, graph=self.use_cuda_graph)
                staged["free"].record(torch.cuda.current_stream(dev))
                return y
            if self.use_cuda_graph and self.graph_buckets:
                m = mask.to(device=dev, dtype=dt).contiguous()
                lengths_dev = torch.empty(B, dtype=torch.int32, device=dev)
                call("fcv_mask_lengths", m.data_ptr(), _dtype_code(dt), B, T, lengths_dev.data_ptr(), _stream(dev))
                lengths = lengths_dev.cpu().tolist()
                y = self.forward_bucketed(lengths, x, mu, t, spks, cond, streaming)
                if y is not None:
                    return y
                layout = self.prepare_layout(lengths, T, streaming, dev, lengths_dev)
                return self.forward_layout(layout, x, mu, t, spks, cond)
            layout = self.layout_from_mask(mask.to(dev), streaming)
            return self.forward_layout(layout, x, mu, t, spks, cond, graph=self.use_cuda_graph)

    def _staging(self, B: int, T: int, dt: torch.dtype, dev: torch.device) -> dict:
        """The next of two persistent device buffer sets for host inputs of one (B, T)
        shape, with its upload-done and compute-done events (FIFO of 8 shapes)."""
        key = (B, T)
        pair = self._stage.get(key)
        if pair is None:
            if len(self._stage) >= 8:
                torch.cuda.synchronize(dev)  # nothing may still read the evicted buffers
                self._stage.popitem(last=False)
            pair = [0, []]
            for _ in range(2):
                pair[1].append({"x": torch.empty(B, MEL, T, dtype=dt, device=dev),
                                "mu": torch.empty(B, MEL, T, dtype=dt, device=dev),
                                "cond": torch.empty(B, MEL, T, dtype=dt, device=dev),
                                "spks": torch.empty(B, MEL, dtype=dt, device=dev),
                                "t": torch.empty(B, dtype=dt, device=dev),
                                "ready": torch.cuda.Event(), "free": torch.cuda.Event()})
                # the allocator may hand out memory that work queued on the compute stream still
                # reads or writes: the copy stream must not touch it before that work is done
                pair[1][-1]["free"].record(torch.cuda.current_stream(dev))
            self._stage[key] = pair
        st = pair[1][pair[0]]
        pair[0] ^= 1
        return st

    def _copy_stream_for(self, dev: torch.device) -> torch.cuda.Stream:
        if self._copy_stream is None:
            self._copy_stream = torch.cuda.Stream(dev)
        return self._copy_stream

    # ------------------------------------------------------------------ bucketed graphs
    def bucket_for(self, lengths: Sequence[int]) -> tuple[int, int] | None:
        """(row capacity, document capacity) of the graph serving this batch, or
        None when no bucket holds it (or a document exceeds the RoPE table)."""
        if not self.graph_buckets:
            return None
        N = sum(lengths)
        if max(lengths, default=0) > ROPE_TABLE_LEN:
            return None
        rows = next((b for b in self.graph_buckets if b >= N), None)
        if rows is None:
            return None
        docs = 2
        while docs < len(lengths):
            docs *= 2
        return rows, docs

    def forward_bucketed(self, lengths: Sequence[int], x, mu, t, spks, cond, streaming: bool,
                         out: torch.Tensor | None = None) -> torch.Tensor | None:
        """Replay the bucket graph that holds this batch (the packed counterpart of
        ``_forward_graph_bucketed`` / ``_forward_graph_bucketed_stream``,
        ``flashinfer_dit.py:742-826``): one captured estimator call serves every
        composition of up to ``docs`` documents and ``rows`` packed rows, so a new
        composition costs a few copies, not a capture.  x, mu, cond are padded
        (B, 80, T) of the weight dtype on the module's device.  Returns the
        (B, 80, T) flow field (padding frames zero), or None when no bucket holds
        the batch."""
        key = self.bucket_for(lengths)
        if key is None:
            return None
        chunk = self._chunk_size if streaming else 0
        gkey = key + (chunk,)
        g = self._bucket_graphs.get(gkey)
        if g is None:
            if len(self._bucket_graphs) >= 16:
                self._bucket_graphs.popitem(last=False)
            g = _BucketGraph(self, key[0], key[1], chunk, x.device)
            self._bucket_graphs[gkey] = g
            self.bucket_captures += 1
        else:
            self._bucket_graphs.move_to_end(gkey)
        return g.run(lengths, x, mu, t, spks, cond, out)


def graph_row_buckets(cuda_graph_buckets: Sequence[float] | None = None,
                      stream_graph_buckets: Sequence[int] | None = None) -> tuple[int, ...] | None:
    """Row capacities for the bucketed graphs from the reference's presets:
    offline buckets in seconds (50 Mel frames per second,
    ``flashinfer_dit.py:154-158``), streaming buckets in frames; each holds one
    CFG pair, so a bucket of F frames is 2F packed rows."""
    rows = set()
    for s in cuda_graph_buckets or ():
        rows.add(2 * round(float(s) * 50))
    for f in stream_graph_buckets or ():
        rows.add(2 * int(f))
    return tuple(sorted(rows)) or None


# Default row ladder for packed batches: steps of 512 rows to 4096, then 1.25x.
DEFAULT_GRAPH_BUCKETS = (512, 1024, 1536, 2048, 2560, 3072, 3584, 4096, 5120, 6144, 7168, 8192, 10240,
                         12288, 14336, 16384, 20480, 24576, 28672, 32768)


def apply_b200(model, dtype: torch.dtype = torch.bfloat16, enable_cuda_graph: bool = False,
               cuda_graph_buckets: Sequence[float] | None = None,
               stream_graph_buckets: Sequence[int] | None = None):
    """Replace a Token2Wav model's estimator with :class:`B200DiT`
    (mirror of ``apply_flashinfer``, ``flashinfer_dit.py:951-988``).  With
    ``enable_cuda_graph`` every call replays a bucketed graph: the reference's
    bucket presets (seconds offline, frames streaming) become row capacities,
    else :data:`DEFAULT_GRAPH_BUCKETS`."""
    reference = model.flow.decoder.estimator
    device = next(reference.parameters()).device
    buckets = None
    if enable_cuda_graph:
        buckets = graph_row_buckets(cuda_graph_buckets, stream_graph_buckets) or DEFAULT_GRAPH_BUCKETS
    est = B200DiT(static_chunk_size=getattr(reference, "static_chunk_size", 50),
                  depth=len(reference.transformer_blocks), use_cuda_graph=enable_cuda_graph,
                  graph_buckets=buckets)
    missing, unexpected = est.load_state_dict(reference.state_dict(), strict=False)
    missing = [k for k in missing if "rope" not in k and "rotary" not in k]
    if missing or unexpected:
        raise RuntimeError(f"B200DiT state-dict mismatch: missing={missing}, unexpected={unexpected}")
    est = est.to(device=device, dtype=dtype).eval()
    est.finalize_weights()
    model.flow.decoder.estimator = est
    return model


class _BucketGraph:
    """One estimator call captured for ``rows`` packed rows and ``docs`` real
    document slots, serving every batch that fits.

    The graph holds the packed layout computation (``fcv_pack_layout`` from a
    device lengths buffer) and the packed-row estimator call.  Per replay the
    host uploads one small block -- lengths, cu_seqlens, the attention work
    list and its length -- and packs the inputs into the static rows.  Rows
    past the batch belong to filler documents (at most ``ROPE_TABLE_LEN`` rows
    each, after the unused zero-length slots): every kernel but attention is
    row-local or document-local, so they never touch real rows, and the work
    list leaves them out of attention.  Results are bit-identical to the eager
    call (no kernel's per-element reduction order depends on the row count)."""

    def __init__(self, model: B200DiT, rows: int, docs: int, chunk: int, device: torch.device):
        self.model, self.rows, self.docs, self.chunk, self.device = model, rows, docs, chunk, device
        dt = model.weight_dtype
        self.n_fill = max(1, -(-rows // ROPE_TABLE_LEN))
        self.n_docs = docs + self.n_fill
        self.tile_cap = -(-rows // 128) + docs
        self.ctas = int(lib().fcv_attn_ctas(self.tile_cap))
        nd = self.n_docs
        # device block: lengths (nd) | cu (nd + 1) | n_tiles (1) | pad | tiles (2 * cap) | schedule, int32
        self.off_cu = nd
        self.off_nt = 2 * nd + 1
        self.off_tiles = (self.off_nt + 2) // 2 * 2
        self.off_sched = self.off_tiles + 2 * self.tile_cap
        self.sched_cap = self.ctas + 1 + 16 * self.tile_cap
        size = self.off_sched + self.sched_cap
        self.meta = torch.zeros(size, dtype=torch.int32, device=device)
        self.host = torch.zeros(size, dtype=torch.int32).pin_memory()
        self.copied = torch.cuda.Event()
        self.x = torch.zeros(rows, MEL, dtype=dt, device=device)
        self.mu = torch.zeros_like(self.x)
        self.cond = torch.zeros_like(self.x)
        self.spks = torch.zeros(nd, MEL, dtype=dt, device=device)
        self.t = torch.zeros(nd, dtype=dt, device=device)
        self.out = torch.zeros(rows, MEL, dtype=dt, device=device)
        self.gather = torch.empty(rows, dtype=torch.int64, device=device)
        self.doc_ids = torch.empty(rows, dtype=torch.int32, device=device)
        self.positions = torch.empty(rows, dtype=torch.int32, device=device)
        self.cu = torch.empty(nd + 1, dtype=torch.int32, device=device)
        self.gap_rows = torch.empty(rows + 30 * (nd + 1), dtype=torch.int32, device=device)
        need = int(lib().fcv_dit_workspace_bytes(rows, nd, model.depth, _dtype_code(dt)))
        # zeroed once: rows no kernel writes for a batch stay finite
        self.workspace = torch.zeros(max(need, 256), dtype=torch.uint8, device=device)
        self.batch = DitBatch()
        b = self.batch
        b.B, b.T, b.N, b.max_len, b.chunk = nd, rows, rows, min(rows, ROPE_TABLE_LEN), chunk
        b.x, b.mu, b.cond, b.spks, b.t = (self.x.data_ptr(), self.mu.data_ptr(), self.cond.data_ptr(),
                                          self.spks.data_ptr(), self.t.data_ptr())
        b.cu_seqlens, b.doc_ids, b.positions = self.cu.data_ptr(), self.doc_ids.data_ptr(), self.positions.data_ptr()
        b.gap_rows = self.gap_rows.data_ptr()
        b.attn_tiles = self.meta.data_ptr() + 4 * self.off_tiles
        b.n_attn_tiles = self.tile_cap
        b.n_attn_tiles_dev = self.meta.data_ptr() + 4 * self.off_nt
        b.attn_sched = self.meta.data_ptr() + 4 * self.off_sched
        b.attn_sched_ctas = self.ctas
        b.out, b.out_f32, b.packed = self.out.data_ptr(), 0, 1
        self._fill_host([])  # an empty batch: everything is filler
        self.meta.copy_(self.host)
        stream = _stream(device)
        self._body(stream)  # first launches (function attributes) outside the capture
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._body(_stream(device))

    def _body(self, stream: int) -> None:
        call("fcv_pack_layout", self.meta.data_ptr(), self.n_docs, self.rows, self.rows, self.gather.data_ptr(),
             self.doc_ids.data_ptr(), self.positions.data_ptr(), self.cu.data_ptr(), self.gap_rows.data_ptr(),
             stream)
        call("fcv_dit_forward", ctypes.byref(self.model.weights_struct()), ctypes.byref(self.batch),
             self.workspace.data_ptr(), self.workspace.numel(), stream)

    def _fill_host(self, lengths: Sequence[int]) -> int:
        """Lengths (real, zero slots, filler), cu_seqlens and the work list into
        the pinned block; returns the real row count."""
        B, N = len(lengths), sum(lengths)
        fill, rest = [], self.rows - N
        for _ in range(self.n_fill):
            f = min(rest, ROPE_TABLE_LEN)
            fill.append(f)
            rest -= f
        ext = list(lengths) + [0] * (self.docs - B) + fill
        h = self.host
        h[:self.n_docs] = torch.tensor(ext, dtype=torch.int32)
        cu = [0]
        for v in ext:
            cu.append(cu[-1] + v)
        h[self.off_cu:self.off_cu + self.n_docs + 1] = torch.tensor(cu, dtype=torch.int32)
        n_tiles = 0
        lens = (ctypes.c_int32 * max(B, 1))(*lengths)
        base = h.data_ptr()
        if B:
            cap = sum((L + 127) // 128 for L in lengths)
            n_tiles = call("fcv_attn_tiles", ctypes.addressof(lens), B, self.chunk, base + 4 * self.off_tiles, cap)
        h[self.off_nt] = n_tiles
        call("fcv_attn_schedule", ctypes.addressof(lens), B, self.chunk, base + 4 * self.off_tiles, n_tiles,
             self.ctas, base + 4 * self.off_sched, self.sched_cap)
        return N

    def run(self, lengths: Sequence[int], x, mu, t, spks, cond, out: torch.Tensor | None = None) -> torch.Tensor:
        lengths = [int(v) for v in lengths]
        B, T = len(lengths), int(x.shape[2])
        dev, stream = self.device, _stream(self.device)
        self.copied.synchronize()  # the previous upload has left the pinned block
        N = self._fill_host(lengths)
        self.meta.copy_(self.host, non_blocking=True)
        self.copied.record()
        cu_real = self.meta[self.off_cu:self.off_cu + B + 1]
        dcode = _dtype_code(self.model.weight_dtype)
        max_len = max(lengths, default=0)
        for src, dst in ((x, self.x), (mu, self.mu), (cond, self.cond)):
            call("fcv_pack_rows", src.data_ptr(), dcode, MEL * T, T, cu_real.data_ptr(), B, max_len,
                 dst.data_ptr(), dcode, stream)
        self.spks[:B].copy_(spks)
        self.spks[B:].zero_()
        self.t[:B].copy_(t)
        self.t[B:].zero_()
        self.graph.replay()
        if out is None:
            out = torch.empty(B, MEL, T, dtype=self.model.weight_dtype, device=dev)
        # rows -> (B, 80, T), padding frames written as zeros
        call("fcv_unpack_output", self.out.data_ptr(), dcode, cu_real.data_ptr(), B, T, N, out.data_ptr(), stream)
        return out
