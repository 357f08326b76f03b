"""Flow inference on the B200 estimator: the CFG Euler solver and the packed front end.

``solve_euler_batched`` mirrors the reference's padded solver
(``faster_cosyvoice/token2wav/flashinfer_flow.py:16-74``): cosine schedule in the
input dtype, the ``[cond; uncond]`` stack with mu, speaker embedding and condition
zeroed in the second half, ``x.repeat(2)``, ``d = (1 + r) d_c - r d_u`` and
``x += dt d``.  Differences that only remove work: the packed layout is computed
once per call (the mask is the same for all steps), the CFG combine, the Euler
update and the next step's repeated input are one fused kernel
(``fcv_cfg_euler``), and the sample is carried in float32 between steps.

``flow_inference_batched`` / ``flow_inference_batched_streaming`` mirror the
reference's batched flow inference (``flashinfer_flow.py:118-281``) with the
whole front end device-packed: tokens, mu, condition, noise and the ODE state
live as packed rows (one row per mel frame, requests back to back), so no
padded (B, 80, T) tensor exists anywhere between the token ids and the
generated Mel, and the per-request Python loops of the reference become one
C-ABI call each (``fcv_flow_frontend``, ``fcv_speaker_projection``,
``fcv_prompt_rows``, ``fcv_pack_rows``).
"""

from __future__ import annotations

import ctypes
import math
from collections.abc import Sequence

import torch
import torch.nn as nn

from . import _lib
from ._lib import FlowWeights, call
from .model import B200DiT, PrefixState, _dtype_code, _stream


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
            est.forward_layout(layout, x_in, mu_in, t_in, spk_in, cond_in, out=d,
                               shared_mods=est.shared_modulations(float(t)))
            nxt = x_in.data_ptr() if k < num_timesteps else None
            call("fcv_cfg_euler", x.data_ptr(), d.data_ptr(), _lib.DTYPE_F32, R, T, float(step), rate, nxt,
                 _dtype_code(dt_w), stream)
            t = t + step
            if k < num_timesteps:
                step = span[k + 1] - t
        return x.to(sdtype)


# ---------------------------------------------------------------------------
# The flow module (inference side of CausalMaskedDiffWithDiT)
# ---------------------------------------------------------------------------

class _PreLookahead(nn.Module):
    """Parameters of ``PreLookaheadLayer`` (``upsample_encoder.py:55-69``):
    conv1 (in -> channels, kernel ``pre_lookahead_len + 1``) and conv2
    (channels -> in, kernel 3).  Its forward runs inside ``fcv_flow_frontend``."""

    def __init__(self, in_channels: int = 80, channels: int = 1024, pre_lookahead_len: int = 3):
        super().__init__()
        self.in_channels = in_channels
        self.channels = channels
        self.pre_lookahead_len = pre_lookahead_len
        self.conv1 = nn.Conv1d(in_channels, channels, kernel_size=pre_lookahead_len + 1, stride=1, padding=0)
        self.conv2 = nn.Conv1d(channels, in_channels, kernel_size=3, stride=1, padding=0)


class _FlowDecoder(nn.Module):
    """Inference state of ``CausalConditionalCFM`` (``flow_matching.py:196-200``):
    the estimator, the guidance rate and the fixed noise prefix, drawn right
    after the constructor reseeds the generator with 0 (as the reference's
    ``set_all_random_seed(0)`` does for torch)."""

    def __init__(self, estimator: B200DiT, inference_cfg_rate: float = 0.7):
        super().__init__()
        self.estimator = estimator
        self.inference_cfg_rate = inference_cfg_rate
        torch.manual_seed(0)
        self.register_buffer("rand_noise", torch.randn([1, 80, 50 * 300]), persistent=False)


class B200Flow(nn.Module):
    """The inference side of ``CausalMaskedDiffWithDiT`` (``flow.py:281-313``,
    built as ``builders.py:33-45``) over a :class:`B200DiT`.

    Module tree and parameter creation order follow the reference (the DiT,
    then the CFM's reseed and noise prefix, then the pre-lookahead convolutions,
    the token table and the speaker projection), so a reference flow's state
    dict loads unchanged and construction after ``torch.manual_seed(s)``
    reproduces the reference's random initialisation.  The batched entry points
    below accept either this module or the reference's own flow module whose
    estimator was replaced by a finalized :class:`B200DiT` (``apply_b200``)."""

    def __init__(self, estimator: B200DiT | None = None, depth: int = 22, vocab_size: int = 6561,
                 input_size: int = 80, output_size: int = 80, spk_embed_dim: int = 192,
                 token_mel_ratio: int = 2, pre_lookahead_len: int = 3, lookahead_channels: int = 1024,
                 inference_cfg_rate: float = 0.7, static_chunk_size: int = 50):
        super().__init__()
        if estimator is None:
            estimator = B200DiT(depth=depth, static_chunk_size=static_chunk_size)
        decoder = _FlowDecoder(estimator, inference_cfg_rate)
        pre = _PreLookahead(input_size, lookahead_channels, pre_lookahead_len)
        self.input_size = input_size
        self.output_size = output_size
        self.vocab_size = vocab_size
        self.input_embedding = nn.Embedding(vocab_size, input_size)
        self.spk_embed_affine_layer = nn.Linear(spk_embed_dim, output_size)
        self.pre_lookahead_len = pre_lookahead_len
        self.pre_lookahead_layer = pre
        self.decoder = decoder
        self.token_mel_ratio = token_mel_ratio


class _FrontEnd:
    """Device copies of the front-end weights in the layouts the kernels read
    (prepared once per flow module, device and dtype, like ``finalize_weights``)."""

    def __init__(self, flow, device: torch.device, dtype: torch.dtype):
        pl = flow.pre_lookahead_layer
        if pl.conv1.kernel_size[0] != 4 or pl.conv2.kernel_size[0] != 3 or pl.conv1.out_channels != 1024:
            raise ValueError("the packed front end implements PreLookaheadLayer(80, 1024, pre_lookahead_len=3)")
        if flow.input_embedding.weight.shape[1] != 80 or flow.spk_embed_affine_layer.out_features != 80:
            raise ValueError("the packed front end implements 80-channel token features and speaker rows")
        self.device, self.dtype = device, dtype
        det = lambda t: t.detach().to(device)  # noqa: E731
        self.embed = det(flow.input_embedding.weight).to(dtype).contiguous()
        w1 = det(pl.conv1.weight)  # (1024, 80, 4) -> [o, k*80 + c]
        self.conv1_w = w1.permute(0, 2, 1).reshape(w1.shape[0], -1).to(dtype).contiguous()
        self.conv1_b = det(pl.conv1.bias).float().contiguous()
        w2 = det(pl.conv2.weight)  # (80, 1024, 3) -> [o, k*1024 + c]
        self.conv2_w = w2.permute(0, 2, 1).reshape(w2.shape[0], -1).to(dtype).contiguous()
        self.conv2_b = det(pl.conv2.bias).float().contiguous()
        self.spk_w = det(flow.spk_embed_affine_layer.weight).to(dtype).contiguous()
        self.spk_b = det(flow.spk_embed_affine_layer.bias).float().contiguous()
        self.vocab = int(self.embed.shape[0])
        self.lookahead = int(pl.pre_lookahead_len)
        noise = getattr(flow.decoder, "rand_noise", None)
        # the reference moves the prefix to the device and casts it to the flow dtype (flashinfer_flow.py:266)
        self.rand_noise = None if noise is None else noise.detach().to(device).to(dtype).contiguous()
        self.struct = FlowWeights()
        self.struct.dtype = _dtype_code(dtype)
        self.struct.vocab = self.vocab
        self.struct.embed = self.embed.data_ptr()
        self.struct.conv1_w = self.conv1_w.data_ptr()
        self.struct.conv1_b = self.conv1_b.data_ptr()
        self.struct.conv2_w = self.conv2_w.data_ptr()
        self.struct.conv2_b = self.conv2_b.data_ptr()
        self.workspace = None

    def workspace_for(self, n_out: int) -> torch.Tensor:
        need = int(_lib.lib().fcv_flow_workspace_bytes(n_out, _dtype_code(self.dtype)))
        if self.workspace is None or self.workspace.numel() < need:
            self.workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=self.device)
        return self.workspace


def prepare_frontend(flow) -> _FrontEnd:
    """The flow's prepared front end for its estimator's device and dtype."""
    est = flow.decoder.estimator
    if not isinstance(est, B200DiT):
        raise TypeError("flow.decoder.estimator must be a B200DiT (see apply_b200)")
    dev, dt = est.proj_out.weight.device, est.weight_dtype
    fe = getattr(flow, "_b200_frontend", None)
    if fe is None or fe.device != dev or fe.dtype != dt:
        fe = _FrontEnd(flow, dev, dt)
        flow._b200_frontend = fe
    return fe


# ---------------------------------------------------------------------------
# Packed solver and batched flow inference
# ---------------------------------------------------------------------------

@torch.inference_mode()
def solve_euler_packed(decoder, noise_rows: torch.Tensor, mu_rows: torch.Tensor, lengths: Sequence[int],
                       speaker_embeddings: torch.Tensor, condition_rows: torch.Tensor,
                       num_timesteps: int = 10, streaming: bool = False) -> torch.Tensor:
    """The CFG Euler solver of ``flashinfer_flow.py:16-74`` on packed rows.

    ``noise_rows``, ``mu_rows``, ``condition_rows``: (N, 80) with request r in
    rows ``[sum(lengths[:r]), sum(lengths[:r+1]))``; ``speaker_embeddings``
    (R, 80).  The ``[cond; uncond]`` stack is 2R documents over 2N rows.
    Returns the float32 sample rows (N, 80)."""
    est: B200DiT = decoder.estimator
    if not isinstance(est, B200DiT):
        raise TypeError("decoder.estimator must be a B200DiT")
    rate = float(decoder.inference_cfg_rate)
    dev = est.proj_out.weight.device
    dt_w = est.weight_dtype
    lengths = [int(v) for v in lengths]
    R, N = len(lengths), sum(lengths)
    with torch.cuda.device(dev):
        x = noise_rows.to(device=dev, dtype=torch.float32).clone()
        if N == 0:
            return x
        span = cosine_schedule(num_timesteps, speaker_embeddings.dtype)
        t = span[0]
        step = span[1] - span[0]
        layout = est.prepare_layout(lengths + lengths, max(lengths), streaming, dev)
        mu_in = torch.zeros(2 * N, 80, dtype=dt_w, device=dev)
        mu_in[:N].copy_(mu_rows)
        cond_in = torch.zeros(2 * N, 80, dtype=dt_w, device=dev)
        cond_in[:N].copy_(condition_rows)
        spk_in = torch.zeros(2 * R, 80, dtype=dt_w, device=dev)
        spk_in[:R].copy_(speaker_embeddings)
        x_in = torch.empty(2 * N, 80, dtype=dt_w, device=dev)
        x_in[:N].copy_(x)
        x_in[N:].copy_(x)
        d = torch.empty(2 * N, 80, dtype=torch.float32, device=dev)
        t_in = torch.empty(2 * R, dtype=dt_w, device=dev)
        stream = _stream(dev)
        for k in range(1, num_timesteps + 1):
            t_in.fill_(float(t))
            est.forward_layout(layout, x_in, mu_in, t_in, spk_in, cond_in, out=d, packed=True,
                               shared_mods=est.shared_modulations(float(t)))
            nxt = x_in.data_ptr() if k < num_timesteps else None
            # rows (N, 80) are one flat run of 80*N values: the kernel's (R=1, 80, T=N) view
            call("fcv_cfg_euler", x.data_ptr(), d.data_ptr(), _lib.DTYPE_F32, 1, N, float(step), rate, nxt,
                 _dtype_code(dt_w), stream)
            t = t + step
            if k < num_timesteps:
                step = span[k + 1] - t
        return x


def _int_rows(values: Sequence[int]) -> list[int]:
    cu = [0]
    for v in values:
        cu.append(cu[-1] + int(v))
    return cu


def _packed_front(flow, fe: _FrontEnd, token_list, prompt_features, out_lens):
    """Upload tokens and offsets once, run the front end: mu rows, prompt
    condition rows and the request offsets."""
    dev, dt = fe.device, fe.dtype
    R = len(token_list)
    ratio = int(flow.token_mel_ratio)
    in_lens = [len(t) for t in token_list]
    flat = [int(v) for tl in token_list for v in tl]
    if flat and max(flat) >= fe.vocab:
        raise IndexError(f"token id {max(flat)} out of range for a table of {fe.vocab} rows")
    tok_cu, out_cu = _int_rows(in_lens), _int_rows(out_lens)
    mel_lens = [ratio * v for v in out_lens]
    mel_cu = _int_rows(mel_lens)
    prompt_lens = [int(p.shape[1]) for p in prompt_features]
    for r, (lp, lm) in enumerate(zip(prompt_lens, mel_lens)):
        if lp > lm:
            raise ValueError(f"prompt of request {r} has {lp} frames but the request only {lm}")
    p_cu = _int_rows(prompt_lens)
    host = torch.tensor(flat + tok_cu + out_cu + mel_cu + p_cu, dtype=torch.int32).pin_memory()
    idx = host.to(dev, non_blocking=True)
    n_tok = len(flat)
    tokens = idx[:max(n_tok, 1)]
    o = n_tok
    tok_cu_d, out_cu_d, mel_cu_d, p_cu_d = (idx[o + i * (R + 1): o + (i + 1) * (R + 1)] for i in range(4))
    n_out, n_mel = out_cu[-1], mel_cu[-1]
    stream = _stream(dev)
    mu = torch.empty(max(n_mel, 1), 80, dtype=dt, device=dev)[:n_mel]
    ws = fe.workspace_for(n_out)
    call("fcv_flow_frontend", ctypes.byref(fe.struct), tokens.data_ptr(), tok_cu_d.data_ptr(), out_cu_d.data_ptr(),
         R, n_out, max(out_lens) if out_lens else 0, ratio, ws.data_ptr(), ws.numel(), mu.data_ptr(), stream)
    cond = torch.empty(max(n_mel, 1), 80, dtype=dt, device=dev)[:n_mel]
    prompt = (torch.cat([p[0] for p in prompt_features], 0) if sum(prompt_lens) else
              torch.zeros(1, 80)).to(device=dev, dtype=dt).contiguous()
    call("fcv_prompt_rows", prompt.data_ptr(), p_cu_d.data_ptr(), mel_cu_d.data_ptr(), R,
         max(mel_lens) if mel_lens else 0, cond.data_ptr(), _dtype_code(dt), stream)
    return mu, cond, mel_lens, mel_cu, mel_cu_d, prompt_lens


def _speaker_rows(fe: _FrontEnd, spk: torch.Tensor) -> torch.Tensor:
    R = spk.shape[0]
    out = torch.empty(max(R, 1), 80, dtype=fe.dtype, device=fe.device)[:R]
    spk = spk.to(fe.device).contiguous()
    call("fcv_speaker_projection", spk.data_ptr(), _dtype_code(spk.dtype), R, int(spk.shape[1]), fe.spk_w.data_ptr(),
         fe.spk_b.data_ptr(), 80, out.data_ptr(), _dtype_code(fe.dtype), _stream(fe.device))
    return out


def _split(x: torch.Tensor, mel_cu, prompt_lens) -> list[torch.Tensor]:
    """Generated Mel of every request, (1, 80, n_mel - prompt) float32 views
    (``flashinfer_flow.py:180-184, 277-281``)."""
    return [x[mel_cu[r] + prompt_lens[r]: mel_cu[r + 1]].t().unsqueeze(0) for r in range(len(prompt_lens))]


@torch.inference_mode()
def flow_inference_batched(flow, token_list: Sequence[Sequence[int]], prompt_features: Sequence[torch.Tensor],
                           speaker_embeddings: torch.Tensor, noise: torch.Tensor | None = None,
                           num_timesteps: int = 10) -> list[torch.Tensor]:
    """Offline flow inference for variable-length requests
    (``flow_inference_batched``, ``flashinfer_flow.py:118-184``), device-packed.

    ``token_list``: prompt + generated speech tokens per request;
    ``prompt_features``: (1, prompt_len, 80) Mel per request;
    ``speaker_embeddings``: (R, 192).  Returns (1, 80, generated_len) float32
    per request.  ``noise`` (R, 80, max_mel) replaces the solver's
    ``torch.randn`` start (drawn exactly as the reference draws it when absent)."""
    fe = prepare_frontend(flow)
    dev, dt = fe.device, fe.dtype
    R = len(token_list)
    with torch.cuda.device(dev):
        # F.normalize of the embedding cast to the flow dtype (flashinfer_flow.py:145)
        spk = _speaker_rows(fe, speaker_embeddings.to(device=dev, dtype=dt))
        out_lens = [len(t) for t in token_list]
        mu, cond, mel_lens, mel_cu, mel_cu_d, prompt_lens = _packed_front(flow, fe, token_list, prompt_features,
                                                                          out_lens)
        max_mel = max(mel_lens) if mel_lens else 0
        if noise is None:
            noise = torch.randn(R, 80, max_mel, device=dev, dtype=dt)
        noise = noise.to(dev).contiguous()
        x0 = torch.empty(max(mel_cu[-1], 1), 80, dtype=torch.float32, device=dev)[:mel_cu[-1]]
        call("fcv_pack_rows", noise.data_ptr(), _dtype_code(noise.dtype), 80 * int(noise.shape[2]),
             int(noise.shape[2]), mel_cu_d.data_ptr(), R, max_mel, x0.data_ptr(), _lib.DTYPE_F32, _stream(dev))
        x = solve_euler_packed(flow.decoder, x0, mu, mel_lens, spk, cond, num_timesteps, streaming=False)
        return _split(x, mel_cu, prompt_lens)


class PrefixCache:
    """Cached state of streaming flows for prefix reuse.

    The reference recomputes every frame of a stream at every call
    (``flashinfer_flow.py:215-221``).  A frame in a chunk that was complete in
    the previous call keeps a bit-identical trajectory (chunk-causal attention,
    causal position convolutions, lookahead tokens that are the real next
    tokens, the fixed noise prefix), so a call only needs its rows from the
    first incomplete chunk on, given per ODE step and DiT block the earlier
    frames' keys and values, per step the two position convolutions' 30-row
    left context, and the final sample of the earlier frames.  This object
    holds that state for up to ``max_streams`` streams of at most
    ``max_frames`` Mel frames (prompt included): ``steps x depth x
    (2 x max_streams x max_frames) x 2048`` K/V values (both CFG documents of a
    stream), about 0.9 MB per frame and document over 10 steps and 22 blocks."""

    def __init__(self, flow, max_streams: int, max_frames: int, num_timesteps: int = 10):
        est = flow.decoder.estimator
        if not isinstance(est, B200DiT):
            raise TypeError("flow.decoder.estimator must be a B200DiT")
        self.device, self.dtype = est.proj_out.weight.device, est.weight_dtype
        self.steps, self.max_streams = int(num_timesteps), int(max_streams)
        self.cap = -(-int(max_frames) // 64) * 64
        self.chunk = int(est.static_chunk_size)
        self.layer_rows = 2 * self.max_streams * self.cap
        # zeroed once: attention loads whole 64-key tiles, and the rows past a document's
        # keys must hold finite values (their probabilities are 0, but 0 x NaN is NaN)
        self.kv = torch.zeros(self.steps, est.depth, self.layer_rows, 2048, dtype=self.dtype, device=self.device)
        self.ctx = torch.zeros(self.steps, 2 * self.max_streams, 2, 30, 1024, dtype=self.dtype, device=self.device)
        self.final = torch.zeros(self.max_streams, self.cap, 80, dtype=torch.float32, device=self.device)
        self._state: dict = {}  # stream id -> [slot, stable frames]
        self._free = list(range(self.max_streams))[::-1]

    def stable_frames(self, stream_id) -> int:
        """Frames of a stream whose state is cached (0 for an unknown stream)."""
        st = self._state.get(stream_id)
        return 0 if st is None else st[1]

    def release(self, stream_id) -> None:
        """Forget a stream (its slot is reused)."""
        st = self._state.pop(stream_id, None)
        if st is not None:
            self._free.append(st[0])

    def _acquire(self, stream_id) -> list:
        st = self._state.get(stream_id)
        if st is None:
            if not self._free:
                raise RuntimeError(f"prefix cache full ({self.max_streams} streams)")
            slot = self._free.pop()
            self.ctx[:, 2 * slot:2 * slot + 2].zero_()  # a fresh stream's convolutions see zeros
            st = self._state[stream_id] = [slot, 0]
        return st


@torch.inference_mode()
def _solve_euler_prefix(decoder, cache: PrefixCache, x0: torch.Tensor, mu: torch.Tensor, cond: torch.Tensor,
                        spk: torch.Tensor, new_lens: list[int], pos0: list[int], slots: list[int],
                        next_stable: list[int], num_timesteps: int) -> torch.Tensor:
    """The streaming CFG Euler solver on the new rows only (chunk-causal mask),
    every estimator call continuing the cached prefixes; returns the new rows'
    final samples (float32)."""
    est: B200DiT = decoder.estimator
    rate = float(decoder.inference_cfg_rate)
    dev, dt_w = cache.device, cache.dtype
    R, N = len(new_lens), sum(new_lens)
    x = x0.to(torch.float32).clone()
    if N == 0:
        return x
    span = cosine_schedule(num_timesteps, spk.dtype)
    t = span[0]
    step = span[1] - span[0]
    layout = est.prepare_layout(new_lens + new_lens, max(new_lens), True, dev)
    # both CFG documents of request r: cache slots 2 slot_r and 2 slot_r + 1
    docs = [2 * s for s in slots] + [2 * s + 1 for s in slots]
    meta = torch.tensor(pos0 + pos0 + [d * cache.cap for d in docs] + docs
                        + [n - p for n, p in zip(next_stable, pos0)] * 2, dtype=torch.int32).to(dev)
    pos0_d, kvb_d, slot_d, row0_d = meta[:2 * R], meta[2 * R:4 * R], meta[4 * R:6 * R], meta[6 * R:]
    positions = layout.positions.clone()
    call("fcv_offset_positions", positions.data_ptr(), layout.document_ids.data_ptr(), pos0_d.data_ptr(), 2 * N,
         _stream(dev))
    slot_idx = slot_d.long()
    max_pos = max(p + n for p, n in zip(pos0, new_lens))
    mu_in = torch.zeros(2 * N, 80, dtype=dt_w, device=dev)
    mu_in[:N].copy_(mu)
    cond_in = torch.zeros(2 * N, 80, dtype=dt_w, device=dev)
    cond_in[:N].copy_(cond)
    spk_in = torch.zeros(2 * R, 80, dtype=dt_w, device=dev)
    spk_in[:R].copy_(spk)
    x_in = torch.empty(2 * N, 80, dtype=dt_w, device=dev)
    x_in[:N].copy_(x)
    x_in[N:].copy_(x)
    d = torch.empty(2 * N, 80, dtype=torch.float32, device=dev)
    t_in = torch.empty(2 * R, dtype=dt_w, device=dev)
    stream = _stream(dev)
    for k in range(1, num_timesteps + 1):
        t_in.fill_(float(t))
        ctx_in = cache.ctx[k - 1].index_select(0, slot_idx)
        ctx_out = torch.empty_like(ctx_in)
        prefix = PrefixState(positions, pos0_d, kvb_d, cache.kv[k - 1], cache.layer_rows, ctx_in, ctx_out, row0_d,
                             max_pos)
        est.forward_layout(layout, x_in, mu_in, t_in, spk_in, cond_in, out=d, packed=True, prefix=prefix,
                           shared_mods=est.shared_modulations(float(t)))
        cache.ctx[k - 1].index_copy_(0, slot_idx, ctx_out)
        nxt = x_in.data_ptr() if k < num_timesteps else None
        call("fcv_cfg_euler", x.data_ptr(), d.data_ptr(), _lib.DTYPE_F32, 1, N, float(step), rate, nxt,
             _dtype_code(dt_w), stream)
        t = t + step
        if k < num_timesteps:
            step = span[k + 1] - t
    return x


@torch.inference_mode()
def flow_inference_batched_streaming(flow, token_list: Sequence[Sequence[int]],
                                     prompt_features: Sequence[torch.Tensor], speaker_embeddings: torch.Tensor,
                                     finalize_list: Sequence[bool], num_timesteps: int = 10,
                                     cache: PrefixCache | None = None,
                                     stream_ids: Sequence | None = None) -> list[torch.Tensor]:
    """Full-prefix streaming flow inference for several streams
    (``flow_inference_batched_streaming``, ``flashinfer_flow.py:187-281``),
    device-packed: a non-final stream's last ``pre_lookahead_len`` tokens are
    lookahead context only, the start is the decoder's fixed noise prefix and
    the estimator uses the chunk-causal mask.

    With a :class:`PrefixCache` and one ``stream_ids`` entry per request (the
    same id on every call of a stream) only the rows from each stream's first
    incomplete chunk on are computed; the result is bit-identical to the full
    recomputation.  A stream's tokens may only grow between its calls, and its
    prompt and speaker embedding must stay the same (the cached state depends on
    them).  A finalised stream is released from the cache."""
    if cache is not None:
        return _streaming_with_cache(flow, token_list, prompt_features, speaker_embeddings, finalize_list,
                                     num_timesteps, cache, stream_ids)
    if len(token_list) != len(finalize_list):
        raise ValueError("token_list and finalize_list must have the same length")
    fe = prepare_frontend(flow)
    dev, dt = fe.device, fe.dtype
    R = len(token_list)
    with torch.cuda.device(dev):
        # F.normalize in float32, then the projection in the flow dtype (flashinfer_flow.py:219-220)
        spk = _speaker_rows(fe, speaker_embeddings.to(device=dev, dtype=torch.float32))
        out_lens = []
        for r, (tl, fin) in enumerate(zip(token_list, finalize_list)):
            if not fin and len(tl) < fe.lookahead:
                raise ValueError(f"non-final stream {r} has fewer than {fe.lookahead} lookahead tokens")
            out_lens.append(len(tl) if fin else len(tl) - fe.lookahead)
        mu, cond, mel_lens, mel_cu, mel_cu_d, prompt_lens = _packed_front(flow, fe, token_list, prompt_features,
                                                                          out_lens)
        max_mel = max(mel_lens) if mel_lens else 0
        if fe.rand_noise is None or fe.rand_noise.shape[2] < max_mel:
            raise ValueError("the decoder's noise prefix is shorter than the longest stream")
        x0 = torch.empty(max(mel_cu[-1], 1), 80, dtype=torch.float32, device=dev)[:mel_cu[-1]]
        call("fcv_pack_rows", fe.rand_noise.data_ptr(), _dtype_code(dt), 0, int(fe.rand_noise.shape[2]),
             mel_cu_d.data_ptr(), R, max_mel, x0.data_ptr(), _lib.DTYPE_F32, _stream(dev))
        x = solve_euler_packed(flow.decoder, x0, mu, mel_lens, spk, cond, num_timesteps, streaming=True)
        return _split(x, mel_cu, prompt_lens)


def _streaming_with_cache(flow, token_list, prompt_features, speaker_embeddings, finalize_list, num_timesteps,
                          cache: PrefixCache, stream_ids) -> list[torch.Tensor]:
    if len(token_list) != len(finalize_list):
        raise ValueError("token_list and finalize_list must have the same length")
    if stream_ids is None or len(stream_ids) != len(token_list) or len(set(stream_ids)) != len(stream_ids):
        raise ValueError("one distinct stream id per request is required with a prefix cache")
    if num_timesteps != cache.steps:
        raise ValueError(f"the cache holds {cache.steps} ODE steps, not {num_timesteps}")
    fe = prepare_frontend(flow)
    dev, dt = fe.device, fe.dtype
    if dev != cache.device or dt != cache.dtype:
        raise ValueError("the prefix cache belongs to another device or dtype")
    R = len(token_list)
    with torch.cuda.device(dev):
        spk = _speaker_rows(fe, speaker_embeddings.to(device=dev, dtype=torch.float32))
        out_lens = []
        for r, (tl, fin) in enumerate(zip(token_list, finalize_list)):
            if not fin and len(tl) < fe.lookahead:
                raise ValueError(f"non-final stream {r} has fewer than {fe.lookahead} lookahead tokens")
            out_lens.append(len(tl) if fin else len(tl) - fe.lookahead)
        mu, cond, mel_lens, mel_cu, mel_cu_d, prompt_lens = _packed_front(flow, fe, token_list, prompt_features,
                                                                          out_lens)
        max_mel = max(mel_lens) if mel_lens else 0
        if fe.rand_noise is None or fe.rand_noise.shape[2] < max_mel:
            raise ValueError("the decoder's noise prefix is shorter than the longest stream")
        states = [cache._acquire(sid) for sid in stream_ids]
        for r, st in enumerate(states):
            if mel_lens[r] > cache.cap:
                raise ValueError(f"stream {stream_ids[r]!r} has {mel_lens[r]} frames, the cache holds {cache.cap}")
            if mel_lens[r] < st[1]:
                raise ValueError(f"stream {stream_ids[r]!r} shrank below its cached {st[1]} frames")
        pos0 = [st[1] for st in states]
        new_lens = [L - p for L, p in zip(mel_lens, pos0)]
        nxt = [L if fin else (L // cache.chunk) * cache.chunk for L, fin in zip(mel_lens, finalize_list)]
        # full noise rows as the non-cached path forms them, then the new rows of every request
        x0_all = torch.empty(max(mel_cu[-1], 1), 80, dtype=torch.float32, device=dev)[:mel_cu[-1]]
        call("fcv_pack_rows", fe.rand_noise.data_ptr(), _dtype_code(dt), 0, int(fe.rand_noise.shape[2]),
             mel_cu_d.data_ptr(), R, max_mel, x0_all.data_ptr(), _lib.DTYPE_F32, _stream(dev))
        idx = torch.cat([torch.arange(mel_cu[r] + pos0[r], mel_cu[r + 1]) for r in range(R)]).to(dev) \
            if sum(new_lens) else torch.zeros(0, dtype=torch.long, device=dev)
        x_new = _solve_euler_prefix(flow.decoder, cache, x0_all.index_select(0, idx), mu.index_select(0, idx),
                                    cond.index_select(0, idx), spk, new_lens, pos0, [st[0] for st in states], nxt,
                                    num_timesteps)
        outs, o = [], 0
        for r, st in enumerate(states):
            slot, n = st[0], new_lens[r]
            rows = torch.cat([cache.final[slot, :pos0[r]], x_new[o:o + n]])
            cache.final[slot, pos0[r]:nxt[r]].copy_(x_new[o:o + nxt[r] - pos0[r]])
            st[1] = nxt[r]
            outs.append(rows[prompt_lens[r]:].t().unsqueeze(0).contiguous())
            o += n
        for sid, fin in zip(stream_ids, finalize_list):
            if fin:
                cache.release(sid)
        return outs
