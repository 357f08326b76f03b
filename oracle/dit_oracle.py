"""CPU oracle for the packed DiT estimator hot path -- TEST INFRASTRUCTURE ONLY.

This module is a numpy restatement of the reference algorithm.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline arm may import it,
and only as the checker (or the timed CPU baseline).  The product path in
``faster-cosyvoice_b200`` never imports it and has no CPU fallback.

Every function cites the reference file:line it restates (paths are relative to
the reference project root, ``faster_cosyvoice/token2wav/...``).

Pinning: the functions here are checked against golden vectors produced by the
reference's own torch code (``tests/golden/make_golden.py`` imports the
reference DiT, mask utilities, pack-layout and Euler solver and records their
outputs); ``tests/test_oracle_golden.py`` runs that check.  The one part of the
reference that is not importable anywhere is the third-party
``x_transformers==2.23.5`` rotary helper (``pyproject.toml:20``); its semantics
are pinned only through the reference's in-repo restatements
(``flashinfer_dit.py:262-273, 586-594``; ``flashinfer_kernels.py:167-192``).

Numerics: everything is computed in float32 (numpy IEEE arithmetic, BLAS
matmuls).  ``emulate_bf16_time=True`` reproduces the one place where the
reference's reduced-precision path changes the *semantics* rather than adding
rounding noise: ``SinusPositionEmbedding`` computes ``scale * t`` in the input
dtype (``modules.py:81``), so a bf16 estimator sees ``bf16(1000*t)``, and the
sinusoid is cast back to the input dtype (``modules.py:614``).
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass

import numpy as np

DIM = 1024
HEADS = 16
DIM_HEAD = 64
FF_INNER = 2048
MEL = 80
ROPE_DIM = 64
CONV_K = 31
CONV_GROUPS = 16
LN_EPS = 1e-6
CFG_RATE = 0.7


# ---------------------------------------------------------------------------
# bf16 helpers (round-to-nearest-even, as torch's float->bfloat16 cast)
# ---------------------------------------------------------------------------

def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); returns float32."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) << 16
    out = r.astype(np.uint32).view(np.float32)
    nan = np.isnan(a)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


# ---------------------------------------------------------------------------
# Pack layout: flashinfer_dit.py:364-405, flashinfer_attention.py:82-86
# ---------------------------------------------------------------------------

@dataclass
class PackedLayout:
    lengths: np.ndarray  # (B,) int64
    gather_indices: np.ndarray  # (N,) int64, row*T + [0, L_row)
    document_ids: np.ndarray  # (N,) int32
    positions: np.ndarray  # (N,) int32
    cu_seqlens: np.ndarray  # (B+1,) int32


def lengths_from_mask(mask: np.ndarray) -> np.ndarray:
    """Document lengths from a (B,1,T) 0/1 mask (``flashinfer_dit.py:460``).

    The reference sums the mask in the activation dtype; this counts the ones
    exactly (integers), which equals the reference for every length that its
    dtype represents exactly (fp16: all lengths <= 2048 and even lengths to
    4096; fp32: all)."""
    m = np.asarray(mask)
    return (m[:, 0, :] > 0.5).sum(-1).astype(np.int64)


def pack_layout(lengths, padded_length: int) -> PackedLayout:
    """Restates ``FlashInferDiT._get_packed_layout`` (``flashinfer_dit.py:376-392``)
    and ``RaggedAttentionRunner._make_indptr`` (``flashinfer_attention.py:82-86``)."""
    lengths = np.asarray(lengths, dtype=np.int64).reshape(-1)
    T = int(padded_length)
    if lengths.size:
        gather = np.concatenate(
            [np.arange(r * T, r * T + int(L), dtype=np.int64) for r, L in enumerate(lengths)]
        )
        positions = np.concatenate([np.arange(int(L), dtype=np.int32) for L in lengths])
    else:
        gather = np.zeros(0, np.int64)
        positions = np.zeros(0, np.int32)
    doc_ids = np.repeat(np.arange(lengths.size, dtype=np.int32), lengths)
    cu = np.zeros(lengths.size + 1, dtype=np.int32)
    cu[1:] = np.cumsum(lengths)
    return PackedLayout(lengths, gather, doc_ids, positions, cu)


def chunk_causal_mask_flat(lengths, chunk: int) -> np.ndarray:
    """Flattened per-document chunk mask (``flashinfer_attention.py:16-33``):
    key k visible from query q iff ``k // chunk <= q // chunk``."""
    out = []
    for L in np.asarray(lengths).reshape(-1):
        p = np.arange(int(L))
        out.append((p[None, :] // chunk <= p[:, None] // chunk).reshape(-1))
    return np.concatenate(out) if out else np.zeros(0, bool)


def visible_pairs(lengths, chunk: int | None) -> int:
    """Number of visible (q, k) pairs P used by the FLOP model."""
    total = 0
    for L in np.asarray(lengths).reshape(-1):
        L = int(L)
        if chunk is None or chunk <= 0:
            total += L * L
        else:
            q = np.arange(L)
            total += int(np.minimum(L, (q // chunk + 1) * chunk).sum())
    return total


# ---------------------------------------------------------------------------
# Parameters (state-dict keys of the reference DiT, dit.py:104-143)
# ---------------------------------------------------------------------------

def block_key(i: int, name: str) -> str:
    return f"transformer_blocks.{i}.{name}"


def count_blocks(params: dict) -> int:
    n = 0
    while block_key(n, "attn.to_q.weight") in params:
        n += 1
    return n


# ---------------------------------------------------------------------------
# Building blocks
# ---------------------------------------------------------------------------

def _linear(x, w, b=None):
    y = x @ w.T
    if b is not None:
        y = y + b
    return y.astype(np.float32, copy=False)


def _silu(x):
    return (x / (1.0 + np.exp(-x))).astype(np.float32)


def _mish(x):
    # x * tanh(softplus(x)), softplus computed stably
    sp = np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0))))
    return (x * np.tanh(sp)).astype(np.float32)


def _gelu_tanh(x):
    c = math.sqrt(2.0 / math.pi)
    return (0.5 * x * (1.0 + np.tanh(c * (x + 0.044715 * x * x * x)))).astype(np.float32)


def layer_norm(x):
    """Affine-free LayerNorm, eps 1e-6 (``modules.py:237, 513``)."""
    mu = x.mean(-1, keepdims=True, dtype=np.float64).astype(np.float32)
    c = x - mu
    var = (c.astype(np.float64) ** 2).mean(-1, keepdims=True).astype(np.float32)
    return (c / np.sqrt(var + np.float32(LN_EPS))).astype(np.float32)


def layer_norm_modulate(h, shift, scale_plus_one):
    """``flashinfer_kernels.py:83-108``: LN(h) * scale' + shift with scale' = 1 + scale."""
    return (layer_norm(h) * scale_plus_one + shift).astype(np.float32)


def gate_residual_layer_norm_modulate(h, gate, r, shift, scale_plus_one):
    """``flashinfer_kernels.py:110-145``: h += gate*r; norm = LN(h)*scale' + shift."""
    h2 = (h + gate * r).astype(np.float32)
    return h2, layer_norm_modulate(h2, shift, scale_plus_one)


def sinus_embed(t, dim=256, scale=1000.0, emulate_bf16_time=False):
    """``SinusPositionEmbedding.forward`` (``modules.py:76-83``) followed by the
    cast to the input dtype in ``TimestepEmbedding.forward`` (``modules.py:614``)."""
    t = np.asarray(t, np.float32).reshape(-1)
    half = dim // 2
    e = math.log(10000) / (half - 1)
    freqs = np.exp(np.arange(half, dtype=np.float32) * np.float32(-e)).astype(np.float32)
    st = (np.float32(scale) * t).astype(np.float32)
    if emulate_bf16_time:
        st = bf16_round(st)
    arg = (st[:, None] * freqs[None, :]).astype(np.float32)
    emb = np.concatenate([np.sin(arg), np.cos(arg)], -1).astype(np.float32)
    if emulate_bf16_time:
        emb = bf16_round(emb)
    return emb


def time_embedding(params, t, emulate_bf16_time=False):
    """``TimestepEmbedding`` (``modules.py:606-616``): sinusoid -> Linear -> SiLU -> Linear."""
    h = sinus_embed(t, emulate_bf16_time=emulate_bf16_time)
    h = _linear(h, params["time_embed.time_mlp.0.weight"], params["time_embed.time_mlp.0.bias"])
    h = _silu(h)
    return _linear(h, params["time_embed.time_mlp.2.weight"], params["time_embed.time_mlp.2.bias"])


def modulations(params, temb, depth):
    """Per-block AdaLN-Zero chunks (``modules.py:239-244``) and the final
    (scale, shift) (``modules.py:260-265``).  Scale chunks are returned as
    ``1 + scale`` (the fold at ``flashinfer_dit.py:253-260``)."""
    s = _silu(temb)
    blocks = []
    for i in range(depth):
        e = _linear(s, params[block_key(i, "attn_norm.linear.weight")],
                    params[block_key(i, "attn_norm.linear.bias")])
        sh_a, sc_a, g_a, sh_f, sc_f, g_f = np.split(e, 6, axis=-1)
        blocks.append((sh_a, 1.0 + sc_a, g_a, sh_f, 1.0 + sc_f, g_f))
    e = _linear(s, params["norm_out.linear.weight"], params["norm_out.linear.bias"])
    sc, sh = np.split(e, 2, axis=-1)
    return blocks, (sh, 1.0 + sc)


def rope_tables(max_len: int):
    """Partial-RoPE angles (``flashinfer_dit.py:262-273``): theta[p, j] = p * 10000^(-2j/64)."""
    inv = (1.0 / (10000.0 ** (np.arange(0, ROPE_DIM, 2, dtype=np.float32) / ROPE_DIM))).astype(np.float32)
    th = (np.arange(max_len, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    return np.cos(th).astype(np.float32), np.sin(th).astype(np.float32)


def apply_partial_rope(x, positions):
    """Rotate columns [0, 64) of a (n, 1024) Q or K block on interleaved pairs
    (``flashinfer_kernels.py:224-249``; x_transformers ``apply_rotary_pos_emb``)."""
    cos, sin = rope_tables(int(positions.max()) + 1 if positions.size else 1)
    c = cos[positions]
    s = sin[positions]
    a = x[:, 0:ROPE_DIM:2]
    b = x[:, 1:ROPE_DIM:2]
    out = x.copy()
    out[:, 0:ROPE_DIM:2] = a * c - b * s
    out[:, 1:ROPE_DIM:2] = b * c + a * s
    return out


def causal_group_conv(h, w, b):
    """One ``Conv1d(1024, 1024, 31, groups=16)`` with causal left zero pad 30
    (``modules.py:134-139``) on one document h (L, 1024)."""
    L = h.shape[0]
    G, cpg = CONV_GROUPS, DIM // CONV_GROUPS
    hp = np.concatenate([np.zeros((CONV_K - 1, DIM), np.float32), h], 0)
    out = np.empty((L, DIM), np.float32)
    # windows: (L, K, C) via stride tricks
    win = np.lib.stride_tricks.sliding_window_view(hp, CONV_K, axis=0)  # (L, C, K)
    for g in range(G):
        wg = w[g * cpg:(g + 1) * cpg]  # (cpg_out, cpg_in, K)
        xg = win[:, g * cpg:(g + 1) * cpg, :]  # (L, cpg_in, K)
        out[:, g * cpg:(g + 1) * cpg] = np.einsum("lck,ock->lo", xg, wg, optimize=True)
    return (out + b).astype(np.float32)


def input_embed(params, x, cond, mu, spk):
    """``InputEmbedding.forward`` (``dit.py:84-98``) on one document: x, cond, mu
    (L, 80), spk (80,) -> (L, 1024), including ``CausalConvPositionEmbedding``
    (``modules.py:129-144``) and its residual."""
    L = x.shape[0]
    cat = np.concatenate([x, cond, mu, np.broadcast_to(spk, (L, MEL))], -1).astype(np.float32)
    h = _linear(cat, params["input_embed.proj.weight"], params["input_embed.proj.bias"])
    c1 = _mish(causal_group_conv(h, params["input_embed.conv_pos_embed.conv1.0.weight"],
                                 params["input_embed.conv_pos_embed.conv1.0.bias"]))
    c2 = _mish(causal_group_conv(c1, params["input_embed.conv_pos_embed.conv2.0.weight"],
                                 params["input_embed.conv_pos_embed.conv2.0.bias"]))
    return (c2 + h).astype(np.float32)


_POOL = None


def _head_pool():
    """Threads for the per-head attention loop (numpy releases the GIL in its
    BLAS calls and ufuncs; no processes are forked)."""
    global _POOL
    if _POOL is None:
        from concurrent.futures import ThreadPoolExecutor

        _POOL = ThreadPoolExecutor(max_workers=min(HEADS, os.cpu_count() or 1))
    return _POOL


def attention_doc(q, k, v, chunk: int | None, threaded_heads: bool = True):
    """Per-document multi-head attention with scale 1/8 and the optional
    chunk-causal mask (``modules.py:349-407``; mask ``mask.py:127-158, 223-229``).

    One head per thread (``threaded_heads``; else the heads in turn, for callers
    that already run documents in parallel), plain 2-D BLAS matmuls on one BLAS thread:
    s = (q/8) k^T (+ the 0/-inf chunk mask), p = exp(s - rowmax),
    o = (p v) / rowsum(p).  Scaling q by 1/8 is exact in float32."""
    L = q.shape[0]
    qh = np.ascontiguousarray((q * np.float32(DIM_HEAD ** -0.5)).reshape(L, HEADS, DIM_HEAD).transpose(1, 0, 2),
                              dtype=np.float32)
    kt = np.ascontiguousarray(k.reshape(L, HEADS, DIM_HEAD).transpose(1, 2, 0), dtype=np.float32)
    vh = np.ascontiguousarray(v.reshape(L, HEADS, DIM_HEAD).transpose(1, 0, 2), dtype=np.float32)
    add = None
    if chunk:
        p = np.arange(L)
        add = np.where((p[None, :] // chunk) <= (p[:, None] // chunk), np.float32(0), np.float32(-np.inf))
        add = add.astype(np.float32)
    out = np.empty((L, HEADS, DIM_HEAD), np.float32)

    def head(h):
        s = qh[h] @ kt[h]
        if add is not None:
            s += add
        s -= s.max(-1, keepdims=True)
        np.exp(s, out=s)
        out[:, h] = (s @ vh[h]) / s.sum(-1, keepdims=True)

    if not threaded_heads:
        for h in range(HEADS):
            head(h)
        return out.reshape(L, DIM)
    with _blas_threads(1):
        list(_head_pool().map(head, range(HEADS)))
    return out.reshape(L, DIM)


class _blas_threads:
    """Limit the BLAS thread pool inside a block (no-op without threadpoolctl)."""

    def __init__(self, n: int):
        self.n, self.limit = n, None

    def __enter__(self):
        try:
            from threadpoolctl import threadpool_limits

            self.limit = threadpool_limits(limits=self.n, user_api="blas")
        except Exception:
            self.limit = None
        return self

    def __exit__(self, *exc):
        if self.limit is not None:
            self.limit.restore_original_limits()


# ---------------------------------------------------------------------------
# The estimator
# ---------------------------------------------------------------------------

def _doc_forward(params, depth, blocks, final, d, doc, chunk, threaded_heads):
    """One document of :func:`dit_forward_docs` (its modulation rows are row d)."""
    x, mu, cond, spk = doc
    fsh, fsc = final
    L = x.shape[1]
    h = input_embed(params, x.T.astype(np.float32), cond.T.astype(np.float32),
                    mu.T.astype(np.float32), np.asarray(spk, np.float32))
    pos = np.arange(L, dtype=np.int32)
    for i in range(depth):
        sh_a, sc_a, g_a, sh_f, sc_f, g_f = (m[d] for m in blocks[i])
        norm = layer_norm_modulate(h, sh_a, sc_a)
        wq = np.concatenate([params[block_key(i, f"attn.to_{n}.weight")] for n in "qkv"], 0)
        bq = np.concatenate([params[block_key(i, f"attn.to_{n}.bias")] for n in "qkv"], 0)
        qkv = _linear(norm, wq, bq)
        q = apply_partial_rope(qkv[:, :DIM], pos)
        k = apply_partial_rope(qkv[:, DIM:2 * DIM], pos)
        v = qkv[:, 2 * DIM:]
        o = attention_doc(q, k, v, chunk, threaded_heads)
        a = _linear(o, params[block_key(i, "attn.to_out.0.weight")],
                    params[block_key(i, "attn.to_out.0.bias")])
        h, ffin = gate_residual_layer_norm_modulate(h, g_a, a, sh_f, sc_f)
        f = _gelu_tanh(_linear(ffin, params[block_key(i, "ff.ff.0.0.weight")],
                               params[block_key(i, "ff.ff.0.0.bias")]))
        f = _linear(f, params[block_key(i, "ff.ff.2.weight")], params[block_key(i, "ff.ff.2.bias")])
        h = (h + g_f * f).astype(np.float32)
    norm = layer_norm_modulate(h, fsh[d], fsc[d])
    out = _linear(norm, params["proj_out.weight"], params["proj_out.bias"])
    return out.T.copy()


def dit_forward_docs(params, docs, t, chunk: int | None = None, emulate_bf16_time=False):
    """DiT forward over a list of documents.

    ``docs`` is a list of (x, mu, cond, spk) with x/mu/cond of shape (80, L_i)
    and spk (80,); ``t`` has one value per document.  Returns a list of
    (80, L_i) float32 outputs.  Semantics: ``DiT.forward`` (``dit.py:145-176``)
    restricted to the valid frames of each padded row, which is exactly what
    ``FlashInferDiT._forward_packed`` (``flashinfer_dit.py:447-543``) computes.

    Documents are independent.  Long ones (>= 1024 frames) run one after the
    other with all BLAS threads and one thread per attention head; the short
    ones run on parallel threads (longest first) with one BLAS thread each.
    The arithmetic of each document is the same either way.
    """
    depth = count_blocks(params)
    temb = time_embedding(params, np.asarray(t, np.float32), emulate_bf16_time)
    blocks, final = modulations(params, temb, depth)
    outs = [None] * len(docs)
    short = []
    for d, doc in enumerate(docs):
        if doc[0].shape[1] >= 1024 or len(docs) == 1:
            outs[d] = _doc_forward(params, depth, blocks, final, d, doc, chunk, True)
        else:
            short.append(d)
    if short:
        from concurrent.futures import ThreadPoolExecutor

        short.sort(key=lambda d: -docs[d][0].shape[1])

        def run(d):
            outs[d] = _doc_forward(params, depth, blocks, final, d, docs[d], chunk, False)

        with _blas_threads(1), ThreadPoolExecutor(max_workers=min(len(short), os.cpu_count() or 1)) as pool:
            list(pool.map(run, short))
    return outs


def dit_forward_padded(params, x, mask, mu, t, spks, cond, streaming=False, chunk=50,
                       emulate_bf16_time=False):
    """Padded-batch interface of ``DiT.forward`` / ``FlashInferDiT.forward``:
    x, mu, cond (B, 80, T), mask (B, 1, T), t (B,), spks (B, 80) -> (B, 80, T).
    Padding frames of the result are zero (the packed path's unpack,
    ``flashinfer_dit.py:536-543``)."""
    x = np.asarray(x, np.float32)
    B, _, T = x.shape
    lengths = lengths_from_mask(mask)
    docs = [(x[b, :, :L], np.asarray(mu[b, :, :L], np.float32), np.asarray(cond[b, :, :L], np.float32),
             np.asarray(spks[b], np.float32)) for b, L in enumerate(lengths)]
    outs = dit_forward_docs(params, docs, np.asarray(t, np.float32).reshape(-1),
                            chunk if streaming else None, emulate_bf16_time)
    y = np.zeros((B, MEL, T), np.float32)
    for b, L in enumerate(lengths):
        y[b, :, :L] = outs[b]
    return y


# ---------------------------------------------------------------------------
# Euler / CFG solver: flashinfer_flow.py:16-74
# ---------------------------------------------------------------------------

def cosine_time_span(num_steps: int = 10, emulate_bf16=False):
    """``torch.linspace(0, 1, n+1)`` then ``1 - cos(t*pi/2)`` in the input dtype
    (``flashinfer_flow.py:34-41``)."""
    ts = np.array([k / num_steps for k in range(num_steps + 1)], np.float32)
    if emulate_bf16:
        ts = bf16_round(ts)
        arg = bf16_round((ts * np.float32(0.5)).astype(np.float32))
        arg = bf16_round((arg * np.float32(math.pi)).astype(np.float32))
        c = bf16_round(np.cos(arg).astype(np.float32))
        return bf16_round((np.float32(1.0) - c).astype(np.float32))
    return (np.float32(1.0) - np.cos(ts * np.float32(0.5) * np.float32(math.pi))).astype(np.float32)


def solve_euler_docs(params, noise_docs, mu_docs, cond_docs, spks, num_steps=10,
                     streaming=False, chunk=50, cfg_rate=CFG_RATE, emulate_bf16=False,
                     bf16_sample=False, bf16_schedule=None):
    """CFG-doubled Euler solver over documents (``flashinfer_flow.py:16-74``):
    the unconditional half has mu, spks and cond zeroed (``:45-51``), the
    sample is repeated (``:55``), ``d = (1+r) d_c - r d_u`` (``:66-69``),
    ``x += dt d`` with the cosine schedule (``:34-43, 70-73``).  fp32.

    ``emulate_bf16=True`` reproduces the semantics of a bf16 solver call: the
    schedule, t and dt are computed in bf16 (the solver works in
    ``speaker_embeddings.dtype``, ``:34-43, 70-73``), the estimator sees
    bf16-rounded inputs and ``bf16(1000 t)``; the sample itself stays float32.

    ``bf16_schedule=False`` (with ``emulate_bf16``) keeps the schedule, t and dt
    in float32 -- a solver call whose speaker rows are float32 -- while the
    bf16 estimator still sees bf16(t) and bf16(1000 bf16(t)).

    ``bf16_sample=True`` (with ``emulate_bf16``) also follows the reference
    solver's own bf16 arithmetic: the sample starts as bf16(noise) and every
    operation of the CFG combine and the Euler update (``:57-70``) -- the scaled
    halves, their difference, the step and the sum -- is rounded to bf16, the
    estimator output being bf16 as well."""
    sched16 = emulate_bf16 if bf16_schedule is None else (emulate_bf16 and bf16_schedule)
    ts = cosine_time_span(num_steps, sched16)
    rnd = (lambda v: np.float32(bf16_round(np.asarray(v, np.float32)))) if sched16 else np.float32
    inp = bf16_round if emulate_bf16 else (lambda a: a)
    R = len(noise_docs)
    xs = [np.asarray(n, np.float32).copy() for n in noise_docs]
    b16 = bf16_round if (emulate_bf16 and bf16_sample) else (lambda a: a)
    xs = [b16(x) for x in xs]
    t = ts[0]
    dt = rnd(ts[1] - ts[0])
    for step in range(1, num_steps + 1):
        docs = [(inp(xs[i]), inp(mu_docs[i]), inp(cond_docs[i]), inp(spks[i])) for i in range(R)]
        docs += [(inp(xs[i]), np.zeros_like(mu_docs[i]), np.zeros_like(cond_docs[i]),
                  np.zeros_like(spks[i])) for i in range(R)]
        tt = np.full(2 * R, bf16_round(np.float32(t)) if emulate_bf16 else t, np.float32)
        d = dit_forward_docs(params, docs, tt, chunk if streaming else None, emulate_bf16_time=emulate_bf16)
        for i in range(R):
            if emulate_bf16 and bf16_sample:
                a = bf16_round(np.float32(1.0 + cfg_rate) * bf16_round(d[i]))
                b = bf16_round(np.float32(cfg_rate) * bf16_round(d[R + i]))
                xs[i] = bf16_round(xs[i] + bf16_round(dt * bf16_round(a - b)))
                continue
            der = (np.float32(1.0 + cfg_rate) * d[i] - np.float32(cfg_rate) * d[R + i]).astype(np.float32)
            xs[i] = (xs[i] + dt * der).astype(np.float32)
        t = rnd(t + dt)
        if step < num_steps:
            dt = rnd(ts[step + 1] - t)
    return xs


# ---------------------------------------------------------------------------
# FLOP model
# ---------------------------------------------------------------------------

def estimator_flops(lengths, chunk: int | None, depth: int = 22) -> int:
    """Algorithmic FLOPs of one estimator call over packed documents:
    per row 22*(QKV 6.29M + out 2.10M + FF 8.39M) + embed 0.66M + conv 8.13M
    + proj_out 0.16M; attention 4*H*dh = 4096 FLOPs per visible (q,k) pair and
    layer; per sequence the AdaLN projection and the time MLP."""
    lengths = np.asarray(lengths).reshape(-1)
    N = int(lengths.sum())
    per_row = depth * (2 * DIM * 3 * DIM + 2 * DIM * DIM + 2 * 2 * DIM * FF_INNER) \
        + 2 * 320 * DIM + 2 * 2 * DIM * (CONV_K * DIM // CONV_GROUPS) + 2 * DIM * MEL
    P = visible_pairs(lengths, chunk)
    per_seq = 2 * DIM * (depth * 6 * DIM + 2 * DIM) + 2 * (256 * DIM + DIM * DIM)
    return N * per_row + depth * 4 * HEADS * DIM_HEAD * P + lengths.size * per_seq
