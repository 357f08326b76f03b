"""CPU oracle for the packed flow front end -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's batched flow inference
(``faster_cosyvoice/token2wav/flashinfer_flow.py:118-281``): token embedding,
the pre-lookahead convolutions, repeat-interleave to the mel rate, the speaker
projection, the prompt condition and the CFG Euler ODE over the estimator.
Only ``tests/`` and ``bench.py``'s CPU arm may import it, and only as the
checker; the product path never does.

Pinning: ``tests/test_oracle_golden.py`` checks every function here against
``tests/golden/flow_frontend.npz``, which ``tests/golden/make_golden.py``
records from the reference's own ``flow_inference_batched`` and
``flow_inference_batched_streaming`` (and their front-end intermediates) on a
``CausalMaskedDiffWithDiT`` built as ``builders.py:16-45`` does.

Numerics: float32 throughout (numpy IEEE arithmetic, BLAS matmuls).
"""

from __future__ import annotations

import numpy as np

from . import dit_oracle as D

LOOKAHEAD = 3       # pre_lookahead_len (builders.py:41)
TOKEN_MEL_RATIO = 2  # token_mel_ratio (builders.py:41)
LRELU_SLOPE = 0.01  # F.leaky_relu default (upsample_encoder.py:84)


def token_embed(table: np.ndarray, tokens) -> np.ndarray:
    """``input_embedding(clamp(token, min=0))`` (``flashinfer_flow.py:148``,
    ``flow.py:381``): rows of the (vocab, 80) table."""
    return table[np.maximum(np.asarray(tokens, np.int64), 0)].astype(np.float32)


def pre_lookahead(emb: np.ndarray, w1, b1, w2, b2, n_out: int, emulate_bf16: bool = False) -> np.ndarray:
    """``PreLookaheadLayer.forward`` (``upsample_encoder.py:71-92``) on one document.

    ``emb`` (L_in, 80) holds the embedded tokens, the context tokens of a
    non-final stream included; ``n_out`` = L_in for a final stream or an offline
    document (three zero rows padded on the right, ``:79``) and L_in - 3 when the
    last three rows are context (``:83``).  conv1 (kernel 4, no padding) reads
    rows p..p+3, zeros past L_in; LeakyReLU; conv2 (kernel 3) is causal with two
    zero rows on the left (``:86-87``); the residual adds emb[:n_out] (``:91``).
    ``emulate_bf16``: the hidden activation is stored in bf16 between the two
    convolutions, as a bf16 module does (fp32 accumulation inside each)."""
    L, C = emb.shape
    k1 = w1.shape[2]
    k2 = w2.shape[2]
    hid = w1.shape[0]
    pad = np.zeros((max(0, n_out + k1 - 1 - L), C), np.float32)
    src = np.concatenate([emb, pad], 0)
    a1 = np.concatenate([src[k:k + n_out] for k in range(k1)], 1)               # [p, k*C + c]
    w1r = np.transpose(w1, (0, 2, 1)).reshape(hid, k1 * C).astype(np.float32)  # [o, k*C + c]
    h1 = (a1 @ w1r.T + b1).astype(np.float32)
    h1 = np.where(h1 >= 0, h1, np.float32(LRELU_SLOPE) * h1).astype(np.float32)
    if emulate_bf16:
        h1 = D.bf16_round(h1)
    hp = np.concatenate([np.zeros((k2 - 1, hid), np.float32), h1], 0)
    a2 = np.concatenate([hp[k:k + n_out] for k in range(k2)], 1)
    w2r = np.transpose(w2, (0, 2, 1)).reshape(w2.shape[0], k2 * hid).astype(np.float32)
    out = (a2 @ w2r.T + b2).astype(np.float32)
    return (out + emb[:n_out]).astype(np.float32)


def frontend_mu(fe: dict, tokens, finalize: bool = True, ratio: int = TOKEN_MEL_RATIO,
                emulate_bf16: bool = False) -> np.ndarray:
    """mu rows (ratio * n_out, 80) of one document: ``_streaming_token_features``
    (``flashinfer_flow.py:167-184``) and, with ``finalize=True``, the per-document
    rows of the batched offline front end (``:144-152``).  ``emulate_bf16``: the
    rows are stored in bf16 (the estimator's input type)."""
    emb = token_embed(fe["input_embedding.weight"], tokens)
    n_out = emb.shape[0] if finalize else emb.shape[0] - LOOKAHEAD
    h = pre_lookahead(emb, fe["pre_lookahead_layer.conv1.weight"], fe["pre_lookahead_layer.conv1.bias"],
                      fe["pre_lookahead_layer.conv2.weight"], fe["pre_lookahead_layer.conv2.bias"], n_out,
                      emulate_bf16)
    if emulate_bf16:
        h = D.bf16_round(h)
    return np.repeat(h, ratio, axis=0)


def speaker_projection(fe: dict, spk: np.ndarray, emulate_bf16: bool = False) -> np.ndarray:
    """``spk_embed_affine_layer(F.normalize(spk, dim=1))`` (``flashinfer_flow.py:145-146``).
    ``emulate_bf16``: the normalised vector and the result are stored in bf16."""
    spk = np.asarray(spk, np.float32)
    n = np.sqrt((spk.astype(np.float64) ** 2).sum(1, keepdims=True))
    x = (spk / np.maximum(n, 1e-12)).astype(np.float32)
    if emulate_bf16:
        x = D.bf16_round(x)
    y = (x @ fe["spk_embed_affine_layer.weight"].T + fe["spk_embed_affine_layer.bias"]).astype(np.float32)
    return D.bf16_round(y) if emulate_bf16 else y


def prompt_condition(prompt: np.ndarray, n_mel: int) -> np.ndarray:
    """One document's condition (n_mel, 80): prompt Mel rows first, zeros after
    (``_copy_prompt_features``, ``flashinfer_flow.py:95-115``)."""
    c = np.zeros((n_mel, prompt.shape[1]), np.float32)
    c[:prompt.shape[0]] = prompt
    return c


def flow_inference_docs(fe: dict, dit_params: dict, token_lists, prompts, spk, noise_docs,
                        finalize=None, streaming: bool = False, num_steps: int = 10,
                        emulate_bf16: bool = False):
    """Batched flow inference over documents (``flashinfer_flow.py:118-164`` offline,
    ``:187-281`` streaming with ``finalize``): returns the generated Mel of every
    request, (80, n_mel - prompt_len) each.  ``noise_docs`` are (80, n_mel).
    ``emulate_bf16``: the storage points and time semantics of a bf16 flow
    (front-end rows, speaker rows, prompt rows and noise in bf16; the solver as
    ``solve_euler_docs(emulate_bf16=True)``), arithmetic in fp32."""
    R = len(token_lists)
    fin = [True] * R if finalize is None else list(finalize)
    rnd = D.bf16_round if emulate_bf16 else (lambda a: a)
    spk_p = speaker_projection(fe, spk, emulate_bf16)
    mu = [frontend_mu(fe, token_lists[i], fin[i], emulate_bf16=emulate_bf16) for i in range(R)]
    cond = [rnd(prompt_condition(prompts[i], mu[i].shape[0])) for i in range(R)]
    xs = D.solve_euler_docs(dit_params, [rnd(np.asarray(n, np.float32)) for n in noise_docs],
                            [m.T.copy() for m in mu], [c.T.copy() for c in cond], list(spk_p),
                            num_steps=num_steps, streaming=streaming, emulate_bf16=emulate_bf16)
    return [xs[i][:, prompts[i].shape[0]:] for i in range(R)]
