"""Device-packed flow front end on the GPU, through the C ABI (fcv_flow_frontend,
fcv_speaker_projection, fcv_prompt_rows, fcv_pack_rows, fcv_dit_forward with
packed rows), against the reference's own outputs (tests/golden/flow_frontend.npz,
recorded from flashinfer_flow.py:118-281) and the oracle."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import ensure_built, flow_case, load_golden, make_flow, make_model, rel_l2

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _built():
    ensure_built()
    yield
    from fcv_b200 import ops

    assert ops.device_error() == 0


def _flow(dtype):
    f = make_flow(4, 2).to(DEV, dtype)
    f.decoder.estimator.finalize_weights()
    return f


def _inputs(c, dtype=torch.float32):
    prompts = [torch.tensor(p, device=DEV).unsqueeze(0) for p in c["prompts"]]
    spk = torch.tensor(c["spk"], device=DEV)
    return [t.tolist() for t in c["tokens"]], prompts, spk


@pytest.mark.parametrize("dtype,tol", [("float32", 1e-5), ("bfloat16", 1e-2)])
@pytest.mark.parametrize("mode", ["offline", "streaming"])
def test_frontend_rows_match_reference(dtype, tol, mode):
    """mu rows (embedding, pre-lookahead convolutions, repeat-interleave), the
    speaker projection and the prompt condition rows vs the reference."""
    from fcv_b200 import flow as FL

    dt = getattr(torch, dtype)
    flow = _flow(dt)
    c = flow_case(load_golden("flow_frontend"), mode)
    tokens, prompts, spk = _inputs(c)
    fe = FL.prepare_frontend(flow)
    fin = c["finalize"] or [True] * len(tokens)
    out_lens = [len(t) if f else len(t) - 3 for t, f in zip(tokens, fin)]
    mu, cond, mel_lens, mel_cu, _, prompt_lens = FL._packed_front(flow, fe, tokens, prompts, out_lens)
    spk_rows = FL._speaker_rows(fe, spk.to(dt) if mode == "offline" else spk)
    torch.cuda.synchronize()
    assert mel_lens == [m.shape[0] for m in c["mu"]]
    mu = mu.float().cpu().numpy()
    for i, ref in enumerate(c["mu"]):
        assert rel_l2(mu[mel_cu[i]:mel_cu[i + 1]], ref) <= tol, (mode, i)
    assert rel_l2(spk_rows.float().cpu().numpy(), c["spk_proj"]) <= tol
    cond = cond.float().cpu().numpy()
    for i, p in enumerate(c["prompts"]):
        rows = cond[mel_cu[i]:mel_cu[i + 1]]
        assert np.array_equal(rows[:p.shape[0]], torch.tensor(p).to(dt).float().numpy()), (mode, i)
        assert not np.any(rows[p.shape[0]:]), (mode, i)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("mode", ["offline", "streaming"])
def test_flow_inference_matches_reference(dtype, mode):
    """The whole device-packed flow inference (10-step CFG ODE included) on the
    reference's weights, tokens, prompts, speakers and noise; max-abs gate 2e-2.

    float32: against the reference's own flow_inference_batched / _streaming
    output (golden), max-abs 1e-4.  bfloat16: against the oracle on the same
    bf16 weights with the semantics of a bf16 flow (schedule, t and dt in bf16
    because the solver works in the speaker-row dtype, flashinfer_flow.py:34-43;
    bf16(1000 t) in the estimator, modules.py:81; bf16 storage of mu, speaker,
    prompt rows and noise), max-abs 2e-2; and within 5e-2 of the float32 golden."""
    from fcv_b200.flow import flow_inference_batched, flow_inference_batched_streaming
    from oracle import flow_oracle as F

    dt = getattr(torch, dtype)
    flow = _flow(dt)
    z = load_golden("flow_frontend")
    c = flow_case(z, mode)
    tokens, prompts, spk = _inputs(c)
    n_mel = [m.shape[0] for m in c["mu"]]
    if mode == "offline":
        noise = torch.tensor(z["offline_noise"], device=DEV).to(dt)
        outs = flow_inference_batched(flow, tokens, prompts, spk, noise=noise)
        noise_docs = [noise[i, :, :n].float().cpu().numpy() for i, n in enumerate(n_mel)]
    else:
        outs = flow_inference_batched_streaming(flow, tokens, prompts, spk, c["finalize"])
        noise_docs = [flow.decoder.rand_noise[0, :, :n].float().cpu().numpy() for n in n_mel]
    assert len(outs) == len(c["out"])
    refs = [o.T for o in c["out"]]
    if dt == torch.bfloat16:
        sd = {k: v.detach().float().cpu().numpy() for k, v in flow.state_dict().items()}
        fe = {k: v for k, v in sd.items() if not k.startswith("decoder.")}
        dit = {k[len("decoder.estimator."):]: v for k, v in sd.items() if k.startswith("decoder.estimator.")}
        emu = F.flow_inference_docs(fe, dit, c["tokens"], c["prompts"], c["spk"], noise_docs,
                                    finalize=c["finalize"], streaming=mode == "streaming", emulate_bf16=True)
    for i, o in enumerate(outs):
        assert tuple(o.shape) == (1, 80, refs[i].shape[1]) and o.dtype == torch.float32, (mode, i)
        y = o[0].cpu().numpy()
        if dt == torch.float32:
            err = np.abs(y - refs[i]).max()
            assert err <= 1e-4, (mode, i, err)
        else:
            err = np.abs(y - emu[i]).max()
            assert err <= 2e-2, (mode, i, err)
            assert np.abs(y - refs[i]).max() <= 5e-2, (mode, i)


def test_flow_inference_rejects_bad_requests():
    from fcv_b200.flow import flow_inference_batched, flow_inference_batched_streaming

    flow = _flow(torch.float32)
    spk = torch.zeros(1, 192, device=DEV)
    with pytest.raises(IndexError):
        flow_inference_batched(flow, [[1, 2, 6561]], [torch.zeros(1, 2, 80, device=DEV)], spk)
    with pytest.raises(ValueError):
        flow_inference_batched(flow, [[1, 2, 3]], [torch.zeros(1, 7, 80, device=DEV)], spk)
    with pytest.raises(ValueError):
        flow_inference_batched_streaming(flow, [[1, 2]], [torch.zeros(1, 0, 80, device=DEV)], spk, [False])
    with pytest.raises(ValueError):
        flow_inference_batched_streaming(flow, [[1, 2, 3, 4]], [torch.zeros(1, 0, 80, device=DEV)], spk, [])


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_packed_rows_estimator_equals_padded_bit_exact(dtype):
    """fcv_dit_forward on packed (N, 80) rows gives exactly the padded path's
    valid frames: only the input gather and the output store differ."""
    dt = getattr(torch, dtype)
    model = make_model(2, 2).to(DEV, dt)
    model.finalize_weights()
    rng = np.random.default_rng(41)
    lengths = [173, 1, 60, 251]
    B, T = len(lengths), max(lengths)
    x, mu, cond = (torch.tensor(rng.standard_normal((B, 80, T)), device=DEV).to(dt) for _ in range(3))
    spks = torch.tensor(rng.standard_normal((B, 80)), device=DEV).to(dt)
    t = torch.tensor(rng.uniform(size=B), device=DEV).to(dt)
    for streaming in (False, True):
        lay = model.prepare_layout(lengths, T, streaming, torch.device(DEV))
        pad = model.forward_layout(lay, x, mu, t, spks, cond, out=torch.empty(B, 80, T, device=DEV))
        rows = lambda a: torch.cat([a[b, :, :L].t() for b, L in enumerate(lengths)]).contiguous()  # noqa: E731
        packed = model.forward_layout(lay, rows(x), rows(mu), t, spks, rows(cond),
                                      out=torch.empty(sum(lengths), 80, device=DEV), packed=True)
        assert torch.equal(packed, rows(pad)), (dtype, streaming)


@pytest.mark.parametrize("src_dtype", ["float32", "bfloat16"])
def test_pack_rows_bit_exact(src_dtype):
    """fcv_pack_rows: channel-major (B, 80, T) -> packed rows, and the broadcast
    form (batch stride 0) used for the fixed noise prefix."""
    from fcv_b200 import _lib
    from fcv_b200._lib import call
    from fcv_b200.model import _dtype_code

    dt = getattr(torch, src_dtype)
    lengths = [37, 0, 1, 70, 33]
    B, T = len(lengths), 75
    src = torch.randn(B, 80, T, device=DEV).to(dt)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=DEV)
    N = sum(lengths)
    out = torch.empty(N, 80, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    call("fcv_pack_rows", src.data_ptr(), _dtype_code(dt), 80 * T, T, cu.data_ptr(), B, max(lengths),
         out.data_ptr(), _lib.DTYPE_F32, stream)
    ref = torch.cat([src[b, :, :L].t() for b, L in enumerate(lengths)]).float()
    assert torch.equal(out, ref)
    call("fcv_pack_rows", src.data_ptr(), _dtype_code(dt), 0, T, cu.data_ptr(), B, max(lengths),
         out.data_ptr(), _lib.DTYPE_F32, stream)
    ref = torch.cat([src[0, :, :L].t() for L in lengths]).float()
    assert torch.equal(out, ref)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_streaming_prefix_trajectory_is_stable_across_calls(dtype):
    """Semantics behind streaming prefix reuse (flashinfer_flow.py:215-221 recomputes
    the whole prefix every call): with the chunk-causal mask, the causal position
    convolution, lookahead context tokens that are the real next tokens and the
    fixed noise prefix, a frame in a chunk that was complete in the previous call
    follows the same 10-step trajectory in the next call, so its output is
    bit-identical; frames of the previous call's partial chunk change (they now
    see the rest of their chunk)."""
    from fcv_b200.flow import flow_inference_batched_streaming

    dt = getattr(torch, dtype)
    flow = _flow(dt)
    rng = np.random.default_rng(77)
    tokens = rng.integers(0, 6561, size=200).tolist()
    prompt = torch.tensor(rng.standard_normal((1, 30, 80)), device=DEV, dtype=torch.float32)
    spk = torch.tensor(rng.standard_normal((1, 192)), device=DEV, dtype=torch.float32)
    prev = None
    for n_tok in (63, 88, 113):  # 60, 85, 110 tokens + 3 lookahead tokens of context
        out = flow_inference_batched_streaming(flow, [tokens[:n_tok]], [prompt], spk, [False])[0][0]
        mel = 2 * (n_tok - 3)
        assert out.shape[1] == mel - 30
        if prev is not None:
            prev_mel = prev.shape[1] + 30
            stable = (prev_mel // 50) * 50 - 30  # generated frames in the previous call's complete chunks
            assert torch.equal(out[:, :stable], prev[:, :stable]), (dtype, n_tok)
            if prev_mel % 50:
                assert not torch.equal(out[:, stable:prev.shape[1]], prev[:, stable:]), (dtype, n_tok)
        prev = out


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_prefix_cache_matches_full_recompute_bit_exact(dtype):
    """Streaming prefix reuse: with a PrefixCache each call computes only the
    rows from every stream's first incomplete chunk on (keys of earlier frames,
    convolution context and final samples come from the cache), and the
    generated Mel equals the full recomputation of flashinfer_flow.py:187-281
    bit for bit -- two streams of different lengths batched together over three
    calls, the last one finalising the first stream."""
    from fcv_b200.flow import PrefixCache, flow_inference_batched_streaming

    dt = getattr(torch, dtype)
    flow = _flow(dt)
    cache = PrefixCache(flow, max_streams=3, max_frames=400)
    rng = np.random.default_rng(91)
    toks = {s: rng.integers(0, 6561, size=200).tolist() for s in ("a", "b")}
    prompts = [torch.tensor(rng.standard_normal((1, n, 80)), device=DEV, dtype=torch.float32) for n in (30, 17)]
    spk = torch.tensor(rng.standard_normal((2, 192)), device=DEV, dtype=torch.float32)
    for call_i, (na, nb) in enumerate(((63, 40), (88, 65), (113, 90))):
        tl = [toks["a"][:na], toks["b"][:nb]]
        fin = [call_i == 2, False]
        ref = flow_inference_batched_streaming(flow, tl, prompts, spk, fin)
        got = flow_inference_batched_streaming(flow, tl, prompts, spk, fin, cache=cache, stream_ids=["a", "b"])
        for r in range(2):
            assert got[r].shape == ref[r].shape, (dtype, call_i, r)
            assert torch.equal(got[r], ref[r]), (dtype, call_i, r, (got[r] - ref[r]).abs().max().item())
    assert cache.stable_frames("a") == 0  # finalised and released
    assert cache.stable_frames("b") == (2 * (90 - 3) // 50) * 50


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_interleaved_streams_match_solo_runs_bit_exact(dtype):
    """Restates the reference's interleave gate (tests/gpu/test_stream_flashinfer.py:63-90,
    bit-exact there too) on this build's streaming flow: two sessions advanced call by
    call in alternation on one model instance and one PrefixCache give exactly what each
    session gives when it runs alone with a cache of its own -- the cache keeps each
    stream's state under its id and nothing leaks between streams."""
    from fcv_b200.flow import PrefixCache, flow_inference_batched_streaming

    dt = getattr(torch, dtype)
    flow = _flow(dt)
    rng = np.random.default_rng(23)
    toks = {s: rng.integers(0, 6561, size=200).tolist() for s in ("a", "b")}
    prompts = {"a": torch.tensor(rng.standard_normal((1, 30, 80)), device=DEV, dtype=torch.float32),
               "b": torch.tensor(rng.standard_normal((1, 21, 80)), device=DEV, dtype=torch.float32)}
    spk = {s: torch.tensor(rng.standard_normal((1, 192)), device=DEV, dtype=torch.float32) for s in ("a", "b")}
    steps = {"a": (63, 88, 113), "b": (40, 65, 90)}

    def advance(cache, s, k):
        fin = k == len(steps[s]) - 1
        return flow_inference_batched_streaming(flow, [toks[s][:steps[s][k]]], [prompts[s]], spk[s], [fin],
                                                cache=cache, stream_ids=[s])[0]

    solo = {}
    for s in ("a", "b"):
        cache = PrefixCache(flow, max_streams=2, max_frames=400)
        solo[s] = [advance(cache, s, k) for k in range(3)]
    cache = PrefixCache(flow, max_streams=2, max_frames=400)
    for k in range(3):
        for s in ("a", "b"):
            out = advance(cache, s, k)
            assert out.shape == solo[s][k].shape, (dtype, s, k)
            assert torch.equal(out, solo[s][k]), (dtype, s, k, (out - solo[s][k]).abs().max().item())
    assert cache.stable_frames("a") == 0 and cache.stable_frames("b") == 0  # both finalised and released
