"""Whole-estimator parity on the GPU (B200DiT -> fcv_dit_forward through the C ABI).

Gates (north star): fp32 rel-L2 <= 1e-5 and bf16 rel-L2 <= 1e-2 against the
reference torch (padded SDPA) path on identical seeded inputs -- the golden
vectors under tests/golden/ were produced by the reference itself -- and the
10-step ODE mel within max-abs 2e-2.  Only valid frames are compared; the
padding frames of our output must be exactly zero."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import ensure_built, load_golden, make_model, numpy_params, rel_l2
from oracle import dit_oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
DEV = "cuda:0"


@pytest.fixture(scope="module", autouse=True)
def _built():
    ensure_built()
    yield
    from fcv_b200 import ops

    assert ops.device_error() == 0


def _model(seed, depth, dtype):
    m = make_model(seed, depth).to(DEV, dtype)
    m.finalize_weights()
    return m


def _run(model, z, streaming, dtype):
    T = lambda a: torch.tensor(a, device=DEV).to(dtype)  # noqa: E731
    with torch.inference_mode():
        y = model(T(z["x"]), T(z["mask"]), T(z["mu"]), T(z["t"]), T(z["spks"]), T(z["cond"]), streaming=streaming)
    return y.float().cpu().numpy()


@pytest.mark.parametrize("name", ["dit_block_fp32", "dit_depth2_edge", "dit_depth22_cfg"])
def test_fp32_matches_reference_golden(name):
    z = load_golden(name)
    model = _model(int(z["seed"]), int(z["depth"]), torch.float32)
    for streaming, key in ((False, "out_offline"), (True, "out_streaming")):
        y = _run(model, z, streaming, torch.float32)
        for b, L in enumerate(z["lengths"]):
            assert rel_l2(y[b, :, :L], z[key][b, :, :L]) <= 1e-5, (name, streaming, b)
            assert not np.any(y[b, :, L:]), "padding frames must be zero"


@pytest.mark.parametrize("name", ["dit_block_fp32", "dit_depth2_edge", "dit_depth22_cfg"])
def test_bf16_matches_reference_within_1e2(name):
    """bf16 estimator vs the reference on the same bf16-rounded weights and
    inputs; the reference side is the oracle (pinned to the reference's golden
    outputs) run in fp32 with the reference's bf16 time-argument rounding."""
    z = load_golden(name)
    model = _model(int(z["seed"]), int(z["depth"]), torch.bfloat16)
    params = {k: v.float().cpu().numpy() for k, v in model.state_dict().items()}
    zb = {k: (O.bf16_round(v) if k in ("x", "mu", "cond", "spks", "t") else v) for k, v in z.items()}
    for streaming in (False, True):
        y = _run(model, z, streaming, torch.bfloat16)
        ref = O.dit_forward_padded(params, zb["x"], zb["mask"], zb["mu"], zb["t"], zb["spks"], zb["cond"],
                                   streaming=streaming, emulate_bf16_time=True)
        for b, L in enumerate(z["lengths"]):
            e = rel_l2(y[b, :, :L], ref[b, :, :L])
            assert e <= 1e-2, (name, streaming, b, e)


@pytest.mark.parametrize("dtype,tol,modes", [("bfloat16", 1e-2, (False, True)), ("float32", 1e-5, (False,))])
def test_long_documents_match_oracle(dtype, tol, modes):
    """The gates at the benchmark's document lengths: two requests of 600 and
    257 frames under CFG (second half with mu, spks and cond zeroed, as
    flashinfer_flow.py:45-51 stacks them), 22 blocks, so every query tile sees
    up to ten key tiles.  The oracle runs on the same bf16-rounded weights and
    inputs; in bf16 mode with the reference's bf16 time-argument rounding."""
    dt = getattr(torch, dtype)
    model = _model(11, 22, dt)
    params = numpy_params(model)  # the weights exactly as the model holds them (bf16 values in bf16 mode)
    rng = np.random.default_rng(12)
    req = [600, 257]
    lengths = req + req
    B, T = len(lengths), max(lengths)
    z = {k: np.zeros((B, 80, T), np.float32) for k in ("x", "mu", "cond")}
    z["spks"] = np.zeros((B, 80), np.float32)
    for r, L in enumerate(req):
        z["x"][r, :, :L] = z["x"][r + 2, :, :L] = rng.standard_normal((80, L))
        z["mu"][r, :, :L] = rng.standard_normal((80, L))
        z["cond"][r, :, :L] = rng.standard_normal((80, L))
        z["spks"][r] = rng.standard_normal(80)
    z["t"] = rng.uniform(size=2).astype(np.float32)[[0, 1, 0, 1]]
    z["mask"] = np.zeros((B, 1, T), np.float32)
    for b, L in enumerate(lengths):
        z["mask"][b, 0, :L] = 1
    z = {k: O.bf16_round(v) for k, v in z.items()}
    for streaming in modes:
        y = _run(model, z, streaming, dt)
        ref = O.dit_forward_padded(params, z["x"], z["mask"], z["mu"], z["t"], z["spks"], z["cond"],
                                   streaming=streaming, emulate_bf16_time=dt == torch.bfloat16)
        for b, L in enumerate(lengths):
            e = rel_l2(y[b, :, :L], ref[b, :, :L])
            assert e <= tol, (dtype, streaming, b, e)
            assert not np.any(y[b, :, L:]), "padding frames must be zero"


def test_batch_composition_invariance_bit_exact():
    """A document's output does not depend on its neighbours in the packed
    batch (reference invariant: flashinfer_attention.py:104-107,
    tests/gpu/test_stream_flashinfer.py:87-90)."""
    model = _model(2, 2, torch.bfloat16)
    rng = np.random.default_rng(3)
    lengths = [173, 60, 251, 1, 129]
    T = 260
    B = len(lengths)
    x = torch.tensor(rng.standard_normal((B, 80, T)), device=DEV, dtype=torch.bfloat16)
    mu = torch.tensor(rng.standard_normal((B, 80, T)), device=DEV, dtype=torch.bfloat16)
    cond = torch.tensor(rng.standard_normal((B, 80, T)), device=DEV, dtype=torch.bfloat16)
    spks = torch.tensor(rng.standard_normal((B, 80)), device=DEV, dtype=torch.bfloat16)
    t = torch.tensor(rng.uniform(size=B), device=DEV, dtype=torch.bfloat16)
    mask = torch.zeros(B, 1, T, device=DEV, dtype=torch.bfloat16)
    for b, L in enumerate(lengths):
        mask[b, 0, :L] = 1
    with torch.inference_mode():
        for streaming in (True, False):
            packed = model(x, mask, mu, t, spks, cond, streaming=streaming)
            for b, L in enumerate(lengths):
                solo = model(x[b:b + 1, :, :L].contiguous(), mask[b:b + 1, :, :L].contiguous(),
                             mu[b:b + 1, :, :L].contiguous(), t[b:b + 1], spks[b:b + 1],
                             cond[b:b + 1, :, :L].contiguous(), streaming=streaming)
                assert torch.equal(packed[b:b + 1, :, :L], solo), (streaming, b)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_empty_sequences_give_zero_output_and_leave_the_others_unchanged(dtype):
    """Sequences whose mask is all zero (length 0: the reference's packed path gives
    them no rows, flashinfer_dit.py:364-405, 460) come out as exact zeros, in any
    position of the batch, and the other sequences' outputs equal those of the batch
    without them, bit for bit -- offline and streaming, fp32 and bf16.  A batch in
    which every sequence is empty returns an all-zero padded output."""
    dt = getattr(torch, dtype)
    model = _model(4, 2, dt)
    rng = np.random.default_rng(12)
    lengths = [0, 90, 0, 1, 130, 0]
    T = 140
    B = len(lengths)
    x = torch.tensor(rng.standard_normal((B, 80, T)), device=DEV, dtype=dt)
    mu = torch.tensor(rng.standard_normal((B, 80, T)), device=DEV, dtype=dt)
    cond = torch.tensor(rng.standard_normal((B, 80, T)), device=DEV, dtype=dt)
    spks = torch.tensor(rng.standard_normal((B, 80)), device=DEV, dtype=dt)
    t = torch.tensor(rng.uniform(size=B), device=DEV, dtype=dt)
    mask = torch.zeros(B, 1, T, device=DEV, dtype=dt)
    for b, L in enumerate(lengths):
        mask[b, 0, :L] = 1
    keep = [b for b, L in enumerate(lengths) if L > 0]
    with torch.inference_mode():
        for streaming in (False, True):
            y = model(x, mask, mu, t, spks, cond, streaming=streaming)
            assert torch.isfinite(y).all()
            for b, L in enumerate(lengths):
                if L == 0:
                    assert not torch.any(y[b]), (dtype, streaming, b)
            ref = model(x[keep], mask[keep], mu[keep], t[keep], spks[keep], cond[keep], streaming=streaming)
            assert torch.equal(y[keep], ref), (dtype, streaming)
            # a batch with no frames at all: the whole padded output is zero
            empty = torch.zeros_like(mask)
            y0 = model(x, empty, mu, t, spks, cond, streaming=streaming)
            assert y0.shape == (B, 80, T) and not torch.any(y0), (dtype, streaming)


def test_gate_a_streaming_prefix_stability():
    """Reference Gate A (tests/gpu/test_flashinfer_streaming_estimator.py:58-89):
    with the chunk-50 mask the first floor(160/50)*50 = 150 output frames for
    T=160 equal those for T=200; with the full mask they must differ."""
    model = _model(0, 22, torch.bfloat16)
    g = torch.Generator().manual_seed(1234)
    T_new, T_old, stable = 200, 160, 150
    x = torch.randn(2, 80, T_new, generator=g).to(DEV, torch.bfloat16)
    mu = torch.randn(2, 80, T_new, generator=g).to(DEV, torch.bfloat16)
    cond = torch.randn(2, 80, T_new, generator=g).to(DEV, torch.bfloat16)
    spks = torch.randn(2, 80, generator=g).to(DEV, torch.bfloat16)
    t = torch.rand(1, generator=g).to(DEV, torch.bfloat16).expand(2).contiguous()
    mask = torch.ones(2, 1, T_new, device=DEV, dtype=torch.bfloat16)

    def run(T, streaming):
        return model(x[:, :, :T].contiguous(), mask[:, :, :T].contiguous(), mu[:, :, :T].contiguous(), t, spks,
                     cond[:, :, :T].contiguous(), streaming=streaming)

    with torch.inference_mode():
        d_s = (run(T_old, True)[:, :, :stable] - run(T_new, True)[:, :, :stable]).abs().max().item()
        d_o = (run(T_old, False)[:, :, :stable] - run(T_new, False)[:, :, :stable]).abs().max().item()
    assert d_s <= 1e-3, d_s
    assert d_o > 5e-3, d_o


@pytest.mark.parametrize("dtype,tol", [("float32", 1e-4), ("bfloat16", 2e-2)])
def test_ode_matches_reference_golden(dtype, tol):
    """10-step CFG Euler (flashinfer_flow.py:16-74) vs the reference's own
    solve_euler_batched output (golden), streaming and offline."""
    import types

    from fcv_b200.flow import solve_euler_batched

    dt = getattr(torch, dtype)
    z = load_golden("ode")
    model = _model(3, 2, dt)
    decoder = types.SimpleNamespace(estimator=model, inference_cfg_rate=0.7)
    args = [torch.tensor(z[k], device=DEV) for k in ("noise", "mu", "mask", "spks", "cond")]
    for streaming, key in ((True, "out_streaming"), (False, "out_offline")):
        y = solve_euler_batched(decoder, *args, num_timesteps=10, streaming=streaming).float().cpu().numpy()
        for i, L in enumerate(z["lengths"]):
            err = np.abs(y[i, :, :L] - z[key][i, :, :L]).max()
            assert err <= tol, (dtype, key, i, err)


def test_forward_rejects_missing_conditions():
    model = _model(0, 1, torch.float32)
    x = torch.zeros(1, 80, 10, device=DEV)
    with pytest.raises(ValueError):
        model(x, torch.ones(1, 1, 10, device=DEV), x, torch.zeros(1, device=DEV), None, x)
    with pytest.raises(RuntimeError):
        model.finalize_weights()


def test_cuda_graph_path_matches_eager_and_follows_new_inputs():
    """use_cuda_graph=True (the reference's enable_cuda_graph) replays a captured
    estimator call; results equal the eager path bit for bit, and a replay with
    new values in the same buffers follows the new inputs."""
    model = _model(4, 2, torch.bfloat16)
    rng = np.random.default_rng(9)
    lengths = [150, 77, 150, 77]
    T = 150
    B = len(lengths)

    def batch():
        a = lambda *s: torch.tensor(rng.standard_normal(s), device=DEV, dtype=torch.bfloat16)  # noqa: E731
        return a(B, 80, T), a(B, 80, T), a(B, 80, T), a(B, 80), torch.tensor(rng.uniform(size=B), device=DEV,
                                                                           dtype=torch.bfloat16)

    mask = torch.zeros(B, 1, T, device=DEV, dtype=torch.bfloat16)
    for b, L in enumerate(lengths):
        mask[b, 0, :L] = 1
    x, mu, cond, spks, t = batch()
    with torch.inference_mode():
        eager = model(x, mask, mu, t, spks, cond, streaming=True).clone()
        model.use_cuda_graph = True
        g1 = model(x, mask, mu, t, spks, cond, streaming=True).clone()
        assert torch.equal(g1, eager)
        x2, mu2, cond2, spks2, t2 = batch()
        x.copy_(x2), mu.copy_(mu2), cond.copy_(cond2), spks.copy_(spks2), t.copy_(t2)
        g2 = model(x, mask, mu, t, spks, cond, streaming=True).clone()
        model.use_cuda_graph = False
        e2 = model(x, mask, mu, t, spks, cond, streaming=True)
    assert torch.equal(g2, e2) and not torch.equal(g2, g1)


@pytest.mark.parametrize("streaming", [False, True])
def test_bucketed_graph_serves_many_compositions_bit_exact(streaming):
    """One captured graph per (row bucket, document bucket, mask) serves every
    batch composition that fits it (the packed counterpart of the reference's
    graph buckets, flashinfer_dit.py:742-826); results equal the eager call bit
    for bit, and batches beyond the largest bucket run eagerly."""
    model = _model(5, 2, torch.bfloat16)
    model.graph_buckets = (512, 1024)
    rng = np.random.default_rng(17)
    compositions = [[150, 77, 150, 77], [100, 20, 100, 20], [300, 300], [33, 1, 200, 33, 1, 200],
                    [1, 1], [700, 700]]
    for lengths in compositions:
        B, T = len(lengths), max(lengths) + 3
        x, mu, cond = (torch.tensor(rng.standard_normal((B, 80, T)), device=DEV, dtype=torch.bfloat16)
                       for _ in range(3))
        spks = torch.tensor(rng.standard_normal((B, 80)), device=DEV, dtype=torch.bfloat16)
        t = torch.tensor(rng.uniform(size=B), device=DEV, dtype=torch.bfloat16)
        mask = torch.zeros(B, 1, T, device=DEV, dtype=torch.bfloat16)
        for b, L in enumerate(lengths):
            mask[b, 0, :L] = 1
        with torch.inference_mode():
            model.use_cuda_graph = False
            ref = model(x, mask, mu, t, spks, cond, streaming=streaming)
            model.use_cuda_graph = True
            got = model(x, mask, mu, t, spks, cond, streaming=streaming)
        assert torch.equal(got, ref), (lengths, streaming)
    # (512 rows, 4 docs), (1024, 2), (512, 8), (512, 2); [700, 700] exceeds every bucket
    assert model.bucket_captures == 4
    assert len(model._bucket_graphs) == 4


@pytest.mark.parametrize("streaming", [False, True])
def test_attention_schedule_does_not_change_results(streaming):
    """The balanced (LPT) attention schedule only reassigns items to CTAs:
    estimator outputs are bit-identical to the round-robin deal."""
    model = _model(6, 2, torch.bfloat16)
    rng = np.random.default_rng(23)
    lengths = [int(v) for v in rng.integers(150, 601, size=6)] * 2 + [1, 700]
    B, T = len(lengths), max(lengths)
    x, mu, cond = (torch.tensor(rng.standard_normal((B, 80, T)), device=DEV, dtype=torch.bfloat16) for _ in range(3))
    spks = torch.tensor(rng.standard_normal((B, 80)), device=DEV, dtype=torch.bfloat16)
    t = torch.tensor(rng.uniform(size=B), device=DEV, dtype=torch.bfloat16)
    lay = model.prepare_layout(lengths, T, streaming, torch.device(DEV))
    assert lay.attn_sched is not None and lay.attn_ctas > 0
    with torch.inference_mode():
        model.use_attn_schedule = True
        a = model.forward_layout(lay, x, mu, t, spks, cond)
        model.use_attn_schedule = False
        b = model.forward_layout(lay, x, mu, t, spks, cond)
    model.use_attn_schedule = True
    assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_shared_modulation_row_equals_per_document_time_embedding(dtype):
    """When every document has the same t (the ODE solver's case), the cached
    modulation row of that t (fcv_dit_modulations, broadcast with stride 0)
    gives exactly the per-document time embedding + AdaLN GEMM result."""
    dt = getattr(torch, dtype)
    model = _model(7, 2, dt)
    rng = np.random.default_rng(29)
    lengths = [150, 77, 150, 77]
    B, T = len(lengths), max(lengths)
    x, mu, cond = (torch.tensor(rng.standard_normal((B, 80, T)), device=DEV).to(dt) for _ in range(3))
    spks = torch.tensor(rng.standard_normal((B, 80)), device=DEV).to(dt)
    t = torch.full((B,), 0.3071, device=DEV, dtype=dt)
    lay = model.prepare_layout(lengths, T, False, torch.device(DEV))
    with torch.inference_mode():
        a = model.forward_layout(lay, x, mu, t, spks, cond)
        b = model.forward_layout(lay, x, mu, t, spks, cond, shared_mods=model.shared_modulations(0.3071))
    assert torch.equal(a, b)
    assert len(model._mod_cache) == 1


def test_host_inputs_match_device_inputs():
    """forward() on host tensors (pinned or not; lengths counted from the host
    mask, inputs staged into persistent device buffers) gives exactly the
    device-tensor result, eagerly, through the per-layout graph and through the
    bucketed graph; a replay with new host values follows them."""
    model = _model(8, 2, torch.bfloat16)
    rng = np.random.default_rng(33)
    lengths = [120, 57, 120, 57]
    B, T = len(lengths), 124
    host = {k: torch.tensor(rng.standard_normal((B, 80, T)), dtype=torch.bfloat16) for k in ("x", "mu", "cond")}
    host["spks"] = torch.tensor(rng.standard_normal((B, 80)), dtype=torch.bfloat16)
    host["t"] = torch.tensor(rng.uniform(size=B), dtype=torch.bfloat16)
    host["mask"] = torch.zeros(B, 1, T, dtype=torch.bfloat16)
    for b, L in enumerate(lengths):
        host["mask"][b, 0, :L] = 1
    order = ("x", "mask", "mu", "t", "spks", "cond")
    dev = {k: v.to(DEV) for k, v in host.items()}
    pinned = {k: v.pin_memory() for k, v in host.items()}
    with torch.inference_mode():
        for graph, buckets in ((False, None), (True, None), (True, (512,))):
            model.use_cuda_graph, model.graph_buckets = graph, buckets
            ref = model(*(dev[k] for k in order)).clone()
            for src in (host, pinned):
                got = model(*(src[k] for k in order))
                torch.cuda.synchronize()
                assert torch.equal(got, ref), (graph, buckets, src is pinned)
        pinned["x"].mul_(0.5)
        got = model(*(pinned[k] for k in order))
        torch.cuda.synchronize()
        ref = model(*(pinned[k].to(DEV) for k in order))
        assert torch.equal(got, ref)
    model.use_cuda_graph, model.graph_buckets = False, None
