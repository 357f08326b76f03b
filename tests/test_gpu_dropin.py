"""The drop-in boundary exercised through the reference's own callers.

The reference installs its estimator by replacing ``model.flow.decoder.estimator``
(``token2wav/token2wav.py:92-101`` via ``apply_flashinfer``,
``flashinfer_dit.py:951-988``) and reaches it only through
``ConditionalCFM.forward_estimator`` (``cosyvoice/flow/flow_matching.py:126-128``)
called from ``flashinfer_flow.solve_euler_batched`` (``flashinfer_flow.py:16-74``).
Here the reference's own ``CausalConditionalCFM`` (``flow_matching.py:196-200``)
is built around the reference's own ``DiT`` (``dit.py:104-143``) in a holder shaped
like ``CosyVoice3Token2Wav`` (``.flow.decoder.estimator``); ``apply_b200`` swaps in
``B200DiT``; the reference's unmodified solver then runs the 10-step CFG ODE.

Gates: fp32 max-abs <= 1e-4 against the oracle solver (pinned to the reference's
golden ODE outputs).  bf16: the reference solver then works in bf16 because it
follows the speaker rows' dtype (``flashinfer_flow.py:34-43, 55-70``) -- t, dt
and the sample itself are bf16, rounded at every step -- and is compared with the
oracle run with exactly those bf16 semantics; since the sample is bf16, one unit
in the last place at |x| >= 4 is already 0.03, so the 2e-2 bound applies to
|err| / (1 + |ref|).  And the reference's streaming gate
(``tests/gpu/test_stream_batched.py:88-103``: a multi-request packed batch matches
each request's one-request batch, atol 1e-3), here on the solver path: the packed
batch equals the per-request calls bit for bit.

The reference package comes from the offline install in ``baseline/_ref`` (its
``x_transformers`` RoPE dependency restated by ``tests/golden/_xt_shim``).
"""

from __future__ import annotations

import sys
import types
from pathlib import Path

import numpy as np
import pytest

from conftest import ensure_built, numpy_params
from oracle import dit_oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
DEV = "cuda:0"
ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"
LENGTHS = [260, 120, 75]  # requests of one packed streaming batch (chunk 50)
DEPTH = 4


@pytest.fixture(scope="module")
def reference():
    if not (REF / "faster_cosyvoice").is_dir():
        pytest.skip("the reference is not installed in baseline/_ref")
    for p in (str(REF), str(ROOT / "tests" / "golden" / "_xt_shim")):
        if p not in sys.path:
            sys.path.insert(0, p)
    ensure_built()
    from faster_cosyvoice.token2wav import flashinfer_flow
    from faster_cosyvoice.token2wav.cosyvoice.flow.DiT.dit import DiT
    from faster_cosyvoice.token2wav.cosyvoice.flow.flow_matching import CausalConditionalCFM

    return types.SimpleNamespace(flow=flashinfer_flow, DiT=DiT, CFM=CausalConditionalCFM)


def _token2wav_like(reference, dtype):
    """A holder shaped like CosyVoice3Token2Wav with the reference's CFM and DiT
    (seeded random init), on the GPU, after apply_b200."""
    from fcv_b200.model import B200DiT, apply_b200

    torch.manual_seed(8)
    dit = reference.DiT(dim=1024, depth=DEPTH, heads=16, dim_head=64, ff_mult=2, mel_dim=80, mu_dim=80, spk_dim=80,
                        out_channels=80, static_chunk_size=50, num_decoding_left_chunks=-1).eval()
    cfm = types.SimpleNamespace(sigma_min=1e-6, solver="euler", t_scheduler="cosine", training_cfg_rate=0.2,
                                inference_cfg_rate=0.7, reg_loss_type="l1")
    decoder = reference.CFM(in_channels=240, cfm_params=cfm, n_spks=1, spk_emb_dim=80, estimator=dit).to(DEV).eval()
    holder = types.SimpleNamespace(flow=types.SimpleNamespace(decoder=decoder))
    ref_sd = {k: v.detach().float().cpu().clone() for k, v in dit.state_dict().items()}
    apply_b200(holder, dtype=dtype)
    assert isinstance(decoder.estimator, B200DiT)
    return decoder, ref_sd


def _inputs(decoder):
    rng = np.random.default_rng(19)
    R, T = len(LENGTHS), max(LENGTHS)
    mu = np.zeros((R, 80, T), np.float32)
    cond = np.zeros((R, 80, T), np.float32)
    mask = np.zeros((R, 1, T), np.float32)
    for i, L in enumerate(LENGTHS):
        mu[i, :, :L] = rng.standard_normal((80, L))
        cond[i, :, :L] = rng.standard_normal((80, L))
        mask[i, 0, :L] = 1
    spks = rng.standard_normal((R, 80)).astype(np.float32)
    noise = decoder.rand_noise[:, :, :T].float().cpu().expand(R, -1, -1).numpy().copy()  # flashinfer_flow.py:266
    return dict(noise=noise, mu=mu, mask=mask, spks=spks, cond=cond)


def _solve(reference, decoder, z, dtype, idx=None):
    idx = list(range(len(LENGTHS))) if idx is None else idx
    T = max(LENGTHS[i] for i in idx)
    sel = lambda a: torch.tensor(a[idx][..., :T] if a.ndim == 3 else a[idx], device=DEV)  # noqa: E731
    y = reference.flow.solve_euler_batched(decoder, sel(z["noise"]), sel(z["mu"]), sel(z["mask"]),
                                           sel(z["spks"]).to(dtype), sel(z["cond"]), num_timesteps=10,
                                           streaming=True)
    return y.float()


@pytest.mark.parametrize("dtype,tol", [("float32", 1e-4), ("bfloat16", 2e-2)])
def test_reference_solver_over_applied_b200(reference, dtype, tol):
    dt = getattr(torch, dtype)
    decoder, ref_sd = _token2wav_like(reference, dt)
    est = decoder.estimator
    # apply_b200 loaded the reference's own weights: the same values, in the estimator dtype
    for k, v in est.state_dict().items():
        if k in ref_sd:
            assert torch.equal(v.float().cpu(), ref_sd[k].to(dt).float()), k
    z = _inputs(decoder)
    y = _solve(reference, decoder, z, dt).cpu().numpy()
    params = numpy_params(est)
    cut = lambda a: [a[i, :, :L] for i, L in enumerate(LENGTHS)]  # noqa: E731
    bf = dt == torch.bfloat16
    ref = O.solve_euler_docs(params, cut(z["noise"]), cut(z["mu"]), cut(z["cond"]), list(z["spks"]), 10,
                             streaming=True, emulate_bf16=bf, bf16_sample=bf)
    for i, L in enumerate(LENGTHS):
        diff = np.abs(y[i, :, :L] - ref[i])
        err = (diff / (1.0 + np.abs(ref[i]))).max() if bf else diff.max()
        assert err <= tol, (dtype, i, L, err)


def test_packed_batch_equals_single_request_batches_on_the_solver_path(reference):
    """Restates the reference's streaming gate (tests/gpu/test_stream_batched.py:88-103)
    on the reference solver over B200DiT: every request of a packed 3-request
    batch equals its own one-request batch, bit for bit (the reference allows
    atol 1e-3)."""
    decoder, _ = _token2wav_like(reference, torch.bfloat16)
    z = _inputs(decoder)
    packed = _solve(reference, decoder, z, torch.bfloat16)
    for i, L in enumerate(LENGTHS):
        alone = _solve(reference, decoder, z, torch.bfloat16, [i])
        assert alone.shape[-1] == L
        assert torch.equal(packed[i, :, :L], alone[0]), i
        assert torch.allclose(packed[i, :, :L], alone[0], atol=1e-3)
