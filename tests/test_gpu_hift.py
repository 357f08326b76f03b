"""HiFT vocoder on the GPU through the C ABI (``fcv_hift_forward``) against the
numpy oracle and the reference's own outputs (``tests/golden/hift_case.npz``).

Tolerances (float32 like the reference module, float64 f0 predictor):
speech rel-L2 <= 1e-4, excitation rel-L2 <= 1e-5, f0 within 1e-6 relative.
Packed batches must equal per-request calls bit for bit.  Every test runs on both
convolution paths: the residual blocks on the tensor cores (split-tf32 operands)
and all convolutions on the SIMT float32 kernel."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import cuda_available, ensure_built, hift_inputs, rel_l2
from oracle import hift_oracle as H

pytestmark = pytest.mark.gpu

SPEECH_TOL, SOURCE_TOL, F0_TOL = 1e-4, 1e-5, 1e-6


@pytest.fixture(scope="module", params=[True, False], ids=["tensor_cores", "simt"])
def vocoder(request):
    if not cuda_available():
        pytest.skip("needs a CUDA device")
    ensure_built()
    from fcv_b200.hift import B200HiFT

    sd, W, noise, z = hift_inputs()
    return B200HiFT(sd, noise, "cuda:0", tensor_cores=request.param), W, noise, z


@pytest.mark.parametrize("case", ["off0", "off1", "str0"])
def test_hift_matches_reference_golden(vocoder, case):
    import torch

    voc, W, noise, z = vocoder
    mel = torch.from_numpy(z[f"{case}_mel"])[None].cuda()
    fin = bool(z[f"{case}_finalize"])
    speech, s = voc.inference(mel, finalize=fin)
    speech, s = speech.cpu().numpy()[0], s.cpu().numpy()[0, 0]
    assert speech.shape == z[f"{case}_speech"].shape
    assert s.shape == z[f"{case}_s"].shape
    assert rel_l2(s, z[f"{case}_s"]) <= SOURCE_TOL
    assert rel_l2(speech, z[f"{case}_speech"]) <= SPEECH_TOL
    ref, ref_s, _ = H.inference(z[f"{case}_mel"].T.copy(), W, noise.numpy(), fin)
    assert rel_l2(speech, ref) <= SPEECH_TOL
    assert rel_l2(s, ref_s) <= SOURCE_TOL


def test_hift_f0_matches_oracle(vocoder):
    import torch

    from fcv_b200.hift import MEL

    voc, W, noise, z = vocoder
    mels = [z["off0_mel"], z["off1_mel"], z["str0_mel"]]
    fins = [True, True, False]
    lay = voc.layout([m.shape[1] for m in mels], fins)
    rows = voc._pack([torch.from_numpy(m).cuda() for m in mels], lay)
    f0 = torch.empty(lay.rows[1], device="cuda")
    audio, _ = voc.forward_packed(rows, lay, f0_out=f0)
    got = np.split(f0.cpu().numpy(), np.cumsum(lay.counts[1])[:-1])
    for g, m, fin in zip(got, mels, fins):
        ref = H.f0_predict(m.T.copy(), W, fin)
        np.testing.assert_allclose(g, ref, rtol=F0_TOL, atol=0)
    assert rows.shape[1] == MEL


def test_hift_packed_batch_equals_single_requests_bit_exact(vocoder):
    """Documents share convolution tiles in a packed call; every output still
    equals its own single-request call exactly (mixed offline / non-final)."""
    import torch

    voc = vocoder[0]
    rng = np.random.default_rng(11)
    lengths = [17, 9, 20, 12]
    fins = [True, False, True, False]
    mels = [torch.from_numpy((1.5 * rng.standard_normal((1, 80, L)) - 3).astype(np.float32)).cuda() for L in lengths]
    batch, srcs = voc.inference_batched(mels, fins, want_source=True)
    for m, fin, y, s in zip(mels, fins, batch, srcs):
        y1, s1 = voc.inference(m, finalize=fin)
        assert y.shape == y1.shape and s.shape == s1.shape
        assert torch.equal(y, y1) and torch.equal(s, s1)
        assert y.shape[1] == H.out_samples(m.shape[-1], fin)


def test_hift_longer_documents_match_oracle(vocoder):
    import torch

    voc, W, noise, _ = vocoder
    rng = np.random.default_rng(12)
    lengths, fins = [18, 13], [True, False]
    mels = [(1.5 * rng.standard_normal((80, L)) - 3).astype(np.float32) for L in lengths]
    got = voc.inference_batched([torch.from_numpy(m).cuda() for m in mels], fins)
    for g, m, fin in zip(got, mels, fins):
        ref, _, _ = H.inference(m.T.copy(), W, noise.numpy(), fin)
        assert rel_l2(g.cpu().numpy()[0], ref) <= SPEECH_TOL


def test_hift_audio_free_chunk_still_gives_source_and_f0(vocoder):
    """An 8-frame non-final chunk decodes no audio (all of its frames are
    look-ahead) but the reference still returns its excitation ``s`` and f0
    (generator.py:728-740): both must match the oracle, alone and packed with a
    chunk that has audio."""
    import torch

    voc, W, noise, _ = vocoder
    rng = np.random.default_rng(14)
    short = (1.5 * rng.standard_normal((80, 8)) - 3).astype(np.float32)
    longer = (1.5 * rng.standard_normal((80, 15)) - 3).astype(np.float32)
    ref_speech, ref_s, ref_f0 = H.inference(short.T.copy(), W, noise.numpy(), False)
    assert ref_speech.shape == (0,)
    speech, s = voc.inference(torch.from_numpy(short)[None].cuda(), finalize=False)
    assert speech.shape == (1, 0)
    assert rel_l2(s.cpu().numpy()[0, 0], ref_s) <= SOURCE_TOL
    lay = voc.layout([8], [False])
    f0 = torch.full((lay.rows[1],), float("nan"), device="cuda")
    voc.forward_packed(voc._pack([torch.from_numpy(short).cuda()], lay), lay, f0_out=f0)
    np.testing.assert_allclose(f0.cpu().numpy(), ref_f0, rtol=F0_TOL, atol=0)
    both, srcs = voc.inference_batched([torch.from_numpy(short).cuda(), torch.from_numpy(longer).cuda()],
                                       [False, False], want_source=True)
    assert both[0].shape == (1, 0)
    assert torch.equal(srcs[0], s)


def test_hift_rejects_short_chunks_and_short_noise(vocoder):
    import torch

    from fcv_b200._lib import FcvError
    from fcv_b200.hift import B200HiFT

    voc, _, noise, _ = vocoder
    with pytest.raises(ValueError):
        voc.inference(torch.zeros(1, 80, 7, device="cuda"), finalize=False)
    sd, _, _, _ = hift_inputs()
    small = B200HiFT(sd, noise[:480 * 5], "cuda:0")
    with pytest.raises(FcvError):
        small.inference(torch.zeros(1, 80, 6, device="cuda"), finalize=True)
    assert small.inference(torch.zeros(1, 80, 5, device="cuda"), finalize=True)[0].shape == (1, 2400)


def test_hift_tensor_core_path_matches_simt_path():
    """The split-tf32 tensor-core residual convolutions stay within the float32
    speech tolerance of the all-SIMT path on a packed batch (3.2e-5 rel-L2 measured
    on a B200: the tf32 truncation of the remainder, about 2^-21 relative per product)."""
    if not cuda_available():
        pytest.skip("needs a CUDA device")
    ensure_built()
    import torch

    from fcv_b200.hift import B200HiFT

    sd, _, noise, _ = hift_inputs()
    tc, simt = B200HiFT(sd, noise, "cuda:0", True), B200HiFT(sd, noise, "cuda:0", False)
    rng = np.random.default_rng(13)
    mels = [torch.from_numpy((1.5 * rng.standard_normal((80, L)) - 3).astype(np.float32)).cuda() for L in (19, 11)]
    for a, b in zip(tc.inference_batched(mels, [True, False]), simt.inference_batched(mels, [True, False])):
        assert rel_l2(a.cpu().numpy(), b.cpu().numpy()) <= SPEECH_TOL
