"""Host-side logic of the HiFT vocoder, no GPU: the per-level row layout of a
packed batch (the fcv_hift_batch.layout block), output lengths against the
oracle, rejection of too-short non-final chunks, and the convolution order of
the C ABI against the reference's state-dict keys."""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from conftest import hift_inputs
from oracle import hift_oracle as H


def _layout_host():
    from fcv_b200.hift import B200HiFT

    obj = types.SimpleNamespace(device=torch.device("cpu"), _layouts={})
    return lambda n_mel, fin: B200HiFT.layout(obj, n_mel, fin)


def test_layout_rows_per_level():
    lay = _layout_host()([9, 14, 17], [True, True, False])
    # mel, f0, x, source, stft, level0, level1, level2, audio
    assert lay.counts == [[9, 14, 17], [9, 14, 14], [9, 14, 10], [4320, 6720, 6720], [1081, 1681, 1681],
                          [72, 112, 80], [360, 560, 400], [1081, 1681, 1201], [4320, 6720, 4320]]
    block = lay.block.numpy()
    np.testing.assert_array_equal(block[36:], [0, lay.rows[0]])  # offsets of the one pack call
    block = block[:36].reshape(9, 4)
    for a in range(9):
        assert block[a, 0] == 0
        np.testing.assert_array_equal(np.diff(block[a]), lay.counts[a])
        assert block[a, -1] == lay.rows[a]
    assert lay.max_src == 6720


def test_layout_audio_lengths_match_oracle_and_reference_golden():
    _, _, _, z = hift_inputs()
    layout = _layout_host()
    for case in ("off0", "off1", "str0"):
        L, fin = z[f"{case}_mel"].shape[1], bool(z[f"{case}_finalize"])
        lay = layout([L], [fin])
        assert lay.rows[8] == H.out_samples(L, fin) == z[f"{case}_speech"].shape[0]
        assert lay.rows[3] == z[f"{case}_s"].shape[0]


def test_layout_rejects_short_non_final_chunks():
    layout = _layout_host()
    with pytest.raises(ValueError):
        layout([7], [False])
    with pytest.raises(ValueError):
        layout([0], [True])
    assert layout([8], [False]).rows[8] == 0   # 8 frames: one decoded frame, all of it look-ahead


def test_conv_order_covers_the_reference_state_dict():
    from fcv_b200.hift import conv_names

    sd, _, _, _ = hift_inputs()
    names = conv_names()
    assert len(names) == len(set(names)) == 80
    convs = {k.rsplit(".parametrizations", 1)[0] if ".parametrizations." in k else k.rsplit(".", 1)[0]
             for k in sd if k.endswith((".original1", ".weight")) and not k.startswith(("f0_predictor", "m_source"))}
    assert convs == set(names)


def test_oracle_non_final_chunks_are_prefixes_of_the_offline_output():
    """The property the reference checks in its own streaming demo (generator.py:743-752):
    every decode step is causal apart from the look-ahead a non-final chunk consumes, so
    its 480 (L - 8) samples equal the first samples of the offline output of the whole mel."""
    _, W, noise, _ = hift_inputs()
    rng = np.random.default_rng(21)
    mel = (1.5 * rng.standard_normal((20, 80)) - 3).astype(np.float32)
    full, _, _ = H.inference(mel, W, noise.numpy(), True)
    for L in (9, 13, 17):
        part, _, _ = H.inference(mel[:L], W, noise.numpy(), False)
        assert part.shape[0] == H.out_samples(L, False)
        np.testing.assert_allclose(part, full[:part.shape[0]], rtol=0, atol=1e-5)


def test_weight_preparation_on_the_host():
    """B200HiFT built on the CPU: every convolution's padded [k][C_in][C_out] copy holds
    the weight-norm-folded weights, the tensor-core copies split them exactly
    (head + remainder == weight, heads with 13 zero mantissa bits), and the Snake
    inverses are the reference's float32 1 / (alpha + 1e-9)."""
    from fcv_b200.hift import B200HiFT, conv_names

    sd, W, noise, _ = hift_inputs()
    voc = B200HiFT(sd, noise, "cpu", tensor_cores=True)
    by_ptr = {t.data_ptr(): t for t in voc._keep}
    w = voc._w
    for i, name in enumerate(conv_names()):
        ref = torch.from_numpy(W[f"{name}.weight"])                      # (C_out, C_in, k)
        co, ci, k = ref.shape
        pad = by_ptr[w.conv_w[i]]
        assert pad.shape == (k, -(-ci // 16) * 16, -(-co // 64) * 64)
        assert torch.equal(pad[:, :ci, :co], ref.permute(2, 1, 0))
        assert not pad[:, ci:, :].any() and not pad[:, :, co:].any()
        if "resblocks." in name:
            hi, lo = by_ptr[w.tc_w_hi[i]], by_ptr[w.tc_w_lo[i]]
            assert torch.equal(hi + lo, ref.permute(2, 0, 1))
            assert not (hi.view(torch.int32) & 8191).any()
        else:
            assert not w.tc_w_hi[i] and not w.tc_w_lo[i]
        if ".convs1." in name:
            block, s = name.split(".convs1.")
            a = torch.from_numpy(W[f"{block}.activations1.{s}.alpha"])
            assert torch.equal(by_ptr[w.snake_alpha[i]], a)
            assert torch.equal(by_ptr[w.snake_inv[i]], 1.0 / (a + 1e-9))
    f0w = by_ptr[w.f0_w[1]]
    assert f0w.dtype == torch.float64
    assert torch.equal(f0w, torch.from_numpy(W["f0_predictor.condnet.2.weight"]).permute(2, 1, 0))
    assert w.noise_rows == noise.shape[0]
