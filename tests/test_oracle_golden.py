"""Pin the numpy oracle (oracle/dit_oracle.py) to golden vectors produced by the
reference's own code (tests/golden/make_golden.py), and check that the
framework's module tree reproduces the reference's random initialisation."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from conftest import flow_case, golden_fingerprints, hift_inputs, load_golden, make_flow, make_model, numpy_params, rel_l2
from oracle import dit_oracle as O
from oracle import flow_oracle as F
from oracle import hift_oracle as H


def test_pack_layout_matches_reference_bit_exact():
    z = load_golden("pack_layout")
    for i in range(int(z["n_cases"])):
        lengths = z[f"c{i}_lengths"]
        lay = O.pack_layout(lengths, int(z[f"c{i}_T"]))
        np.testing.assert_array_equal(lay.gather_indices, z[f"c{i}_gather"])
        assert lay.gather_indices.dtype == z[f"c{i}_gather"].dtype
        np.testing.assert_array_equal(lay.document_ids, z[f"c{i}_doc_ids"])
        np.testing.assert_array_equal(lay.positions, z[f"c{i}_positions"])
        np.testing.assert_array_equal(lay.cu_seqlens, z[f"c{i}_cu"])
        np.testing.assert_array_equal(O.chunk_causal_mask_flat(lengths, 50), z[f"c{i}_mask50"])


def test_lengths_from_mask_counts_exactly():
    m = np.zeros((3, 1, 10), np.float32)
    m[0, 0, :10] = 1
    m[1, 0, :1] = 1
    np.testing.assert_array_equal(O.lengths_from_mask(m), [10, 1, 0])


def test_rownorm_matches_reference():
    z = load_golden("rownorm")
    out = O.layer_norm_modulate(z["h"], z["shift"], z["scale"])
    assert rel_l2(out, z["ln_mod"]) < 1e-6
    h2, norm = O.gate_residual_layer_norm_modulate(z["h"], z["gate"], z["r"], z["shift"], z["scale"])
    np.testing.assert_allclose(h2, z["gres_h"], rtol=1e-6, atol=1e-6)
    assert rel_l2(norm, z["gres_norm"]) < 1e-6


def test_time_sinusoid_matches_reference_fp32_and_bf16():
    z = load_golden("time_embed")
    s32 = O.sinus_embed(z["t_bf16"], emulate_bf16_time=False)
    # |arg| reaches 1000 rad, so one ulp of the fp32 frequency moves sin by ~6e-5
    np.testing.assert_allclose(s32, z["sin_f32"], atol=2e-4)
    s16 = O.sinus_embed(z["t_bf16"], emulate_bf16_time=True)
    # bf16 semantics: the argument 1000*t is rounded to bf16 before the sinusoid
    np.testing.assert_allclose(s16, z["sin_bf16"], atol=1e-2)
    assert np.mean(np.abs(s16 - z["sin_bf16"]) > 0) < 0.05


@pytest.mark.parametrize("key,seed,depth", [("seed0_depth1", 0, 1), ("seed2_depth2", 2, 2),
                                            ("seed3_depth2", 3, 2), ("seed4_depth2", 4, 2),
                                            ("seed1_depth22", 1, 22), ("seed6_depth22", 6, 22)])
def test_module_tree_reproduces_reference_init(key, seed, depth):
    fp = golden_fingerprints()[key]
    sd = make_model(seed, depth).state_dict()
    assert sorted(sd.keys()) == sorted(fp.keys())
    for k, meta in fp.items():
        a = sd[k].detach().contiguous().numpy()
        assert list(a.shape) == meta["shape"], k
        assert hashlib.sha256(a.tobytes()).hexdigest() == meta["sha256"], k


def _dit_case(name, rtol):
    z = load_golden(name)
    params = numpy_params(make_model(int(z["seed"]), int(z["depth"])))
    for streaming, key in ((False, "out_offline"), (True, "out_streaming")):
        y = O.dit_forward_padded(params, z["x"], z["mask"], z["mu"], z["t"], z["spks"], z["cond"],
                                 streaming=streaming)
        for b, L in enumerate(z["lengths"]):
            assert rel_l2(y[b, :, :L], z[key][b, :, :L]) < rtol, (name, streaming, b)


def test_dit_single_block_fp32_matches_reference():
    _dit_case("dit_block_fp32", 1e-5)


def test_dit_depth2_ragged_edge_matches_reference():
    _dit_case("dit_depth2_edge", 1e-5)


def test_dit_depth22_cfg_matches_reference():
    _dit_case("dit_depth22_cfg", 1e-4)


def test_ode_matches_reference():
    z = load_golden("ode")
    params = numpy_params(make_model(3, 2))
    lengths = z["lengths"]
    noise = [z["noise"][i, :, :L] for i, L in enumerate(lengths)]
    mu = [z["mu"][i, :, :L] for i, L in enumerate(lengths)]
    cond = [z["cond"][i, :, :L] for i, L in enumerate(lengths)]
    for streaming, key in ((True, "out_streaming"), (False, "out_offline")):
        xs = O.solve_euler_docs(params, noise, mu, cond, list(z["spks"]), 10, streaming=streaming)
        for i, L in enumerate(lengths):
            assert np.abs(xs[i] - z[key][i, :, :L]).max() < 1e-4, (key, i)


def test_ode_config3_lengths_matches_reference():
    """The oracle's CFG Euler solver against the reference's own
    solve_euler_batched on the full 22-layer DiT at four of config 3's document
    lengths (157-518 frames), streaming chunk-50 mask, 10 steps, float32."""
    z = load_golden("ode_config3")
    params = numpy_params(make_model(int(z["seed"]), int(z["depth"])))
    lengths = z["lengths"]
    noise = [z["noise"][i, :, :L] for i, L in enumerate(lengths)]
    mu = [z["mu"][i, :, :L] for i, L in enumerate(lengths)]
    cond = [z["cond"][i, :, :L] for i, L in enumerate(lengths)]
    xs = O.solve_euler_docs(params, noise, mu, cond, list(z["spks"]), 10, streaming=True)
    for i, L in enumerate(lengths):
        assert np.abs(xs[i] - z["out_streaming"][i, :, :L]).max() < 1e-4, i


def test_flop_model_matches_closed_form():
    # the estimator FLOPs per NFE in closed form: 378,044,416 per packed row (22 blocks of
    # 2^24 in the four block GEMMs, plus input projection, the two convolutions and
    # proj_out), 4096 per visible (q, k) pair and block, and the time MLP and AdaLN per sequence
    f1 = O.estimator_flops([1], None, 22)
    per_seq = 2 * 1024 * 137216 + 2 * (256 * 1024 + 1024 * 1024)
    assert f1 == 378044416 + 22 * 4096 * 1 + per_seq
    assert O.visible_pairs([100], 50) == 50 * 50 + 50 * 100


# ---------------------------------------------------------------- packed flow front end

def _flow_params():
    flow = make_flow(4, 2)
    sd = {k: v.detach().float().numpy() for k, v in flow.state_dict().items()}
    fe = {k: v for k, v in sd.items() if not k.startswith("decoder.")}
    dit = {k[len("decoder.estimator."):]: v for k, v in sd.items() if k.startswith("decoder.estimator.")}
    return flow, fe, dit


def test_flow_module_reproduces_reference_init():
    """B200Flow's front-end parameters and noise prefix equal the reference's
    CausalMaskedDiffWithDiT built as builders.py:16-45 does (same RNG order)."""
    flow, fe, _ = _flow_params()
    fp = golden_fingerprints()["flow_seed4_depth2_frontend"]
    assert sorted(fe.keys()) == sorted(fp.keys())
    for k, meta in fp.items():
        assert list(fe[k].shape) == meta["shape"], k
        assert hashlib.sha256(np.ascontiguousarray(fe[k]).tobytes()).hexdigest() == meta["sha256"], k
    z = load_golden("flow_frontend")
    assert np.array_equal(flow.decoder.rand_noise[0, :, :8].numpy(), z["rand_noise_head"])


@pytest.mark.parametrize("mode", ["offline", "streaming"])
def test_flow_frontend_oracle_matches_reference(mode):
    """Token embedding + PreLookaheadLayer + repeat-interleave and the speaker
    projection vs the reference's own modules (flashinfer_flow.py:144-153, 167-184)."""
    _, fe, _ = _flow_params()
    c = flow_case(load_golden("flow_frontend"), mode)
    fin = c["finalize"] or [True] * len(c["tokens"])
    for i, toks in enumerate(c["tokens"]):
        mu = F.frontend_mu(fe, toks, fin[i])
        assert mu.shape == c["mu"][i].shape, (mode, i)
        np.testing.assert_allclose(mu, c["mu"][i], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(F.speaker_projection(fe, c["spk"]), c["spk_proj"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("mode", ["offline", "streaming"])
def test_flow_inference_oracle_matches_reference(mode):
    """The whole batched flow inference (flashinfer_flow.py:118-281) on a
    depth-2 flow: the generated Mel of every request."""
    flow, fe, dit = _flow_params()
    z = load_golden("flow_frontend")
    c = flow_case(z, mode)
    fin = c["finalize"] or [True] * len(c["tokens"])
    n_mel = [m.shape[0] for m in c["mu"]]
    if mode == "offline":
        noise = [z["offline_noise"][i, :, :n] for i, n in enumerate(n_mel)]
    else:
        noise = [flow.decoder.rand_noise[0, :, :n].numpy() for n in n_mel]
    outs = F.flow_inference_docs(fe, dit, c["tokens"], c["prompts"], c["spk"], noise, finalize=fin,
                                 streaming=mode == "streaming")
    for i, o in enumerate(outs):
        assert o.shape == c["out"][i].T.shape, (mode, i)
        assert np.abs(o - c["out"][i].T).max() < 1e-4, (mode, i)


def test_hift_weights_reproduce_golden_state():
    """The seeded generator still yields the weights the HiFT fixture was made with."""
    sd, _, _, _ = hift_inputs()
    import hift_weights as HW
    assert HW.fingerprint(sd) == golden_fingerprints()["hift_seed0"]


@pytest.mark.parametrize("case", ["off0", "off1", "str0"])
def test_hift_oracle_matches_reference(case):
    """The numpy HiFT restatement against the reference's CausalHiFTGenerator.inference
    (offline and non-final chunks): f0 exact, excitation and speech within float32 noise."""
    _, W, noise, z = hift_inputs()
    fin = bool(z[f"{case}_finalize"])
    speech, s, f0 = H.inference(z[f"{case}_mel"].T.copy(), W, noise.numpy(), fin)
    np.testing.assert_array_equal(f0, z[f"{case}_f0"])
    assert speech.shape == z[f"{case}_speech"].shape == (H.out_samples(z[f"{case}_mel"].shape[1], fin),)
    assert rel_l2(s, z[f"{case}_s"]) <= 1e-6
    assert rel_l2(speech, z[f"{case}_speech"]) <= 1e-5
