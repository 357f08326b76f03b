"""Generate the golden vectors under ``tests/golden/`` from the reference itself.

Run in a container where the reference project is present (read-only), with
``FCV_REFERENCE_ROOT`` naming its root (the directory that holds the
``faster_cosyvoice`` package)::

    FCV_REFERENCE_ROOT=<reference root> python tests/golden/make_golden.py

The reference's own code is imported and executed on the CPU in float32:

* ``cosyvoice/flow/DiT/dit.py`` ``DiT`` (padded SDPA path, ``dit.py:145-176``);
* ``flashinfer_dit.FlashInferDiT._get_packed_layout`` (``flashinfer_dit.py:364-405``);
* ``flashinfer_attention.build_chunk_causal_mask`` / ``_make_indptr``
  (``flashinfer_attention.py:16-33, 82-86``);
* ``flashinfer_kernels.layer_norm_modulate_torch`` (``flashinfer_kernels.py:288-296``);
* ``flashinfer_flow.solve_euler_batched`` (``flashinfer_flow.py:16-74``) with
  ``CausalConditionalCFM`` (``flow_matching.py:196-200``): a depth-2 case and the
  full 22-layer DiT at config-3 lengths (``python tests/golden/make_golden.py ode3``
  regenerates only the latter);
* ``modules.TimestepEmbedding`` in bf16 (``modules.py:71-83, 606-616``);
* ``flashinfer_flow.flow_inference_batched`` / ``flow_inference_batched_streaming``
  (``flashinfer_flow.py:118-281``) on a ``CausalMaskedDiffWithDiT`` built as
  ``builders.py:16-45`` does (``python tests/golden/make_golden.py flow`` regenerates
  only this fixture);
* ``cosyvoice/hifigan/generator.py`` ``CausalHiFTGenerator.inference`` built by
  ``builders.py:38-50`` with the seeded weights of ``hift_weights.py``
  (``python tests/golden/make_golden.py hift`` regenerates only this fixture).

``x_transformers`` (pinned 2.23.5, absent here) is replaced by the restatement in
``_xt_shim``; ``omegaconf`` is bypassed by passing a ``SimpleNamespace`` as
``cfm_params`` (and stubbed for ``flow.py``'s default-argument import).  Weights come
from ``torch.manual_seed(seed)`` followed by the reference constructor; their SHA-256 fingerprints are stored so the tests can
check that the framework's own module tree reproduces the same initialisation.

None of the tests import this script or the reference; they read the ``.npz`` /
``.json`` files it writes.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
if not os.environ.get("FCV_REFERENCE_ROOT"):
    raise SystemExit("set FCV_REFERENCE_ROOT to the reference project's root (the directory holding "
                     "the faster_cosyvoice package)")
REF = Path(os.environ["FCV_REFERENCE_ROOT"])
if not (REF / "faster_cosyvoice").is_dir():
    raise SystemExit(f"FCV_REFERENCE_ROOT={REF} holds no faster_cosyvoice package")
sys.path.insert(0, str(HERE / "_xt_shim"))
sys.path.insert(0, str(REF))

from faster_cosyvoice.token2wav.cosyvoice.flow.DiT.dit import DiT  # noqa: E402
from faster_cosyvoice.token2wav.cosyvoice.flow.DiT import modules as ref_modules  # noqa: E402
from faster_cosyvoice.token2wav.cosyvoice.flow.flow_matching import CausalConditionalCFM  # noqa: E402
from faster_cosyvoice.token2wav import flashinfer_attention as ref_attn  # noqa: E402
from faster_cosyvoice.token2wav import flashinfer_dit as ref_fdit  # noqa: E402
from faster_cosyvoice.token2wav import flashinfer_flow as ref_flow  # noqa: E402
from faster_cosyvoice.token2wav import flashinfer_kernels as ref_kernels  # noqa: E402

torch.set_num_threads(max(1, os.cpu_count() or 1))


def build_ref_dit(seed: int, depth: int) -> DiT:
    """``builders.py:17-21`` hyper-parameters, random init from ``seed``."""
    torch.manual_seed(seed)
    return DiT(dim=1024, depth=depth, heads=16, dim_head=64, ff_mult=2, mel_dim=80, mu_dim=80,
               spk_dim=80, out_channels=80, static_chunk_size=50,
               num_decoding_left_chunks=-1).eval()


def fingerprint(model: torch.nn.Module) -> dict:
    out = {}
    for k, v in model.state_dict().items():
        a = v.detach().contiguous().cpu().numpy()
        out[k] = {"shape": list(a.shape), "dtype": str(a.dtype),
                  "sha256": hashlib.sha256(a.tobytes()).hexdigest()}
    return out


def inputs(rng, B, T, lengths, cfg_pairs=False):
    x = rng.standard_normal((B, 80, T)).astype(np.float32)
    mu = rng.standard_normal((B, 80, T)).astype(np.float32)
    cond = rng.standard_normal((B, 80, T)).astype(np.float32)
    spks = rng.standard_normal((B, 80)).astype(np.float32)
    t = rng.uniform(0, 1, size=(B,)).astype(np.float32)
    if cfg_pairs:
        h = B // 2
        x[h:] = x[:h]
        mu[h:] = 0
        cond[h:] = 0
        spks[h:] = 0
        t[h:] = t[:h]
    mask = np.zeros((B, 1, T), np.float32)
    for b, L in enumerate(lengths):
        mask[b, 0, :L] = 1
    return dict(x=x, mu=mu, cond=cond, spks=spks, t=t, mask=mask)


@torch.no_grad()
def run_dit(model, d, streaming):
    T = torch.from_numpy
    y = model(T(d["x"]), T(d["mask"]), T(d["mu"]), T(d["t"]), T(d["spks"]), T(d["cond"]),
              streaming=streaming)
    return y.numpy()


def dit_case(name, seed, depth, lengths, T, cfg_pairs, in_seed):
    model = build_ref_dit(seed, depth)
    rng = np.random.default_rng(in_seed)
    d = inputs(rng, len(lengths), T, lengths, cfg_pairs)
    off = run_dit(model, d, False)
    st = run_dit(model, d, True)
    np.savez_compressed(HERE / f"{name}.npz", **d, lengths=np.asarray(lengths, np.int64),
                        out_offline=off, out_streaming=st, seed=seed, depth=depth)
    return model


def pack_cases():
    cases = [([5], 5), ([3, 7, 1], 7), ([50, 50], 64), ([1], 1), ([120, 77, 77, 120], 130),
             ([199, 1, 64, 51, 100], 200)]
    fake = types.SimpleNamespace(_pack_cache=ref_fdit.OrderedDict())
    runner = types.SimpleNamespace(device=torch.device("cpu"))
    out = {}
    for i, (lengths, T) in enumerate(cases):
        lt = torch.tensor(lengths, dtype=torch.int64)
        lay = ref_fdit.FlashInferDiT._get_packed_layout(fake, lt, T, torch.device("cpu"))
        indptr = ref_attn.RaggedAttentionRunner._make_indptr(runner, lengths)
        m = ref_attn.build_chunk_causal_mask(lengths, 50, "cpu")
        out[f"c{i}_lengths"] = np.asarray(lengths, np.int64)
        out[f"c{i}_T"] = np.int64(T)
        out[f"c{i}_gather"] = lay.gather_indices.numpy()
        out[f"c{i}_doc_ids"] = lay.document_ids.numpy()
        out[f"c{i}_positions"] = lay.positions.numpy()
        out[f"c{i}_cu"] = indptr.numpy()
        out[f"c{i}_mask50"] = m.numpy()
    out["n_cases"] = np.int64(len(cases))
    np.savez_compressed(HERE / "pack_layout.npz", **out)


def rownorm_case():
    rng = np.random.default_rng(11)
    h = (rng.standard_normal((37, 1024)) * 3 + 0.5).astype(np.float32)
    shift = rng.standard_normal((37, 1024)).astype(np.float32)
    scale = (1 + 0.3 * rng.standard_normal((37, 1024))).astype(np.float32)
    gate = rng.standard_normal((37, 1024)).astype(np.float32)
    r = rng.standard_normal((37, 1024)).astype(np.float32)
    T = torch.from_numpy
    out = ref_kernels.layer_norm_modulate_torch(T(h), T(shift), T(scale)).numpy()
    h2 = torch.addcmul(T(h), T(gate), T(r))
    out2 = ref_kernels.layer_norm_modulate_torch(h2, T(shift), T(scale)).numpy()
    np.savez_compressed(HERE / "rownorm.npz", h=h, shift=shift, scale=scale, gate=gate, r=r,
                        ln_mod=out, gres_h=h2.numpy(), gres_norm=out2)


@torch.no_grad()
def time_embed_case():
    te = ref_modules.SinusPositionEmbedding(256)
    rng = np.random.default_rng(5)
    t = torch.from_numpy(rng.uniform(0, 1, size=(64,)).astype(np.float32)).to(torch.bfloat16)
    sin_bf16 = te(t).to(torch.bfloat16).float().numpy()
    sin_f32 = te(t.float()).numpy()
    np.savez_compressed(HERE / "time_embed.npz", t_bf16=t.float().numpy(), sin_bf16=sin_bf16,
                        sin_f32=sin_f32)


@torch.no_grad()
def ode_case():
    model = build_ref_dit(3, 2)
    cfm = types.SimpleNamespace(sigma_min=1e-6, solver="euler", t_scheduler="cosine",
                                training_cfg_rate=0.2, inference_cfg_rate=0.7, reg_loss_type="l1")
    decoder = CausalConditionalCFM(in_channels=240, cfm_params=cfm, n_spks=1, spk_emb_dim=80,
                                   estimator=model)
    lengths = [120, 77]
    T = 120
    rng = np.random.default_rng(21)
    mu = rng.standard_normal((2, 80, T)).astype(np.float32)
    cond = rng.standard_normal((2, 80, T)).astype(np.float32)
    spks = rng.standard_normal((2, 80)).astype(np.float32)
    mask = np.zeros((2, 1, T), np.float32)
    for b, L in enumerate(lengths):
        mask[b, 0, :L] = 1
        mu[b, :, L:] = 0
        cond[b, :, L:] = 0
    noise = decoder.rand_noise[:, :, :T].expand(2, -1, -1).contiguous()
    out = {}
    for streaming in (True, False):
        y = ref_flow.solve_euler_batched(decoder, noise, torch.from_numpy(mu),
                                         torch.from_numpy(mask), torch.from_numpy(spks),
                                         torch.from_numpy(cond), num_timesteps=10,
                                         streaming=streaming)
        out["out_streaming" if streaming else "out_offline"] = y.float().numpy()
    np.savez_compressed(HERE / "ode.npz", mu=mu, cond=cond, spks=spks, mask=mask,
                        lengths=np.asarray(lengths, np.int64), noise=noise.numpy(),
                        rand_noise_head=decoder.rand_noise[0, :, :8].numpy(), **out)


# Four of config 3's request lengths (the median, the longest, the shortest and
# the lower quartile of bench.request_lengths("3")): prompt ~U[100, 400] plus a
# generated chunk of 30, 60 or 120 frames.
ODE3_LENGTHS = [309, 518, 157, 257]


@torch.no_grad()
def ode_config3_case():
    """The reference's ``solve_euler_batched`` (``flashinfer_flow.py:16-74``) at
    config-3 document lengths on the full 22-layer DiT (seed 6), streaming
    chunk-50 mask, 10 steps, CFG 0.7, float32; the noise is the CFM's fixed
    ``rand_noise`` prefix (``flow_matching.py:199-200``), as the streaming flow
    uses it (``flashinfer_flow.py:266``)."""
    model = build_ref_dit(6, 22)
    cfm = types.SimpleNamespace(sigma_min=1e-6, solver="euler", t_scheduler="cosine",
                                training_cfg_rate=0.2, inference_cfg_rate=0.7, reg_loss_type="l1")
    decoder = CausalConditionalCFM(in_channels=240, cfm_params=cfm, n_spks=1, spk_emb_dim=80,
                                   estimator=model)
    lengths = ODE3_LENGTHS
    R, T = len(lengths), max(lengths)
    rng = np.random.default_rng(41)
    mu = rng.standard_normal((R, 80, T)).astype(np.float32)
    cond = rng.standard_normal((R, 80, T)).astype(np.float32)
    spks = rng.standard_normal((R, 80)).astype(np.float32)
    mask = np.zeros((R, 1, T), np.float32)
    for b, L in enumerate(lengths):
        mask[b, 0, :L] = 1
        mu[b, :, L:] = 0
        cond[b, :, L:] = 0
    noise = decoder.rand_noise[:, :, :T].expand(R, -1, -1).contiguous()
    y = ref_flow.solve_euler_batched(decoder, noise, torch.from_numpy(mu), torch.from_numpy(mask),
                                     torch.from_numpy(spks), torch.from_numpy(cond), num_timesteps=10,
                                     streaming=True)
    np.savez_compressed(HERE / "ode_config3.npz", mu=mu, cond=cond, spks=spks, mask=mask,
                        lengths=np.asarray(lengths, np.int64), noise=noise.numpy(),
                        out_streaming=y.float().numpy(), seed=6, depth=22)
    return fingerprint(model)


def build_ref_flow(dit_seed: int, depth: int):
    """``builders.py:16-45`` (DiT depth reduced), random init.  The DiT draws from
    ``dit_seed``; the CFM constructor then reseeds 0 and draws ``rand_noise``
    (``flow_matching.py:199-200``); the front-end modules draw next: the
    ``PreLookaheadLayer`` argument (conv1, conv2), then ``nn.Embedding`` and the
    speaker ``nn.Linear`` inside ``CausalMaskedDiffWithDiT.__init__`` (``flow.py:306-307``).
    ``omegaconf`` (imported by ``flow.py:20`` for a default argument only) is stubbed."""
    if "omegaconf" not in sys.modules:
        stub = types.ModuleType("omegaconf")
        stub.DictConfig = dict
        sys.modules["omegaconf"] = stub
    from faster_cosyvoice.token2wav.cosyvoice.flow.flow import CausalMaskedDiffWithDiT
    from faster_cosyvoice.token2wav.cosyvoice.transformer.upsample_encoder import PreLookaheadLayer

    est = build_ref_dit(dit_seed, depth)
    cfm = types.SimpleNamespace(sigma_min=1e-6, solver="euler", t_scheduler="cosine",
                                training_cfg_rate=0.2, inference_cfg_rate=0.7, reg_loss_type="l1")
    decoder = CausalConditionalCFM(in_channels=240, cfm_params=cfm, n_spks=1, spk_emb_dim=80,
                                   estimator=est)
    flow = CausalMaskedDiffWithDiT(
        input_size=80, output_size=80, spk_embed_dim=192, output_type="mel", vocab_size=6561,
        input_frame_rate=25, only_mask_loss=True, token_mel_ratio=2, pre_lookahead_len=3,
        pre_lookahead_layer=PreLookaheadLayer(in_channels=80, channels=1024, pre_lookahead_len=3),
        decoder=decoder)
    return flow.eval()


def _concat_rows(mats):
    """(L_i, C) matrices -> one (sum L_i, C) array + cu offsets."""
    cu = np.zeros(len(mats) + 1, np.int64)
    for i, m in enumerate(mats):
        cu[i + 1] = cu[i] + m.shape[0]
    return np.concatenate(mats, 0).astype(np.float32), cu


@torch.no_grad()
def flow_case():
    """``flashinfer_flow.flow_inference_batched`` (``flashinfer_flow.py:118-184``) and
    ``flow_inference_batched_streaming`` (``:187-281``) on a depth-2 flow, plus their
    front-end intermediates (speaker projection, repeat-interleaved mu)."""
    flow = build_ref_flow(4, 2)
    rng = np.random.default_rng(31)
    out = {}
    front = {"input_embedding.weight": flow.input_embedding.weight,
             "spk_embed_affine_layer.weight": flow.spk_embed_affine_layer.weight,
             "spk_embed_affine_layer.bias": flow.spk_embed_affine_layer.bias,
             "pre_lookahead_layer.conv1.weight": flow.pre_lookahead_layer.conv1.weight,
             "pre_lookahead_layer.conv1.bias": flow.pre_lookahead_layer.conv1.bias,
             "pre_lookahead_layer.conv2.weight": flow.pre_lookahead_layer.conv2.weight,
             "pre_lookahead_layer.conv2.bias": flow.pre_lookahead_layer.conv2.bias}
    fps = {k: {"shape": list(v.shape), "dtype": "float32",
               "sha256": hashlib.sha256(v.detach().contiguous().numpy().tobytes()).hexdigest()}
           for k, v in front.items()}
    for mode, tok_lens, prompt_lens, finalize in (
            ("offline", [37, 61, 20], [24, 40, 10], None),
            ("streaming", [30, 45, 23], [20, 16, 12], [True, False, False])):
        tokens = [rng.integers(0, 6561, size=L).astype(np.int64) for L in tok_lens]
        tokens[0][5] = -1  # clamp(min=0) path (flashinfer_flow.py:148)
        prompts = [rng.standard_normal((L, 80)).astype(np.float32) for L in prompt_lens]
        spk = rng.standard_normal((len(tok_lens), 192)).astype(np.float32)
        prompt_t = [torch.from_numpy(p).unsqueeze(0) for p in prompts]
        spk_t = torch.from_numpy(spk)
        token_list = [t.tolist() for t in tokens]
        captured = {}
        if mode == "offline":
            orig = torch.randn

            def rec(*a, **k):
                r = orig(*a, **k)
                captured["noise"] = r.clone()
                return r

            torch.manual_seed(2024)
            torch.randn = rec
            try:
                gen = ref_flow.flow_inference_batched(flow, token_list, prompt_t, spk_t)
            finally:
                torch.randn = orig
            # front-end intermediates exactly as flashinfer_flow.py:144-153 forms them
            tok, tok_len = ref_flow._pack_tokens(token_list, torch.device("cpu"))
            mask = (~ref_flow.make_pad_mask(tok_len)).unsqueeze(-1).float()
            feats = flow.input_embedding(torch.clamp(tok, min=0)) * mask
            mu = flow.pre_lookahead_layer(feats).repeat_interleave(2, dim=1)
            mu_docs = [mu[i, :2 * L].numpy() for i, L in enumerate(tok_lens)]
            spk_proj = flow.spk_embed_affine_layer(torch.nn.functional.normalize(spk_t, dim=1)).numpy()
            out[f"{mode}_noise"] = captured["noise"].numpy()
        else:
            gen = ref_flow.flow_inference_batched_streaming(flow, token_list, prompt_t, spk_t, finalize)
            mu_docs = [ref_flow._streaming_token_features(flow, tl, finalize=f, device=torch.device("cpu"))[0].numpy()
                       for tl, f in zip(token_list, finalize)]
            spk_proj = flow.spk_embed_affine_layer(torch.nn.functional.normalize(spk_t, dim=1)).numpy()
            out[f"{mode}_finalize"] = np.asarray(finalize, np.int64)
        tok_cat = np.concatenate(tokens).astype(np.int64)
        out[f"{mode}_tokens"] = tok_cat
        out[f"{mode}_token_lengths"] = np.asarray(tok_lens, np.int64)
        out[f"{mode}_prompt"], out[f"{mode}_prompt_cu"] = _concat_rows(prompts)
        out[f"{mode}_spk"] = spk
        out[f"{mode}_spk_proj"] = spk_proj.astype(np.float32)
        out[f"{mode}_mu"], out[f"{mode}_mu_cu"] = _concat_rows(mu_docs)
        gens = [g[0].float().numpy().T for g in gen]  # (G_i, 80)
        out[f"{mode}_out"], out[f"{mode}_out_cu"] = _concat_rows(gens)
    out["rand_noise_head"] = flow.decoder.rand_noise[0, :, :8].numpy()
    np.savez_compressed(HERE / "flow_frontend.npz", **out)
    return fps


def hift_case():
    """HiFT vocoder: the reference's ``CausalHiFTGenerator`` as ``builders.py:38-50``
    builds it, with the seeded weights and noise table of ``hift_weights.py``,
    run through ``inference`` (``generator.py:728-740``) offline (``finalize=True``)
    and for a non-final streaming chunk (``finalize=False``)."""
    if "omegaconf" not in sys.modules:
        stub = types.ModuleType("omegaconf")
        stub.DictConfig = dict
        sys.modules["omegaconf"] = stub
    from faster_cosyvoice.token2wav.builders import build_hift

    sys.path.insert(0, str(HERE))
    import hift_weights as HW

    torch.manual_seed(0)
    hift = build_hift().eval()
    sd = HW.hift_state(0)
    hift.load_state_dict(sd, strict=True)
    noise = HW.hift_noise(480 * 20, 1)
    hift.m_source.l_sin_gen.sine_waves = noise[None]
    rng = np.random.default_rng(7)
    out = {"noise_rows": np.int64(noise.shape[0])}
    cases = (("off0", 9, True), ("off1", 14, True), ("str0", 17, False))
    for name, L, fin in cases:
        mel = (1.5 * rng.standard_normal((1, 80, L)) - 3.0).astype(np.float32)
        with torch.inference_mode():
            speech, s = hift.inference(speech_feat=torch.from_numpy(mel), finalize=fin)
            f0 = hift.f0_predictor(torch.from_numpy(mel).double(), finalize=fin).float()
        out[f"{name}_mel"] = mel[0]
        out[f"{name}_finalize"] = np.bool_(fin)
        out[f"{name}_speech"] = speech[0].numpy()
        out[f"{name}_s"] = s[0, 0].numpy()
        out[f"{name}_f0"] = f0[0].numpy()
    np.savez_compressed(HERE / "hift_case.npz", **out)
    return HW.fingerprint(sd)


def main():
    if sys.argv[1:] == ["ode3"]:
        fps = json.loads((HERE / "weights_fingerprint.json").read_text())
        fps["seed6_depth22"] = ode_config3_case()
        (HERE / "weights_fingerprint.json").write_text(json.dumps(fps, indent=0, sort_keys=True))
        print("config-3 ODE golden vectors written to", HERE)
        return
    if sys.argv[1:] == ["hift"]:
        fps = json.loads((HERE / "weights_fingerprint.json").read_text())
        fps["hift_seed0"] = hift_case()
        (HERE / "weights_fingerprint.json").write_text(json.dumps(fps, indent=0, sort_keys=True))
        print("hift golden vectors written to", HERE)
        return
    if sys.argv[1:] == ["flow"]:
        fps = json.loads((HERE / "weights_fingerprint.json").read_text())
        fps["flow_seed4_depth2_frontend"] = flow_case()
        fps["seed4_depth2"] = fingerprint(build_ref_dit(4, 2))
        (HERE / "weights_fingerprint.json").write_text(json.dumps(fps, indent=0, sort_keys=True))
        print("flow golden vectors written to", HERE)
        return
    fps = {}
    m = dit_case("dit_block_fp32", seed=0, depth=1, lengths=[300], T=300, cfg_pairs=False, in_seed=100)
    fps["seed0_depth1"] = fingerprint(m)
    m = dit_case("dit_depth22_cfg", seed=1, depth=22, lengths=[150, 77, 150, 77], T=150,
                 cfg_pairs=True, in_seed=101)
    fps["seed1_depth22"] = fingerprint(m)
    m = dit_case("dit_depth2_edge", seed=2, depth=2, lengths=[130, 1, 64, 51], T=130,
                 cfg_pairs=False, in_seed=102)
    fps["seed2_depth2"] = fingerprint(m)
    fps["seed3_depth2"] = fingerprint(build_ref_dit(3, 2))
    fps["seed4_depth2"] = fingerprint(build_ref_dit(4, 2))
    fps["flow_seed4_depth2_frontend"] = flow_case()
    fps["hift_seed0"] = hift_case()
    (HERE / "weights_fingerprint.json").write_text(json.dumps(fps, indent=0, sort_keys=True))
    pack_cases()
    rownorm_case()
    time_embed_case()
    ode_case()
    fps["seed6_depth22"] = ode_config3_case()
    (HERE / "weights_fingerprint.json").write_text(json.dumps(fps, indent=0, sort_keys=True))
    print("golden vectors written to", HERE)


if __name__ == "__main__":
    main()
