#!/usr/bin/env python
"""Benchmark of the packed DiT estimator: mel-frames/s per NFE (one estimator call).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 2|3|4|5] [--impl b200|reference]

Default workload ("config 5", the configuration the
metric is quoted on at 1/2/4/8 GPUs): 22-layer bf16 DiT, 16 requests x 3000 mel
frames with CFG doubling -> 32 sequences, 96,000 packed rows, full (offline)
mask, inputs ~N(0,1), t ~U(0,1), random-init weights from seed 5, one estimator
call per step.  ``--config 2|3|4`` select the other estimator configs.
Synthetic data of the reference's shapes; no dataset is involved.

Under torchrun (N > 1) one fixed request set is sharded across the ranks by
LPT bins of the per-request FLOP cost (strong scaling: the same total work at
every N; no collective on the data path); ``--weak`` runs replicas instead.

``--impl reference`` times the reference's own CPU implementation of the path:
its torch ``DiT`` (installed offline in ``baseline/_ref``), float32, all host
threads, one request as its CFG pair per step in a stratified order over the
config's requests; the oracle port stands in when the install is missing.
Under torchrun only rank 0 runs it.

``--impl reference-gpu`` times the reference's own GPU estimator
(``FlashInferDiT``: Triton row kernels, FlashInfer ragged prefill, cuBLAS; in
float16 as ``apply_flashinfer`` deploys it, ``--ref-dtype bf16`` for bfloat16)
on the same weights and inputs, when the reference has been installed offline
into ``baseline/_ref``; otherwise it prints an ``unavailable`` line.  A
comparison bar only: nothing of it is on the B200 path.

``--latency`` times one estimator call for a single CFG pair (B = 2, 200 / 400 /
800 frames), eager and through the bucketed CUDA graphs, for this build or (with
``--impl reference-gpu``) the reference's ``FlashInferDiT`` with and without its
own graph buckets.

``--stream [--prefix-cache]`` times a streaming session: 32 streams that advance by
25 tokens (50 frames) per call, through ``flow_inference_batched_streaming``,
recomputing the whole prefix (as the reference does) or reusing the cached one.

``--flow`` (configs 2 and 3) times the whole flow inference instead -- token
front end and the 10-step CFG ODE -- through ``flow_inference_batched`` (offline)
or ``flow_inference_batched_streaming`` (streaming); with ``--impl
reference-gpu`` the reference's own functions over ``FlashInferDiT``.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "faster-cosyvoice_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import numpy as np  # noqa: E402

METRIC = "DiT estimator mel-frames/s (per NFE)"
UNIT = "mel-frames/s"


# ---------------------------------------------------------------------------- workloads
def request_lengths(config: str) -> tuple[list[int], int, int]:
    """(request lengths, chunk, seed) of a BASELINE.json config."""
    if config == "2":
        rng = np.random.default_rng(1)
        return [int(v) for v in rng.integers(150, 601, size=8)], 0, 1
    if config == "3":
        rng = np.random.default_rng(2)
        prompt = rng.integers(100, 401, size=32)
        gen = rng.choice([30, 60, 120], size=32)
        return [int(a + b) for a, b in zip(prompt, gen)], 50, 2
    if config == "4":
        rng = np.random.default_rng(3)
        L = np.clip(np.round(rng.lognormal(np.log(400.0), 0.6, size=128)), 50, 3000)
        return [int(v) for v in L], 0, 3
    if config == "5":
        return [3000] * 16, 0, 5
    raise ValueError(f"unknown config {config}")


CONFIG_NAMES = {
    "2": "config2: 22-layer bf16 DiT, 1 NFE, 8 requests x CFG = 16 seqs, L~U[150,600], offline mask",
    "3": "config3: 22-layer bf16 DiT, 1 NFE of the 10-step CFG ODE, 32 requests x CFG = 64 seqs, "
         "L = U[100,400] + {30,60,120}, chunk-50 streaming mask",
    "4": "config4: 22-layer bf16 DiT, 1 NFE, 128 requests x CFG, L~LogNormal(ln 400, 0.6) in [50,3000], offline",
    "5": "config5: 22-layer bf16 DiT, 1 NFE, 16 requests x CFG, L=3000, full mask",
}


def make_batch(req_lengths, seed, device, dtype):
    import torch

    R = len(req_lengths)
    lengths = list(req_lengths) + list(req_lengths)  # [cond; uncond] (flashinfer_flow.py:45-51)
    B = 2 * R
    T = max(lengths)
    g = torch.Generator().manual_seed(1000 + seed)
    x = torch.randn(R, 80, T, generator=g)
    x = torch.cat([x, x], 0)
    mu = torch.cat([torch.randn(R, 80, T, generator=g), torch.zeros(R, 80, T)], 0)
    cond = torch.cat([torch.randn(R, 80, T, generator=g), torch.zeros(R, 80, T)], 0)
    spks = torch.cat([torch.randn(R, 80, generator=g), torch.zeros(R, 80)], 0)
    t = torch.rand(R, generator=g)
    t = torch.cat([t, t], 0)
    mask = torch.zeros(B, 1, T)
    for b, L in enumerate(lengths):
        mask[b, 0, :L] = 1
        x[b, :, L:] = 0
        mu[b, :, L:] = 0
        cond[b, :, L:] = 0
    host = dict(x=x, mask=mask, mu=mu, t=t, spks=spks, cond=cond)
    dev = {k: v.to(device=device, dtype=dtype).contiguous() for k, v in host.items()}
    return lengths, T, host, dev


# ---------------------------------------------------------------------------- clocks
class ClockSampler:
    """NVML sampling of SM clock and throttle reasons during the timed region (read only)."""

    REASONS = {
        0x0000000000000008: "hw_slowdown",
        0x0000000000000020: "sw_thermal_slowdown",
        0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000004: "sw_power_cap",
        0x0000000000000080: "hw_power_brake_slowdown",
    }

    def __init__(self, device_index: int):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml

            pynvml.nvmlInit()
            import torch

            uuid = "GPU-" + str(torch.cuda.get_device_properties(device_index).uuid)
            try:
                self._h = pynvml.nvmlDeviceGetHandleByUUID(uuid)
            except Exception:
                self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self._nv = pynvml
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._h = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for bit, name in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.02)

    def __enter__(self):
        if self._h is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._h is not None:
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------- CPU baseline
def _host_threads() -> int:
    """Let torch and the BLAS pools use every host thread (torchrun pins
    OMP_NUM_THREADS=1); returns the thread count in use."""
    import torch

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(limits=cores)
    except Exception:
        pass
    return torch.get_num_threads()


def stratified_order(lengths) -> list[int]:
    """Request indices in an order whose every prefix spans the length
    distribution: the median, the longest, the shortest, then the quartiles,
    the octiles, ... of the sorted lengths, then everything left."""
    n = len(lengths)
    by_len = sorted(range(n), key=lambda i: (lengths[i], i))
    fr = [0.5, 1.0, 0.0]
    k = 4
    while len(fr) < 4 * n and k <= 4 * n:
        fr += [j / k for j in range(1, k, 2)]
        k *= 2
    seen, order = set(), []
    for f in fr:
        i = by_len[int(round(f * (n - 1)))]
        if i not in seen:
            seen.add(i)
            order.append(i)
    order += [i for i in by_len if i not in seen]
    return order


class ReferenceCpuDiT:
    """The reference's own torch ``DiT`` (``cosyvoice/flow/DiT/dit.py:104-176``,
    padded SDPA path) in float32 on the host cores, from the offline install in
    ``baseline/_ref`` (its RoPE dependency ``x-transformers`` restated by the
    test shim).  One call = one request as its CFG pair (B = 2, the second half
    with mu, spks and cond zeroed, ``flashinfer_flow.py:45-51``), no padding.
    ``available`` is False (with ``why``) when the install is missing."""

    def __init__(self, seed: int, depth: int = 22):
        self.available, self.why, self.model = False, "", None
        ref_root = os.path.join(ROOT, "baseline", "_ref")
        if not os.path.isdir(os.path.join(ref_root, "faster_cosyvoice")):
            self.why = "reference not installed in baseline/_ref"
            return
        for p in (ref_root, os.path.join(ROOT, "tests", "golden", "_xt_shim")):
            if p not in sys.path:
                sys.path.insert(0, p)
        try:
            import torch
            from faster_cosyvoice.token2wav.cosyvoice.flow.DiT.dit import DiT
        except Exception as exc:
            self.why = f"reference import failed: {type(exc).__name__}: {exc}"
            return
        self.cores = _host_threads()
        torch.manual_seed(seed)  # the reference constructor's own random initialisation
        self.model = DiT(dim=1024, depth=depth, heads=16, dim_head=64, ff_mult=2, mel_dim=80, mu_dim=80,
                         spk_dim=80, out_channels=80, static_chunk_size=50, num_decoding_left_chunks=-1).eval()
        self.available = True

    def pair_seconds(self, L: int, streaming: bool, seed: int) -> float:
        import torch

        g = torch.Generator().manual_seed(seed)
        x = torch.randn(1, 80, L, generator=g).repeat(2, 1, 1)
        mu = torch.cat([torch.randn(1, 80, L, generator=g), torch.zeros(1, 80, L)])
        cond = torch.cat([torch.randn(1, 80, L, generator=g), torch.zeros(1, 80, L)])
        spks = torch.cat([torch.randn(1, 80, generator=g), torch.zeros(1, 80)])
        t = torch.rand(1, generator=g).repeat(2)
        mask = torch.ones(2, 1, L)
        with torch.inference_mode():
            t0 = time.perf_counter()
            self.model(x, mask, mu, t, spks, cond, streaming=streaming)
            return time.perf_counter() - t0


def cpu_reference_rate(req_lengths, chunk, seed, budget_s: float):
    """CPU baseline of the b200 arm: the reference torch DiT (``ReferenceCpuDiT``)
    over request pairs in stratified order until ``budget_s`` seconds are spent
    (at least one pair).  Falls back to the oracle port when the reference is
    not installed.  Returns the ``cpu_baseline`` object."""
    ref = ReferenceCpuDiT(seed)
    if not ref.available:
        r, dt, L, cores, sample = cpu_oracle_rate(None, req_lengths, seed, budget_s)
        return {"value": r, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample + f" ({ref.why})",
                "seconds": dt}
    ref.pair_seconds(64, chunk > 0, 0)  # warm-up: thread pools, allocator
    frames, secs, done = 0, 0.0, []
    for i in stratified_order(req_lengths):
        L = int(req_lengths[i])
        secs += ref.pair_seconds(L, chunk > 0, 100 + i)
        frames += 2 * L
        done.append(L)
        if secs >= budget_s:
            break
    sample = (f"{len(done)} of {len(req_lengths)} requests as CFG pairs (B=2, lengths {sorted(done)}), stratified "
              f"over the config's lengths; reference torch DiT, fp32, "
              f"{'chunk-%d streaming' % chunk if chunk else 'offline'} mask")
    return {"value": frames / secs, "unit": UNIT, "cores": ref.cores, "kind": "reference", "sample": sample,
            "seconds": secs}


def cpu_oracle_rate(params, req_lengths, seed, budget_s: float):
    """Time the oracle port of the reference torch DiT (float32, numpy BLAS on
    every host thread) on one document of the workload, trimmed so one pass
    takes about ``budget_s`` seconds (the fallback when the reference itself is
    not installed).  Returns (frames/s, seconds, rows, cores, sample)."""
    from oracle import dit_oracle as O

    if params is None:
        import torch

        from fcv_b200.model import B200DiT

        torch.manual_seed(seed)
        params = {k: v.detach().float().numpy() for k, v in B200DiT(depth=22).eval().state_dict().items()}
    cores = os.cpu_count() or 1
    try:
        # torchrun pins OMP_NUM_THREADS=1; the CPU baseline uses every host thread
        from threadpoolctl import threadpool_info, threadpool_limits

        threadpool_limits(limits=cores)
        cores = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:
        pass
    rng = np.random.default_rng(seed)

    def doc(L):
        return (rng.standard_normal((80, L)).astype(np.float32), rng.standard_normal((80, L)).astype(np.float32),
                rng.standard_normal((80, L)).astype(np.float32), rng.standard_normal(80).astype(np.float32))

    # calibrate on 32 rows, then size the sample to the budget
    t0 = time.perf_counter()
    O.dit_forward_docs(params, [doc(32)], np.array([0.5], np.float32))
    per_row = (time.perf_counter() - t0) / 32
    L = int(max(16, min(req_lengths[0], budget_s / max(per_row, 1e-6))))
    d = doc(L)
    t0 = time.perf_counter()
    O.dit_forward_docs(params, [d], np.array([0.5], np.float32))
    dt = time.perf_counter() - t0
    sample = f"one document of {L} frames (22-layer fp32 oracle port, offline mask)"
    return L / dt, dt, L, cores, sample


# ---------------------------------------------------------------------------- flow inference
def flow_requests(config: str, seed: int):
    """Token, prompt and speaker inputs of the flow workload of a config.  A
    request of L mel frames carries L // 2 speech tokens (token_mel_ratio 2).
    Offline (config 2): its prompt Mel is the first 40 % of its frames.
    Streaming (config 3): the prompt part of L is the prompt Mel, every stream
    is non-final with 3 lookahead tokens of context."""
    import torch

    req, chunk, _ = request_lengths(config)
    rng = np.random.default_rng(500 + seed)
    streaming = chunk > 0
    tokens, prompts = [], []
    if streaming:
        prng = np.random.default_rng(2)
        prompt_mel = prng.integers(100, 401, size=32)
    for i, L in enumerate(req):
        n_tok = L // 2
        lp = int(prompt_mel[i]) if streaming else int(0.4 * 2 * n_tok)
        lp = min(lp, 2 * n_tok)
        tokens.append(rng.integers(0, 6561, size=n_tok + (3 if streaming else 0)).tolist())
        prompts.append(torch.from_numpy(rng.standard_normal((1, lp, 80)).astype(np.float32)))
    spk = torch.from_numpy(rng.standard_normal((len(req), 192)).astype(np.float32))
    finalize = [False] * len(req) if streaming else None
    mel = sum(2 * (len(t) - (3 if streaming else 0)) for t in tokens)
    return tokens, prompts, spk, finalize, mel


def flow_arm(args, impl: str):
    """One JSON line: the whole flow inference (front end + 10-step CFG ODE) of a
    config's requests, this build's device-packed flow or the reference's
    flow_inference_batched[_streaming] over FlashInferDiT (flashinfer_flow.py:118-281)."""
    import types

    import torch

    from fcv_b200.flow import B200Flow, flow_inference_batched, flow_inference_batched_streaming

    req, chunk, seed = request_lengths(args.config)
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    tokens, prompts, spk, finalize, mel = flow_requests(args.config, seed)
    streaming = finalize is not None
    torch.manual_seed(seed)
    ours = B200Flow(depth=22).eval()
    base = {"metric": "flow mel-frames/s (front end + 10-step CFG ODE)", "unit": UNIT,
            "config": {"workload": f"flow inference, {CONFIG_NAMES[args.config]}", "requests": len(req),
                       "mel_frames": mel, "streaming": streaming}}
    if impl == "b200":
        flow = ours.to(device, torch.bfloat16)
        flow.decoder.estimator.finalize_weights()
        dtype = "bf16"

        def run(p, s):
            if streaming:
                return flow_inference_batched_streaming(flow, tokens, p, s, finalize)
            return flow_inference_batched(flow, tokens, p, s)
    else:
        ref_root = os.path.join(ROOT, "baseline", "_ref")
        if not os.path.isdir(os.path.join(ref_root, "faster_cosyvoice")):
            print(json.dumps({**base, "impl": "reference-gpu", "unavailable": "reference not installed in baseline/_ref"}))
            return
        for p in (ref_root, os.path.join(ROOT, "tests", "golden", "_xt_shim")):
            if p not in sys.path:
                sys.path.insert(0, p)
        if "omegaconf" not in sys.modules:  # imported by flow.py for a default argument only
            stub = types.ModuleType("omegaconf")
            stub.DictConfig = dict
            sys.modules["omegaconf"] = stub
        from faster_cosyvoice.token2wav import flashinfer_flow as ref_flow
        from faster_cosyvoice.token2wav.cosyvoice.flow.flow import CausalMaskedDiffWithDiT
        from faster_cosyvoice.token2wav.cosyvoice.flow.flow_matching import CausalConditionalCFM
        from faster_cosyvoice.token2wav.cosyvoice.transformer.upsample_encoder import PreLookaheadLayer
        from faster_cosyvoice.token2wav.flashinfer_dit import FlashInferDiT

        est = FlashInferDiT(device=device, static_chunk_size=50)
        est.load_state_dict(ours.decoder.estimator.state_dict(), strict=False)
        rdt = torch.float16 if args.ref_dtype == "fp16" else torch.bfloat16
        est = est.to(device=device, dtype=rdt).eval()
        est.finalize_weights()
        cfm = types.SimpleNamespace(sigma_min=1e-6, solver="euler", t_scheduler="cosine", training_cfg_rate=0.2,
                                    inference_cfg_rate=0.7, reg_loss_type="l1")
        decoder = CausalConditionalCFM(in_channels=240, cfm_params=cfm, n_spks=1, spk_emb_dim=80, estimator=est)
        flow = CausalMaskedDiffWithDiT(input_size=80, output_size=80, spk_embed_dim=192, output_type="mel",
                                       vocab_size=6561, input_frame_rate=25, only_mask_loss=True, token_mel_ratio=2,
                                       pre_lookahead_len=3,
                                       pre_lookahead_layer=PreLookaheadLayer(in_channels=80, channels=1024,
                                                                             pre_lookahead_len=3),
                                       decoder=decoder)
        front = {k: v for k, v in ours.state_dict().items() if not k.startswith("decoder.")}
        flow.load_state_dict(front, strict=False)
        flow = flow.to(device).to(rdt).eval()
        dtype = "f16" if rdt == torch.float16 else "bf16"

        def run(p, s):
            if streaming:
                return ref_flow.flow_inference_batched_streaming(flow, tokens, p, s, finalize)
            return ref_flow.flow_inference_batched(flow, tokens, p, s)

    p_dev = [p.to(device) for p in prompts]
    s_dev = spk.to(device)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    for _ in range(args.warmup):
        run(p_dev, s_dev)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(0) as clocks:
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record(stream)
            out = run(p_dev, s_dev)
            ev[i][1].record(stream)
        torch.cuda.synchronize()
    ms = [a.elapsed_time(b) for a, b in ev]
    t = float(np.mean(ms))
    line = {**base, "impl": impl if impl == "b200" else "reference-gpu", "value": mel / (t / 1000.0),
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t,
            "higher_is_better": True, "dtype": dtype, "data": "synthetic (seeded tokens, prompts, speakers; "
            "random-init 22-layer DiT and front end)", "step_ms_min": min(ms), "clocks": clocks.summary(),
            "generated_frames": int(sum(o.shape[2] for o in out))}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- vocoder
def vocoder_arm(args, impl: str):
    """One JSON line: the HiFT vocoder over a config's request mels (offline
    finalize=True for config 2, non-final chunks for config 3), this build's one
    packed ``fcv_hift_forward`` call or the reference's per-request
    ``CausalHiFTGenerator.inference`` loop (token2wav.py:130-131, 194-195).
    Synthetic seeded weights and noise table (tests/golden/hift_weights.py), float32."""
    import types

    import torch

    req, chunk, seed = request_lengths(args.config)
    if args.requests > 0:
        req = req[:args.requests]
    finalize = chunk == 0
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import hift_weights as HW

    sd = HW.hift_state(0)
    noise = HW.hift_noise(480 * (max(req) + 8), 1)
    rng = np.random.default_rng(900 + seed)
    mels = [torch.from_numpy((1.5 * rng.standard_normal((1, 80, L)) - 3).astype(np.float32)).to(device) for L in req]
    frames = sum(req)
    base = {"metric": "vocoder mel-frames/s (HiFT decode)", "unit": UNIT,
            "config": {"workload": f"HiFT vocoder, {CONFIG_NAMES[args.config]}", "requests": len(req),
                       "mel_frames": frames, "finalize": finalize}}
    if impl == "b200":
        from fcv_b200.hift import B200HiFT

        voc = B200HiFT(sd, noise, device)

        def run():
            return voc.inference_batched(mels, finalize)
    else:
        ref_root = os.path.join(ROOT, "baseline", "_ref")
        if not os.path.isdir(os.path.join(ref_root, "faster_cosyvoice")):
            print(json.dumps({**base, "impl": "reference-gpu", "unavailable": "reference not installed in baseline/_ref"}))
            return
        for p in (ref_root, os.path.join(ROOT, "tests", "golden", "_xt_shim")):
            if p not in sys.path:
                sys.path.insert(0, p)
        if "omegaconf" not in sys.modules:  # builders.py imports it for the flow's config only
            stub = types.ModuleType("omegaconf")
            stub.DictConfig = dict
            sys.modules["omegaconf"] = stub
        from faster_cosyvoice.token2wav.builders import build_hift

        hift = build_hift()
        hift.load_state_dict(sd, strict=True)
        hift.m_source.l_sin_gen.sine_waves = noise[None]
        hift = hift.to(device).eval()

        def run():
            with torch.inference_mode():
                return [hift.inference(speech_feat=m, finalize=finalize)[0] for m in mels]

    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(0) as clocks:
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record(stream)
            out = run()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
    ms = [a.elapsed_time(b) for a, b in ev]
    t = float(np.mean(ms))
    line = {**base, "impl": impl if impl == "b200" else "reference-gpu", "value": frames / (t / 1000.0),
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t, "step_ms_min": min(ms),
            "higher_is_better": True, "dtype": "f32 (f64 f0 predictor)",
            "data": "synthetic (seeded mels, weights and noise table)", "clocks": clocks.summary(),
            "samples": int(sum(o.shape[-1] for o in out))}
    print(json.dumps(line), flush=True)


def vocoder_cpu_arm(args):
    """The vocoder's CPU reference arm: the numpy port of CausalHiFTGenerator.inference
    (oracle/hift_oracle.py, float32 with a float64 f0 predictor, BLAS on every host
    thread) timed on the config's requests (``--requests`` honoured) one after the
    other, each trimmed to the same length so a step takes a few seconds.  The
    per-frame cost is calibrated after a warm-up call, from two lengths so that the
    fixed per-call cost is subtracted.  Same metric and statistic (mean step time)
    as ``vocoder_arm``; the line's ``sample`` says what was timed."""
    from oracle import hift_oracle as H

    req, chunk, seed = request_lengths(args.config)
    if args.requests > 0:
        req = req[:args.requests]
    finalize = chunk == 0
    cores = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_info, threadpool_limits

        threadpool_limits(limits=cores)
        cores = max([i.get("num_threads", 1) for i in threadpool_info()] or [1])
    except Exception:
        pass
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import hift_weights as HW

    W = HW.folded(HW.hift_state(0))
    noise = HW.hift_noise(480 * (max(req) + 8), 1).numpy()
    rng = np.random.default_rng(900 + seed)
    mels = [(1.5 * rng.standard_normal((L, 80)) - 3).astype(np.float32) for L in req]
    budget = max(0.5, min(6.0, 150.0 / (args.steps + args.warmup)))
    longest = mels[int(np.argmax(req))]
    H.inference(longest[:16], W, noise, finalize)  # warm-up (BLAS threads, allocations)

    def once(L):
        t0 = time.perf_counter()
        H.inference(longest[:L], W, noise, finalize)
        return time.perf_counter() - t0

    l2 = min(48, max(req))
    t16, t48 = once(16), once(l2)
    per_frame = max((t48 - t16) / max(l2 - 16, 1), 1e-6)
    fixed = max(t16 - 16 * per_frame, 0.0)
    # every request trimmed to the same L frames, L sized so the step fits the budget
    L = int(max(16, min(max(req), (budget - fixed * len(req)) / (per_frame * len(req)))))
    use = [m[:min(L, m.shape[0])] for m in mels]
    frames = sum(m.shape[0] for m in use)

    def step():
        for m in use:
            H.inference(m, W, noise, finalize)

    for _ in range(args.warmup):
        step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    value = frames / float(np.mean(times))
    sample = (f"{len(use)} requests, each trimmed to at most {L} mel frames ({frames} frames per step; "
              f"{'offline' if finalize else 'non-final chunks'}, numpy port)")
    line = {"metric": "vocoder mel-frames/s (HiFT decode)", "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * float(np.mean(times)),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (f64 f0 predictor)",
            "data": "synthetic (seeded mels, weights and noise table)",
            "config": {"workload": f"HiFT vocoder, {CONFIG_NAMES[args.config]}", "requests": len(req),
                       "mel_frames": sum(req), "finalize": finalize,
                       "measured_requests": len(use), "measured_mel_frames": frames},
            "impl": "reference",
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- streaming calls
def stream_arm(args, impl: str, cached: bool):
    """One JSON line: a streaming session of 32 streams (config 3's prompts, 100-400
    Mel frames) that each advance by 25 speech tokens (50 frames) per call, all
    calls through flow_inference_batched_streaming (flashinfer_flow.py:187-281).
    Calls 1..3 warm up (and build the cache); the next ``--steps`` calls are
    timed.  Metric: new Mel frames per second (50 per stream per call)."""
    import types

    import torch

    from fcv_b200.flow import B200Flow, PrefixCache, flow_inference_batched_streaming

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    rng = np.random.default_rng(2)
    prompt_mel = [int(v) for v in rng.integers(100, 401, size=32)]
    R = len(prompt_mel)
    calls = 3 + args.steps
    prng = np.random.default_rng(7)
    tokens = [prng.integers(0, 6561, size=pm // 2 + 25 * (calls + 1) + 3).tolist() for pm in prompt_mel]
    prompts = [torch.from_numpy(prng.standard_normal((1, pm, 80)).astype(np.float32)).to(device) for pm in prompt_mel]
    spk = torch.from_numpy(prng.standard_normal((R, 192)).astype(np.float32)).to(device)
    torch.manual_seed(2)
    ours = B200Flow(depth=22).eval()
    if impl == "b200":
        flow = ours.to(device, torch.bfloat16)
        flow.decoder.estimator.finalize_weights()
        max_frames = max(prompt_mel) + 50 * (calls + 1) + 64
        cache = PrefixCache(flow, max_streams=R, max_frames=max_frames) if cached else None
        dtype = "bf16"

        def run(tl):
            if cache is None:
                return flow_inference_batched_streaming(flow, tl, prompts, spk, [False] * R)
            return flow_inference_batched_streaming(flow, tl, prompts, spk, [False] * R, cache=cache,
                                                    stream_ids=list(range(R)))
    else:
        ref_root = os.path.join(ROOT, "baseline", "_ref")
        if not os.path.isdir(os.path.join(ref_root, "faster_cosyvoice")):
            print(json.dumps({"impl": "reference-gpu", "unavailable": "reference not installed in baseline/_ref"}))
            return
        for p in (ref_root, os.path.join(ROOT, "tests", "golden", "_xt_shim")):
            if p not in sys.path:
                sys.path.insert(0, p)
        if "omegaconf" not in sys.modules:
            stub = types.ModuleType("omegaconf")
            stub.DictConfig = dict
            sys.modules["omegaconf"] = stub
        from faster_cosyvoice.token2wav import flashinfer_flow as ref_flow
        from faster_cosyvoice.token2wav.cosyvoice.flow.flow import CausalMaskedDiffWithDiT
        from faster_cosyvoice.token2wav.cosyvoice.flow.flow_matching import CausalConditionalCFM
        from faster_cosyvoice.token2wav.cosyvoice.transformer.upsample_encoder import PreLookaheadLayer
        from faster_cosyvoice.token2wav.flashinfer_dit import FlashInferDiT

        rdt = torch.float16 if args.ref_dtype == "fp16" else torch.bfloat16
        est = FlashInferDiT(device=device, static_chunk_size=50)
        est.load_state_dict(ours.decoder.estimator.state_dict(), strict=False)
        est = est.to(device=device, dtype=rdt).eval()
        est.finalize_weights()
        cfm = types.SimpleNamespace(sigma_min=1e-6, solver="euler", t_scheduler="cosine", training_cfg_rate=0.2,
                                    inference_cfg_rate=0.7, reg_loss_type="l1")
        decoder = CausalConditionalCFM(in_channels=240, cfm_params=cfm, n_spks=1, spk_emb_dim=80, estimator=est)
        flow = CausalMaskedDiffWithDiT(input_size=80, output_size=80, spk_embed_dim=192, output_type="mel",
                                       vocab_size=6561, input_frame_rate=25, only_mask_loss=True, token_mel_ratio=2,
                                       pre_lookahead_len=3,
                                       pre_lookahead_layer=PreLookaheadLayer(in_channels=80, channels=1024,
                                                                             pre_lookahead_len=3),
                                       decoder=decoder)
        flow.load_state_dict({k: v for k, v in ours.state_dict().items() if not k.startswith("decoder.")},
                             strict=False)
        flow = flow.to(device).to(rdt).eval()
        dtype = "f16" if rdt == torch.float16 else "bf16"

        def run(tl):
            return ref_flow.flow_inference_batched_streaming(flow, tl, prompts, spk, [False] * R)

    stream = torch.cuda.current_stream(device)
    times, frames = [], []
    with ClockSampler(0) as clocks:
        for c in range(calls):
            tl = [tokens[r][:prompt_mel[r] // 2 + 25 * (c + 1) + 3] for r in range(R)]
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            run(tl)
            e1.record(stream)
            torch.cuda.synchronize()
            if c >= 3:
                times.append(e0.elapsed_time(e1))
                frames.append(sum(2 * (len(t) - 3) for t in tl))
    t = float(np.mean(times))
    print(json.dumps({"metric": "streaming flow: new mel-frames/s (32 streams, +50 frames per call)",
                      "unit": UNIT, "value": R * 50 / (t / 1000.0), "impl": impl if impl == "b200" else "reference-gpu",
                      "prefix_cache": cached, "ms_per_call": t, "calls_timed": len(times),
                      "frames_per_call_total": float(np.mean(frames)), "dtype": dtype, "clocks": clocks.summary(),
                      "data": "synthetic (config-3 prompt lengths, seeded tokens)"}), flush=True)


# ---------------------------------------------------------------------------- single-request latency
def latency_arm(args, impl: str):
    """One JSON line: latency of one estimator call for one CFG pair (B = 2),
    the case the reference's CUDA-graph buckets serve (flashinfer_dit.py:742-826):
    eager and graph-bucketed, through the module's forward on device-resident
    inputs.  ``wall`` = host time from call to synchronised result (launch cost
    included), ``device`` = CUDA-event time on the stream."""
    import torch

    from fcv_b200.model import DEFAULT_GRAPH_BUCKETS, B200DiT

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    streaming = args.config == "3"
    torch.manual_seed(1)
    ours = B200DiT(depth=22).eval()
    if impl == "b200":
        model = ours.to(device, torch.bfloat16)
        model.finalize_weights()
        model.graph_buckets = DEFAULT_GRAPH_BUCKETS
        dt = torch.bfloat16

        def set_graph(on):
            model.use_cuda_graph = on
    else:
        ref_root = os.path.join(ROOT, "baseline", "_ref")
        if not os.path.isdir(os.path.join(ref_root, "faster_cosyvoice")):
            print(json.dumps({"impl": "reference-gpu", "unavailable": "reference not installed in baseline/_ref"}))
            return
        for p in (ref_root, os.path.join(ROOT, "tests", "golden", "_xt_shim")):
            if p not in sys.path:
                sys.path.insert(0, p)
        from faster_cosyvoice.token2wav.flashinfer_dit import FlashInferDiT

        dt = torch.float16 if args.ref_dtype == "fp16" else torch.bfloat16
        models = {}
        for on in (False, True):
            # offline presets in seconds, streaming presets in frames (config/settings.py:9-10)
            m = FlashInferDiT(device=device, static_chunk_size=50, enable_cuda_graph=on and not streaming,
                              cuda_graph_buckets=(8.0, 12.0, 16.0, 20.0, 24.0) if on and not streaming else None,
                              stream_graph_buckets=(512, 640, 768, 896, 1024, 1280) if on and streaming else None)
            m.load_state_dict(ours.state_dict(), strict=False)
            m = m.to(device=device, dtype=dt).eval()
            m.finalize_weights()
            models[on] = m
        holder = {}

        def set_graph(on):
            holder["m"] = models[on]

        def model(*a, **k):
            return holder["m"](*a, **k)

    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    results = {}
    for L in (200, 400, 800):
        g = torch.Generator().manual_seed(L)
        x = torch.randn(1, 80, L, generator=g).repeat(2, 1, 1)
        mu = torch.cat([torch.randn(1, 80, L, generator=g), torch.zeros(1, 80, L)])
        cond = torch.cat([torch.randn(1, 80, L, generator=g), torch.zeros(1, 80, L)])
        spks = torch.cat([torch.randn(1, 80, generator=g), torch.zeros(1, 80)])
        t = torch.rand(1, generator=g).repeat(2)
        inp = [v.to(device, dt).contiguous() for v in (x, torch.ones(2, 1, L), mu, t, spks, cond)]
        res = {}
        for on in (False, True):
            set_graph(on)
            with torch.inference_mode():
                for _ in range(args.warmup):
                    model(*inp, streaming=streaming)
                torch.cuda.synchronize()
                wall, dev_ms = [], []
                for _ in range(args.steps):
                    flush.zero_()
                    torch.cuda.synchronize()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    t0 = time.perf_counter()
                    e0.record(stream)
                    model(*inp, streaming=streaming)
                    e1.record(stream)
                    torch.cuda.synchronize()
                    wall.append(1000 * (time.perf_counter() - t0))
                    dev_ms.append(e0.elapsed_time(e1))
            res["graph" if on else "eager"] = {"wall_ms": float(statistics.median(wall)),
                                               "device_ms": float(statistics.median(dev_ms))}
        results[f"L={L}"] = res
    print(json.dumps({"metric": "estimator call latency, one CFG pair (B=2)", "unit": "ms",
                      "higher_is_better": False, "impl": impl, "dtype": "bf16" if dt == torch.bfloat16 else "f16",
                      "streaming": streaming, "steps": args.steps, "warmup": args.warmup,
                      "results": results}), flush=True)


# ---------------------------------------------------------------------------- main
def reference_gpu_arm(args, req_lengths, chunk, seed, cfg, strong):
    """The reference's FlashInferDiT (flashinfer_dit.py:98-543, loaded as apply_flashinfer does at
    :951-988) on the B200 with this run's weights and inputs; one JSON line."""
    import torch

    ref_root = os.path.join(ROOT, "baseline", "_ref")
    base = {"metric": METRIC, "unit": UNIT, "impl": "reference-gpu", "config": cfg}
    if not os.path.isdir(os.path.join(ref_root, "faster_cosyvoice")):
        print(json.dumps({**base, "unavailable": "reference not installed in baseline/_ref"}), flush=True)
        return
    if not torch.cuda.is_available():
        print(json.dumps({**base, "unavailable": "no CUDA device"}), flush=True)
        return
    # x-transformers==2.23.5 (the reference's RoPE dependency) is not installed: the RoPE tables come
    # from the test shim that restates them (interleaved pairs, base 10000, rotary dim 64)
    for p in (ref_root, os.path.join(ROOT, "tests", "golden", "_xt_shim")):
        if p not in sys.path:
            sys.path.insert(0, p)
    try:
        from faster_cosyvoice.token2wav.flashinfer_dit import FlashInferDiT
    except Exception as exc:  # missing flashinfer / triton on this box
        print(json.dumps({**base, "unavailable": f"reference import failed: {type(exc).__name__}: {exc}"}),
              flush=True)
        return
    from fcv_b200.model import B200DiT

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    rdt = torch.float16 if args.ref_dtype == "fp16" else torch.bfloat16
    # FlashInferDiT counts each document's length by summing its mask in the activation
    # dtype (flashinfer_dit.py:460).  A length that rounds up past the padded length T
    # makes its packing gather read past the row: in bf16, 3000 rounds to 3008, and on
    # the B200 that raised a device-side assert.  Such a batch is not run again.
    T_pad = max(req_lengths)
    rounded = [int(torch.tensor(float(L), dtype=rdt).item()) for L in req_lengths]
    if any(r > T_pad for r in rounded):
        bad = sorted({(L, r) for L, r in zip(req_lengths, rounded) if r > T_pad})
        print(json.dumps({**base, "unavailable": f"the reference counts lengths in {args.ref_dtype} "
                          f"(flashinfer_dit.py:460): {bad[0][0]} frames round to {bad[0][1]} > T={T_pad}, "
                          "an out-of-range gather that raised a device-side assert on B200"}), flush=True)
        return
    torch.manual_seed(seed)
    sd = B200DiT(depth=22).eval().state_dict()
    ref = FlashInferDiT(device=device, static_chunk_size=50)
    missing, unexpected = ref.load_state_dict(sd, strict=False)
    missing = [k for k in missing if "rope" not in k]
    if missing or unexpected:
        raise RuntimeError(f"state-dict mismatch: missing={missing}, unexpected={unexpected}")
    ref = ref.to(device=device, dtype=rdt).eval()
    ref.finalize_weights()
    lengths, T, host, dev = make_batch(req_lengths, seed, device, rdt)
    streaming = chunk > 0
    N = sum(lengths)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    def step(inp):
        with torch.inference_mode():
            return ref(inp["x"], inp["mask"], inp["mu"], inp["t"], inp["spks"], inp["cond"], streaming=streaming)

    for _ in range(args.warmup):
        step(dev)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(0) as clocks:
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record(stream)
            step(dev)
            ev[i][1].record(stream)
        torch.cuda.synchronize()
    step_ms = [a.elapsed_time(b) for a, b in ev]
    ms = float(np.mean(step_ms))

    pin = {k: v.to(rdt).pin_memory() for k, v in host.items()}
    dev2 = {k: torch.empty_like(v, device=device) for k, v in pin.items()}
    out_h = torch.empty(len(lengths), 80, T, dtype=rdt).pin_memory()

    def e2e_step():
        for k in pin:
            dev2[k].copy_(pin[k], non_blocking=True)
        out_h.copy_(step(dev2), non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    line = {**base, "value": N / (ms / 1000.0), "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong" if strong else "weak",
            "vs_baseline": None, "dtype": "f16" if rdt == torch.float16 else "bf16",
            "data": "synthetic (seeded N(0,1) inputs, random-init weights of the 22-layer DiT)",
            "e2e": {"value": N / (e2e_ms / 1000.0), "unit": UNIT,
                    "h2d_bytes_per_step": int(sum(v.numel() * v.element_size() for v in pin.values())),
                    "d2h_bytes_per_step": int(out_h.numel() * out_h.element_size()),
                    "api": "FlashInferDiT.forward(x, mask, mu, t, spks, cond, streaming) with pinned host buffers"},
            "step_ms_min": min(step_ms), "step_ms_median": float(statistics.median(step_ms)),
            "clocks": clocks.summary(),
            "note": "the reference's own GPU estimator path (packed Triton/FlashInfer path), "
                    "L2 flushed between steps, device-resident inputs for value"}
    print(json.dumps(line), flush=True)


def reference_cpu_arm(args, req_lengths, chunk, seed, cfg, strong):
    """``--impl reference``: the reference's own CPU implementation of the path
    -- its torch ``DiT`` (``dit.py:145-176``), fp32, every host thread -- timed
    per request as its CFG pair.  Step k times request ``order[k % R]`` of a
    stratified order (median, longest, shortest, quartiles, ...), so the steps
    cover the length distribution; value = frames of the timed steps / their
    time.  Warm-up steps run a short pair (thread pools, allocator).  Falls
    back to the oracle port (``kind: "port"``) when the reference is not
    installed."""
    ref = ReferenceCpuDiT(seed)
    base = {"metric": METRIC, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "strong" if strong else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded N(0,1) inputs, random-init weights of the 22-layer DiT)",
            "config": cfg, "impl": "reference"}
    if not ref.available:
        import torch

        from fcv_b200.model import B200DiT

        torch.manual_seed(seed)
        params = {k: v.detach().float().numpy() for k, v in B200DiT(depth=22).eval().state_dict().items()}
        budget = max(0.5, min(6.0, 150.0 / (args.steps + args.warmup)))
        for _ in range(args.warmup):
            cpu_oracle_rate(params, req_lengths, seed, budget)
        rates, times = [], []
        for _ in range(args.steps):
            r, dt, L, cores, sample = cpu_oracle_rate(params, req_lengths, seed, budget)
            rates.append(r)
            times.append(dt)
        value = float(statistics.median(rates))
        line = {**base, "value": value, "ms_per_step": 1000 * float(np.mean(times)),
                "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                                 "sample": sample + f" ({ref.why})"},
                "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    for w in range(args.warmup):
        ref.pair_seconds(64, chunk > 0, w)
    order = stratified_order(req_lengths)
    times, frames, lens = [], 0, []
    for k in range(args.steps):
        i = order[k % len(order)]
        L = int(req_lengths[i])
        times.append(ref.pair_seconds(L, chunk > 0, 100 + i))
        frames += 2 * L
        lens.append(L)
    value = frames / float(sum(times))
    sample = (f"{args.steps} steps, each one request as its CFG pair (B=2, no padding) in stratified order over "
              f"the config's {len(req_lengths)} requests ({len(set(order[:args.steps]))} distinct; lengths "
              f"{min(lens)}-{max(lens)}, {frames} frames); reference torch DiT (baseline/_ref), fp32, "
              f"{'chunk-%d streaming' % chunk if chunk else 'offline'} mask")
    line = {**base, "value": value, "ms_per_step": 1000 * float(np.mean(times)),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": ref.cores, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def gemm_compare(args, req_lengths, seed, cfg):
    """One JSON line: per block GEMM shape of the config (M = packed rows; QKV
    1024 -> 3072 with the RoPE epilogue, out 1024 -> 1024 and FF2 2048 -> 1024
    with the gated-residual epilogue, FF1 1024 -> 2048 with GELU), the mean time
    of 22 back-to-back launches in a CUDA graph for this build's tcgen05 GEMM and
    for cuBLAS through torch ``F.linear`` (bias, bf16 out; the reference's
    ``flashinfer_dit.py:490-512``, with its separate GELU / residual passes left
    out, so cuBLAS is timed on less work).  L2 flushed between graph replays."""
    import torch
    import torch.nn.functional as F

    from fcv_b200 import _lib, ops
    from fcv_b200.model import B200DiT

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    torch.manual_seed(seed)
    model = B200DiT(depth=22).eval().to(device=device, dtype=torch.bfloat16)
    model.finalize_weights()
    lengths = list(req_lengths) + list(req_lengths)
    layout = model.prepare_layout(lengths, max(lengths), False, device)
    N = sum(lengths)
    d = model._derived
    A = torch.randn(N, 2048, device=device, dtype=torch.bfloat16)
    H = torch.zeros(N, 1024, device=device)
    O3 = torch.empty(N, 3072, device=device, dtype=torch.bfloat16)
    O2 = torch.empty(N, 2048, device=device, dtype=torch.bfloat16)
    O1 = torch.empty(N, 1024, device=device, dtype=torch.bfloat16)
    gate = torch.ones(len(lengths), 4096, device=device)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    b16 = {k: d[k].to(torch.bfloat16) for k in ("qkv_b", "o_b", "ff1_b", "ff2_b")}  # cuBLAS bias in bf16
    shapes = {
        "qkv": (1024, 3072, lambda i: ops.linear(A[:, :1024], d["qkv_w"][i], d["qkv_b"][i], epilogue=_lib.EPI_BIAS_ROPE_QKV,
                                                  out=O3, aux=layout.positions, rope_cos=d["rope_cos"],
                                                  rope_sin=d["rope_sin"]),
                lambda i: torch.addmm(b16["qkv_b"][i], A[:, :1024], d["qkv_w"][i].t(), out=O3)),
        "out": (1024, 1024, lambda i: ops.linear(A[:, :1024], d["o_w"][i], d["o_b"][i], epilogue=_lib.EPI_BIAS_GATE_RES,
                                                  out=H, aux=layout.document_ids, gate=gate, gate_stride=4096),
                lambda i: torch.addmm(b16["o_b"][i], A[:, :1024], d["o_w"][i].t(), out=O1)),
        "ff1": (1024, 2048, lambda i: ops.linear(A[:, :1024], d["ff1_w"][i], d["ff1_b"][i], epilogue=_lib.EPI_BIAS_GELU,
                                                  out=O2),
                lambda i: torch.addmm(b16["ff1_b"][i], A[:, :1024], d["ff1_w"][i].t(), out=O2)),
        "ff2": (2048, 1024, lambda i: ops.linear(A, d["ff2_w"][i], d["ff2_b"][i], epilogue=_lib.EPI_BIAS_GATE_RES,
                                                  out=H, aux=layout.document_ids, gate=gate, gate_stride=4096),
                lambda i: torch.addmm(b16["ff2_b"][i], A, d["ff2_w"][i].t(), out=O1)),
    }

    def time_graph(fn, reps):
        fn()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        g.replay()
        torch.cuda.synchronize()
        tot = 0.0
        for _ in range(reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            tot += e0.elapsed_time(e1)
        return tot / reps

    res = {}
    with ClockSampler(0) as clocks:
        for name, (K, Nout, ours, cublas) in shapes.items():
            flops = 2.0 * N * K * Nout
            row = {"M": N, "K": K, "N": Nout}
            for impl, fn in (("b200", ours), ("cublas", cublas)):
                ms = time_graph(lambda: [fn(i) for i in range(22)], max(3, args.steps)) / 22
                row[impl] = {"ms": ms, "tflops": flops / (ms / 1000.0) / 1e12}
            row["speedup"] = row["cublas"]["ms"] / row["b200"]["ms"]
            res[name] = row
    print(json.dumps({"metric": "block GEMM TFLOP/s, this build vs cuBLAS (F.linear), per shape",
                      "config": cfg, "results": res, "clocks": clocks.summary(),
                      "note": "ours includes its fused epilogue (RoPE / gated residual into fp32 h / GELU); "
                              "cuBLAS computes bias + bf16 output only"}), flush=True)


def bin_times(args, req_lengths, chunk, seed, cfg):
    """One JSON line: the config's requests dealt into ``args.bin_times`` LPT bins
    (fcv_b200.shard.lpt_bins, as ``--gpus N`` under torchrun deals them), each bin's
    estimator call timed alone on this one GPU (CUDA-graph replays, median of 6,
    L2 flushed between replays).  The spread of the bins' times is the partition's
    own imbalance, free of per-GPU clock differences between the ranks of a run."""
    import torch

    from fcv_b200.model import B200DiT
    from fcv_b200.shard import bin_loads, lpt_bins

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    torch.manual_seed(seed)
    model = B200DiT(depth=22).eval().to(device=device, dtype=torch.bfloat16)
    model.finalize_weights()
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    bins = lpt_bins(req_lengths, args.bin_times, chunk or None)

    def time_bin(sub):
        lengths, T, _, dev = make_batch(sub, seed, device, torch.bfloat16)
        layout = model.layout_from_mask(dev["mask"], chunk > 0)
        out = torch.empty(len(lengths), 80, T, dtype=torch.bfloat16, device=device)
        run = lambda: model.forward_layout(layout, dev["x"], dev["mu"], dev["t"], dev["spks"], dev["cond"],  # noqa: E731
                                           out=out)
        for _ in range(3):
            run()
        torch.cuda.synchronize()
        ts = []
        for _ in range(6):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            run()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return sorted(ts)[len(ts) // 2]

    with ClockSampler(0) as clocks:
        ms = [time_bin([req_lengths[i] for i in b]) for b in bins]
    loads = bin_loads(req_lengths, bins, chunk or None)
    print(json.dumps({"metric": "LPT bins timed alone on one GPU", "config": cfg, "bins": args.bin_times,
                      "requests_per_bin": [len(b) for b in bins],
                      "rows_per_bin": [2 * sum(req_lengths[i] for i in b) for b in bins],
                      "cost_max_over_mean": max(loads) / (sum(loads) / len(loads)),
                      "ms_per_bin": ms, "time_max_over_mean": max(ms) / (sum(ms) / len(ms)),
                      "clocks": clocks.summary()}), flush=True)


def ncu_case(req_lengths, chunk, seed):
    """One pass of every kernel of the path on a config's inputs, for ncu: the
    packed layout from the device mask (fcv_mask_lengths, fcv_pack_layout), one
    eager estimator call (embed gather, convolutions, AdaLN, the 22 blocks,
    proj_out, unpack and padding zeroing) and one fused CFG + Euler step on its
    output (fcv_cfg_euler).  Prints one line naming the sizes."""
    import torch

    from fcv_b200 import _lib
    from fcv_b200.model import B200DiT

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    torch.manual_seed(seed)
    model = B200DiT(depth=22).eval().to(device=device, dtype=torch.bfloat16)
    model.finalize_weights()
    lengths, T, _, dev = make_batch(req_lengths, seed, device, torch.bfloat16)
    layout = model.layout_from_mask(dev["mask"], chunk > 0)
    out = torch.empty(len(lengths), 80, T, dtype=torch.float32, device=device)
    model.forward_layout(layout, dev["x"], dev["mu"], dev["t"], dev["spks"], dev["cond"], out=out)
    R = len(lengths) // 2
    x = torch.randn(R, 80, T, device=device)
    x_next = torch.empty(2 * R, 80, T, dtype=torch.bfloat16, device=device)
    _lib.call("fcv_cfg_euler", x.data_ptr(), out.data_ptr(), _lib.DTYPE_F32, R, T, 0.1, 0.7, x_next.data_ptr(),
              _lib.DTYPE_BF16, torch.cuda.current_stream(device).cuda_stream)
    torch.cuda.synchronize()
    from fcv_b200 import ops

    err = ops.device_error(device)
    print(json.dumps({"ncu_case": True, "rows": sum(lengths), "sequences": len(lengths), "T": T, "chunk": chunk,
                      "device_error": err}), flush=True)
    if err:
        raise SystemExit(f"device error word {err}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="5", choices=["2", "3", "4", "5"],
                    help="BASELINE.json config (default 5, the config the metric is quoted on at 1/2/4/8 GPUs)")
    ap.add_argument("--weak", action="store_true",
                    help="N > 1: every rank runs its own copy of the batch (replicas) instead of one fixed "
                         "request set sharded across the ranks by LPT bins")
    ap.add_argument("--impl", default="b200", choices=["b200", "reference", "reference-gpu"])
    ap.add_argument("--ref-dtype", default="fp16", choices=["fp16", "bf16"],
                    help="element type of the reference GPU estimator (--impl reference-gpu)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--flow", action="store_true",
                    help="time the whole flow inference (front end + 10-step ODE) of --config 2 (offline) "
                         "or 3 (streaming) instead of one estimator call")
    ap.add_argument("--latency", action="store_true",
                    help="latency of one estimator call for one CFG pair, eager and graph-bucketed "
                         "(--config 3 for the streaming mask)")
    ap.add_argument("--stream", action="store_true",
                    help="a streaming session: 32 streams advancing 50 frames per call (full prefix recomputed)")
    ap.add_argument("--prefix-cache", action="store_true",
                    help="with --stream: reuse the cached prefix (this build only)")
    ap.add_argument("--vocoder", action="store_true",
                    help="time the HiFT vocoder over --config 2 (offline) or 3 (non-final chunks) request mels")
    ap.add_argument("--requests", type=int, default=0,
                    help="use only the first R requests of the config (small cases for profiling)")
    ap.add_argument("--gemm-compare", action="store_true",
                    help="the four block GEMM shapes of the config (M = its packed rows): this build's tcgen05 "
                         "GEMM against cuBLAS (torch F.linear with bias, bf16), CUDA events, L2 flushed")
    ap.add_argument("--bin-times", type=int, default=0,
                    help="deal the config's requests into N LPT bins (as --gpus N does) and time each bin's "
                         "estimator call alone on one GPU")
    ap.add_argument("--ncu-case", action="store_true",
                    help="no timing: one layout from a device mask, one eager estimator call and one CFG + Euler "
                         "step on the config's inputs, each kernel launched once (a target for ncu captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    req_lengths, chunk, seed = request_lengths(args.config)
    if args.requests > 0:
        req_lengths = req_lengths[:args.requests]
    # N > 1: one fixed request set sharded across the ranks by LPT bins (strong
    # scaling, the same total work at every N) unless --weak asks for replicas
    strong = not args.weak
    cfg = {"workload": CONFIG_NAMES[args.config], "requests": len(req_lengths), "sequences": 2 * len(req_lengths),
           "packed_rows": 2 * sum(req_lengths), "chunk": chunk, "seed": seed,
           "parallelism": f"dp{world} ({'LPT request bins of one fixed request set' if strong else 'replicas'}, "
                          "no collective on the data path)",
           "l2": "working set (662 MB of weights per NFE) exceeds the 126 MB L2; L2 also flushed between steps"}

    if args.vocoder:
        if args.config not in ("2", "3"):
            raise SystemExit("--vocoder runs configs 2 (offline) and 3 (streaming)")
        if rank == 0:
            if args.impl == "reference":
                vocoder_cpu_arm(args)
            else:
                vocoder_arm(args, args.impl)
        return

    if args.stream:
        if rank == 0 and args.impl != "reference":
            stream_arm(args, args.impl, args.prefix_cache and args.impl == "b200")
        return

    if args.latency:
        if rank == 0 and args.impl != "reference":
            latency_arm(args, args.impl)
        return

    if args.flow:
        if args.config not in ("2", "3"):
            raise SystemExit("--flow runs configs 2 (offline) and 3 (streaming)")
        if rank == 0 and args.impl != "reference":
            flow_arm(args, args.impl)
        return

    if args.impl == "reference":
        if rank != 0:
            return
        reference_cpu_arm(args, req_lengths, chunk, seed, cfg, strong)
        return

    if args.ncu_case:
        if rank == 0:
            ncu_case(req_lengths, chunk, seed)
        return

    if args.gemm_compare:
        if rank == 0:
            gemm_compare(args, req_lengths, seed, cfg)
        return

    if args.bin_times > 0:
        if rank == 0:
            bin_times(args, req_lengths, chunk, seed, cfg)
        return

    if args.impl == "reference-gpu":
        if rank == 0:
            reference_gpu_arm(args, req_lengths, chunk, seed, cfg, strong)
        return

    import torch
    import torch.distributed as dist

    from fcv_b200 import _lib
    from fcv_b200.model import B200DiT
    from fcv_b200.shard import bin_loads, lpt_bins

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    if strong:
        bins = lpt_bins(req_lengths, world, chunk or None)
        my_req = [req_lengths[i] for i in bins[rank]]
        if not my_req:
            raise SystemExit(f"config {args.config} has {len(req_lengths)} requests, fewer than {world} ranks")
    else:
        my_req = list(req_lengths)

    torch.manual_seed(seed)
    cpu_model = B200DiT(depth=22).eval()
    model = cpu_model.to(device=device, dtype=torch.bfloat16)
    model.finalize_weights()
    lengths, T, host, dev = make_batch(my_req, seed + 17 * rank, device, torch.bfloat16)
    streaming = chunk > 0
    N = sum(lengths)
    layout = model.layout_from_mask(dev["mask"], streaming)
    out = torch.empty(len(lengths), 80, T, dtype=torch.bfloat16, device=device)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    lib = _lib.lib()

    def eager_step():
        model.forward_layout(layout, dev["x"], dev["mu"], dev["t"], dev["spks"], dev["cond"], out=out)

    for _ in range(args.warmup):
        eager_step()
    torch.cuda.synchronize()

    # ---- timed region: the estimator call replayed from a CUDA graph (device-resident
    # inputs), CUDA events per step, L2 flushed between steps.
    stream = torch.cuda.current_stream(device)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    cats = len(_lib.CATEGORIES)
    import ctypes

    ms_arr = (ctypes.c_float * cats)()
    cnt_arr = (ctypes.c_int * cats)()
    launches0 = lib.fcv_launch_count()
    graph, _, _ = model.capture_graph(layout, dev["x"], dev["mu"], dev["t"], dev["spks"], dev["cond"], out=out,
                                      warmup=False)
    launches_per_step = lib.fcv_launch_count() - launches0
    for _ in range(2):
        graph.replay()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clocks:
        for i in range(args.steps):
            flush.zero_()
            ev[i][0].record(stream)
            graph.replay()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
    launches = launches_per_step * args.steps

    # ---- per-kernel-class device time: a second graph of the same call with the
    # library's CUDA-event tracing captured inside, replayed for the same number of
    # steps (flush between steps); the events report the last replay.
    out_t = torch.empty_like(out)
    lib.fcv_profile_enable(1)
    _lib.call("fcv_profile_collect", ctypes.addressof(ms_arr), ctypes.addressof(cnt_arr), cats)  # reset
    tgraph, _, _ = model.capture_graph(layout, dev["x"], dev["mu"], dev["t"], dev["spks"], dev["cond"],
                                       out=out_t, warmup=False)
    lib.fcv_profile_enable(0)
    traced_ms = []
    for i in range(args.steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        tgraph.replay()
        e1.record(stream)
        traced_ms.append((e0, e1))
    torch.cuda.synchronize()
    traced_step_ms = float(np.mean([a.elapsed_time(b) for a, b in traced_ms]))
    _lib.call("fcv_profile_collect", ctypes.addressof(ms_arr), ctypes.addressof(cnt_arr), cats)
    if world > 1:
        dist.barrier()
    # ---- dominant kernels timed alone: CUDA graphs of the 22 x 4 block GEMMs (same shapes,
    # epilogues and weights as the step) and of the 22 attention launches on the same layout,
    # bracketed by one event pair each, so per-launch averages carry no per-kernel event cost.
    from fcv_b200 import ops

    d = model._derived
    gA = torch.randn(N, 2048, device=device, dtype=torch.bfloat16)
    gH = torch.zeros(N, 1024, device=device)
    gO = torch.empty(N, 3072, device=device, dtype=torch.bfloat16)
    gM = torch.empty(N, 2048, device=device, dtype=torch.bfloat16)
    gate = torch.ones(len(lengths), 4096, device=device)

    def gemm_layers():
        for i in range(22):
            ops.linear(gA[:, :1024], d["qkv_w"][i], d["qkv_b"][i], epilogue=_lib.EPI_BIAS_ROPE_QKV, out=gO,
                       aux=layout.positions, rope_cos=d["rope_cos"], rope_sin=d["rope_sin"])
            ops.linear(gA[:, :1024], d["o_w"][i], d["o_b"][i], epilogue=_lib.EPI_BIAS_GATE_RES, out=gH,
                       aux=layout.document_ids, gate=gate, gate_stride=4096)
            ops.linear(gA[:, :1024], d["ff1_w"][i], d["ff1_b"][i], epilogue=_lib.EPI_BIAS_GELU, out=gM)
            ops.linear(gA, d["ff2_w"][i], d["ff2_b"][i], epilogue=_lib.EPI_BIAS_GATE_RES, out=gH,
                       aux=layout.document_ids, gate=gate, gate_stride=4096)

    def attn_layers():
        for i in range(22):
            ops.ragged_attention(gO, layout.cu_seqlens, layout.attn_tiles, layout.n_attn_tiles, layout.chunk,
                                 layout.max_len, layout.attn_sched, layout.attn_ctas)

    def time_graph(fn, reps):
        fn()  # eager warm-up (first-launch attributes)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        g.replay()
        torch.cuda.synchronize()
        tot = 0.0
        for _ in range(reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            g.replay()
            e1.record(stream)
            torch.cuda.synchronize()
            tot += e0.elapsed_time(e1)
        return tot / reps

    # the in-step gated residual reads the gate rows of the modulation GEMM; ones keep h bounded here
    reps = max(3, min(args.steps, 10))
    gemm_graph_ms = time_graph(gemm_layers, reps)
    attn_graph_ms = time_graph(attn_layers, reps)
    del gA, gH, gO, gM

    step_ms = [a.elapsed_time(b) for a, b in ev]
    total_ms = float(sum(step_ms))
    mine = torch.tensor([total_ms, float(N)], dtype=torch.float64, device=device)
    per_rank = [mine]
    if world > 1:
        per_rank = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(per_rank, mine)
    total_ms_max = max(float(v[0].item()) for v in per_rank)
    all_rows = sum(float(v[1].item()) for v in per_rank)
    shard = {"rows_per_rank": [int(v[1].item()) for v in per_rank],
             "ms_per_step_per_rank": [float(v[0].item()) / args.steps for v in per_rank],
             "requests_per_rank": [len(b) for b in bins] if strong and world > 1 else [len(my_req)] * world}
    if strong and world > 1:
        shard["bin_cost_imbalance"] = max(bin_loads(req_lengths, bins, chunk or None)) / (
            sum(bin_loads(req_lengths, bins, chunk or None)) / world)
    value = all_rows * args.steps / (total_ms_max / 1000.0)
    ms_per_step = total_ms_max / args.steps

    # ---- per-kernel-class timing from the events recorded inside the timed region
    prof = {name: {"ms_per_step": float(ms_arr[i]), "launches_per_step": int(cnt_arr[i])}
            for i, name in enumerate(_lib.CATEGORIES)}
    from fcv_b200.flops import estimator_flops, visible_pairs

    gemm_flops_step = 22 * N * (2 ** 24)
    gemm_launches = 88
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        burst, sustained = float(peaks["bf16_tflops"]), float(peaks["bf16_tflops_sustained"])
        peak_src = "of measured (MEASURED_PEAKS.json)"
    except Exception:
        burst, sustained, peak_src = 1590.0, 1400.0, "of fallback"
    gemm_tf = gemm_flops_step / (gemm_graph_ms / 1000.0) / 1e12 if gemm_graph_ms > 0 else None
    attn_flops_step = 22 * 4096 * visible_pairs(lengths, chunk or None)
    attn_tf = attn_flops_step / (attn_graph_ms / 1000.0) / 1e12 if attn_graph_ms > 0 else None
    total_flops = estimator_flops(lengths, chunk or None, 22)
    nfe_tf = total_flops / (ms_per_step / 1000.0) / 1e12
    tr = {}
    try:
        tr = json.load(open(os.path.join(ROOT, "profiles", "traffic.json"))).get(args.config, {})
    except Exception:
        pass
    # The two dominant kernel classes are timed alone (their own CUDA graphs of one
    # step's launches), so both are held against the measured BURST bf16 peak; the
    # whole NFE, timed inside the step loop, against the SUSTAINED one.
    gemm = {"kernel": "tc_gemm_pair_kernel (tcgen05 cta_group::2; QKV, out, FF1, FF2 of each block)",
            "bound": "tensor", "unit": "TFLOP/s", "achieved": gemm_tf, "peak": burst,
            "frac": gemm_tf / burst if gemm_tf else None, "peak_kind": "burst",
            "flops_per_launch": gemm_flops_step / gemm_launches, "avg_launch_ms": gemm_graph_ms / gemm_launches,
            "launches_per_step": gemm_launches, "traffic": tr.get("gemm_bytes_per_launch"),
            "timing": "22 x 4 block GEMMs of this workload in one CUDA graph, CUDA events around the graph, "
                      "L2 flushed between replays; average per launch"}
    attn = {"kernel": "attn_fa_kernel (tcgen05; ragged chunk-masked attention)", "bound": "tensor",
            "unit": "TFLOP/s", "achieved": attn_tf, "peak": burst, "frac": attn_tf / burst if attn_tf else None,
            "peak_kind": "burst", "flops_per_launch": attn_flops_step / 22, "avg_launch_ms": attn_graph_ms / 22,
            "launches_per_step": 22, "traffic": tr.get("attention_bytes_per_launch"),
            "timing": "the 22 attention launches of this workload in one CUDA graph, CUDA events around the graph, "
                      "L2 flushed between replays; average per launch"}
    dom = attn if attn_graph_ms > gemm_graph_ms else gemm
    roofline = {"bound": dom["bound"], "kernel": dom["kernel"], "achieved": dom["achieved"], "peak": dom["peak"],
                "unit": "TFLOP/s", "frac": dom["frac"], "traffic": dom["traffic"],
                "peak_source": f"bf16 burst {peak_src}", "flops_per_launch": dom["flops_per_launch"],
                "avg_launch_ms": dom["avg_launch_ms"], "timing": dom["timing"],
                "dominant": "attention" if dom is attn else "gemm",
                "share_of_step": {"gemm": gemm_graph_ms / max(ms_per_step, 1e-9),
                                  "attention": attn_graph_ms / max(ms_per_step, 1e-9)},
                "gemm": gemm, "attention": attn,
                "nfe_tflops": nfe_tf, "nfe_frac": nfe_tf / sustained, "nfe_peak": sustained,
                "nfe_peak_kind": "sustained (the NFE is timed inside the step loop)"}

    # ---- end to end through the public module API with host buffers
    e2e = None
    if True:
        model.use_cuda_graph = True  # the module's graph path (reference: enable_cuda_graph)
        # pinned host tensors straight into the module: it stages them on the device
        # asynchronously and counts the lengths from the host mask (no device round trip)
        pin = {k: v.to(torch.bfloat16).pin_memory() for k, v in host.items()}
        out_h = torch.empty(len(lengths), 80, T, dtype=torch.bfloat16).pin_memory()
        h2d = sum(v.numel() * v.element_size() for k, v in pin.items() if k != "mask")
        d2h = out_h.numel() * out_h.element_size()

        def e2e_step():
            with torch.inference_mode():
                y = model(pin["x"], pin["mask"], pin["mu"], pin["t"], pin["spks"], pin["cond"],
                          streaming=streaming)
            out_h.copy_(y, non_blocking=True)

        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        et = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(et, op=dist.ReduceOp.MAX)
        e2e = {"value": all_rows * args.steps / (float(et.item()) / 1000.0), "unit": UNIT,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "api": "B200DiT.forward(x, mask, mu, t, spks, cond, streaming) on pinned host tensors "
                      "(inputs staged to the device asynchronously, lengths counted from the host mask), "
                      "use_cuda_graph=True, output read back to pinned host memory"}

    # ---- CPU baseline (rank 0, N=1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_reference_rate(req_lengths, chunk, seed, 15.0)

    if world > 1:
        dist.barrier()
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
                "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded N(0,1) inputs, random-init weights of the 22-layer DiT)",
                "config": cfg, "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "shard": shard,
                "gpu_launches": int(launches), "gpu_launches_note": "kernels per step counted at graph capture x steps",
                "clocks": clocks.summary(),
                "request_frames_per_s": value / 2, "kernel_ms_traced": prof,
                "kernel_ms_traced_note": "per-class device time from event pairs inside a traced graph of the step; "
                                         "each pair adds ~4 us, so these overstate kernel time (see traced_step_ms)",
                "step_ms_min": min(step_ms), "step_ms_median": float(statistics.median(step_ms)),
                "traced_step_ms": traced_step_ms}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
