"""CPU oracle for the HiFT vocoder decode -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of ``CausalHiFTGenerator.inference``
(``faster_cosyvoice/token2wav/cosyvoice/hifigan/generator.py:728-740``) with the
structure that ``builders.py:38-50`` builds: the causal f0 predictor
(``f0_predictor.py:60-103``, float64 like the reference), the neural-source
excitation (``SineGen2`` ``generator.py:214-262`` in causal mode,
``SourceModuleHnNSF.forward`` ``:321-336``), the STFT of the source
(``:413-419``), the decode network (``:678-720``: causal pre-conv, three
nearest-upsample convolutions, source down-sampling, Snake residual blocks
``:116-121``) and the inverse STFT (``:421-427``).  Only ``tests/`` and
``bench.py``'s CPU arm may import it, and only as the checker.

Pinning: ``tests/test_oracle_golden.py`` checks it against
``tests/golden/hift_case.npz``, which ``tests/golden/make_golden.py hift``
records from the reference's own ``CausalHiFTGenerator`` (offline
``finalize=True`` and streaming ``finalize=False`` calls).

Numerics: float32 (numpy IEEE arithmetic, BLAS matmuls), float64 for the f0
predictor.  Rows are time-major: a signal of L steps and C channels is (L, C).
Weights are a dict keyed like the reference's state dict with weight norm
already folded (``<name>.weight`` = g * v / ||v||).
"""

from __future__ import annotations

import numpy as np

F32 = np.float32
SAMPLE_RATE = 24000
UPSAMPLE_RATES = (8, 5, 3)
UPSAMPLE_KERNELS = (16, 11, 7)
HOP = 4
N_FFT = 16
UP_TOTAL = 8 * 5 * 3 * HOP           # 480 samples per mel frame
SOURCE_DOWN = ((30, 15), (6, 3), (1, 1))   # (kernel, stride) per level
SOURCE_RB_KERNELS = (7, 7, 11)
RB_KERNELS = (3, 7, 11)
DILATIONS = (1, 3, 5)
CHANNELS = (256, 128, 64)
LOOK_RIGHT = 4      # conv_pre_look_right (builders.py:48)
F0_LOOK_RIGHT = 3   # CausalConv1d(k=4, 'right').causal_padding (convolution.py:172)


def conv(x: np.ndarray, w: np.ndarray, b: np.ndarray, *, dil: int = 1, stride: int = 1,
         pad_left: int = 0, pad_right: int = 0) -> np.ndarray:
    """Conv1d on time-major rows with explicit zero padding
    (``convolution.py:176-192, 219-226``); ``w`` is (C_out, C_in, k)."""
    dt = x.dtype
    k = w.shape[2]
    xp = np.concatenate([np.zeros((pad_left, x.shape[1]), dt), x, np.zeros((pad_right, x.shape[1]), dt)])
    n_out = (xp.shape[0] - dil * (k - 1) - 1) // stride + 1
    out = np.zeros((n_out, w.shape[0]), dt)
    for j in range(k):
        taps = xp[j * dil: j * dil + stride * (n_out - 1) + 1: stride]
        out += taps @ w[:, :, j].T.astype(dt)
    return out + b.astype(dt)


def snake(x: np.ndarray, alpha: np.ndarray) -> np.ndarray:
    """``Snake.forward`` (``activation.py:73-84``): x + 1/(a + 1e-9) * sin(a x)^2."""
    a = alpha.astype(F32)
    inv = (F32(1.0) / (a + F32(1e-9))).astype(F32)
    s = np.sin(x * a).astype(F32)
    return (x + inv * (s * s)).astype(F32)


def leaky(x: np.ndarray, slope: float) -> np.ndarray:
    return np.where(x >= 0, x, x * F32(slope)).astype(F32)


def f0_predict(mel: np.ndarray, W: dict, finalize: bool) -> np.ndarray:
    """``CausalConvRNNF0Predictor.forward`` (``f0_predictor.py:92-103``) in
    float64 (``generator.py:731-732``) on one (L, 80) mel; returns float32 f0
    of L frames (``finalize``) or L - 3 (the last 3 frames are look-ahead)."""
    x = mel.astype(np.float64)
    p = "f0_predictor.condnet"
    x = conv(x, W[f"{p}.0.weight"].astype(np.float64), W[f"{p}.0.bias"].astype(np.float64),
             pad_right=F0_LOOK_RIGHT if finalize else 0)
    x = np.where(x > 0, x, np.expm1(x))
    for i in (2, 4, 6, 8):
        x = conv(x, W[f"{p}.{i}.weight"].astype(np.float64), W[f"{p}.{i}.bias"].astype(np.float64), pad_left=2)
        x = np.where(x > 0, x, np.expm1(x))
    y = x @ W["f0_predictor.classifier.weight"].astype(np.float64).T + W["f0_predictor.classifier.bias"].astype(np.float64)
    return np.abs(y[:, 0]).astype(F32)


def source(f0: np.ndarray, W: dict, noise: np.ndarray) -> np.ndarray:
    """Excitation ``s`` (480 samples per f0 frame) of ``SourceModuleHnNSF``
    with ``SineGen2`` in causal inference mode (``generator.py:195-262,
    321-336``).

    * The per-sample radian step is constant within a frame (nearest
      upsampling, ``:718``); the linear down-sampling by 480 reads samples
      480 f + 239 and 480 f + 240 with weights 1/2 each, so it returns exactly
      the frame's value and the random initial phase added to sample 0
      (``:208``) never reaches the output.
    * The phase is the float64-accumulated prefix sum of the frame steps
      (``torch.cumsum`` on the CPU accumulates in double), times 2 pi, times
      480, held for the frame's 480 samples (``nearest`` in causal mode).
    * ``noise`` is the module's fixed (samples, 9) uniform table
      (``self.sine_waves``, ``:187``), read from sample 0 of every call."""
    F = f0.shape[0]
    h = np.arange(1, 10, dtype=F32)
    fn = (f0[:, None] * h[None, :]).astype(F32)
    rad = np.remainder((fn / F32(SAMPLE_RATE)).astype(F32), F32(1.0)).astype(F32)
    cum = np.cumsum(rad.astype(np.float64), axis=0).astype(F32)
    phase = ((cum * F32(2.0)).astype(F32) * F32(np.pi)).astype(F32)
    phase = (phase * F32(UP_TOTAL)).astype(F32)
    sines = (np.sin(phase).astype(F32) * F32(0.1)).astype(F32)
    uv = (f0 > F32(10.0)).astype(F32)
    amp = ((uv * F32(0.003)).astype(F32) + (((F32(1.0) - uv) * F32(0.1)).astype(F32) / F32(3.0))).astype(F32)
    frame = np.arange(F * UP_TOTAL) // UP_TOTAL
    sw = (sines[frame] * uv[frame, None]).astype(F32) + (amp[frame, None] * noise[:F * UP_TOTAL]).astype(F32)
    y = sw.astype(F32) @ W["m_source.l_linear.weight"].astype(F32).T + W["m_source.l_linear.bias"].astype(F32)
    return np.tanh(y[:, 0]).astype(F32)


def hann() -> np.ndarray:
    """Periodic Hann window of 16 points (``scipy.signal.get_window('hann', 16,
    fftbins=True)``, ``generator.py:411``) in float32."""
    n = np.arange(N_FFT, dtype=np.float64)
    return (0.5 - 0.5 * np.cos(2 * np.pi * n / N_FFT)).astype(F32)


def stft(s: np.ndarray) -> np.ndarray:
    """``torch.stft(s, 16, 4, 16, hann, center=True, reflect)`` (``generator.py:413-419``)
    as (frames, 18) rows: 9 real parts then 9 imaginary parts."""
    w = hann()
    sp = np.pad(s, (N_FFT // 2, N_FFT // 2), mode="reflect")
    n_frames = s.shape[0] // HOP + 1
    idx = np.arange(n_frames)[:, None] * HOP + np.arange(N_FFT)[None, :]
    spec = np.fft.rfft(sp[idx].astype(np.float64) * w.astype(np.float64), axis=1)
    return np.concatenate([spec.real, spec.imag], axis=1).astype(F32)


def istft(post: np.ndarray) -> np.ndarray:
    """Magnitude/phase head and ``torch.istft`` (``generator.py:421-427, 713-716``):
    mag = clip(exp(x[:9]), 100), phase = sin(x[9:]), centred inverse STFT with
    the window-square envelope; returns 4 * (frames - 1) samples."""
    mag = np.minimum(np.exp(post[:, :9]).astype(F32), F32(100.0))
    ph = np.sin(post[:, 9:]).astype(F32)
    spec = (mag * np.cos(ph)).astype(np.float64) + 1j * (mag * np.sin(ph)).astype(np.float64)
    frames = np.fft.irfft(spec, n=N_FFT, axis=1)
    w = hann().astype(np.float64)
    n_frames = post.shape[0]
    total = N_FFT + HOP * (n_frames - 1)
    y = np.zeros(total)
    env = np.zeros(total)
    for m in range(n_frames):
        y[m * HOP: m * HOP + N_FFT] += frames[m] * w
        env[m * HOP: m * HOP + N_FFT] += w * w
    half = N_FFT // 2
    return (y[half: total - half] / env[half: total - half]).astype(F32)


def resblock(x: np.ndarray, W: dict, prefix: str, k: int) -> np.ndarray:
    """Causal ``ResBlock.forward`` (``generator.py:116-121``)."""
    for s, d in enumerate(DILATIONS):
        xt = snake(x, W[f"{prefix}.activations1.{s}.alpha"])
        xt = conv(xt, W[f"{prefix}.convs1.{s}.weight"], W[f"{prefix}.convs1.{s}.bias"], dil=d, pad_left=(k - 1) * d)
        xt = snake(xt, W[f"{prefix}.activations2.{s}.alpha"])
        xt = conv(xt, W[f"{prefix}.convs2.{s}.weight"], W[f"{prefix}.convs2.{s}.bias"], pad_left=k - 1)
        x = (xt + x).astype(F32)
    return x


def decode(mel: np.ndarray, s: np.ndarray, W: dict, finalize: bool) -> np.ndarray:
    """``CausalHiFTGenerator.decode`` (``generator.py:678-720``) on one
    document: ``mel`` (L, 80), ``s`` the excitation of L frames."""
    spec = stft(s)
    if finalize:
        x = conv(mel, W["conv_pre.weight"], W["conv_pre.bias"], pad_right=LOOK_RIGHT)
    else:
        x = conv(mel, W["conv_pre.weight"], W["conv_pre.bias"])
        spec = spec[:spec.shape[0] - (UP_TOTAL // HOP) * LOOK_RIGHT]
    for i in range(3):
        x = leaky(x, 0.1)
        u, k = UPSAMPLE_RATES[i], UPSAMPLE_KERNELS[i]
        x = conv(np.repeat(x, u, axis=0), W[f"ups.{i}.weight"], W[f"ups.{i}.bias"], pad_left=k - 1)
        if i == 2:
            x = np.concatenate([x[1:2], x])    # ReflectionPad1d((1, 0))
        kd, sd = SOURCE_DOWN[i]
        si = conv(spec, W[f"source_downs.{i}.weight"], W[f"source_downs.{i}.bias"], stride=sd,
                  pad_left=sd - 1 if sd > 1 else 0)
        si = resblock(si, W, f"source_resblocks.{i}", SOURCE_RB_KERNELS[i])
        x = (x + si).astype(F32)
        xs = None
        for j in range(3):
            y = resblock(x, W, f"resblocks.{i * 3 + j}", RB_KERNELS[j])
            xs = y if xs is None else (xs + y).astype(F32)
        x = (xs / F32(3.0)).astype(F32)
    x = leaky(x, 0.01)
    post = conv(x, W["conv_post.weight"], W["conv_post.bias"], pad_left=6)
    y = istft(post)
    if not finalize:
        y = y[:y.shape[0] - UP_TOTAL]
    return np.clip(y, -0.99, 0.99).astype(F32)


def inference(mel: np.ndarray, W: dict, noise: np.ndarray, finalize: bool = True):
    """``CausalHiFTGenerator.inference`` (``generator.py:728-740``) on one
    (L, 80) mel.  Returns (speech, s, f0): speech has 480 L samples
    (``finalize``) or 480 (L - 8); s is the excitation (480 per f0 frame)."""
    f0 = f0_predict(mel, W, finalize)
    s = source(f0, W, noise)
    x = mel if finalize else mel[:mel.shape[0] - F0_LOOK_RIGHT]
    return decode(x, s, W, finalize), s, f0


def out_samples(n_mel: int, finalize: bool) -> int:
    """Speech samples of one call: 480 L offline, 480 (L - 8) for a non-final chunk."""
    return UP_TOTAL * n_mel if finalize else max(0, UP_TOTAL * (n_mel - F0_LOOK_RIGHT - LOOK_RIGHT - 1))
