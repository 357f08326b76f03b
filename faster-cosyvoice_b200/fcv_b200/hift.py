"""B200 HiFT vocoder: ``CausalHiFTGenerator.inference`` over packed requests.

Mirror of the reference's vocoder entry point
(``cosyvoice/hifigan/generator.py:728-740``, built by ``builders.py:38-50``):
``inference(speech_feat, finalize)`` returns ``(speech, s)`` like the reference,
and :meth:`B200HiFT.inference_batched` vocodes many requests in one native call
(``fcv_hift_forward``) instead of one module call per request
(``token2wav.py:130-131, 194-195``).  Weights come from the reference's state
dict (weight norm folded with ``torch._weight_norm``, the op its
parametrization evaluates) and its fixed source-noise table.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Sequence

import torch

from ._lib import HIFT_CONVS, HIFT_LAYOUT_ARRAYS, HiftBatch, HiftWeights, call, lib

MEL = 80
SAMPLES_PER_FRAME = 480
F0_LOOK_RIGHT = 3   # f0_predictor condnet[0] causal_padding (convolution.py:172)
LOOK_RIGHT = 4      # conv_pre_look_right (builders.py:48)
CHANNELS = (256, 128, 64)


def conv_names() -> list[str]:
    """Module path of convolution i of ``fcv_hift_weights`` (index order of the C ABI)."""
    names = ["conv_pre"] + [f"ups.{i}" for i in range(3)] + [f"source_downs.{i}" for i in range(3)]
    for prefix, count in (("source_resblocks", 3), ("resblocks", 9)):
        for n in range(count):
            for s in range(3):
                names += [f"{prefix}.{n}.convs1.{s}", f"{prefix}.{n}.convs2.{s}"]
    names.append("conv_post")
    assert len(names) == HIFT_CONVS
    return names


def _weight(sd: dict, name: str, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Effective weight of a (possibly weight-normed) convolution, computed in
    ``dtype`` like the parametrization of a module held in that dtype (the f0
    predictor runs in float64, ``generator.py:731``)."""
    g = sd.get(f"{name}.parametrizations.weight.original0", sd.get(f"{name}.weight_g"))
    v = sd.get(f"{name}.parametrizations.weight.original1", sd.get(f"{name}.weight_v"))
    if g is not None and v is not None:
        return torch._weight_norm(v.to(dtype).cpu(), g.to(dtype).cpu(), 0)
    return sd[f"{name}.weight"].to(dtype).cpu()


def _round(v: int, m: int) -> int:
    return (v + m - 1) // m * m


@dataclass
class HiftLayout:
    """Row layout of one batch: per-document row counts of every level and the
    device int32 block of their cu arrays (``fcv_hift_batch.layout``)."""
    n_mel: tuple
    finalize: tuple
    counts: list          # 9 lists of per-document rows
    rows: list            # 9 totals
    block: torch.Tensor   # device int32, 9 * (n_docs + 1)
    max_src: int


class B200HiFT:
    """HiFT vocoder on the B200 (``CausalHiFTGenerator`` drop-in for inference)."""

    def __init__(self, state_dict: dict, noise: torch.Tensor, device: str | torch.device = "cuda",
                 tensor_cores: bool = True):
        """``tensor_cores``: run the 72 residual-block convolutions on tcgen05 with
        split-tf32 operands (float32 accuracy), else on the SIMT float32 kernel."""
        self.device = torch.device(device)
        self.tensor_cores = tensor_cores
        sd = {k: v.detach() for k, v in state_dict.items()}
        keep = []
        w = HiftWeights()
        f32 = dict(dtype=torch.float32, device=self.device)
        for i, name in enumerate(conv_names()):
            wt = _weight(sd, name)                                   # (C_out, C_in, k)
            co, ci, k = wt.shape
            pad = torch.zeros(k, _round(ci, 16), _round(co, 64))
            pad[:, :ci, :co] = wt.permute(2, 1, 0)
            bias = torch.zeros(_round(co, 64))
            bias[:co] = sd[f"{name}.bias"].float().cpu()
            keep += [pad.to(**f32).contiguous(), bias.to(**f32)]
            w.conv_w[i], w.conv_b[i] = keep[-2].data_ptr(), keep[-1].data_ptr()
            if tensor_cores and "resblocks." in name:
                kmaj = wt.permute(2, 0, 1).contiguous()                # [k][C_out][C_in]
                hi = ((kmaj.view(torch.int32) + 4096) & -8192).view(torch.float32)  # nearest tf32 head
                keep += [hi.to(**f32), (kmaj - hi).to(**f32)]
                w.tc_w_hi[i], w.tc_w_lo[i] = keep[-2].data_ptr(), keep[-1].data_ptr()
            if ".convs1." in name:
                block, s = name.split(".convs1.")
                for fa, fi, act in (("snake_alpha", "snake_inv", "activations1"),
                                    ("snake2_alpha", "snake2_inv", "activations2")):
                    a = sd[f"{block}.{act}.{s}.alpha"].float().cpu()
                    inv = 1.0 / (a + 1e-9)                             # activation.py:82, float32
                    keep += [a.to(**f32), inv.to(**f32)]
                    getattr(w, fa)[i], getattr(w, fi)[i] = keep[-2].data_ptr(), keep[-1].data_ptr()
        f64 = dict(dtype=torch.float64, device=self.device)
        for j, idx in enumerate((0, 2, 4, 6, 8)):
            name = f"f0_predictor.condnet.{idx}"
            wt = _weight(sd, name, torch.float64)
            keep += [wt.permute(2, 1, 0).contiguous().to(**f64), sd[f"{name}.bias"].double().to(**f64)]
            w.f0_w[j], w.f0_b[j] = keep[-2].data_ptr(), keep[-1].data_ptr()
        keep.append(sd["f0_predictor.classifier.weight"].double().reshape(-1).to(**f64))
        w.f0_cls_w = keep[-1].data_ptr()
        w.f0_cls_b = float(sd["f0_predictor.classifier.bias"].double().reshape(-1)[0])
        keep.append(sd["m_source.l_linear.weight"].float().reshape(-1).to(**f32))
        w.source_w = keep[-1].data_ptr()
        w.source_b = float(sd["m_source.l_linear.bias"].float().reshape(-1)[0])
        nz = noise.detach().reshape(-1, 9).to(**f32).contiguous()
        keep.append(nz)
        w.noise, w.noise_rows = nz.data_ptr(), nz.shape[0]
        self._keep, self._w = keep, w
        self._ws: torch.Tensor | None = None
        self._layouts: dict = {}

    @classmethod
    def from_reference(cls, hift, device: str | torch.device | None = None) -> "B200HiFT":
        """Build from a reference ``CausalHiFTGenerator`` (its state dict and its
        fixed noise table ``m_source.l_sin_gen.sine_waves``, ``generator.py:187``)."""
        dev = device if device is not None else next(hift.parameters()).device
        return cls(hift.state_dict(), hift.m_source.l_sin_gen.sine_waves, dev)

    # ------------------------------------------------------------------ layout
    def layout(self, n_mel: Sequence[int], finalize: Sequence[bool]) -> HiftLayout:
        key = (tuple(int(v) for v in n_mel), tuple(bool(f) for f in finalize))
        lay = self._layouts.get(key)
        if lay is not None:
            return lay
        counts = [[] for _ in range(HIFT_LAYOUT_ARRAYS)]
        for L, fin in zip(*key):
            if L < (1 if fin else F0_LOOK_RIGHT + LOOK_RIGHT + 1):
                raise ValueError(f"a {'final' if fin else 'non-final'} HiFT call needs more mel frames (got {L})")
            f0 = L if fin else L - F0_LOOK_RIGHT
            x = f0 if fin else f0 - LOOK_RIGHT
            audio = SAMPLES_PER_FRAME * x - (0 if fin else SAMPLES_PER_FRAME)
            for a, v in enumerate((L, f0, x, SAMPLES_PER_FRAME * f0, 120 * f0 + 1, 8 * x, 40 * x, 120 * x + 1, audio)):
                counts[a].append(v)
        cu = []
        rows = []
        for c in counts:
            t = torch.zeros(len(c) + 1, dtype=torch.int64)
            t[1:] = torch.cumsum(torch.tensor(c, dtype=torch.int64), 0)
            if int(t[-1]) >= 2 ** 31:
                raise ValueError("HiFT batch too large for int32 row offsets")
            cu.append(t)
            rows.append(int(t[-1]))
        # the nine cu arrays, then [0, total mel rows]: the row offsets of the one
        # pack call that transposes all requests' (80, sum L) mels into rows
        block = torch.cat(cu + [torch.tensor([0, rows[0]], dtype=torch.int64)]).to(torch.int32).to(self.device)
        lay = HiftLayout(key[0], key[1], counts, rows, block, max(counts[3], default=0))
        if len(self._layouts) >= 64:
            self._layouts.pop(next(iter(self._layouts)))
        self._layouts[key] = lay
        return lay

    def _workspace(self, rows: list) -> torch.Tensor:
        need = int(lib().fcv_hift_workspace_bytes((ctypes.c_int * HIFT_LAYOUT_ARRAYS)(*rows)))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(max(need, 256), dtype=torch.uint8, device=self.device)
        return self._ws

    # ------------------------------------------------------------------ forward
    def forward_packed(self, mel_rows: torch.Tensor, lay: HiftLayout, want_source: bool = False,
                       f0_out: torch.Tensor | None = None):
        """Vocode packed mel rows (sum of n_mel, 80) float32 on the device.
        Returns (packed speech, packed excitation or None); ``f0_out`` (float32,
        ``lay.rows[1]``) receives the predicted f0 of every frame."""
        audio = torch.empty(max(lay.rows[8], 1), dtype=torch.float32, device=self.device)
        src = torch.empty(max(lay.rows[3], 1), dtype=torch.float32, device=self.device) if want_source else None
        b = HiftBatch()
        b.n_docs = len(lay.n_mel)
        b.mel = mel_rows.data_ptr()
        b.layout = lay.block.data_ptr()
        for i, v in enumerate(lay.rows):
            b.rows[i] = v
        b.max_src = lay.max_src
        b.audio = audio.data_ptr()
        b.source = src.data_ptr() if src is not None else None
        if f0_out is not None:
            if f0_out.dtype != torch.float32 or f0_out.numel() < lay.rows[1] or not f0_out.is_contiguous():
                raise ValueError("f0_out must be a contiguous float32 tensor of the batch's f0 frames")
            b.f0 = f0_out.data_ptr()
        ws = self._workspace(lay.rows)
        call("fcv_hift_forward", ctypes.byref(self._w), ctypes.byref(b), ws.data_ptr(), ws.numel(),
             torch.cuda.current_stream(self.device).cuda_stream)
        return audio[:lay.rows[8]], (src[:lay.rows[3]] if src is not None else None)

    def _pack(self, mels: Sequence[torch.Tensor], lay: HiftLayout) -> torch.Tensor:
        """(80, L_i) request mels -> packed (sum L_i, 80) rows: the mels side by side
        as one (80, sum L_i) matrix, transposed by a single ``fcv_pack_rows`` call
        whose row offsets [0, sum L_i] sit at the end of the layout block."""
        total = lay.rows[0]
        rows = torch.empty(max(total, 1), MEL, dtype=torch.float32, device=self.device)
        if total == 0:
            return rows
        flat = [m.reshape(MEL, -1).to(device=self.device, dtype=torch.float32) for m in mels]
        wide = flat[0].contiguous() if len(flat) == 1 else torch.cat(flat, 1)
        cu = lay.block[HIFT_LAYOUT_ARRAYS * (len(lay.n_mel) + 1):]
        call("fcv_pack_rows", wide.data_ptr(), 0, 0, total, cu.data_ptr(), 1, total, rows.data_ptr(), 0,
             torch.cuda.current_stream(self.device).cuda_stream)
        return rows

    def inference_batched(self, mels: Sequence[torch.Tensor], finalize: bool | Sequence[bool] = True,
                          want_source: bool = False):
        """Vocode many requests in one call.  ``mels``: (1, 80, L_i) or (80, L_i)
        tensors.  Returns a list of (1, n_i) speech tensors (and of (1, 1, m_i)
        excitations with ``want_source``), each what ``inference`` would return."""
        fin = [bool(finalize)] * len(mels) if isinstance(finalize, bool) else [bool(f) for f in finalize]
        if len(fin) != len(mels):
            raise ValueError("one finalize flag per request")
        n_mel = [int(m.shape[-1]) for m in mels]
        with torch.cuda.device(self.device):
            lay = self.layout(n_mel, fin)
            audio, src = self.forward_packed(self._pack(mels, lay), lay, want_source)
        speech = [a.unsqueeze(0) for a in torch.split(audio, lay.counts[8])]
        if not want_source:
            return speech
        return speech, [s.reshape(1, 1, -1) for s in torch.split(src, lay.counts[3])]

    @torch.inference_mode()
    def inference(self, speech_feat: torch.Tensor, finalize: bool = True):
        """``CausalHiFTGenerator.inference`` (``generator.py:728-740``) for a
        (1, 80, L) mel: returns (speech (1, n), s (1, 1, m))."""
        if speech_feat.dim() != 3 or speech_feat.shape[0] != 1 or speech_feat.shape[1] != MEL:
            raise ValueError("speech_feat must be (1, 80, L)")
        speech, src = self.inference_batched([speech_feat], finalize, want_source=True)
        return speech[0], src[0]

    def install(self, token2wav) -> None:
        """Serve ``token2wav.hift.inference`` from this vocoder (the calls of
        ``token2wav.py:130-131`` and ``:194-195``)."""
        token2wav.hift.inference = self.inference
