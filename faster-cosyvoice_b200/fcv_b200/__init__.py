"""fcv_b200 -- B200-native packed DiT estimator for CosyVoice3 token2wav.

Drop-in replacement for the reference's ``FlashInferDiT`` estimator path
(``faster_cosyvoice/token2wav/flashinfer_dit.py``): same module interface and
state dict, all GPU work in hand-written sm_100a CUDA behind a C ABI
(``include/fcv_b200.h``, ``libfcv_b200.so``).
"""

from .model import B200DiT, PackedLayout, apply_b200  # noqa: F401
from .flow import solve_euler_batched  # noqa: F401

__all__ = ["B200DiT", "PackedLayout", "apply_b200", "solve_euler_batched"]
