"""ctypes binding of ``libfcv_b200.so`` (the C ABI declared in ``include/fcv_b200.h``).

The shared library is built in-tree by :func:`fcv_b200.build.build` (nvcc,
``-gencode arch=compute_100a,code=sm_100a``).  There is no fallback: if the
library is missing or fails to load, every entry point raises.
"""

from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libfcv_b200.so")

FCV_OK = 0
FCV_EINVAL = -1
FCV_EUNSUPPORTED = -2
FCV_ECUDA = -3
FCV_EDEVICE = -4

DTYPE_F32 = 0
DTYPE_BF16 = 1

NOALLOC_MAX_B = 512  # FCV_NOALLOC_MAX_B

EPI_BIAS = 0
EPI_BIAS_GELU = 1
EPI_BIAS_ROPE_QKV = 2
EPI_BIAS_GATE_RES = 3
EPI_BIAS_F32 = 4

CATEGORIES = ("gemm_qkv", "gemm_out", "gemm_ff1", "gemm_ff2", "attention", "ln_modulate", "embed",
              "adaln", "output")

# Exported entry points (kept in sync with include/fcv_b200.h; a CPU test checks both).
EXPORTS = (
    "fcv_version",
    "fcv_last_error",
    "fcv_device_error",
    "fcv_selftest_wait_expiry",
    "fcv_mask_lengths",
    "fcv_pack_layout",
    "fcv_unpack_output",
    "fcv_ln_modulate",
    "fcv_gate_res_ln_modulate",
    "fcv_gemm",
    "fcv_attention",
    "fcv_attn_tiles",
    "fcv_attn_ctas",
    "fcv_attn_schedule",
    "fcv_time_embed",
    "fcv_time_embed_noalloc",
    "fcv_cfg_euler",
    "fcv_profile_enable",
    "fcv_profile_collect",
    "fcv_launch_count",
    "fcv_dit_workspace_bytes",
    "fcv_dit_forward",
    "fcv_offset_positions",
    "fcv_dit_modulations",
    "fcv_flow_workspace_bytes",
    "fcv_flow_frontend",
    "fcv_speaker_projection",
    "fcv_prompt_rows",
    "fcv_pack_rows",
    "fcv_hift_workspace_bytes",
    "fcv_hift_forward",
)


class FcvError(RuntimeError):
    """A C-ABI call returned a non-zero status."""

    def __init__(self, what: str, status: int, message: str):
        super().__init__(f"{what} failed with status {status}: {message}")
        self.status = status


class DitWeights(ctypes.Structure):
    _fields_ = [
        ("depth", ctypes.c_int),
        ("dtype", ctypes.c_int),
        ("time_w1", ctypes.c_void_p),
        ("time_b1", ctypes.c_void_p),
        ("time_w2", ctypes.c_void_p),
        ("time_b2", ctypes.c_void_p),
        ("ada_w", ctypes.c_void_p),
        ("ada_b", ctypes.c_void_p),
        ("in_w", ctypes.c_void_p),
        ("in_b", ctypes.c_void_p),
        ("conv1_w", ctypes.c_void_p),
        ("conv1_b", ctypes.c_void_p),
        ("conv2_w", ctypes.c_void_p),
        ("conv2_b", ctypes.c_void_p),
        ("qkv_w", ctypes.c_void_p),
        ("qkv_b", ctypes.c_void_p),
        ("o_w", ctypes.c_void_p),
        ("o_b", ctypes.c_void_p),
        ("ff1_w", ctypes.c_void_p),
        ("ff1_b", ctypes.c_void_p),
        ("ff2_w", ctypes.c_void_p),
        ("ff2_b", ctypes.c_void_p),
        ("out_w", ctypes.c_void_p),
        ("out_b", ctypes.c_void_p),
        ("rope_cos", ctypes.c_void_p),
        ("rope_sin", ctypes.c_void_p),
        ("rope_max_len", ctypes.c_int),
    ]


class DitBatch(ctypes.Structure):
    _fields_ = [
        ("B", ctypes.c_int),
        ("T", ctypes.c_int),
        ("N", ctypes.c_int),
        ("max_len", ctypes.c_int),
        ("chunk", ctypes.c_int),
        ("x", ctypes.c_void_p),
        ("mu", ctypes.c_void_p),
        ("cond", ctypes.c_void_p),
        ("spks", ctypes.c_void_p),
        ("t", ctypes.c_void_p),
        ("cu_seqlens", ctypes.c_void_p),
        ("doc_ids", ctypes.c_void_p),
        ("positions", ctypes.c_void_p),
        ("gap_rows", ctypes.c_void_p),
        ("attn_tiles", ctypes.c_void_p),
        ("n_attn_tiles", ctypes.c_int),
        ("out", ctypes.c_void_p),
        ("out_f32", ctypes.c_int),
        ("packed", ctypes.c_int),
        ("n_attn_tiles_dev", ctypes.c_void_p),
        ("attn_sched", ctypes.c_void_p),
        ("attn_sched_ctas", ctypes.c_int),
        ("doc_pos0", ctypes.c_void_p),
        ("doc_kv_base", ctypes.c_void_p),
        ("kv_cache", ctypes.c_void_p),
        ("kv_layer_rows", ctypes.c_long),
        ("conv_ctx", ctypes.c_void_p),
        ("conv_ctx_out", ctypes.c_void_p),
        ("ctx_row0", ctypes.c_void_p),
        ("shared_mods", ctypes.c_void_p),
    ]


class FlowWeights(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int),
        ("vocab", ctypes.c_int),
        ("embed", ctypes.c_void_p),
        ("conv1_w", ctypes.c_void_p),
        ("conv1_b", ctypes.c_void_p),
        ("conv2_w", ctypes.c_void_p),
        ("conv2_b", ctypes.c_void_p),
    ]


HIFT_CONVS = 80
HIFT_LAYOUT_ARRAYS = 9


class HiftWeights(ctypes.Structure):
    _fields_ = [
        ("conv_w", ctypes.c_void_p * HIFT_CONVS),
        ("conv_b", ctypes.c_void_p * HIFT_CONVS),
        ("snake_alpha", ctypes.c_void_p * HIFT_CONVS),
        ("snake_inv", ctypes.c_void_p * HIFT_CONVS),
        ("snake2_alpha", ctypes.c_void_p * HIFT_CONVS),
        ("snake2_inv", ctypes.c_void_p * HIFT_CONVS),
        ("tc_w_hi", ctypes.c_void_p * HIFT_CONVS),
        ("tc_w_lo", ctypes.c_void_p * HIFT_CONVS),
        ("f0_w", ctypes.c_void_p * 5),
        ("f0_b", ctypes.c_void_p * 5),
        ("f0_cls_w", ctypes.c_void_p),
        ("f0_cls_b", ctypes.c_double),
        ("source_w", ctypes.c_void_p),
        ("source_b", ctypes.c_float),
        ("noise", ctypes.c_void_p),
        ("noise_rows", ctypes.c_longlong),
    ]


class HiftBatch(ctypes.Structure):
    _fields_ = [
        ("n_docs", ctypes.c_int),
        ("mel", ctypes.c_void_p),
        ("layout", ctypes.c_void_p),
        ("rows", ctypes.c_int * HIFT_LAYOUT_ARRAYS),
        ("max_src", ctypes.c_int),
        ("audio", ctypes.c_void_p),
        ("source", ctypes.c_void_p),
        ("f0", ctypes.c_void_p),
    ]


_lock = threading.Lock()
_lib = None

_vp = ctypes.c_void_p
_i = ctypes.c_int
_l = ctypes.c_long

_SIGNATURES = {
    "fcv_version": (_i, []),
    "fcv_last_error": (ctypes.c_char_p, []),
    "fcv_device_error": (_i, [ctypes.POINTER(ctypes.c_int), _vp]),
    "fcv_selftest_wait_expiry": (_i, [ctypes.c_ulonglong, _vp, _vp]),
    "fcv_mask_lengths": (_i, [_vp, _i, _i, _i, _vp, _vp]),
    "fcv_pack_layout": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp]),
    "fcv_unpack_output": (_i, [_vp, _i, _vp, _i, _i, _i, _vp, _vp]),
    "fcv_ln_modulate": (_i, [_vp, _i, _vp, _vp, _vp, _l, _i, _vp, _i, _vp]),
    "fcv_gate_res_ln_modulate": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _l, _i, _vp, _vp, _i, _vp]),
    "fcv_gemm": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _l, _vp, _vp, _vp]),
    "fcv_attention": (_i, [_vp, _i, _vp, _i, _i, _i, _i, _vp, _i, _vp, _i, _vp, _vp]),
    "fcv_attn_tiles": (_i, [_vp, _i, _i, _vp, _i]),
    "fcv_attn_ctas": (_i, [_i]),
    "fcv_attn_schedule": (_i, [_vp, _i, _i, _vp, _i, _i, _vp, _i]),
    "fcv_time_embed": (_i, [ctypes.POINTER(DitWeights), _vp, _i, _vp, _vp, _vp]),
    "fcv_time_embed_noalloc": (_i, [ctypes.POINTER(DitWeights), _vp, _i, _vp, _vp, _vp]),
    "fcv_cfg_euler": (_i, [_vp, _vp, _i, _i, _i, ctypes.c_float, ctypes.c_float, _vp, _i, _vp]),
    "fcv_profile_enable": (_i, [_i]),
    "fcv_profile_collect": (_i, [_vp, _vp, _i]),
    "fcv_launch_count": (ctypes.c_long, []),
    "fcv_dit_workspace_bytes": (ctypes.c_size_t, [_i, _i, _i, _i]),
    "fcv_dit_forward": (_i, [ctypes.POINTER(DitWeights), ctypes.POINTER(DitBatch), _vp, ctypes.c_size_t, _vp]),
    "fcv_offset_positions": (_i, [_vp, _vp, _vp, _i, _vp]),
    "fcv_dit_modulations": (_i, [ctypes.POINTER(DitWeights), _vp, _vp, _vp, ctypes.c_size_t, _vp]),
    "fcv_flow_workspace_bytes": (ctypes.c_size_t, [_i, _i]),
    "fcv_flow_frontend": (_i, [ctypes.POINTER(FlowWeights), _vp, _vp, _vp, _i, _i, _i, _i, _vp, ctypes.c_size_t,
                               _vp, _vp]),
    "fcv_speaker_projection": (_i, [_vp, _i, _i, _i, _vp, _vp, _i, _vp, _i, _vp]),
    "fcv_prompt_rows": (_i, [_vp, _vp, _vp, _i, _i, _vp, _i, _vp]),
    "fcv_pack_rows": (_i, [_vp, _i, _l, _i, _vp, _i, _i, _vp, _i, _vp]),
    "fcv_hift_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(ctypes.c_int)]),
    "fcv_hift_forward": (_i, [ctypes.POINTER(HiftWeights), ctypes.POINTER(HiftBatch), _vp, ctypes.c_size_t, _vp]),
}


def lib() -> ctypes.CDLL:
    """Load the in-tree shared library (raises if it is missing)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build the CUDA extension first "
                    "(python -c 'import __graft_entry__; __graft_entry__.build()')"
                )
            handle = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(status: int, what: str) -> int:
    if status < 0:
        msg = lib().fcv_last_error()
        raise FcvError(what, status, msg.decode() if msg else "")
    return status


def call(name: str, *args) -> int:
    """Invoke entry point ``name`` and raise FcvError on a negative status."""
    return check(getattr(lib(), name)(*args), name)
