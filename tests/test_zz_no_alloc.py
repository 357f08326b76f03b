"""The allocation-free time-embedding entry point (fcv_time_embed_noalloc).

Some callers cannot allocate device memory: a host that binds only the C ABI
and has no device allocator, code running during CUDA-graph stream capture
(where cudaMalloc is not allowed), or a real-time audio thread that must not
enter the allocator.  For them the library keeps the scratch rows of the time
embedding in its own static device array; the caller passes only inputs and
outputs.  This test calls that entry point through the C ABI twice in a row
(different batch sizes and timesteps) and checks each result against the
regular entry point, fcv_time_embed, which takes caller-provided scratch, and
both against the reference semantics (the oracle's TimestepEmbedding,
modules.py:606-616, with the bf16 time rounding of modules.py:81 in bf16 mode):
rel-L2 <= 1e-5 in float32, <= 1e-2 in bf16.  It also checks that a batch above
the static limit is refused.

The file is named so that pytest collects it last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import ensure_built, make_model, numpy_params, rel_l2
from oracle import dit_oracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
DEV = "cuda:0"


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_noalloc_time_embed_matches_regular_entry_point(dtype):
    ensure_built()
    from fcv_b200 import _lib

    lib = _lib.lib()
    dt = getattr(torch, dtype)
    model = make_model(5, 1).to(DEV, dt)
    model.finalize_weights()
    w = model.weights_struct()
    params = numpy_params(model)  # the weights exactly as the model holds them
    tol = 1e-5 if dt == torch.float32 else 1e-2
    stream = torch.cuda.current_stream(DEV).cuda_stream
    g = torch.Generator().manual_seed(11)
    for B in (37, 5):  # two calls in a row; the second reuses the static scratch
        t = torch.rand(B, generator=g).to(DEV, dt)
        temb_ref = torch.empty(B, 1024, device=DEV)
        silu_ref = torch.empty(B * 2304, device=DEV, dtype=dt)  # outputs + caller scratch
        _lib.call("fcv_time_embed", ctypes.byref(w), t.data_ptr(), B, temb_ref.data_ptr(), silu_ref.data_ptr(),
                  stream)
        temb = torch.empty(B, 1024, device=DEV)
        silu = torch.empty(B, 1024, device=DEV, dtype=dt)  # outputs only
        _lib.call("fcv_time_embed_noalloc", ctypes.byref(w), t.data_ptr(), B, temb.data_ptr(), silu.data_ptr(),
                  stream)
        torch.cuda.synchronize()
        a, b = temb.cpu().numpy(), temb_ref.cpu().numpy()
        # same kernels on the same inputs: identical up to the 1e-6 relative tolerance of the fp32 checks
        assert np.linalg.norm(a - b) <= 1e-6 * max(np.linalg.norm(b), 1e-30)
        s_a = silu.float().cpu().numpy().reshape(-1)
        s_b = silu_ref[:B * 1024].float().cpu().numpy()
        assert np.linalg.norm(s_a - s_b) <= 1e-6 * max(np.linalg.norm(s_b), 1e-30)
        assert np.isfinite(a).all()
        ref = O.time_embedding(params, t.float().cpu().numpy(), emulate_bf16_time=dt == torch.bfloat16)
        assert rel_l2(b, ref) <= tol, ("fcv_time_embed", dtype, B, rel_l2(b, ref))
        assert rel_l2(a, ref) <= tol, ("fcv_time_embed_noalloc", dtype, B, rel_l2(a, ref))
        silu_ref = ref / (1.0 + np.exp(-ref))
        assert rel_l2(s_a, silu_ref.reshape(-1)) <= tol


def test_noalloc_time_embed_rejects_batch_above_limit():
    ensure_built()
    from fcv_b200 import _lib

    lib = _lib.lib()
    model = make_model(5, 1).to(DEV, torch.bfloat16)
    model.finalize_weights()
    B = _lib.NOALLOC_MAX_B + 1
    t = torch.zeros(B, device=DEV, dtype=torch.bfloat16)
    temb = torch.empty(B, 1024, device=DEV)
    silu = torch.empty(B, 1024, device=DEV, dtype=torch.bfloat16)
    rc = lib.fcv_time_embed_noalloc(ctypes.byref(model.weights_struct()), t.data_ptr(), B, temb.data_ptr(),
                                    silu.data_ptr(), torch.cuda.current_stream(DEV).cuda_stream)
    assert rc == _lib.FCV_EINVAL
    assert b"static scratch limit" in lib.fcv_last_error()
