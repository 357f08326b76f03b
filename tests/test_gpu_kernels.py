"""Per-kernel parity on the GPU, through the C ABI.

Integer work (layout) is compared bit-exactly with the oracle / golden
vectors; floating-point kernels against a plain PyTorch fp32 computation of the
same op.  Tolerances: fp32 kernels 1e-5 relative; bf16 kernels are judged on
their bf16 output rounding (|err| <= 1e-2 * max|ref| or rel-L2 <= 5e-3)."""

from __future__ import annotations

import math
import time

import numpy as np
import pytest

from conftest import ensure_built, load_golden, rel_l2
from oracle import dit_oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _lib():
    ensure_built()
    from fcv_b200 import _lib as L

    L.lib()
    yield
    from fcv_b200 import ops

    assert ops.device_error() == 0


DEV = "cuda:0"


def _ops():
    from fcv_b200 import ops

    return ops


# ---------------------------------------------------------------- bounded waits

def test_bounded_wait_expires_with_an_error_code_and_the_context_survives():
    """Every pipelined kernel here (GEMM, convolution, attention) waits on mbarriers
    with a time limit, so a stalled pipeline ends with an error word the host reads
    instead of a hung GPU.  fcv_selftest_wait_expiry runs that wait on a barrier that
    nothing completes (limit 20 ms): both waiters return false, the first code (901)
    reaches the host, reading it clears it, and the context still computes (a GEMM
    checked against torch right after)."""
    from fcv_b200 import _lib
    from fcv_b200._lib import call

    ops = _ops()
    assert ops.device_error() == 0
    observed = torch.full((2,), 7, dtype=torch.int32, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    t0 = time.perf_counter()
    call("fcv_selftest_wait_expiry", 20_000_000, observed.data_ptr(), stream)
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert observed.tolist() == [0, 0]
    assert 0.015 < elapsed < 2.0, elapsed
    assert ops.device_error() == 901
    assert ops.device_error() == 0  # read and cleared
    x = torch.randn(300, 1024, device=DEV).to(torch.bfloat16)
    w = torch.randn(256, 1024, device=DEV).to(torch.bfloat16)
    y = ops.linear(x, w, epilogue=_lib.EPI_BIAS_F32)
    ref = x.float() @ w.float().t()
    assert rel_l2(y.cpu().numpy(), ref.cpu().numpy()) < 1e-5
    assert ops.device_error() == 0


# ---------------------------------------------------------------- layout (bit-exact)

def test_pack_layout_bit_exact_against_reference_golden():
    ops = _ops()
    z = load_golden("pack_layout")
    for i in range(int(z["n_cases"])):
        lengths = z[f"c{i}_lengths"].astype(np.int32)
        T = int(z[f"c{i}_T"])
        N = int(lengths.sum())
        g, d, p, cu, gap = ops.pack_layout(torch.tensor(lengths, device=DEV), T, N)
        np.testing.assert_array_equal(g.cpu().numpy(), z[f"c{i}_gather"])
        np.testing.assert_array_equal(d.cpu().numpy(), z[f"c{i}_doc_ids"])
        np.testing.assert_array_equal(p.cpu().numpy(), z[f"c{i}_positions"])
        np.testing.assert_array_equal(cu.cpu().numpy(), z[f"c{i}_cu"])
        # gapped layout: every document behind 30 zero rows
        exp = np.full(N + 30 * (len(lengths) + 1), -1, np.int32)
        off = 0
        for b, L in enumerate(lengths):
            start = off + 30 * (b + 1)
            exp[start:start + L] = np.arange(off, off + L)
            off += L
        np.testing.assert_array_equal(gap.cpu().numpy(), exp)


def test_pack_layout_zero_length_and_large_batch():
    ops = _ops()
    rng = np.random.default_rng(0)
    lengths = rng.integers(0, 40, size=3000).astype(np.int32)
    lengths[:5] = 0
    lengths[-1] = 0
    T = 64
    N = int(lengths.sum())
    g, d, p, cu, gap = ops.pack_layout(torch.tensor(lengths, device=DEV), T, N)
    ref = O.pack_layout(lengths, T)
    np.testing.assert_array_equal(g.cpu().numpy(), ref.gather_indices)
    np.testing.assert_array_equal(d.cpu().numpy(), ref.document_ids)
    np.testing.assert_array_equal(p.cpu().numpy(), ref.positions)
    np.testing.assert_array_equal(cu.cpu().numpy(), ref.cu_seqlens)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_mask_lengths(dtype):
    ops = _ops()
    lengths = [300, 1, 0, 4095, 3001]
    T = 4100
    m = torch.zeros(len(lengths), 1, T, dtype=getattr(torch, dtype), device=DEV)
    for b, L in enumerate(lengths):
        m[b, 0, :L] = 1
    assert ops.mask_lengths(m).cpu().tolist() == lengths


# ---------------------------------------------------------------- row kernels

@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_ln_modulate_and_gate_residual_vs_reference_golden(dtype):
    ops = _ops()
    z = load_golden("rownorm")
    dt = getattr(torch, dtype)
    n = z["h"].shape[0]
    h = torch.tensor(z["h"], device=DEV).to(dt)
    # modulation rows: one document per row, stride 2048 (shift | scale)
    mods = torch.zeros(n, 2048, device=DEV)
    mods[:, :1024] = torch.tensor(z["shift"])
    mods[:, 1024:] = torch.tensor(z["scale"])
    doc = torch.arange(n, dtype=torch.int32, device=DEV)
    out = ops.layer_norm_modulate_packed(h, mods[:, :1024], mods[:, 1024:], doc, 2048)
    ref = O.layer_norm_modulate(h.float().cpu().numpy(), z["shift"], z["scale"])
    tol = 1e-5 if dtype == "float32" else 5e-3
    assert rel_l2(out.float().cpu().numpy(), ref) < tol
    gmods = torch.zeros(n, 4096, device=DEV)
    gmods[:, :1024] = torch.tensor(z["gate"])
    gmods[:, 1024:2048] = torch.tensor(z["shift"])
    gmods[:, 2048:3072] = torch.tensor(z["scale"])
    r = torch.tensor(z["r"], device=DEV).to(dt)
    h2, norm = ops.gate_residual_layer_norm_modulate_packed(h, gmods[:, :1024], r, gmods[:, 1024:2048],
                                                            gmods[:, 2048:3072], doc, 4096)
    rh, rn = O.gate_residual_layer_norm_modulate(h.float().cpu().numpy(), z["gate"], r.float().cpu().numpy(),
                                                 z["shift"], z["scale"])
    assert rel_l2(h2.float().cpu().numpy(), rh) < tol
    assert rel_l2(norm.float().cpu().numpy(), rn) < tol


# ---------------------------------------------------------------- GEMM

def _gemm_inputs(M, N, K, dt, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    A = torch.randn(M, K, generator=g).to(DEV, dt)
    W = (torch.randn(N, K, generator=g) / math.sqrt(K)).to(DEV, dt)
    b = torch.randn(N, generator=g).to(DEV)
    return A, W, b


def _ref_gemm(A, W, b):
    return A.float() @ W.float().T + b


def _close(out, ref, dtype):
    out = out.float()
    if dtype == torch.float32:
        assert rel_l2(out.cpu().numpy(), ref.cpu().numpy()) < 1e-5
    else:
        err = (out - ref).abs().max().item()
        assert err <= 1e-2 * ref.abs().max().item() + 1e-3, err
        assert rel_l2(out.cpu().numpy(), ref.cpu().numpy()) < 5e-3


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
@pytest.mark.parametrize("M,N,K", [(1, 3072, 1024), (129, 1024, 1024), (300, 2048, 1024),
                                   (257, 1024, 2048), (1000, 80, 1024), (200, 1024, 320),
                                   (6000, 1024, 1024), (40000, 1024, 1024), (16, 137216, 1024),
                                   (6578, 3072, 1024)])
def test_gemm_bias(dtype, M, N, K):
    ops = _ops()
    dt = getattr(torch, dtype)
    if dtype == "float32" and M * N > 50_000_000:
        pytest.skip("fp32 CUDA-core path: large shapes covered by bf16")
    A, W, b = _gemm_inputs(M, N, K, dt)
    out = ops.linear(A, W, b)
    _close(out, _ref_gemm(A, W, b), dt)


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_gemm_gelu_and_f32(dtype):
    from fcv_b200 import _lib as L

    ops = _ops()
    dt = getattr(torch, dtype)
    A, W, b = _gemm_inputs(333, 2048, 1024, dt, 1)
    ref = _ref_gemm(A, W, b)
    _close(ops.linear(A, W, b, epilogue=L.EPI_BIAS_GELU), torch.nn.functional.gelu(ref, approximate="tanh"), dt)
    out = ops.linear(A, W, b, epilogue=L.EPI_BIAS_F32)
    assert out.dtype == torch.float32
    _close(out, ref, dt)


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
def test_gemm_rope_epilogue(dtype):
    from fcv_b200 import _lib as L

    ops = _ops()
    dt = getattr(torch, dtype)
    lengths = [100, 37, 150]
    N = sum(lengths)
    A, W, b = _gemm_inputs(N, 3072, 1024, dt, 2)
    pos_np = np.concatenate([np.arange(L) for L in lengths]).astype(np.int32)
    pos = torch.tensor(pos_np, device=DEV)
    cos, sin = O.rope_tables(4096)
    out = ops.linear(A, W, b, epilogue=L.EPI_BIAS_ROPE_QKV, aux=pos, rope_cos=torch.tensor(cos, device=DEV),
                     rope_sin=torch.tensor(sin, device=DEV))
    ref = _ref_gemm(A, W, b).cpu().numpy()
    ref[:, :1024] = O.apply_partial_rope(ref[:, :1024], pos_np)
    ref[:, 1024:2048] = O.apply_partial_rope(ref[:, 1024:2048], pos_np)
    _close(out, torch.tensor(ref, device=DEV), dt)


@pytest.mark.parametrize("dtype,lengths", [("bfloat16", [64, 200, 1]), ("float32", [64, 200, 1]),
                                           ("bfloat16", [3000, 1, 3577])])
def test_gemm_gate_residual_epilogue(dtype, lengths):
    """Gated residual into fp32 h; the 6578-row case runs several full waves of
    256 x 256 tiles and splits the last wave's tiles into 256 x 128 pieces."""
    from fcv_b200 import _lib as L

    ops = _ops()
    dt = getattr(torch, dtype)
    N = sum(lengths)
    A, W, b = _gemm_inputs(N, 1024, 2048, dt, 3)
    doc = torch.tensor(np.repeat(np.arange(3), lengths).astype(np.int32), device=DEV)
    mods = torch.randn(3, 5000, device=DEV)
    gate = mods[:, 100:]  # row stride 5000, offset 100 floats (16-byte aligned)
    h = torch.randn(N, 1024, device=DEV)
    ref = h + gate[doc.long(), :1024] * _ref_gemm(A, W, b)
    ops.linear(A, W, b, epilogue=L.EPI_BIAS_GATE_RES, out=h, aux=doc, gate=gate, gate_stride=5000)
    if dt == torch.float32:
        assert rel_l2(h.cpu().numpy(), ref.cpu().numpy()) < 1e-5
    else:
        assert (h - ref).abs().max().item() < 2e-2 * ref.abs().max().item()


def test_gemm_rejects_bad_arguments_without_launching():
    from fcv_b200 import _lib as L

    ops = _ops()
    A = torch.randn(10, 100, device=DEV, dtype=torch.bfloat16)  # K=100 is not a multiple of 64
    W = torch.randn(64, 100, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(L.FcvError):
        ops.linear(A, W)


# ---------------------------------------------------------------- attention

def _ref_attention(qkv, lengths, chunk):
    out = torch.zeros(qkv.shape[0], 1024, device=qkv.device)
    off = 0
    for L in lengths:
        q = qkv[off:off + L, :1024].float().view(L, 16, 64).transpose(0, 1)
        k = qkv[off:off + L, 1024:2048].float().view(L, 16, 64).transpose(0, 1)
        v = qkv[off:off + L, 2048:].float().view(L, 16, 64).transpose(0, 1)
        s = q @ k.transpose(1, 2) / 8.0
        if chunk:
            p = torch.arange(L, device=qkv.device)
            vis = (p[None, :] // chunk) <= (p[:, None] // chunk)
            s = s.masked_fill(~vis, float("-inf"))
        o = torch.softmax(s, -1) @ v
        out[off:off + L] = o.transpose(0, 1).reshape(L, 1024)
        off += L
    return out


@pytest.mark.parametrize("dtype", ["bfloat16", "float32"])
@pytest.mark.parametrize("chunk", [0, 50])
def test_ragged_attention(dtype, chunk):
    ops = _ops()
    dt = getattr(torch, dtype)
    lengths = [1, 7, 128, 129, 300, 1000, 50, 51]
    N = sum(lengths)
    g = torch.Generator().manual_seed(7)
    qkv = (torch.randn(N, 3072, generator=g) * 1.5).to(DEV, dt)
    _, _, _, cu, _ = ops.pack_layout(torch.tensor(lengths, dtype=torch.int32, device=DEV), max(lengths), N)
    tiles, n = ops.attention_tiles(lengths, chunk, DEV)
    out = ops.ragged_attention(qkv, cu, tiles, n, chunk)
    ref = _ref_attention(qkv, lengths, chunk)
    if dt == torch.float32:
        assert rel_l2(out.cpu().numpy(), ref.cpu().numpy()) < 1e-5
    else:
        # bf16 output: its own rounding is up to 2^-8 relative; P is rounded to bf16 too
        err = ((out.float() - ref).abs() / (1.0 + ref.abs())).max().item()
        assert err < 1e-2, err
        assert rel_l2(out.float().cpu().numpy(), ref.cpu().numpy()) < 5e-3


@pytest.mark.parametrize("key_boost", [60.0, 300.0])
@pytest.mark.parametrize("chunk", [0, 50])
def test_attention_logits_rising_far_above_the_first_key_tile(key_boost, chunk):
    """The bf16 kernel takes a row's reference maximum on its first 64-key tile
    and rescales only when a later tile's exponentials would pass 2^32.  Here
    every query has 4 in dimension 0 of each head and every 37th key of the
    second half of each document has `key_boost` there: those logits sit ~43
    (boost 60: the tile sum passes 2^32) or ~216 (boost 300: the exponentials
    overflow to inf) log2 units above everything before them, so the row is
    rescaled and the tile redone.  Within bf16 rounding of torch fp32, with the
    streaming mask too (early rows never see the boosted keys)."""
    ops = _ops()
    lengths = [700, 300, 1000, 129]
    N = sum(lengths)
    g = torch.Generator().manual_seed(11)
    qkv = torch.randn(N, 3072, generator=g) * 0.5
    qkv[:, 0:1024:64] = 4.0
    off = 0
    for L in lengths:
        qkv[torch.arange(off + L // 2, off + L, 37), 1024:2048:64] = key_boost
        off += L
    qkv = qkv.to(DEV, torch.bfloat16)
    _, _, _, cu, _ = ops.pack_layout(torch.tensor(lengths, dtype=torch.int32, device=DEV), max(lengths), N)
    tiles, n = ops.attention_tiles(lengths, chunk, DEV)
    out = ops.ragged_attention(qkv, cu, tiles, n, chunk)
    ref = _ref_attention(qkv, lengths, chunk)
    assert torch.isfinite(out.float()).all()
    err = ((out.float() - ref).abs() / (1.0 + ref.abs())).max().item()
    assert err < 1e-2, err
    assert rel_l2(out.float().cpu().numpy(), ref.cpu().numpy()) < 5e-3


def test_attention_tiles_cover_every_query_row_once():
    ops = _ops()
    lengths = [1, 127, 128, 129, 1000, 0, 3000]
    for chunk in (0, 50):
        tiles, n = ops.attention_tiles(lengths, chunk, "cpu")
        seen = set()
        for d, q0 in tiles.view(-1, 2)[:n].tolist():
            for q in range(q0, min(q0 + 384, lengths[d])):  # a work-list entry: three 128-row query tiles
                assert (d, q) not in seen
                seen.add((d, q))
        assert len(seen) == sum(lengths)


# ---------------------------------------------------------------- ODE step

def test_cfg_euler_step():
    ops = _ops()
    R, T = 3, 77
    x = torch.randn(R, 80, T, device=DEV)
    d = torch.randn(2 * R, 80, T, device=DEV).to(torch.bfloat16)
    x0 = x.clone()
    nxt = torch.empty(2 * R, 80, T, device=DEV, dtype=torch.bfloat16)
    ops.cfg_euler_(x, d, 0.125, 0.7, nxt)
    ref = x0 + 0.125 * (1.7 * d[:R].float() - 0.7 * d[R:].float())
    assert (x - ref).abs().max().item() < 1e-5
    assert torch.equal(nxt[:R], x.to(torch.bfloat16)) and torch.equal(nxt[R:], x.to(torch.bfloat16))
