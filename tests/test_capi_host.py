"""CPU checks of the C-ABI library and the host logic (no GPU needed).

* the library cross-compiles for sm_100a, loads, and exports exactly the
  entry points ``include/fcv_b200.h`` declares;
* argument validation fails with a status and a message before any CUDA call;
* host-only entry points (attention work list, workspace sizing) compute;
* the layout ("plan") cache mirrors the reference's pool semantics
  (tests/test_plan_pool.py in the reference).
"""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

from conftest import ROOT, ensure_built

HEADER = ROOT / "include" / "fcv_b200.h"


def header_functions() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(fcv_[a-z0-9_]+)\s*\(", text))


@pytest.fixture(scope="module")
def lib():
    ensure_built()
    from fcv_b200 import _lib

    return _lib.lib()


def test_library_exports_every_declared_entry_point(lib):
    from fcv_b200 import _lib

    declared = header_functions()
    assert declared == set(_lib.EXPORTS)
    so = _lib.LIB_PATH
    out = subprocess.run(["nm", "-D", "--defined-only", so], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (fcv_[a-z0-9_]+)", out))
    assert declared <= exported, declared - exported
    for name in declared:
        assert hasattr(lib, name)


def test_version_and_error_paths_without_gpu(lib):
    assert lib.fcv_version() >= 1
    rc = lib.fcv_gemm(None, None, None, 1, 1, 1, 1, 0, None, None, None, 0, None, None, None)
    assert rc == -1
    assert b"fcv_gemm" in lib.fcv_last_error()
    assert lib.fcv_dit_forward(None, None, None, 0, None) == -1
    assert lib.fcv_attention(None, 1, None, 0, 0, 0, 0, None, 0, None, 0, None, None) == -1
    assert lib.fcv_ln_modulate(None, 0, None, None, None, 0, 0, None, 0, None) == -1
    assert lib.fcv_selftest_wait_expiry(1000, None, None) == -1  # no observed buffer
    assert lib.fcv_selftest_wait_expiry(0, 16, None) == -1  # limit outside (0, 4 s]
    assert lib.fcv_selftest_wait_expiry(5_000_000_000, 16, None) == -1
    assert b"fcv_selftest_wait_expiry" in lib.fcv_last_error()
    assert lib.fcv_pack_layout(None, 0, 0, 0, None, None, None, None, None, None) == -1


def test_alignment_rules_rejected_before_any_launch(lib):
    """Operands read with 16-byte vector or bulk copies are checked on the host
    (the pointers below are never dereferenced: the calls return first)."""
    a16, odd = 0x10000, 0x10004
    # LayerNorm-modulate streams h rows with 1-D bulk copies: h must be 16-byte aligned
    rc = lib.fcv_ln_modulate(odd, 0, a16, a16, a16, 4096, 8, a16, 1, None)
    assert rc == -1 and b"16-byte aligned" in lib.fcv_last_error()
    # modulation rows are read as float4
    rc = lib.fcv_ln_modulate(a16, 0, odd, a16, a16, 4096, 8, a16, 1, None)
    assert rc == -1 and b"16-byte aligned" in lib.fcv_last_error()
    # RoPE tables are read as float4 in the QKV epilogue
    rc = lib.fcv_gemm(a16, a16, None, 8, 3072, 1024, 1, 2, a16, a16, None, 0, odd, a16, None)
    assert rc == -1 and b"RoPE tables must be 16-byte aligned" in lib.fcv_last_error()


def test_workspace_bytes_grows_with_rows(lib):
    a = lib.fcv_dit_workspace_bytes(1000, 4, 22, 1)
    b = lib.fcv_dit_workspace_bytes(2000, 4, 22, 1)
    c = lib.fcv_dit_workspace_bytes(1000, 4, 22, 0)
    assert 0 < a < b and a < c
    assert lib.fcv_dit_workspace_bytes(-1, 4, 22, 1) == 0


def _tiles(lib, lengths, chunk):
    cap = sum((L + 127) // 128 for L in lengths)
    buf = (ctypes.c_int32 * (2 * max(cap, 1)))()
    lens = (ctypes.c_int32 * len(lengths))(*lengths)
    n = lib.fcv_attn_tiles(ctypes.addressof(lens), len(lengths), chunk, ctypes.addressof(buf), cap)
    return n, np.array(list(buf)[:2 * n]).reshape(-1, 2)


@pytest.mark.parametrize("chunk", [0, 50])
def test_attention_work_list_covers_rows_and_orders_by_cost(lib, chunk):
    lengths = [1, 127, 128, 129, 1000, 0, 3000, 64]
    n, tiles = _tiles(lib, lengths, chunk)
    seen = set()
    costs = []
    for d, q0 in tiles:
        rows = min(384, lengths[d] - q0)  # a work-list entry: up to three 128-row query tiles
        assert rows > 0 and q0 % 384 == 0
        for q in range(q0, q0 + rows):
            assert (d, q) not in seen
            seen.add((d, q))
        q_last = q0 + rows - 1
        kv = lengths[d] if not chunk else min(lengths[d], (q_last // chunk + 1) * chunk)
        costs.append(rows * kv)
    assert len(seen) == sum(lengths)
    assert costs == sorted(costs, reverse=True)


def test_attention_work_list_capacity_error(lib):
    lens = (ctypes.c_int32 * 1)(1000)
    buf = (ctypes.c_int32 * 4)()
    assert lib.fcv_attn_tiles(ctypes.addressof(lens), 1, 0, ctypes.addressof(buf), 2) == -1


def test_layout_cache_fifo_and_no_replan(monkeypatch, lib):
    """Recurring batch compositions reuse their prepared layout (no re-plan);
    the cache is a bounded FIFO of 64 (flashinfer_dit.py:62, 400-404)."""
    import torch

    from fcv_b200 import model as M

    real_call = M.call

    def fake_call(name, *args):
        if name == "fcv_pack_layout":
            return 0
        return real_call(name, *args)

    monkeypatch.setattr(M, "call", fake_call)
    dit = M.B200DiT(depth=1)
    cpu = torch.device("cpu")
    monkeypatch.setattr(M, "_stream", lambda device: 0)
    a = dit.prepare_layout([100, 100], 100, True, cpu)
    b = dit.prepare_layout([200, 200], 200, True, cpu)
    assert a is not b and dit.plan_calls == 2
    assert dit.prepare_layout([100, 100], 100, True, cpu) is a
    assert dit.prepare_layout([200, 200], 200, True, cpu) is b
    assert dit.plan_calls == 2
    # streaming and offline are different plans (chunk mask vs full)
    assert dit.prepare_layout([100, 100], 100, False, cpu) is not a
    for i in range(64):
        dit.prepare_layout([i + 1], 64, False, cpu)
    assert len(dit._layouts) == 64
    assert dit.prepare_layout([100, 100], 100, True, cpu) is not a  # evicted, re-planned
    with pytest.raises(ValueError):
        dit.prepare_layout([5, 300], 100, True, cpu)


def test_graph_bucket_presets_become_row_capacities():
    """The reference's presets (seconds offline at 50 frames/s, frames streaming;
    config/settings.py:9-10) hold one CFG pair: F frames -> 2F packed rows."""
    from fcv_b200.model import DEFAULT_GRAPH_BUCKETS, graph_row_buckets

    assert graph_row_buckets((8.0, 12.0), (512, 640)) == (800, 1024, 1200, 1280)
    assert graph_row_buckets(None, None) is None
    assert list(DEFAULT_GRAPH_BUCKETS) == sorted(DEFAULT_GRAPH_BUCKETS)


@pytest.mark.parametrize("chunk", [0, 50])
def test_attention_schedule_assigns_every_item_once_and_balances(lib, chunk):
    """fcv_attn_schedule: a permutation of the 16 * n_tiles items grouped by CTA,
    longest first to the least loaded CTA; its worst CTA carries no more work
    than round robin's (config-2 lengths, one CTA per SM: 148 on a B200).  The
    cost of an item is the 128 x 64 tiles of its (up to three) query tiles + 1."""
    rng = np.random.default_rng(1)
    req = [int(v) for v in rng.integers(150, 601, size=8)]
    lengths = req + req + [1, 0, 3000]
    n, tiles = _tiles(lib, lengths, chunk)
    ctas = lib.fcv_attn_ctas(n)
    assert ctas == min(16 * n, 148)
    cap = ctas + 1 + 16 * n
    buf = (ctypes.c_int32 * cap)()
    lens = (ctypes.c_int32 * len(lengths))(*lengths)
    flat = (ctypes.c_int32 * (2 * n))(*tiles.reshape(-1).tolist())
    assert lib.fcv_attn_schedule(ctypes.addressof(lens), len(lengths), chunk, ctypes.addressof(flat), n, ctas,
                                 ctypes.addressof(buf), cap) == cap
    s = np.array(list(buf))
    off, items = s[:ctas + 1], s[ctas + 1:]
    assert off[0] == 0 and off[-1] == 16 * n and np.all(np.diff(off) >= 0)
    assert sorted(items.tolist()) == list(range(16 * n))

    def key_tiles(L, q_last):
        kv = min(L, (q_last // chunk + 1) * chunk) if chunk else L
        return -(-kv // 64)

    def cost(it):
        d, q0 = tiles[it // 16]
        L = lengths[d]
        return 1 + sum(key_tiles(L, min(q0 + 128 * (u + 1), L) - 1) for u in range(3) if q0 + 128 * u < L)

    lpt = max(sum(cost(i) for i in items[off[c]:off[c + 1]]) for c in range(ctas))
    rr = max(sum(cost(i) for i in range(c, 16 * n, ctas)) for c in range(ctas))
    assert lpt <= rr
    assert lib.fcv_attn_schedule(ctypes.addressof(lens), len(lengths), chunk, ctypes.addressof(flat), n, ctas,
                                 ctypes.addressof(buf), cap - 1) == -1
