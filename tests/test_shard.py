"""Request sharding across ranks: LPT bins, 2-rank gloo exchange on CPU, and
host-side failure propagation (a rank that raises fails the batch on every
rank; nothing runs on a GPU)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from fcv_b200.shard import bin_loads, lpt_bins, request_cost


def test_lpt_bins_partition_and_balance():
    rng = np.random.default_rng(3)
    lengths = [int(v) for v in np.clip(np.round(rng.lognormal(np.log(400), 0.6, 128)), 50, 3000)]
    for n in (1, 2, 4, 8):
        bins = lpt_bins(lengths, n)
        flat = sorted(i for b in bins for i in b)
        assert flat == list(range(len(lengths)))
        loads = bin_loads(lengths, bins)
        # LPT bound: max load <= mean + largest single item
        assert max(loads) <= sum(loads) / n + max(request_cost(L) for L in lengths)
    assert lpt_bins([3000] * 16, 8) == [[k, k + 8] for k in range(8)]


def test_benchmark_configs_shard_evenly():
    """The request sets bench.py shards under --gpus N: config 5 (16 x 3000 frames)
    splits into bins of exactly equal cost at 2, 4 and 8 ranks, and config 4's 128
    log-normal requests into bins within 0.5 % of the mean cost."""
    import bench

    c5 = bench.request_lengths("5")[0]
    c4 = bench.request_lengths("4")[0]
    for n in (2, 4, 8):
        loads = bin_loads(c5, lpt_bins(c5, n))
        assert max(loads) == min(loads)
        loads = bin_loads(c4, lpt_bins(c4, n))
        assert max(loads) / (sum(loads) / n) < 1.005, (n, max(loads) / (sum(loads) / n))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, fail_rank, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from fcv_b200.shard import ShardError, run_sharded

    lengths = [5, 300, 17, 120, 64, 1, 999, 250]

    def run_local(idx):
        if rank == fail_rank:
            raise ValueError("injected failure")
        return [(i, lengths[i] * 3 + rank * 0) for i in idx]

    try:
        out = run_sharded(lengths, run_local)
        q.put((rank, "ok", out))
    except ShardError as e:
        q.put((rank, "shard_error", sorted(e.failures)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fail_rank", [-1, 1])
def test_two_rank_gloo_exchange_and_failure(fail_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, fail_rank, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    lengths = [5, 300, 17, 120, 64, 1, 999, 250]
    for rank, kind, payload in results:
        if fail_rank < 0:
            assert kind == "ok"
            assert payload == [(i, L * 3) for i, L in enumerate(lengths)]
        else:
            assert kind == "shard_error" and payload == [fail_rank]
