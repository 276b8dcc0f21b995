"""The multi-GPU plumbing of bench.py on CPU: two (and three) gloo ranks.

Every (batch, head) pair is independent, so ranks share nothing on the data
path: each takes a contiguous range of units, and the only collectives are
the max-over-ranks of the timings and the gather of verification errors.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, ws, port, units, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(ws), LOCAL_RANK=str(rank))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=ws,
                            timeout=datetime.timedelta(seconds=60))
    try:
        env = bench.dist_env()
        lo, hi = bench.shard(units, ws, rank)
        # each rank "processes" its units: a per-unit result that depends only
        # on the unit index, summed locally (no data-path collective)
        local = sum((u * 2654435761) % 1000003 for u in range(lo, hi))
        t_ms = 10.0 + rank  # a per-rank time: the job time is the slowest rank
        t_max = bench.max_over_ranks(t_ms, torch.device("cpu"), ws)
        errs = bench.gather_max([0.001 * (rank + 1), 0.5 - 0.1 * rank], torch.device("cpu"), ws)
        per_rank = bench.gather_all([1000.0 + rank, 2.0 * rank], torch.device("cpu"), ws)
        assert per_rank == [[1000.0 + r, 2.0 * r] for r in range(ws)]
        q.put((rank, env, lo, hi, local, t_max, errs))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("ws,units", [(2, 1024), (2, 7), (3, 1000)])
def test_shards_cover_units_once_and_reduce_over_ranks(ws, units):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, ws, port, units, q)) for r in range(ws)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(ws))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # contiguous, disjoint, covering, sizes differ by at most one
    bounds = [(r[2], r[3]) for r in res]
    assert bounds[0][0] == 0 and bounds[-1][1] == units
    for (a_lo, a_hi), (b_lo, b_hi) in zip(bounds, bounds[1:]):
        assert a_hi == b_lo
    sizes = [hi - lo for lo, hi in bounds]
    assert max(sizes) - min(sizes) <= 1
    # the union of the shards' work equals the whole job's
    assert sum(r[4] for r in res) == sum((u * 2654435761) % 1000003 for u in range(units))
    for rank, env, *_rest, t_max, errs in res:
        assert env == (ws, rank, rank)
        assert t_max == 10.0 + (ws - 1)
        assert errs == pytest.approx([0.001 * ws, 0.5])


def test_single_rank_needs_no_process_group():
    assert bench.shard(1024, 1, 0) == (0, 1024)
    assert bench.max_over_ranks(3.5, torch.device("cpu"), 1) == 3.5
    assert bench.gather_max([1.0, 2.0], torch.device("cpu"), 1) == [1.0, 2.0]
    assert bench.gather_all([1.0, 2.0], torch.device("cpu"), 1) == [[1.0, 2.0]]


def test_per_head_parameters_follow_the_shard():
    """The headline suite flattens (batch, head) into units u = b*H + h and
    shards them; unit u must carry head u % H's parameter."""
    H = 16
    vals = torch.arange(H, dtype=torch.float32) * 10
    for ws in (1, 2, 4, 8):
        got = torch.cat([bench._flat_param(vals, *bench.shard(4 * H, ws, r), H)
                         for r in range(ws)])
        assert torch.equal(got, vals.repeat(4))
