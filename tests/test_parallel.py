"""Data-parallel host logic on CPU: shard/merge round trip, the spawned-worker runner (including a failing
shard), and the bench's max-over-ranks reduction on a world-size-2 gloo process group."""

import os
import socket

import numpy as np
import pytest

from viktor_b200.parallel import ShardError, merge_shards, run_sharded, shard_indices


@pytest.mark.parametrize("mode", ["strided", "contiguous"])
@pytest.mark.parametrize("n,world", [(16384, 8), (10, 3), (2, 4), (0, 2)])
def test_shard_merge_round_trip(mode, n, world):
    rows = np.arange(n * 3).reshape(n, 3)
    parts = [rows[shard_indices(n, world, r, mode)] for r in range(world)]
    assert sum(len(p) for p in parts) == n
    assert np.array_equal(merge_shards(parts, n, mode), rows) if n else True
    seen = np.concatenate([shard_indices(n, world, r, mode) for r in range(world)])
    assert np.array_equal(np.sort(seen), np.arange(n))


def fake_decode(rank, world, indices, fail_rank, how="raise"):
    """Stands in for a per-GPU engine: 'tokens' are a function of the chunk index only."""
    if rank == fail_rank:
        if how == "exit0":
            os._exit(0)  # leaves without a result and without an error code
        raise RuntimeError("simulated device failure")
    return np.stack([np.arange(5) + 100 * i for i in indices]) if len(indices) else np.zeros((0, 5), int)


def test_run_sharded_gathers_in_order():
    n, world = 11, 2
    parts = run_sharded(fake_decode, n, world, args=(-1,))
    out = merge_shards(parts, n)
    assert np.array_equal(out, np.stack([np.arange(5) + 100 * i for i in range(n)]))


def test_run_sharded_reports_the_failing_shard():
    with pytest.raises(ShardError) as e:
        run_sharded(fake_decode, 8, 2, args=(1,), timeout=120)
    assert e.value.rank == 1


def test_run_sharded_reports_a_worker_that_exits_without_result():
    """A worker that ends with exit code 0 but never answered fails its shard within seconds (not at the
    call's timeout)."""
    import time
    t0 = time.monotonic()
    with pytest.raises(ShardError) as e:
        run_sharded(fake_decode, 8, 2, args=(0, "exit0"), timeout=600)
    assert e.value.rank == 0
    assert time.monotonic() - t0 < 60


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, q):
    import torch.distributed as dist
    from viktor_b200.parallel import reduce_bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q.put((rank, reduce_bench(1.0 + rank, 0.5 * (rank + 1), 0.1, 1000 * (rank + 1))))
    finally:
        dist.destroy_process_group()


def test_reduce_bench_on_gloo_world_of_two():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=30)
    for r in range(2):
        e, d, pf, b = res[r]
        assert (e, d, pf, b) == (2.0, 1.0, 0.1, 3000)


def _gloo_gather_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from viktor_b200.parallel import gather_tokens
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        tok = torch.arange(12, dtype=torch.int64).reshape(3, 4) + 1000 * rank
        tok[0, 0] = 342  # the largest 4-mer token id survives the int16 transport
        got = gather_tokens(tok)
        q.put((rank, None if got is None else got.numpy()))
    finally:
        dist.destroy_process_group()


def test_gather_tokens_on_gloo_world_of_two():
    """The final token gather: rank 0 receives every rank's [rows, cols] tokens in rank order, others None."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_gather_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=30)
    assert res[1] is None
    want = np.concatenate([np.arange(12).reshape(3, 4) + 1000 * r for r in range(2)])
    want[0, 0] = want[3, 0] = 342
    assert res[0].dtype == np.int16 and np.array_equal(res[0], want)
