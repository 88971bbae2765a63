"""Data-parallel decoding across the GPUs of one host.

Chunks are independent, so the batch is sharded across processes, one per GPU, each with its own engine,
weights and KV cache; there is no collective on the data path and the token arrays are gathered on the host
at the end (the pattern of scripts/evaluate.py:127-138, and of `sharded_calls` in scripts/train.py:297-305).

* ``shard_indices`` / ``merge_shards``: which chunks a rank decodes, and the inverse (strided, as the reference,
  or contiguous).
* ``run_sharded``: spawn one worker process per device, call ``worker(rank, world, indices, *args)`` in each,
  collect the results in rank order.  A worker that raises, exits or does not answer makes the call raise
  ``ShardError`` naming the rank (the other workers are stopped), so a caller never gets a silently partial
  result.
* ``gather_tokens``: the final gather of every rank's token array onto one host (rank 0), over the process
  group (NCCL over NVLink between GPUs), then one copy into pinned host memory.
* ``reduce_bench``: the timing reduction used by ``bench.py`` under ``torch.distributed`` (max of the elapsed
  times, sum of the bases), written against any backend (NCCL on GPUs, gloo on CPU in the tests).
"""

from __future__ import annotations

import multiprocessing as mp
import queue
import traceback

import numpy as np


class ShardError(RuntimeError):
    """A data-parallel worker failed; ``rank`` names it."""

    def __init__(self, rank, message):
        super().__init__(f"shard {rank} failed: {message}")
        self.rank = rank


def shard_indices(n: int, world: int, rank: int, mode: str = "strided") -> np.ndarray:
    """Chunk indices decoded by ``rank`` of ``world``: strided (rank, rank + world, ...) or contiguous blocks."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if mode == "strided":
        return np.arange(rank, n, world)
    if mode == "contiguous":
        lo, hi = n * rank // world, n * (rank + 1) // world
        return np.arange(lo, hi)
    raise ValueError(f"unknown shard mode {mode!r}")


def merge_shards(parts, n: int, mode: str = "strided") -> np.ndarray:
    """Inverse of ``shard_indices``: parts[r] holds rank r's rows in its index order; returns all n rows."""
    world = len(parts)
    out = None
    for r, part in enumerate(parts):
        part = np.asarray(part)
        idx = shard_indices(n, world, r, mode)
        if len(idx) != len(part):
            raise ValueError(f"shard {r}: {len(part)} rows, expected {len(idx)}")
        if out is None:
            out = np.empty((n,) + part.shape[1:], dtype=part.dtype)
        out[idx] = part
    return out


def _worker_main(worker, rank, world, indices, args, results):
    try:
        results.put((rank, True, worker(rank, world, indices, *args)))
    except BaseException:  # report anything, including KeyboardInterrupt / SystemExit
        results.put((rank, False, traceback.format_exc(limit=8)))


def run_sharded(worker, n_items: int, world: int, args=(), mode: str = "strided", timeout: float = 3600.0):
    """Runs ``worker(rank, world, indices, *args)`` in ``world`` spawned processes and returns the list of their
    results in rank order.  ``worker`` must be importable (module level).  Raises ``ShardError`` if a worker
    raises, dies without answering, or the whole call exceeds ``timeout`` seconds."""
    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    procs = []
    for r in range(world):
        p = ctx.Process(target=_worker_main,
                        args=(worker, r, world, shard_indices(n_items, world, r, mode), tuple(args), results),
                        daemon=True)
        p.start()
        procs.append(p)
    out = [None] * world
    got = 0

    def take(item):
        nonlocal got
        rank, ok, payload = item
        if not ok:
            raise ShardError(rank, payload.strip().splitlines()[-1] if payload else "error")
        if out[rank] is None:
            out[rank] = (payload,)
            got += 1

    try:
        import time
        deadline = time.monotonic() + timeout
        while got < world:
            try:
                take(results.get(timeout=0.5))
            except queue.Empty:
                dead = [r for r, p in enumerate(procs) if out[r] is None and not p.is_alive()]
                if dead:
                    # a worker that finished without a result in hand: its result may still be in the queue's pipe
                    # (the feeder flushes it on exit), so drain for a moment before declaring the shard failed
                    drain_until = time.monotonic() + 2.0
                    while got < world and time.monotonic() < drain_until:
                        try:
                            take(results.get(timeout=0.2))
                        except queue.Empty:
                            pass
                    for r in dead:
                        if out[r] is None:
                            raise ShardError(r, f"process exited with code {procs[r].exitcode} without a result")
                if time.monotonic() > deadline:
                    missing = [r for r in range(world) if out[r] is None]
                    raise ShardError(missing[0], f"no result after {timeout:.0f} s")
                continue
    finally:
        for p in procs:
            if p.is_alive() and any(o is None for o in out):
                p.terminate()
            p.join(timeout=5)
    return [o[0] for o in out]


def gather_tokens(tokens, dst: int = 0, host_out=None):
    """The final host gather of a data-parallel decode under ``torch.distributed``: every rank passes its token
    array ``tokens`` [rows, cols] (the same shape on every rank, on the rank's device for NCCL or on the CPU for
    gloo); rank ``dst`` gets the ranks' arrays concatenated in rank order as one CPU int16 tensor [world * rows,
    cols] (token ids < 32768; the 4-mer vocabulary has 343), the other ranks get None.  Tokens cross NVLink as
    int16 (a quarter of the engine's int64 buffer) and reach the host in one copy into pinned memory
    (``host_out``, a pinned int16 tensor of the gathered shape, when given; else a new one)."""
    import torch
    import torch.distributed as dist
    world, rank = dist.get_world_size(), dist.get_rank()
    # int16 travels as its bytes: neither NCCL nor gloo has a 16-bit integer type, and a gather only moves bytes
    t8 = tokens.to(torch.int16).contiguous().view(torch.uint8)
    parts = [torch.empty_like(t8) for _ in range(world)] if rank == dst else None
    dist.gather(t8, parts, dst=dst)
    if rank != dst:
        return None
    allt = torch.cat(parts).view(torch.int16)
    if allt.is_cuda:
        host = host_out if host_out is not None else torch.empty(allt.shape, dtype=allt.dtype, pin_memory=True)
        host.copy_(allt, non_blocking=True)
        torch.cuda.current_stream(allt.device).synchronize()
        return host
    return allt


def reduce_bench(elapsed_s: float, decode_s: float, prefill_s: float, bases: int, device=None):
    """Max over ranks of the elapsed / decode / prefill seconds and the sum of the decoded bases (the numbers a
    data-parallel bench reports).  Uses the default process group of ``torch.distributed``."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([elapsed_s, decode_s, prefill_s], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    b = torch.tensor([bases], dtype=torch.long, device=device)
    dist.all_reduce(b)
    e, d, p = t.tolist()
    return e, d, p, int(b.item())
