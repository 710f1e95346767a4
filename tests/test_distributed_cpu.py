"""Multi-rank host logic on CPU: gloo process groups of world size 2 (and
3), the oracle standing in for the selection kernels.  Covers the sharded
eviction exchange (local candidates -> all-gather -> merge), the decode
partition, and failure detection: a rank that dies before the collective
makes the survivor's collective fail within the group timeout instead of
hanging."""

from __future__ import annotations

import os
import socket
import sys
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import PKG, ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_local(scores, k, off):
    from oracle import oracle as O
    s = scores.numpy()
    keys = np.sort(O.pack_candidate_keys(s, np.arange(s.size) + off))[:min(k, s.size)]
    return torch.from_numpy(keys.view(np.int64).copy())


def _oracle_merge(keys, k):
    from oracle import oracle as O
    return torch.from_numpy(O.merge_candidate_keys(keys.numpy().view(np.uint64), k))


def _worker(rank, world, port, mode, scores, k, q):
    try:
        for p in (str(PKG), str(ROOT)):
            sys.path.insert(0, p)
        from pagedkv_fusion.distributed import shard_block_range, sharded_eviction_select
        import torch.distributed as dist
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=timedelta(seconds=8))
        if mode == "die" and rank == 1:
            os._exit(0)  # leaves between steps, before the collective
        lo, hi = shard_block_range(scores.size, rank, world)
        local = torch.from_numpy(scores[lo:hi].copy())
        try:
            idx = sharded_eviction_select(local, k, lo, scores.size,
                                          local_candidates=_oracle_local, merge=_oracle_merge)
            q.put((rank, "ok", idx.numpy()))
        except Exception as exc:  # the survivor of "die" lands here
            q.put((rank, "error", type(exc).__name__))
        dist.destroy_process_group()
    except Exception:
        q.put((rank, "crash", traceback.format_exc()))


def _run(world, mode, scores, k, timeout=60):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, scores, k, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = []
    expected = world if mode != "die" else world - 1
    for _ in range(expected):
        results.append(q.get(timeout=timeout))
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return sorted(results, key=lambda r: r[0])


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_eviction_matches_global_selection(world):
    from oracle import oracle as O
    from pagedkv_fusion import problems
    rec, freq, att, msk = problems.eviction_problem(seed=0, num_blocks=3001, ties=True)
    scores = O.eviction_scores(rec, freq, att, msk)
    for k in (1, 450, 3001):
        want = O.select_eviction_candidates(scores, k)
        res = _run(world, "ok", scores, k)
        assert [r[1] for r in res] == ["ok"] * world, res
        for _, _, got in res:
            np.testing.assert_array_equal(got, want)


def test_rank_failure_surfaces_as_error_not_hang():
    from oracle import oracle as O
    scores = O.eviction_scores(*__import__("pagedkv_fusion.problems", fromlist=["x"])
                               .eviction_problem(seed=1, num_blocks=500))
    res = _run(2, "die", scores, 50, timeout=90)
    assert res[0][0] == 0 and res[0][1] == "error", res


def test_shard_block_range_covers_everything():
    from pagedkv_fusion.distributed import shard_block_range
    for n in (0, 1, 7, 16384, 16385):
        for w in (1, 2, 3, 8):
            ranges = [shard_block_range(n, r, w) for r in range(w)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [hi - lo for lo, hi in ranges]
            assert max(sizes) - min(sizes) <= 1


def test_decode_partition_is_balanced_and_complete():
    from pagedkv_fusion import problems
    from pagedkv_fusion.distributed import shard_sequences
    lens = problems.large_head_seq_lens(0)
    assert lens.min() >= 1024 and lens.max() <= 8192 and (lens % 16 == 0).all()
    for w in (1, 2, 4, 8):
        shards = shard_sequences(lens, w)
        allidx = np.sort(np.concatenate(shards))
        np.testing.assert_array_equal(allidx, np.arange(lens.size))
        loads = [int(lens[s].sum()) for s in shards]
        assert max(loads) - min(loads) <= int(lens.max())
