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


def _coverage(shards, S, Hkv):
    """(sequence, kv head) -> how many ranks hold it."""
    cnt = np.zeros((S, Hkv), dtype=np.int64)
    for sh in shards:
        for s in sh.seqs:
            cnt[s, sh.kv_lo:sh.kv_hi] += 1
    return cnt


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_decode_plan_by_sequence_when_sequences_balance(world):
    """The 512-sequence large-head batch stays sequence-sharded: every
    (sequence, KV head) on exactly one rank, ranks within 2 % of even."""
    from pagedkv_fusion import problems
    from pagedkv_fusion.distributed import plan_decode_shards
    lens = problems.large_head_seq_lens(0)
    shards = plan_decode_shards(lens, 40, 40, world)
    assert len(shards) == world
    assert all(sh.head_split == 1 and (sh.kv_lo, sh.kv_hi) == (0, 40) for sh in shards)
    assert (_coverage(shards, lens.size, 40) == 1).all()
    loads = [sh.tokens(lens) * sh.kv_heads for sh in shards]
    assert max(loads) <= 1.02 * sum(loads) / world


@pytest.mark.parametrize("world", [2, 4, 8])
def test_decode_plan_splits_heads_when_one_sequence_dominates(world):
    """Four sequences of which one holds 53 % of the tokens: sequence
    sharding alone would leave one rank with over half the work, so the
    ranks split the KV heads (40 / world each) and every rank does exactly
    1 / world of the work."""
    from pagedkv_fusion import problems
    from pagedkv_fusion.distributed import plan_decode_shards
    lens = problems.long_context_seq_lens()
    shards = plan_decode_shards(lens, 40, 40, world)
    assert shards[0].head_split == world
    assert (_coverage(shards, lens.size, 40) == 1).all()
    loads = {sh.tokens(lens) * sh.kv_heads for sh in shards}
    assert loads == {int(lens.sum()) * 40 // world}
    # GQA: query heads follow their KV heads
    gq = plan_decode_shards(lens, 32, 8, world)
    for sh in gq:
        assert sh.heads == (sh.kv_lo * 4, sh.kv_hi * 4)


def test_decode_plan_mixed_split_and_uneven_heads():
    """A dominant sequence with KV heads that do not divide by the world
    size: the planner uses the largest head split that divides both (here 2
    of 4 ranks per sequence group) and still covers every (sequence, head)
    once."""
    from pagedkv_fusion.distributed import plan_decode_shards
    lens = np.array([9000, 3000, 2000, 1000, 500], dtype=np.int32)
    shards = plan_decode_shards(lens, 6, 6, 4)
    assert shards[0].head_split == 2
    assert (_coverage(shards, lens.size, 6) == 1).all()
    with pytest.raises(ValueError):
        plan_decode_shards(lens, 6, 4, 2)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_head_and_sequence_shards_reassemble_the_decode(world):
    """Cutting a global cache into the planner's shards, decoding each shard
    with the oracle and stitching the outputs gives the global decode."""
    import torch
    from oracle import oracle as O
    from pagedkv_fusion import problems
    from pagedkv_fusion.distributed import (gather_decode_outputs, local_decode_inputs,
                                            plan_decode_shards)
    rng = np.random.default_rng(world)
    q, k, v, bt, sl, sm = problems.make_paged_kv_problem(rng, 5, 16, 8, 64, 16, 300)
    big = int(np.argmax((bt >= 0).sum(axis=1)))
    sl[:] = np.minimum(sl, 40)
    sl[big] = int((bt[big] >= 0).sum()) * 16  # one long sequence dominates
    kq, ks = O.quantize_kv_per_block(k)
    vq, vs = O.quantize_kv_per_block(v)
    want = O.paged_attention(q, kq, ks, vq, vs, bt, sl, sm)
    shards = plan_decode_shards(sl, 16, 8, world)
    assert shards[0].head_split > 1
    T = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    outs = []
    for sh in shards:
        lq, lk, lks, lv, lvs, lbt, lsl = local_decode_inputs(sh, T(q), T(kq), T(ks), T(vq),
                                                             T(vs), T(bt), T(sl))
        assert lk.shape[2] == sh.kv_heads and lq.shape[1] == sh.kv_heads * 2
        outs.append(T(O.paged_attention(lq.numpy(), lk.numpy(), lks.numpy(), lv.numpy(),
                                        lvs.numpy(), lbt.numpy(), lsl.numpy(), sm)))
    got = gather_decode_outputs(shards, outs, 5, 16).numpy()
    np.testing.assert_allclose(got, want, rtol=1e-6, atol=1e-6)
