"""Two ranks on two GPUs (NCCL): the sharded eviction exchange with the real
kernels, sequence-sharded decode, and head-sharded decode of a batch in
which one sequence dominates, against the oracle.

Needs two visible GPUs; skips otherwise (the single-GPU suite covers the
kernels, tests/test_distributed_cpu.py the exchange logic on gloo)."""

from __future__ import annotations

import socket
import sys
import traceback
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import PKG, ROOT

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    try:
        for p in (str(PKG), str(ROOT)):
            sys.path.insert(0, p)
        import torch.distributed as dist
        from oracle import oracle as O
        from pagedkv_fusion import _C, problems
        from pagedkv_fusion.distributed import (local_decode_inputs, plan_decode_shards,
                                                shard_block_range, shard_sequences,
                                                sharded_eviction_select)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        # eviction over 3 x 16,384 blocks with forced ties
        n = 3 * 16384
        rec, freq, att, msk = problems.eviction_problem(seed=4, num_blocks=n, ties=True)
        lo, hi = shard_block_range(n, rank, world)
        local = _C.eviction_scores(*(torch.from_numpy(a[lo:hi]).to(dev)
                                     for a in (rec, freq, att, msk)))
        k = int(0.15 * n)
        idx = sharded_eviction_select(local, k, lo, n).cpu().numpy()
        want = O.select_eviction_candidates(O.eviction_scores(rec, freq, att, msk), k)
        ev_ok = bool(np.array_equal(idx, want))
        # decode: 12 sequences sharded by tokens; each rank decodes its own
        qf, kf, vf, bt, sl, sm = problems.make_paged_kv_problem(np.random.default_rng(6), 12, 8,
                                                                8, 128, 16, 900)
        kq, ks = O.quantize_kv_per_block(kf)
        vq, vs = O.quantize_kv_per_block(vf)
        mine = shard_sequences(sl, world)[rank]
        d = [torch.from_numpy(np.ascontiguousarray(a)).to(dev)
             for a in (qf[mine], kq, ks, vq, vs, bt[mine], sl[mine])]
        got = _C.quant_paged_attention(*d, sm).cpu().numpy()
        want_d = O.paged_attention(qf[mine], kq, ks, vq, vs, bt[mine], sl[mine], sm)
        err = float(np.abs(got - want_d).max() / max(np.abs(want_d).max(), 1e-30))
        # decode split by KV head: one long sequence dominates the batch
        rng = np.random.default_rng(8)
        qf, kf, vf, bt, sl, sm = problems.make_paged_kv_problem(rng, 4, 16, 8, 128, 16, 700)
        big = int(np.argmax((bt >= 0).sum(axis=1)))
        sl[:] = np.minimum(sl, 48)
        sl[big] = int((bt[big] >= 0).sum()) * 16
        kq, ks = O.quantize_kv_per_block(kf)
        vq, vs = O.quantize_kv_per_block(vf)
        shards = plan_decode_shards(sl, 16, 8, world)
        sh = shards[rank]
        T = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        local = local_decode_inputs(sh, T(qf), T(kq), T(ks), T(vq), T(vs), T(bt), T(sl))
        got_h = _C.quant_paged_attention(*local, sm).cpu().numpy()
        h0, h1 = sh.heads
        want_h = O.paged_attention(qf, kq, ks, vq, vs, bt, sl, sm)[sh.seqs][:, h0:h1]
        err_h = float(np.abs(got_h - want_h).max() / max(np.abs(want_h).max(), 1e-30))
        head_ok = sh.head_split == world and sh.kv_heads == 8 // world
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ev_ok and head_ok, max(err, err_h)))
    except Exception:
        q.put((rank, "crash", traceback.format_exc()))


def test_two_gpus_sharded_eviction_and_decode():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=300) for _ in procs), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert r[1] != "crash", r[2]
        assert r[1] is True, f"rank {r[0]}: sharded eviction differs from the oracle"
        assert r[2] <= 1e-3, f"rank {r[0]}: decode max rel error {r[2]}"


def _compose_worker(rank, world, port, q):
    try:
        for p in (str(PKG), str(ROOT)):
            sys.path.insert(0, p)
        import torch.distributed as dist
        from oracle import c_oracle
        from oracle import oracle as O
        from pagedkv_fusion import problems
        from pagedkv_fusion.compose import evict_quantize_decode
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=timedelta(seconds=60), device_id=dev)
        # rank r owns an independent problem; global block ids concatenate
        # the ranks' blocks in rank order
        probs = [problems.composition_problem(30 + r, num_seqs=20, lo=1, hi=800)
                 for r in range(world)]
        sizes = [p[1].shape[0] for p in probs]
        offsets = np.concatenate([[0], np.cumsum(sizes)])
        total = int(offsets[-1])
        n_ev = int(0.15 * total)
        (qh, k, v, rec, freq, att, val, bt, sl, sm) = probs[rank]
        d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        out, ids, tables, lens = evict_quantize_decode(
            d(qh), d(k), d(v), d(rec), d(freq), d(att), d(val), d(bt), d(sl), n_ev, sm,
            block_offset=int(offsets[rank]), total_blocks=total)
        scores = np.concatenate([O.eviction_scores(*p[3:7]) for p in probs])
        want_ids = O.select_eviction_candidates(scores, n_ev)
        ids_ok = bool(np.array_equal(ids.cpu().numpy(), want_ids))
        mask = O.mark_blocks(want_ids, int(offsets[rank]), sizes[rank])
        want_t, want_l = O.compact_block_tables(bt, sl, mask, k.shape[1])
        tab_ok = bool(np.array_equal(tables.cpu().numpy(), want_t)
                      and np.array_equal(lens.cpu().numpy(), want_l))
        kq, ks = O.quantize_kv_per_block(k.astype(np.float32))
        vq, vs = O.quantize_kv_per_block(v.astype(np.float32))
        want = c_oracle.paged_attention(qh, kq, ks, vq, vs, want_t, want_l, sm)
        got = out.cpu().numpy()
        err = float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ids_ok and tab_ok, err))
    except Exception:
        q.put((rank, "crash", traceback.format_exc()))


def test_two_gpus_evict_quantize_decode():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_compose_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=300) for _ in procs), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for r in res:
        assert r[1] != "crash", r[2]
        assert r[1] is True, f"rank {r[0]}: evicted ids or compacted tables differ"
        assert r[2] <= 1e-3, f"rank {r[0]}: decode max rel error {r[2]}"
