"""Multi-GPU partitioning of the two hot paths (one process per GPU).

The reference is single-GPU (integration/vllm/pagedkv_fusion_backend.py:23).
Across the GPUs of one box this build partitions work so that only one step
exchanges data:

* Decode shards by sequence, and by KV head where sequences alone cannot
  balance the ranks (``plan_decode_shards``).  The ranks form
  ``world / f`` sequence groups of ``f`` ranks each; sequences are spread
  over the groups by tokens (greedy longest-first, ``shard_sequences``) and
  the ``f`` ranks of a group split the KV heads (and their query heads)
  evenly.  ``f`` is the smallest divisor of the world size (and of the KV
  head count) that brings the busiest rank within a tolerance of an even
  share, so a batch of comparable sequences stays sequence-sharded and a
  batch in which one sequence dominates is split by head.  Every rank
  owns its shard's blocks (its heads only) with a local block numbering
  and decodes them with no communication.
* Quantize shards with the blocks it writes (no communication).
* Eviction shards the block pool into contiguous id ranges
  (``shard_block_range``).  Each rank scores its range and keeps its
  min(k, n_local) smallest candidates as 64-bit keys ``orderable(score) <<
  32 | global_id``; one all-gather over NVLink brings every rank's candidates
  to every rank, and each runs the same deterministic merge, so the global
  bottom-k is bit-identical everywhere.  The global answer is a subset of
  the union because every block outside a rank's local bottom-k has at
  least k smaller keys on that rank alone.

``torch.distributed`` (NCCL on GPUs, gloo in the CPU tests) carries the
all-gather; the selection kernels come from ``pagedkv_fusion._C`` unless a
caller passes replacements (the CPU tests pass the oracle's).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import numpy as np
import torch
import torch.distributed as dist

from .problems import balanced_shards

__all__ = [
    "DecodeShard",
    "plan_decode_shards",
    "local_decode_inputs",
    "gather_decode_outputs",
    "shard_sequences",
    "shard_block_range",
    "PAD_KEY",
    "sharded_eviction_select",
]

# Sorts after every real candidate key (real ids are < 2**32 - 1).
PAD_KEY = -1  # int64 bit pattern of 0xFFFF_FFFF_FFFF_FFFF


def shard_sequences(seq_lens, world_size: int) -> list[np.ndarray]:
    """Sequence indices per rank, balanced by total tokens."""
    return balanced_shards(seq_lens, world_size)


@dataclass(frozen=True)
class DecodeShard:
    """One rank's part of a decode step: the sequences ``seqs`` (ascending
    global indices) over the KV heads ``[kv_lo, kv_hi)`` and the query heads
    ``[kv_lo * group, kv_hi * group)`` that attend to them."""

    seqs: np.ndarray
    kv_lo: int
    kv_hi: int
    group: int
    head_split: int  # ranks sharing each sequence group (1: by sequence only)

    @property
    def kv_heads(self) -> int:
        return self.kv_hi - self.kv_lo

    @property
    def heads(self) -> tuple[int, int]:
        return self.kv_lo * self.group, self.kv_hi * self.group

    def tokens(self, seq_lens) -> int:
        return int(np.asarray(seq_lens, dtype=np.int64)[self.seqs].sum())


def plan_decode_shards(seq_lens, num_heads: int, num_kv_heads: int, world_size: int,
                       tolerance: float = 0.02) -> list[DecodeShard]:
    """Decode partition over ``world_size`` ranks: by sequence, and by KV head
    where a sequence dominates.

    For each head split ``f`` (divisors of ``world_size`` that also divide
    ``num_kv_heads``, ascending) the sequences go to ``world_size / f``
    groups by tokens, and a rank's work is its group's tokens times
    ``num_kv_heads / f`` heads.  The first ``f`` whose busiest rank is within
    ``tolerance`` of the even share is used; if none is, the ``f`` with the
    lightest busiest rank (the smaller ``f`` on ties).  Rank ``r`` takes
    group ``r // f`` and head slice ``r % f``.
    """
    if world_size < 1:
        raise ValueError("world_size must be positive")
    if num_kv_heads < 1 or num_heads % num_kv_heads:
        raise ValueError("num_heads must be a positive multiple of num_kv_heads")
    lens = np.asarray(seq_lens, dtype=np.int64)
    ideal = float(lens.sum()) * num_kv_heads / world_size
    best = None
    for f in range(1, world_size + 1):
        if world_size % f or num_kv_heads % f:
            continue
        groups = shard_sequences(lens, world_size // f)
        load = max(int(lens[g].sum()) for g in groups) * (num_kv_heads // f)
        if best is None or load < best[0]:
            best = (load, f, groups)
        if load <= (1.0 + tolerance) * ideal:
            best = (load, f, groups)
            break
    _, f, groups = best
    per = num_kv_heads // f
    group = num_heads // num_kv_heads
    return [DecodeShard(seqs=groups[r // f], kv_lo=(r % f) * per, kv_hi=(r % f + 1) * per,
                        group=group, head_split=f) for r in range(world_size)]


def local_decode_inputs(shard: DecodeShard, q, k_cache, k_scale, v_cache, v_scale,
                        block_tables, seq_lens):
    """A rank's decode inputs cut from a global paged cache: the shard's
    sequences, their pages only (renumbered ``0 .. n-1`` in first-use
    order) and the shard's KV heads / query heads.  Tensors stay on their
    device; ``block_tables`` / ``seq_lens`` may be host or device tensors.
    Returns ``(q, k_cache, k_scale, v_cache, v_scale, block_tables,
    seq_lens)`` ready for ``quant_paged_attention``.  (A serving system
    places each rank's blocks there to begin with; this is for a cache
    that was built on one device.)"""
    dev = k_cache.device
    bs = k_cache.shape[1]
    seqs = torch.as_tensor(shard.seqs, dtype=torch.long)
    bt = torch.as_tensor(block_tables).cpu()[seqs]
    sl = torch.as_tensor(seq_lens).cpu().to(torch.int64)[seqs]
    pages = ((sl.clamp(min=0) + bs - 1) // bs).clamp(max=bt.shape[1] if bt.dim() == 2 else 0)
    cols = torch.arange(bt.shape[1]) if bt.numel() else torch.zeros(0, dtype=torch.long)
    used = cols[None, :] < pages[:, None]
    ids = bt[used].to(torch.int64)
    uniq, inv = torch.unique(ids, return_inverse=True)
    local_bt = torch.full(bt.shape, -1, dtype=torch.int32)
    local_bt[used] = inv.to(torch.int32)
    width = max(1, int(pages.max()) if len(pages) else 1)
    local_bt = local_bt[:, :width].contiguous()
    h0, h1 = shard.heads
    idx = uniq.to(dev)
    cut = lambda c: c.index_select(0, idx)[:, :, shard.kv_lo:shard.kv_hi].contiguous()
    cut_s = lambda s: s.index_select(0, idx)[:, shard.kv_lo:shard.kv_hi].contiguous()
    return (q.index_select(0, seqs.to(q.device))[:, h0:h1].contiguous(), cut(k_cache),
            cut_s(k_scale), cut(v_cache), cut_s(v_scale), local_bt.to(dev),
            sl.to(torch.int32).to(dev))


def gather_decode_outputs(shards: list[DecodeShard], outs, num_seqs: int, num_heads: int):
    """Stitches the ranks' decode outputs (``outs[r]`` of shape
    ``[len(shards[r].seqs), heads of shard r, D]``) into ``[num_seqs,
    num_heads, D]`` on the first output's device.  Outside the timed decode
    path: a caller that needs every output on one device gathers them
    (e.g. with ``all_gather_object`` or point-to-point copies) first."""
    D = outs[0].shape[-1]
    full = torch.zeros((num_seqs, num_heads, D), dtype=outs[0].dtype, device=outs[0].device)
    for sh, o in zip(shards, outs):
        if len(sh.seqs) == 0:
            continue
        h0, h1 = sh.heads
        full[torch.as_tensor(sh.seqs, device=full.device), h0:h1] = o.to(full.device)
    return full


def shard_block_range(num_blocks: int, rank: int, world_size: int) -> tuple[int, int]:
    """Contiguous block-id range ``[lo, hi)`` owned by ``rank``."""
    base, extra = divmod(int(num_blocks), int(world_size))
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def sharded_eviction_select(local_scores: torch.Tensor, k: int, id_offset: int,
                            num_blocks_total: int, group=None,
                            local_candidates: Callable | None = None,
                            merge: Callable | None = None) -> torch.Tensor:
    """Global ``select_eviction_candidates`` over blocks sharded by range.

    ``local_scores`` holds this rank's scores for global ids ``[id_offset,
    id_offset + n_local)``.  Returns the int64 ids of the global k lowest
    (score, id) on every rank.  Every rank must call this with the same
    ``k`` and ``num_blocks_total``.
    """
    if k < 0:
        raise ValueError("k must be non-negative")
    if id_offset + local_scores.numel() > (1 << 32) - 1:
        raise ValueError("global block ids must stay below 2**32 - 1")
    if local_candidates is None or merge is None:
        from . import _C
        local_candidates = local_candidates or _C.eviction_local_candidates
        merge = merge or _C.eviction_merge
    k_eff = min(int(k), int(num_blocks_total))
    keys = local_candidates(local_scores, k_eff, id_offset)
    if keys.numel() < k_eff:  # equal-size all-gather: pad with the largest key
        pad = torch.full((k_eff - keys.numel(),), PAD_KEY, dtype=torch.int64,
                         device=keys.device)
        keys = torch.cat([keys, pad])
    world = dist.get_world_size(group)
    gathered = torch.empty(world * k_eff, dtype=torch.int64, device=keys.device)
    dist.all_gather_into_tensor(gathered, keys, group=group)
    return merge(gathered, k_eff)
