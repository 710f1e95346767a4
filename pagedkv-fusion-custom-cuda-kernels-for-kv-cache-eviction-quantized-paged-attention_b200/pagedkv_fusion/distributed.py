"""Multi-GPU partitioning of the two hot paths (one process per GPU).

The reference is single-GPU (integration/vllm/pagedkv_fusion_backend.py:23).
Across the GPUs of one box this build partitions work so that only one step
exchanges data:

* Decode shards by sequence.  ``shard_sequences`` balances total tokens over
  ranks (greedy longest-first); every rank owns its sequences' blocks with a
  local block numbering and decodes them with no communication.
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

from typing import Callable

import numpy as np
import torch
import torch.distributed as dist

from .problems import balanced_shards

__all__ = [
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
