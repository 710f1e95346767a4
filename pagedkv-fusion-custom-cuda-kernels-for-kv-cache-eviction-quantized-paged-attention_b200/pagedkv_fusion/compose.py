"""One serving step that composes the hot paths: score every KV block,
evict the globally lowest-scoring fraction, quantize the surviving blocks
to the paged INT8 cache, and decode over block tables from which the
evicted blocks are removed.

The reference composes these steps only in a demo that scores and selects,
then quantizes every block and decodes over the unchanged tables
(``scripts/run_end_to_end_demo.py:74-116``).  Here eviction takes effect:
each sequence keeps the tokens of its surviving blocks, in order.

Every stage runs on the GPU through the native library; across ranks the
selection is the sharded one of ``pagedkv_fusion.distributed`` (one
all-gather of candidate keys), everything else is rank-local.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _C
from .distributed import sharded_eviction_select

STAGES = ("score", "select", "quantize", "compact", "decode")


def evict_quantize_decode(q, k_src, v_src, recency, frequency, attn_weights, valid_mask,
                          block_tables, seq_lens, num_evict: int, sm_scale: float,
                          k_cache=None, k_scale=None, v_cache=None, v_scale=None,
                          block_offset: int = 0, total_blocks: Optional[int] = None,
                          group=None, events: Optional[list] = None):
    """Runs the composed step on the current CUDA stream.

    ``k_src`` / ``v_src``: this rank's blocks ``[nb, bs, Hkv, D]`` (fp16,
    bf16 or fp32) with global ids ``block_offset + i``; the block tables
    index them locally.  ``recency`` / ``frequency`` ``[nb]``,
    ``attn_weights`` ``[nb, bs]`` float32 and ``valid_mask`` bool are their
    eviction statistics.  ``num_evict`` blocks are evicted out of
    ``total_blocks`` (default: ``nb``, one rank); with ``total_blocks`` the
    selection runs across the ranks of ``group``.  ``k_cache`` ... ``v_scale``
    are the INT8 cache to fill (allocated when None).  ``events``: a list
    that receives one CUDA event before the first stage and one after each
    of ``STAGES``.

    Returns ``(out, evicted_ids, tables, lens)``: the decode output, the
    global ids of the evicted blocks (identical on every rank), and the
    compacted tables / lengths that were decoded.
    """
    nb, bs = attn_weights.shape
    dev = k_src.device

    def mark():
        if events is not None:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            events.append(e)

    if k_cache is None:
        k_cache = torch.empty(k_src.shape, dtype=torch.int8, device=dev)
        v_cache = torch.empty(v_src.shape, dtype=torch.int8, device=dev)
        k_scale = torch.empty(k_src.shape[0], k_src.shape[2], dtype=torch.float32, device=dev)
        v_scale = torch.empty_like(k_scale)
    mark()
    scores = _C.eviction_scores(recency, frequency, attn_weights, valid_mask)
    mark()
    if total_blocks is None:
        ids = _C.eviction_select(scores, num_evict)
    else:
        ids = sharded_eviction_select(scores, num_evict, block_offset, total_blocks, group=group)
    evicted = _C.mark_blocks(ids, block_offset, nb)
    mark()
    _C.quantize_kv_per_block_except(k_src, evicted, k_cache, k_scale)
    _C.quantize_kv_per_block_except(v_src, evicted, v_cache, v_scale)
    mark()
    tables, lens = _C.compact_block_tables(block_tables, seq_lens, evicted, nb, bs)
    mark()
    out = _C.quant_paged_attention(q, k_cache, k_scale, v_cache, v_scale, tables, lens, sm_scale)
    mark()
    return out, ids, tables, lens
