"""vLLM-shaped decode backend on the native kernels.

Same classes, methods and arguments as the reference's adapter
``integration/vllm/pagedkv_fusion_backend.py`` (:37-123):
``PagedKVFusionMetadata`` (the per-step decode metadata) and
``PagedKVFusionBackend`` with ``write_to_cache``, ``decode_forward`` and
``forward(..., is_prefill=...)``, so a vLLM patch written against the
reference picks this module up unchanged.

What differs is underneath:

* ``write_to_cache`` is one native scatter-quantize (two kernel launches,
  no host synchronization) instead of a Python loop over destination blocks
  with a ``torch.unique`` and per-block indexing; the codes and scales are
  the reference loop's, bit for bit (each call quantizes the tokens it
  writes into one block with one per-(block, head) scale, which replaces
  the block's stored scale).
* ``decode_forward`` runs on views of the ``[2, NB, bs, Hkv, D]`` cache (no
  copies) and reaches the GQA tensor-core kernel for groups of 2/4/8 query
  heads per KV head, so each KV head's pages are read once per group.
* ``capture_decode`` returns an :class:`~pagedkv_fusion.ops.DecodePlan`
  for a CUDA-graph decode loop at a fixed batch shape.

Like the reference, prefill steps go to the fallback backend; ``supports``
tells a caller which decode shapes the kernels take.
"""

from __future__ import annotations

import dataclasses
from typing import Any

import torch

from . import ops

__all__ = ["PagedKVFusionMetadata", "PagedKVFusionBackend"]


@dataclasses.dataclass
class PagedKVFusionMetadata:
    """Decode-step metadata, as vLLM's model runner passes it to attention
    backends (reference ``pagedkv_fusion_backend.py:37-45``)."""

    block_tables: torch.Tensor   # [num_seqs, max_blocks_per_seq] int32, -1 = unused
    seq_lens: torch.Tensor       # [num_seqs] int32
    k_scale: torch.Tensor        # [num_blocks, num_kv_heads] float32
    v_scale: torch.Tensor        # [num_blocks, num_kv_heads] float32


class PagedKVFusionBackend:
    """Opt-in decode attention backend over the INT8 paged cache
    (reference ``pagedkv_fusion_backend.py:48-123``)."""

    supports_prefill = False
    supports_decode = True

    def __init__(self, fallback_backend: Any):
        self.fallback = fallback_backend

    @staticmethod
    def supports(query: torch.Tensor, kv_cache_int8: torch.Tensor) -> bool:
        """Whether the decode kernels take these shapes (the launch checks of
        ``pkv_quant_paged_attention``): float32 ``query [S, H, D]``, int8
        ``kv_cache_int8 [2, NB, bs, Hkv, D]`` with D a multiple of 32 up to
        256, bs <= 64 and H a multiple of Hkv."""
        if query.dim() != 3 or kv_cache_int8.dim() != 5 or kv_cache_int8.shape[0] != 2:
            return False
        _, H, D = query.shape
        _, _, bs, hkv, dk = kv_cache_int8.shape
        return (query.dtype == torch.float32 and kv_cache_int8.dtype == torch.int8
                and dk == D and D % 32 == 0 and 0 < D <= 256 and 0 < bs <= 64
                and hkv > 0 and H % hkv == 0)

    def write_to_cache(
        self,
        key: torch.Tensor,            # [num_tokens, num_kv_heads, head_dim]
        value: torch.Tensor,
        kv_cache_int8: torch.Tensor,  # [2, num_blocks, block_size, nkv, hd]
        scale_cache: torch.Tensor,    # [2, num_blocks, num_kv_heads]
        slot_mapping: torch.Tensor,   # [num_tokens] -> block * block_size + offset
        block_size: int,
    ) -> None:
        """Quantizes new K/V tokens and scatters them into the paged INT8
        cache in place, on the current stream."""
        ops._lib().write_to_cache(key, value, kv_cache_int8, scale_cache, slot_mapping,
                                  block_size)

    def decode_forward(
        self,
        query: torch.Tensor,          # [num_seqs, num_heads, head_dim]
        kv_cache_int8: torch.Tensor,  # [2, num_blocks, block_size, nkv, hd]
        scale_cache: torch.Tensor,    # [2, num_blocks, num_kv_heads]
        metadata: PagedKVFusionMetadata,
        scale: float,
    ) -> torch.Tensor:
        """Decode-step attention over the INT8 cache: ``[num_seqs,
        num_heads, head_dim]`` float32.  ``metadata.k_scale`` /
        ``v_scale`` are not read: the scales come from ``scale_cache``, as in
        the reference adapter."""
        return ops.quant_paged_attention(
            query,
            kv_cache_int8[0], scale_cache[0],
            kv_cache_int8[1], scale_cache[1],
            metadata.block_tables, metadata.seq_lens,
            scale,
        )

    def capture_decode(
        self,
        query: torch.Tensor,
        kv_cache_int8: torch.Tensor,
        scale_cache: torch.Tensor,
        metadata: PagedKVFusionMetadata,
        scale: float,
    ) -> ops.DecodePlan:
        """``decode_forward`` as a CUDA graph bound to these buffers: update
        ``query`` / ``metadata.block_tables`` / ``metadata.seq_lens`` in
        place (and the cache through :meth:`write_to_cache`), then call the
        plan's ``run()``."""
        return ops.DecodePlan(query, kv_cache_int8[0], scale_cache[0], kv_cache_int8[1],
                              scale_cache[1], metadata.block_tables, metadata.seq_lens, scale)

    def forward(self, *args, is_prefill: bool, **kwargs):
        """Prefill (and a build without the native library) goes to the
        fallback backend; decode runs :meth:`decode_forward`."""
        if is_prefill or ops.backend_in_use() != "cuda":
            return self.fallback.forward(*args, **kwargs)
        return self.decode_forward(*args, **kwargs)
