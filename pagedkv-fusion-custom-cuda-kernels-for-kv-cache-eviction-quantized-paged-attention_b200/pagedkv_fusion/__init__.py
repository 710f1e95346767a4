"""PagedKV-Fusion for NVIDIA B200 (sm_100a).

INT8 paged decode attention with per-(block, head) scales, and fused KV
block eviction scoring with deterministic bottom-k selection, behind the
reference package's public API::

    from pagedkv_fusion import ops
    scores = ops.eviction_scores(recency, frequency, attn_weights, valid_mask)
    idx = ops.select_eviction_candidates(scores, k)
    out = ops.quant_paged_attention(q, k_q, k_s, v_q, v_s, block_tables, seq_lens, sm_scale)

    from pagedkv_fusion.quantize import quantize_kv_per_block

All arithmetic runs in hand-written CUDA kernels for sm_100a, loaded from
``lib/libpagedkv_sm100.so`` through ``pagedkv_fusion._C``.
"""

__version__ = "1.0.0"

__all__ = ["__version__"]
