"""Per-(block, head) symmetric INT8 quantization of paged KV caches.

Same functions as the reference's ``pagedkv_fusion/quantize.py`` (:15-36).
``quantize_kv_per_block`` runs one native kernel (absmax, IEEE-divided
scale, round-half-even codes) instead of the reference's ~7 ATen ops and
full-size temporaries; its codes are bit-identical to the NumPy reference.
Host inputs are staged to the current CUDA device and the results are
returned on the caller's device.
"""

from __future__ import annotations

import torch

from . import ops

__all__ = ["quantize_kv_per_block", "dequantize_kv_per_block"]


def quantize_kv_per_block(kv: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantize ``kv [num_blocks, block_size, num_kv_heads, head_dim]``
    (float32 / float16 / bfloat16) to INT8 with per-(block, head) scales.

    Returns ``(q, scale)``: int8 codes of the same shape and float32
    ``[num_blocks, num_kv_heads]`` scales.
    """
    if kv.dim() != 4:
        raise ValueError(f"expected 4D [nb, bs, nkv, hd], got {tuple(kv.shape)}")
    C = ops._lib()
    if kv.is_cuda:
        return C.quantize_kv_per_block(kv)
    src = kv if kv.dtype in (torch.float32, torch.float16, torch.bfloat16) else kv.float()
    dev = torch.device("cuda", torch.cuda.current_device())
    q, scale = C.quantize_kv_per_block(src.to(dev, non_blocking=src.is_pinned()))
    return q.to(kv.device), scale.to(kv.device)


def dequantize_kv_per_block(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`quantize_kv_per_block` (up to rounding error).

    A convenience for inspection; decode never materializes it (the
    attention kernel dequantizes in registers).
    """
    return q.float() * scale[:, None, :, None].float()
