"""Public operator API -- same entry points as the reference's
``pagedkv_fusion/ops.py`` (ops.py:40-141), with one execution path.

The reference dispatches to its CUDA extension when every input is a CUDA
tensor and otherwise falls back to NumPy.  Here every call runs the sm_100a
kernels of ``libpagedkv_sm100.so``:

* CUDA tensors are used in place (outputs stay on the device, work is
  enqueued on the current stream, nothing synchronizes);
* host inputs (NumPy arrays or CPU tensors) are copied to the current CUDA
  device, processed there, and the result is returned in the caller's
  container type after one device-to-host copy -- the same return types as
  the reference's fallback, without a CPU implementation behind them.

There is no CPU fallback: without the library or without a CUDA device the
call raises ``RuntimeError``.
"""

from __future__ import annotations

from typing import Any

import numpy as np
import torch

try:
    from pagedkv_fusion import _C  # type: ignore[attr-defined]
    _IMPORT_ERROR: Exception | None = None
except ImportError as exc:  # pragma: no cover - exercised only without a build
    _C = None
    _IMPORT_ERROR = exc

__all__ = [
    "backend_in_use",
    "eviction_scores",
    "select_eviction_candidates",
    "eviction_scores_and_candidates",
    "EvictionPlan",
    "attention_stats",
    "quant_paged_attention",
    "DecodePlan",
]


def backend_in_use() -> str:
    """'cuda' when the native library is loaded (reference ops.py:40-42)."""
    return "cuda" if _C is not None else "unavailable"


_DEVICE_OK = False


def _lib():
    global _DEVICE_OK
    if _C is None:
        raise RuntimeError(f"pagedkv_fusion native library unavailable: {_IMPORT_ERROR}")
    if not _DEVICE_OK:
        if not torch.cuda.is_available():
            raise RuntimeError("pagedkv_fusion requires a CUDA device (sm_100a); none is visible")
        _DEVICE_OK = True
    return _C


def _all_cuda(*args) -> bool:
    for a in args:
        if not (isinstance(a, torch.Tensor) and a.is_cuda):
            return False
    return True


class _Staging:
    """Moves host inputs to the current CUDA device and results back."""

    def __init__(self, *args: Any):
        self.device = next((a.device for a in args if isinstance(a, torch.Tensor) and a.is_cuda),
                           torch.device("cuda", torch.cuda.current_device()))
        self.host_kind = None
        for a in args:
            if isinstance(a, torch.Tensor) and not a.is_cuda:
                self.host_kind = self.host_kind or ("torch", a.device)
            elif not isinstance(a, torch.Tensor):
                self.host_kind = self.host_kind or ("numpy", None)

    def to_device(self, a: Any, dtype: torch.dtype | None = None) -> torch.Tensor:
        t = a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(a))
        if dtype is not None and t.dtype != dtype:
            t = t.to(dtype)
        if not t.is_cuda:
            t = t.to(self.device, non_blocking=t.is_pinned())
        return t

    def back(self, t: torch.Tensor):
        if self.host_kind is None:
            return t
        # pinned destination, asynchronous copy, then wait on this stream only
        host = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        host.copy_(t, non_blocking=True)
        torch.cuda.current_stream(t.device).synchronize()
        if self.host_kind[0] == "numpy":
            return host.numpy()
        return host


# ---------------------------------------------------------------------------
# Eviction scoring and selection
# ---------------------------------------------------------------------------

def eviction_scores(recency, frequency, attn_weights, valid_mask, w_recency: float = 0.4,
                    w_frequency: float = 0.3, w_attention: float = 0.3):
    """Fused eviction score per KV block (lower = evict first).

    Semantics of ``eviction_scores_ref`` (reference.py:38-71), bit for bit.
    """
    C = _lib()
    if _all_cuda(recency, frequency, attn_weights, valid_mask):
        return C.eviction_scores(recency, frequency, attn_weights, valid_mask, w_recency,
                                 w_frequency, w_attention)
    st = _Staging(recency, frequency, attn_weights, valid_mask)
    out = C.eviction_scores(st.to_device(recency, torch.float32),
                            st.to_device(frequency, torch.float32),
                            st.to_device(attn_weights, torch.float32),
                            st.to_device(valid_mask, torch.bool),
                            w_recency, w_frequency, w_attention)
    return st.back(out)


def select_eviction_candidates(scores, k: int):
    """Indices (int64) of the k lowest-scoring blocks, ascending by score,
    ties by lower block id (reference.py:74-81).

    Unlike the reference's GPU branch (``torch.topk``, ops.py:97-98) the tie
    order is deterministic and identical to the NumPy reference.
    """
    C = _lib()
    if _all_cuda(scores):
        return C.eviction_select(scores, int(k))
    st = _Staging(scores)
    return st.back(C.eviction_select(st.to_device(scores, torch.float32), int(k)))


def eviction_scores_and_candidates(recency, frequency, attn_weights, valid_mask, k: int,
                                   w_recency: float = 0.4, w_frequency: float = 0.3,
                                   w_attention: float = 0.3):
    """``(scores, indices)`` from one native call: the composition
    ``select_eviction_candidates(eviction_scores(...), k)``."""
    C = _lib()
    if _all_cuda(recency, frequency, attn_weights, valid_mask):
        return C.eviction_scores_select(recency, frequency, attn_weights, valid_mask, int(k),
                                        w_recency, w_frequency, w_attention)
    st = _Staging(recency, frequency, attn_weights, valid_mask)
    scores, idx = C.eviction_scores_select(st.to_device(recency, torch.float32),
                                           st.to_device(frequency, torch.float32),
                                           st.to_device(attn_weights, torch.float32),
                                           st.to_device(valid_mask, torch.bool), int(k),
                                           w_recency, w_frequency, w_attention)
    return st.back(scores), st.back(idx)


def attention_stats(k, q, sm_scale: float):
    """Per-token attention weights of a key pool for the eviction score
    (``attn_weights``): mean over KV heads of exp(s - max s) with
    s = sm_scale * q_h . K[b, t, h].  ``k`` ``[nb, bs, Hkv, 128]``, ``q``
    ``[Hkv, 128]``; returns float32 ``[nb, bs]`` in (0, 1]."""
    C = _lib()
    if _all_cuda(k, q):
        return C.attention_stats(k, q, sm_scale)
    st = _Staging(k, q)
    kd = k if isinstance(k, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(k))
    return st.back(C.attention_stats(kd.to(st.device), st.to_device(q, torch.float32), sm_scale))


class EvictionPlan:
    """``eviction_scores_and_candidates`` captured once as a CUDA graph over
    fixed statistics buffers, for a serving loop that updates
    ``recency`` / ``frequency`` / ``attn_weights`` / ``valid_mask`` in place
    each step and then calls :meth:`run`.  A replay skips the per-call
    argument checks, allocations and launch of the eager call; the results
    land in the same ``scores`` / ``indices`` tensors every time.

    The buffers must be CUDA tensors that stay alive (and keep their
    storage) while the plan is used.
    """

    def __init__(self, recency, frequency, attn_weights, valid_mask, k: int,
                 w_recency: float = 0.4, w_frequency: float = 0.3, w_attention: float = 0.3):
        C = _lib()
        if not _all_cuda(recency, frequency, attn_weights, valid_mask):
            raise RuntimeError("EvictionPlan needs CUDA tensors (it binds their storage)")
        self._inputs = (recency, frequency, attn_weights, valid_mask)
        args = (recency, frequency, attn_weights, valid_mask, int(k), w_recency, w_frequency,
                w_attention)
        side = torch.cuda.Stream(device=recency.device)
        side.wait_stream(torch.cuda.current_stream(recency.device))
        with torch.cuda.stream(side):
            C.eviction_scores_select(*args)  # first call: cluster set-up, workspace sizes
        torch.cuda.current_stream(recency.device).wait_stream(side)
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._graph):
            self.scores, self.indices = C.eviction_scores_select(*args)

    def run(self):
        """Replays the capture on the current stream; returns ``(scores, indices)``."""
        self._graph.replay()
        return self.scores, self.indices


# ---------------------------------------------------------------------------
# Quantized paged attention
# ---------------------------------------------------------------------------

def quant_paged_attention(q, k_cache_q, k_scale, v_cache_q, v_scale, block_tables, seq_lens,
                          sm_scale: float):
    """Decode-step paged attention over an INT8 paged KV cache.

    Semantics of ``paged_attention_ref`` (reference.py:140-173); fp32
    accumulation, within 1e-3 relative of the reference.
    """
    C = _lib()
    if _all_cuda(q, k_cache_q, k_scale, v_cache_q, v_scale, block_tables, seq_lens):
        return C.quant_paged_attention(q, k_cache_q, k_scale, v_cache_q, v_scale, block_tables,
                                       seq_lens, sm_scale)
    st = _Staging(q, k_cache_q, k_scale, v_cache_q, v_scale, block_tables, seq_lens)
    out = C.quant_paged_attention(st.to_device(q, torch.float32), st.to_device(k_cache_q),
                                  st.to_device(k_scale, torch.float32), st.to_device(v_cache_q),
                                  st.to_device(v_scale, torch.float32),
                                  st.to_device(block_tables, torch.int32),
                                  st.to_device(seq_lens, torch.int32), sm_scale)
    return st.back(out)


class DecodePlan:
    """``quant_paged_attention`` captured once as a CUDA graph over fixed
    buffers, for a decode loop whose batch shape stays put: each step the
    caller writes the new queries into ``q`` and the new tables / lengths
    into ``block_tables`` / ``seq_lens`` (in place), appends to the caches,
    then calls :meth:`run`.  A replay skips the argument checks, the
    workspace allocation and the host-side launch work of the eager call;
    the output lands in the same ``out`` tensor every time.

    All inputs must be contiguous CUDA tensors that keep their storage while
    the plan is used (``seq_lens`` int32).  The kernel choice is made for
    the capture's shapes; lengths up to ``block_tables``' width are
    handled by the same graph.
    """

    def __init__(self, q, k_cache_q, k_scale, v_cache_q, v_scale, block_tables, seq_lens,
                 sm_scale: float):
        C = _lib()
        bufs = (q, k_cache_q, k_scale, v_cache_q, v_scale, block_tables, seq_lens)
        if not _all_cuda(*bufs):
            raise RuntimeError("DecodePlan needs CUDA tensors (it binds their storage)")
        if not all(t.is_contiguous() for t in bufs):
            raise RuntimeError("DecodePlan needs contiguous tensors (a copy would not be rebound)")
        if q.dtype != torch.float32 or block_tables.dtype != torch.int32 or \
                seq_lens.dtype != torch.int32:
            raise RuntimeError("DecodePlan needs float32 q and int32 block_tables / seq_lens")
        self._inputs = bufs
        args = bufs + (float(sm_scale),)
        dev = q.device
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            C.quant_paged_attention(*args)  # kernel attributes, tensor maps
        torch.cuda.current_stream(dev).wait_stream(side)
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self._graph):
            self.out = C.quant_paged_attention(*args)

    def run(self):
        """Replays the capture on the current stream; returns ``out``."""
        self._graph.replay()
        return self.out
