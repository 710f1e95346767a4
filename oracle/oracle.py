"""CPU oracle for the PagedKV-Fusion hot paths (TEST INFRASTRUCTURE ONLY).

This module restates, in NumPy, the algorithms of the reference package
``pagedkv_fusion/reference.py`` (PagedKV-Fusion v0.1.1).  It exists so that
the CUDA product can be checked on the same seeded inputs; it is never part
of the product path.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` may import it.

Pinning: every function here is checked against golden vectors produced by
importing the reference package itself (``tests/golden/make_golden.py``);
the integer/bit outputs (eviction scores, eviction indices, int8 codes,
scales) must match those vectors bit for bit, attention outputs to 1e-6.

Numerical contract restated from the reference (NumPy >= 1.24 semantics):

* eviction score  (reference.py:38-71)
    a[t]   = attn[b, t] if valid[b, t] else +0.0f
    S      = numpy pairwise float32 sum of a[0:bs]      (reference.py:60)
    mean   = float32(float64(S) / n_valid), 0 if n_valid == 0  (:61-66)
    score  = (f32(w_r*rec) + f32(w_f*freq)) + f32(w_a*mean)     (:67-71)
  where the Python-float weights are rounded to float32 first (NumPy weak
  scalar promotion) and every product / sum is rounded separately (no FMA).
* selection (reference.py:74-81): ascending score, ties by lower block id,
  NaN after every number, -0.0 == +0.0; int64 result of length min(k, n).
* quantization (reference.py:88-105): absmax per (block, head); scale =
  absmax / 127 (float32 IEEE division) or 1.0 when absmax == 0; codes =
  clip(round_half_even(x / scale), -127, 127) as int8.
* paged attention (reference.py:117-173): gather ceil(L/bs) pages through
  the block table, dequantize with the per-(block, head) scale, truncate to
  L tokens, softmax(q.K^T * sm_scale) @ V per query head with GQA mapping
  kv_head = h // (H / Hkv).
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "eviction_scores",
    "select_eviction_candidates",
    "orderable_keys",
    "pack_candidate_keys",
    "merge_candidate_keys",
    "quantize_kv_per_block",
    "dequantize_kv_per_block",
    "paged_attention",
    "dense_attention",
    "write_to_cache",
    "mark_blocks",
    "compact_block_tables",
    "evict_quantize_decode",
    "attention_stats",
]


# ---------------------------------------------------------------------------
# Eviction scoring and selection
# ---------------------------------------------------------------------------

def eviction_scores(recency, frequency, attn_weights, valid_mask,
                    w_recency=0.4, w_frequency=0.3, w_attention=0.3):
    """Per-block eviction score (lower = evict first).

    Restates ``eviction_scores_ref`` (reference.py:38-71).  The masked sum
    is a NumPy float32 reduction over the token axis, which NumPy evaluates
    with its pairwise scheme (8 interleaved accumulators, a fixed tree, then
    a sequential tail; recursive halving above 128 terms).  ``pairwise_sum``
    below spells that order out and the tests check both agree.
    """
    rec = np.ascontiguousarray(recency, dtype=np.float32)
    freq = np.ascontiguousarray(frequency, dtype=np.float32)
    attn = np.ascontiguousarray(attn_weights, dtype=np.float32)
    valid = np.ascontiguousarray(valid_mask, dtype=bool)
    masked = np.where(valid, attn, np.float32(0.0))
    total = masked.sum(axis=1, dtype=np.float32)
    n_valid = valid.sum(axis=1)
    mean = np.zeros_like(total)
    nz = n_valid > 0
    # float64 quotient rounded once to float32 == IEEE float32 division here
    mean[nz] = (total[nz].astype(np.float64) / n_valid[nz]).astype(np.float32)
    wr, wf, wa = np.float32(w_recency), np.float32(w_frequency), np.float32(w_attention)
    return ((wr * rec + wf * freq) + wa * mean).astype(np.float32)


def pairwise_sum(values: np.ndarray) -> np.float32:
    """NumPy's float32 pairwise summation order, written out term by term.

    Used by the tests to document (and pin) the exact order the CUDA kernel
    reproduces; ``eviction_scores`` itself calls NumPy directly.  NumPy's
    ``sum(axis=1)`` adds this value to an output initialised to +0.0, which
    only matters for a row of -0.0 values.
    """
    x = np.asarray(values, dtype=np.float32)
    n = x.shape[0]
    if n < 8:
        acc = np.float32(0.0)
        for v in x:
            acc = np.float32(acc + v)
        return acc
    if n <= 128:
        r = [np.float32(v) for v in x[:8]]
        i = 8
        stop = n - (n % 8)
        while i < stop:
            for j in range(8):
                r[j] = np.float32(r[j] + x[i + j])
            i += 8
        acc = np.float32(np.float32(np.float32(r[0] + r[1]) + np.float32(r[2] + r[3]))
                         + np.float32(np.float32(r[4] + r[5]) + np.float32(r[6] + r[7])))
        while i < n:
            acc = np.float32(acc + x[i])
            i += 1
        return acc
    half = n // 2
    half -= half % 8
    return np.float32(pairwise_sum(x[:half]) + pairwise_sum(x[half:]))


def orderable_keys(scores) -> np.ndarray:
    """Map float32 scores to uint32 keys whose unsigned order is the
    selection order of ``select_eviction_candidates_ref`` (reference.py:80):
    -0.0 is folded onto +0.0 and every NaN maps to the largest key."""
    s = np.ascontiguousarray(scores, dtype=np.float32)
    bits = s.view(np.uint32).copy()
    bits[bits == np.uint32(0x80000000)] = 0
    neg = (bits & np.uint32(0x80000000)) != 0
    keys = np.where(neg, ~bits, bits | np.uint32(0x80000000)).astype(np.uint32)
    keys[np.isnan(s)] = np.uint32(0xFFFFFFFF)
    return keys


def pack_candidate_keys(scores, ids) -> np.ndarray:
    """64-bit candidate keys ``orderable(score) << 32 | id`` (ids < 2**32)."""
    k = orderable_keys(scores).astype(np.uint64)
    return (k << np.uint64(32)) | np.asarray(ids, dtype=np.uint64)


def select_eviction_candidates(scores, k: int) -> np.ndarray:
    """Indices of the k lowest-scoring blocks, ascending by (score, id).

    Restates ``select_eviction_candidates_ref`` (reference.py:74-81) as a
    sort of unique 64-bit keys, which makes the tie rule explicit.
    """
    s = np.ascontiguousarray(scores, dtype=np.float32)
    n = s.shape[0]
    if k < 0:
        raise ValueError("k must be non-negative")
    keys = pack_candidate_keys(s, np.arange(n, dtype=np.uint64))
    order = np.sort(keys)[:min(k, n)]
    return (order & np.uint64(0xFFFFFFFF)).astype(np.int64)


def merge_candidate_keys(keys, k: int) -> np.ndarray:
    """Global selection from gathered 64-bit candidate keys (multi-GPU
    merge): the k smallest keys, returned as int64 block ids."""
    keys = np.sort(np.asarray(keys, dtype=np.uint64))[:k]
    return (keys & np.uint64(0xFFFFFFFF)).astype(np.int64)


# ---------------------------------------------------------------------------
# Per-(block, head) INT8 quantization
# ---------------------------------------------------------------------------

def quantize_kv_per_block(kv):
    """Symmetric per-(block, head) INT8 quantization.

    Restates ``quantize_kv_per_block_ref`` (reference.py:88-105) and its
    torch twin (quantize.py:15-31): fp16/bf16 input is widened to float32
    exactly before any arithmetic.
    """
    x = np.asarray(kv, dtype=np.float32)
    if x.ndim != 4:
        raise ValueError(f"expected [nb, bs, nkv, hd], got {x.shape}")
    absmax = np.abs(x).max(axis=(1, 3)) if x.size else np.zeros(
        (x.shape[0], x.shape[2]), np.float32)
    scale = np.where(absmax > 0, absmax / np.float32(127.0),
                     np.float32(1.0)).astype(np.float32)
    q = np.rint(x / scale[:, None, :, None])
    q = np.clip(q, -127, 127).astype(np.int8)
    return q, scale


def dequantize_kv_per_block(q, scale):
    """Inverse of :func:`quantize_kv_per_block` (reference.py:108-110)."""
    return (np.asarray(q).astype(np.float32)
            * np.asarray(scale, np.float32)[:, None, :, None]).astype(np.float32)


# ---------------------------------------------------------------------------
# Decode-step paged attention
# ---------------------------------------------------------------------------

def dense_attention(q, k, v, sm_scale):
    """Single-token softmax attention over a dense KV with GQA
    (reference.py:117-137), vectorised over query heads."""
    num_heads, head_dim = q.shape
    num_kv_heads = k.shape[1]
    group = num_heads // num_kv_heads
    q = np.asarray(q, dtype=np.float32)
    out = np.empty((num_heads, head_dim), dtype=np.float32)
    for j in range(num_kv_heads):
        # all query heads of KV head j at once: [L, D] @ [D, G]
        qs = q[j * group:(j + 1) * group]
        logits = (k[:, j, :] @ qs.T) * np.float32(sm_scale)          # [L, G]
        logits -= logits.max(axis=0, keepdims=True)
        p = np.exp(logits)
        p /= p.sum(axis=0, keepdims=True)
        out[j * group:(j + 1) * group] = p.T @ v[:, j, :]
    return out


def paged_attention(q, k_cache_q, k_scale, v_cache_q, v_scale,
                    block_tables, seq_lens, sm_scale):
    """Decode attention over the INT8 paged cache (reference.py:140-173).

    A sequence of length 0 yields zeros (the CUDA path's documented
    behaviour; the reference raises on it).  Tokens beyond the block-table
    width are not attended (the reference would index past the table).
    """
    q = np.asarray(q, dtype=np.float32)
    num_seqs = q.shape[0]
    bs = k_cache_q.shape[1]
    out = np.zeros(q.shape, dtype=np.float32)
    for s in range(num_seqs):
        L = min(max(int(seq_lens[s]), 0), block_tables.shape[1] * bs)
        if L == 0:
            continue
        n = (L + bs - 1) // bs
        pages = np.asarray(block_tables[s, :n], dtype=np.int64)
        if (pages < 0).any() or (pages >= k_cache_q.shape[0]).any():
            raise IndexError(f"sequence {s}: block id out of range")
        k = (k_cache_q[pages].astype(np.float32)
             * np.asarray(k_scale, np.float32)[pages][:, None, :, None])
        v = (v_cache_q[pages].astype(np.float32)
             * np.asarray(v_scale, np.float32)[pages][:, None, :, None])
        k = k.reshape(-1, *k.shape[2:])[:L]
        v = v.reshape(-1, *v.shape[2:])[:L]
        out[s] = dense_attention(q[s], k, v, sm_scale)
    return out


# ---------------------------------------------------------------------------
# Cache write (vLLM-shaped backend)
# ---------------------------------------------------------------------------

def write_to_cache(key, value, kv_cache_int8, scale_cache, slot_mapping,
                   block_size):
    """Quantize new tokens and scatter them into the paged INT8 cache.

    Restates ``PagedKVFusionBackend.write_to_cache``
    (integration/vllm/pagedkv_fusion_backend.py:63-95): the tokens of one
    call that land in the same physical block are quantized together as a
    single synthetic block (one scale per head from only those tokens), and
    that scale overwrites ``scale_cache[:, block]``.  Updates in place.
    """
    key = np.asarray(key, dtype=np.float32)
    value = np.asarray(value, dtype=np.float32)
    slots = np.asarray(slot_mapping, dtype=np.int64)
    blocks = slots // block_size
    for b in np.unique(blocks):
        sel = blocks == b
        offs = slots[sel] % block_size
        kq, ks = quantize_kv_per_block(key[sel][None])
        vq, vs = quantize_kv_per_block(value[sel][None])
        kv_cache_int8[0, b, offs] = kq[0]
        kv_cache_int8[1, b, offs] = vq[0]
        scale_cache[0, b] = ks[0]
        scale_cache[1, b] = vs[0]


# ---------------------------------------------------------------------------
# Evict -> quantize -> decode composition.  The reference has no such step:
# its demo (scripts/run_end_to_end_demo.py:74-116) scores and selects, then
# quantizes every block and decodes over the unchanged tables.  These
# functions define the composition the CUDA path implements, built from the
# pinned functions above.
# ---------------------------------------------------------------------------

def mark_blocks(ids, id_offset: int, num_blocks: int) -> np.ndarray:
    """uint8 mask with 1 at id - id_offset for the ids in this range."""
    mask = np.zeros(int(num_blocks), dtype=np.uint8)
    local = np.asarray(ids, dtype=np.int64) - int(id_offset)
    mask[local[(local >= 0) & (local < num_blocks)]] = 1
    return mask


def compact_block_tables(block_tables, seq_lens, evicted, block_size: int):
    """Drops evicted blocks from each sequence's pages, keeping order.

    Page p of the first ceil(L/bs) (clamped to the table width) holds bs
    tokens, the last one the remainder; the kept pages are written in order,
    the rest of the row becomes -1, and the new length is the kept tokens.
    Ids outside the mask's range are kept.
    """
    bt = np.asarray(block_tables, dtype=np.int32)
    S, M = bt.shape
    out = np.full_like(bt, -1)
    lens = np.zeros(S, dtype=np.int32)
    ev = np.asarray(evicted)
    for s in range(S):
        L = max(int(seq_lens[s]), 0)
        pages = min((L + block_size - 1) // block_size, M)
        kept, tokens = 0, 0
        for p in range(pages):
            bid = int(bt[s, p])
            if 0 <= bid < ev.shape[0] and ev[bid]:
                continue
            out[s, kept] = bid
            kept += 1
            tokens += (min(L, pages * block_size) - p * block_size) if p == pages - 1 \
                else block_size
        lens[s] = tokens
    return out, lens


def evict_quantize_decode(q, k, v, recency, frequency, attn_weights, valid_mask,
                          block_tables, seq_lens, num_evict: int, sm_scale):
    """One composed step: score every block, evict the num_evict lowest
    (score, id), quantize the cache, decode over the compacted tables.
    Returns (out, evicted_ids, tables, lens)."""
    scores = eviction_scores(recency, frequency, attn_weights, valid_mask)
    ids = select_eviction_candidates(scores, num_evict)
    mask = mark_blocks(ids, 0, k.shape[0])
    kq, ks = quantize_kv_per_block(k)
    vq, vs = quantize_kv_per_block(v)
    tables, lens = compact_block_tables(block_tables, seq_lens, mask, k.shape[1])
    out = paged_attention(q, kq, ks, vq, vs, tables, lens, sm_scale)
    return out, ids, tables, lens


# ---------------------------------------------------------------------------
# Attention statistics derived from the keys (no reference counterpart: the
# reference's eviction statistics are given arrays, reference.py:38-71).
# Definition of this library, restated here in float64.
# ---------------------------------------------------------------------------

def attention_stats(k, q, sm_scale):
    """attn[b, t] = mean_h exp(s_h[b, t] - max s_h), s_h = sm_scale * q_h . K[b, t, h].

    ``k`` [nb, bs, Hkv, D] (any float dtype), ``q`` [Hkv, D]; float32 [nb, bs].
    """
    kk = np.asarray(k, dtype=np.float64)
    qq = np.asarray(q, dtype=np.float64)
    s = np.einsum("bthd,hd->bth", kk, qq) * float(sm_scale)
    m = s.reshape(-1, s.shape[2]).max(axis=0)
    return np.exp(s - m[None, None, :]).mean(axis=2).astype(np.float32)
