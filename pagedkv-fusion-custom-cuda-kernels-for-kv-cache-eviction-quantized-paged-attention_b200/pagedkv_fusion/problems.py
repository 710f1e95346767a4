"""Seeded synthetic paged-KV problems (shared by tests and the benchmark).

``make_paged_kv_problem`` keeps the signature, defaults and random-stream
order of ``pagedkv_fusion/testing_utils.py:18-52`` in the reference, so the
same seed yields the same arrays: the reference's own test shapes can be
regenerated here and compared with golden outputs recorded from it.

The ``workload_*`` helpers build the named benchmark workloads:

* decode 8 x 512        -- 8 seqs of 512 tokens, 8/8 heads, D=128, bs=16,
                           256 permuted blocks (CPU-runnable case)
* eviction 16K          -- 16,384 blocks of 16 tokens, k = 2,458
* decode heavy 64 x 2K  -- 64 seqs of 2,048 tokens, 8/8 heads, 0.1 % of K
                           entries x10 before quantization
* decode large-head     -- 512 seqs, L ~ U[1024, 8192] (multiple of 16),
                           40/40 heads, ~147K blocks (~24 GB INT8 KV)
* decode long-context    -- 4 seqs of 256K / 128K / 64K / 32K tokens, 40/40
                           heads (the longest holds over half of the
                           tokens: no split by sequence balances ranks)
* evict -> quantize -> decode composition -- 1,024 seqs, L ~ U[4096, 32768]
                           (multiple of 16), 8/8 heads, fp16 K/V, 15 % of
                           the blocks evicted (``composition_seq_lens``;
                           ``composition_problem`` builds small instances)

``device_paged_cache`` builds any of the decode workloads' INT8 caches
directly on a CUDA device (N(0,1) data quantized by the native kernel).
"""

from __future__ import annotations

import math

import numpy as np

__all__ = [
    "make_paged_kv_problem",
    "decode_small_problem",
    "eviction_problem",
    "decode_heavy_tail_problem",
    "large_head_seq_lens",
    "long_context_seq_lens",
    "composition_seq_lens",
    "composition_problem",
    "balanced_shards",
    "device_paged_cache",
]


def make_paged_kv_problem(rng: np.random.Generator, num_seqs: int = 4,
                          num_heads: int = 8, num_kv_heads: int = 4,
                          head_dim: int = 64, block_size: int = 16,
                          max_seq_len: int = 200, kv_scale: float = 1.0):
    """Random decode problem with a shuffled physical block order.

    Returns ``(q, k, v, block_tables, seq_lens, sm_scale)`` with fp32 K/V of
    shape ``[num_blocks, block_size, num_kv_heads, head_dim]``; three spare
    blocks are never referenced.  Same draws, in the same order, as the
    reference generator (testing_utils.py:38-52).
    """
    seq_lens = rng.integers(1, max_seq_len + 1, size=num_seqs).astype(np.int32)
    pages = (seq_lens + block_size - 1) // block_size
    total = int(pages.sum()) + 3
    width = int(pages.max())
    perm = rng.permutation(total)
    tables = np.full((num_seqs, width), -1, dtype=np.int32)
    starts = np.concatenate([[0], np.cumsum(pages)])
    for s in range(num_seqs):
        tables[s, :pages[s]] = perm[starts[s]:starts[s + 1]]
    q = rng.standard_normal((num_seqs, num_heads, head_dim)).astype(np.float32)
    shape = (total, block_size, num_kv_heads, head_dim)
    k = (kv_scale * rng.standard_normal(shape)).astype(np.float32)
    v = (kv_scale * rng.standard_normal(shape)).astype(np.float32)
    return q, k, v, tables, seq_lens, 1.0 / np.sqrt(head_dim)


def decode_small_problem(seed: int = 0):
    """8 seqs x 512 tokens, 8/8 heads, D=128, bs=16 over 256 permuted blocks.

    Returns fp32 ``(q, k, v, block_tables, seq_lens, sm_scale)``.
    """
    rng = np.random.default_rng(seed)
    k = rng.standard_normal((256, 16, 8, 128), dtype=np.float32)
    v = rng.standard_normal((256, 16, 8, 128), dtype=np.float32)
    q = rng.standard_normal((8, 8, 128), dtype=np.float32)
    tables = rng.permutation(256).astype(np.int32).reshape(8, 32)
    seq_lens = np.full(8, 512, dtype=np.int32)
    return q, k, v, tables, seq_lens, 1.0 / math.sqrt(128)


def eviction_problem(seed: int = 0, num_blocks: int = 16384, block_size: int = 16,
                     mask: str = "all", ties: bool = False):
    """Eviction statistics for ``num_blocks`` blocks.

    ``mask='all'`` marks every token valid (the reference benchmark's
    choice, bench_eviction.py:33-36); ``mask='random'`` keeps ~80 % valid
    (tests/test_eviction.py:15).  ``ties=True`` puts attention mass on a
    1/64 grid and recency/frequency on a 1/16 grid, forcing many equal
    scores so the id tie-break is exercised.
    """
    rng = np.random.default_rng(seed)
    recency = rng.random(num_blocks, dtype=np.float32)
    frequency = rng.random(num_blocks, dtype=np.float32)
    attn = rng.random((num_blocks, block_size), dtype=np.float32)
    if mask == "all":
        valid = np.ones((num_blocks, block_size), dtype=bool)
    elif mask == "random":
        valid = rng.random((num_blocks, block_size)) > 0.2
    else:
        raise ValueError(mask)
    if ties:
        attn = (np.floor(attn * 64) / 64).astype(np.float32)
        recency = (np.floor(recency * 16) / 16).astype(np.float32)
        frequency = (np.floor(frequency * 16) / 16).astype(np.float32)
    return recency, frequency, attn, valid


def decode_heavy_tail_problem(seed: int = 0, num_seqs: int = 64, seq_len: int = 2048,
                              heads: int = 8, head_dim: int = 128, block_size: int = 16):
    """64 x 2048 decode with heavy-tailed K (0.1 % of entries x10).

    Outlier recipe as in benchmarks/bench_quant_attention.py:67-70.
    Returns fp32 ``(q, k, v, block_tables, seq_lens, sm_scale)``.
    """
    rng = np.random.default_rng(seed)
    pages = num_seqs * seq_len // block_size
    shape = (pages, block_size, heads, head_dim)
    k = rng.standard_normal(shape, dtype=np.float32)
    v = rng.standard_normal(shape, dtype=np.float32)
    spike = rng.random(shape) < 0.001
    k = np.where(spike, k * np.float32(10), k).astype(np.float32)
    q = rng.standard_normal((num_seqs, heads, head_dim), dtype=np.float32)
    tables = rng.permutation(pages).astype(np.int32).reshape(num_seqs, -1)
    seq_lens = np.full(num_seqs, seq_len, dtype=np.int32)
    return q, k, v, tables, seq_lens, 1.0 / math.sqrt(head_dim)


def large_head_seq_lens(seed: int = 0, num_seqs: int = 512, lo: int = 1024,
                        hi: int = 8192, block_size: int = 16) -> np.ndarray:
    """Sequence lengths uniform in [lo, hi], rounded to multiples of 16."""
    rng = np.random.default_rng(seed)
    raw = rng.uniform(lo, hi, size=num_seqs)
    lens = (np.rint(raw / block_size) * block_size).astype(np.int64)
    return np.clip(lens, lo, hi).astype(np.int32)


def long_context_seq_lens() -> np.ndarray:
    """Four long sequences of 262,144 / 131,072 / 65,536 / 32,768 tokens.
    The longest is 53 % of all tokens, so sharding by sequence alone cannot
    give ranks equal work beyond one GPU."""
    return np.array([262144, 131072, 65536, 32768], dtype=np.int32)


def composition_seq_lens(seed: int = 0, num_seqs: int = 1024, lo: int = 4096,
                         hi: int = 32768, block_size: int = 16) -> np.ndarray:
    """Sequence lengths uniform in [lo, hi], rounded to multiples of 16."""
    return large_head_seq_lens(seed, num_seqs, lo, hi, block_size)


def composition_problem(seed: int = 0, num_seqs: int = 6, lo: int = 1, hi: int = 300,
                        heads: int = 8, kv_heads: int = 8, head_dim: int = 128,
                        block_size: int = 16, spare_blocks: int = 5):
    """A small instance of the evict -> quantize -> decode step.

    Ragged lengths in [lo, hi] (a partial last page is common), a shuffled
    block order with ``spare_blocks`` never-referenced blocks, fp16 K/V
    ~N(0,1) and the eviction statistics of ``eviction_problem``.  Returns
    ``(q, k, v, recency, frequency, attn, valid, block_tables, seq_lens,
    sm_scale)``; K/V are float16 numpy arrays.
    """
    rng = np.random.default_rng(seed)
    seq_lens = rng.integers(lo, hi + 1, size=num_seqs).astype(np.int32)
    pages = (seq_lens + block_size - 1) // block_size
    nb = int(pages.sum()) + spare_blocks
    perm = rng.permutation(nb).astype(np.int32)
    tables = np.full((num_seqs, int(pages.max())), -1, dtype=np.int32)
    starts = np.concatenate([[0], np.cumsum(pages)])
    for s_ in range(num_seqs):
        tables[s_, :pages[s_]] = perm[starts[s_]:starts[s_ + 1]]
    shape = (nb, block_size, kv_heads, head_dim)
    k = rng.standard_normal(shape, dtype=np.float32).astype(np.float16)
    v = rng.standard_normal(shape, dtype=np.float32).astype(np.float16)
    q = rng.standard_normal((num_seqs, heads, head_dim), dtype=np.float32)
    recency = rng.random(nb, dtype=np.float32)
    frequency = rng.random(nb, dtype=np.float32)
    attn = rng.random((nb, block_size), dtype=np.float32)
    valid = rng.random((nb, block_size)) > 0.2
    return (q, k, v, recency, frequency, attn, valid, tables, seq_lens,
            1.0 / math.sqrt(head_dim))


def balanced_shards(seq_lens, world_size: int) -> list[np.ndarray]:
    """Partition sequence indices over ranks, balancing total tokens.

    Greedy longest-processing-time: sequences in descending length go to
    the currently lightest rank (ties to the lower rank).  Each shard is
    returned sorted ascending so a rank's output rows keep global order.
    """
    lens = np.asarray(seq_lens, dtype=np.int64)
    order = sorted(range(len(lens)), key=lambda i: (-int(lens[i]), i))
    loads = [0] * world_size
    shards: list[list[int]] = [[] for _ in range(world_size)]
    for i in order:
        r = min(range(world_size), key=lambda j: (loads[j], j))
        shards[r].append(i)
        loads[r] += int(lens[i])
    return [np.array(sorted(s), dtype=np.int64) for s in shards]


def device_paged_cache(seq_lens, kv_heads: int, num_heads: int, device, seed: int,
                       heavy: bool = False, block_size: int = 16, head_dim: int = 128):
    """An INT8 paged cache for ``seq_lens`` built on a CUDA device.

    K and V are drawn N(0,1) in fp32 chunks of about 1 GB (K entries x10
    with probability 0.001 when ``heavy``, the heavy-tail recipe) and
    quantized per (block, head) by the native kernel straight into the
    cache; the block order is a seeded random permutation, as in the
    reference's generator.  Returns ``(q, k_cache, k_scale, v_cache,
    v_scale, block_tables, num_blocks)`` with ``q`` ``[S, num_heads, D]``
    on the device and ``block_tables`` a host int32 array ``[S, max pages]``
    (-1 padded).
    """
    import torch

    from . import _C
    lens = np.asarray(seq_lens, dtype=np.int64)
    pages = (lens + block_size - 1) // block_size
    nb = int(pages.sum())
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    kc = torch.empty((nb, block_size, kv_heads, head_dim), dtype=torch.int8, device=device)
    vc = torch.empty_like(kc)
    ks = torch.empty((nb, kv_heads), dtype=torch.float32, device=device)
    vs = torch.empty_like(ks)
    chunk = max(1, (1 << 28) // (block_size * kv_heads * head_dim))
    for cache, scale, spiky in ((kc, ks, heavy), (vc, vs, False)):
        for lo in range(0, nb, chunk):
            hi = min(nb, lo + chunk)
            x = torch.randn((hi - lo, block_size, kv_heads, head_dim), generator=g, device=device)
            if spiky:
                spike = torch.rand(x.shape, generator=g, device=device) < 0.001
                x = torch.where(spike, x * 10, x)
            _C.quantize_kv_per_block(x, out_q=cache[lo:hi], out_scale=scale[lo:hi])
            del x
    rng = np.random.default_rng(seed)
    perm = rng.permutation(nb).astype(np.int32)
    bt = np.full((len(lens), max(1, int(pages.max()) if len(lens) else 1)), -1, dtype=np.int32)
    starts = np.concatenate([[0], np.cumsum(pages)])
    for s in range(len(lens)):
        bt[s, :pages[s]] = perm[starts[s]:starts[s + 1]]
    q = torch.randn((len(lens), num_heads, head_dim), generator=g, device=device)
    return q, kc, ks, vc, vs, bt, nb
