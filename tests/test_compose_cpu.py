"""The evict -> quantize -> decode composition's oracle pieces on the CPU:
the table compaction and the mask, checked by properties and against the
pinned oracle functions they are built from."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import ROOT  # noqa: F401  (sets sys.path)
from oracle import oracle as O
from pagedkv_fusion import problems


def _pages(L, bs, M):
    return min((max(L, 0) + bs - 1) // bs, M)


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_compaction_properties(seed):
    prob = problems.composition_problem(seed, num_seqs=9, lo=1, hi=200)
    bt, sl = prob[7], prob[8]
    nb, bs = prob[1].shape[0], prob[1].shape[1]
    rng = np.random.default_rng(100 + seed)
    ev = (rng.random(nb) < 0.3).astype(np.uint8)
    out, lens = O.compact_block_tables(bt, sl, ev, bs)
    for s in range(bt.shape[0]):
        n = _pages(int(sl[s]), bs, bt.shape[1])
        pages = bt[s, :n]
        keep = [p for p in pages if not ev[p]]
        assert list(out[s, :len(keep)]) == keep              # order kept
        assert (out[s, len(keep):] == -1).all()
        last = int(sl[s]) - (n - 1) * bs
        want = sum(bs if i < n - 1 else last for i, p in enumerate(pages) if not ev[p])
        assert lens[s] == want
        assert (len(keep) - 1) * bs < lens[s] <= len(keep) * bs or lens[s] == 0


def test_compaction_identity_and_total_eviction():
    prob = problems.composition_problem(3, num_seqs=5)
    bt, sl = prob[7], prob[8]
    nb, bs = prob[1].shape[0], prob[1].shape[1]
    out, lens = O.compact_block_tables(bt, sl, np.zeros(nb, np.uint8), bs)
    assert np.array_equal(lens, sl)
    for s in range(bt.shape[0]):
        n = _pages(int(sl[s]), bs, bt.shape[1])
        assert np.array_equal(out[s, :n], bt[s, :n]) and (out[s, n:] == -1).all()
    out, lens = O.compact_block_tables(bt, sl, np.ones(nb, np.uint8), bs)
    assert (lens == 0).all() and (out == -1).all()


def test_compaction_clamps_to_table_width_and_keeps_foreign_ids():
    bt = np.array([[4, 7, -1], [2, 99, 5]], dtype=np.int32)
    sl = np.array([40, 48], dtype=np.int32)  # 3 pages each
    ev = np.zeros(10, np.uint8)
    ev[7] = 1
    out, lens = O.compact_block_tables(bt, sl, ev, 16)
    # row 0: page 7 evicted; the last page's id -1 lies outside the mask's
    # range, so it is kept (decode reports it) with its 8 tokens
    assert list(out[0]) == [4, -1, -1] and lens[0] == 16 + 8
    # row 1: 99 is outside the mask: kept; all three pages full
    assert list(out[1]) == [2, 99, 5] and lens[1] == 48
    sl_long = np.array([100, 48], dtype=np.int32)  # beyond the 3-page table
    _, lens = O.compact_block_tables(bt, sl_long, ev, 16)
    assert lens[0] == 16 + 16  # 3 full pages covered, page 7 evicted


def test_mark_blocks_range():
    m = O.mark_blocks(np.array([3, 10, 12, 19, 20, 2], np.int64), 10, 10)
    assert list(np.nonzero(m)[0]) == [0, 2, 9]


def test_composition_without_eviction_is_plain_decode():
    (q, k, v, rec, freq, att, val, bt, sl, sm) = problems.composition_problem(
        5, num_seqs=3, hi=120, head_dim=64)
    out, ids, tables, lens = O.evict_quantize_decode(q, k, v, rec, freq, att, val, bt, sl, 0, sm)
    assert ids.size == 0 and np.array_equal(lens, sl)
    kq, ks = O.quantize_kv_per_block(k)
    vq, vs = O.quantize_kv_per_block(v)
    assert np.array_equal(out, O.paged_attention(q, kq, ks, vq, vs, bt, sl, sm))


def test_composition_evicts_the_lowest_scores():
    (q, k, v, rec, freq, att, val, bt, sl, sm) = problems.composition_problem(
        6, num_seqs=4, hi=150, head_dim=64)
    n_ev = k.shape[0] // 4
    out, ids, tables, lens = O.evict_quantize_decode(q, k, v, rec, freq, att, val, bt, sl,
                                                     n_ev, sm)
    scores = O.eviction_scores(rec, freq, att, val)
    assert np.array_equal(ids, O.select_eviction_candidates(scores, n_ev))
    assert not np.isin(tables[tables >= 0], ids).any()
    assert out.shape == q.shape and np.isfinite(out).all()


def test_report_memory_section_matches_reference_arithmetic():
    """The report's memory rows (pure arithmetic) carry the reference
    driver's keys and values (benchmarks/bench_quant_attention.py:36-56)."""
    from pagedkv_fusion import report
    rows = report.measure_memory([dict(num_blocks=4096, block_size=16, num_kv_heads=8,
                                       head_dim=128)])
    r = rows[0]
    assert set(r) >= {"fp16_MiB", "int8_MiB", "savings_pct", "num_blocks"}
    assert r["fp16_MiB"] == 2 * 4096 * 16 * 8 * 128 * 2 / 2**20
    assert r["int8_MiB"] == (2 * 4096 * 16 * 8 * 128 + 2 * 4096 * 8 * 4) / 2**20
    assert abs(r["savings_pct"] - 100 * (1 - r["int8_MiB"] / r["fp16_MiB"])) < 1e-12


def test_attention_stats_definition_properties():
    rng = np.random.default_rng(9)
    k = rng.standard_normal((40, 16, 4, 128)).astype(np.float16)
    q = rng.standard_normal((4, 128)).astype(np.float32)
    a = O.attention_stats(k, q, 1 / np.sqrt(128))
    assert a.shape == (40, 16) and a.dtype == np.float32
    assert (a > 0).all() and (a <= 1).all()
    # each head's most-attended token contributes exp(0) = 1 to its mean
    s = np.einsum("bthd,hd->bth", k.astype(np.float64), q.astype(np.float64))
    for h in range(4):
        b, t = np.unravel_index(np.argmax(s[:, :, h]), s.shape[:2])
        assert a[b, t] >= 1 / 4 - 1e-7
    # a larger query sharpens the distribution: the mean weight drops
    assert O.attention_stats(k, q * 4, 1 / np.sqrt(128)).mean() < a.mean()


def test_profile_driver_targets_and_no_device():
    """The profiling driver (counterpart of the reference's
    scripts/profile_kernels.py) knows its four targets and refuses to run
    without a device instead of falling back to anything."""
    import torch
    from pagedkv_fusion import profile_kernels as pk
    assert sorted(pk.KERNELS) == ["attention", "eviction", "quantize", "stats"]
    if torch.cuda.is_available():
        pytest.skip("a device is visible")
    with pytest.raises(SystemExit):
        pk.main(["attention", "--num-seqs", "2", "--seq-len", "64"])
