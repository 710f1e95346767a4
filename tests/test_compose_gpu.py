"""The evict -> quantize -> decode composition on the GPU, stage by stage
and whole, against the oracle: masks, compacted tables and lengths, int8
codes / scales and evicted ids bit-exact; the decode output within the
attention tolerance of the double-precision C oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import c_oracle
from oracle import oracle as O
from pagedkv_fusion import problems

pytestmark = pytest.mark.gpu

ATTN_RTOL = ATTN_ATOL = 2e-4
ATTN_MAXREL = 1e-3


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def assert_attention_close(got, want):
    got = got.cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=ATTN_RTOL, atol=ATTN_ATOL)
    assert float(np.abs(got - want).max()) / max(float(np.abs(want).max()), 1e-30) <= ATTN_MAXREL


def test_mark_blocks(cuda):
    rng = np.random.default_rng(0)
    ids = rng.integers(-5, 3000, size=700).astype(np.int64)
    for off, nb in ((0, 3000), (1000, 1000), (2990, 4), (5000, 10)):
        got = cuda.mark_blocks(dev(ids), off, nb).cpu().numpy()
        assert np.array_equal(got, O.mark_blocks(ids, off, nb))
    assert cuda.mark_blocks(dev(np.zeros(0, np.int64)), 0, 7).cpu().numpy().sum() == 0


@pytest.mark.parametrize("seed,frac", [(0, 0.15), (1, 0.5), (2, 0.0), (3, 1.0)])
def test_compact_block_tables(cuda, seed, frac):
    prob = problems.composition_problem(seed, num_seqs=70, lo=0, hi=700)
    bt, sl = prob[7], prob[8]
    nb, bs = prob[1].shape[0], prob[1].shape[1]
    ev = (np.random.default_rng(50 + seed).random(nb) < frac).astype(np.uint8)
    tables, lens = cuda.compact_block_tables(dev(bt), dev(sl), dev(ev), nb, bs)
    want_t, want_l = O.compact_block_tables(bt, sl, ev, bs)
    assert np.array_equal(tables.cpu().numpy(), want_t)
    assert np.array_equal(lens.cpu().numpy(), want_l)


def test_compact_keeps_foreign_ids_and_reports_overlong(cuda):
    bt = np.array([[4, 7, -1], [2, 99, 5], [1, 3, 6]], dtype=np.int32)
    sl = np.array([40, 48, 100], dtype=np.int32)  # row 2 needs 7 pages, has 3
    ev = np.zeros(10, np.uint8)
    ev[[7, 3]] = 1
    cuda.read_device_error(reset=True)
    tables, lens = cuda.compact_block_tables(dev(bt), dev(sl), dev(ev), 10, 16)
    assert cuda.read_device_error(reset=True) == 4  # PKV_DEVERR_SEQ_TOO_LONG
    want_t, want_l = O.compact_block_tables(bt, sl, ev, 16)
    assert np.array_equal(tables.cpu().numpy(), want_t)
    assert np.array_equal(lens.cpu().numpy(), want_l)
    assert list(want_l) == [24, 48, 32]


@pytest.mark.parametrize("head_dim,dtype", [(128, torch.float16), (128, torch.float32),
                                            (64, torch.float16), (128, torch.bfloat16)])
def test_quantize_except_leaves_skipped_blocks(cuda, head_dim, dtype):
    rng = np.random.default_rng(head_dim)
    x = torch.from_numpy(rng.standard_normal((37, 16, 4, head_dim), dtype=np.float32)).to(dtype)
    skip = (rng.random(37) < 0.4).astype(np.uint8)
    xq = torch.full(x.shape, 77, dtype=torch.int8, device="cuda")
    xs = torch.full((37, 4), 3.0, dtype=torch.float32, device="cuda")
    cuda.quantize_kv_per_block_except(x.cuda(), dev(skip), xq, xs)
    wq, ws = O.quantize_kv_per_block(x.float().numpy())
    gq, gs = xq.cpu().numpy(), xs.cpu().numpy()
    keep = skip == 0
    assert np.array_equal(gq[keep], wq[keep])
    assert np.array_equal(gs[keep].view(np.uint32), ws[keep].view(np.uint32))
    assert (gq[~keep] == 77).all() and (gs[~keep] == 3.0).all()


@pytest.mark.parametrize("seed,frac,heads", [(0, 0.15, 8), (1, 0.4, 8), (2, 0.0, 8),
                                             (3, 0.15, 32), (4, 1.0, 8)])
def test_evict_quantize_decode_matches_oracle(cuda, seed, frac, heads):
    from pagedkv_fusion.compose import STAGES, evict_quantize_decode
    (q, k, v, rec, freq, att, val, bt, sl, sm) = problems.composition_problem(
        seed, num_seqs=24, lo=1, hi=900, heads=heads, kv_heads=8)
    nb = k.shape[0]
    n_ev = int(frac * nb)
    events = []
    out, ids, tables, lens = evict_quantize_decode(
        dev(q), dev(k), dev(v), dev(rec), dev(freq), dev(att), dev(val), dev(bt), dev(sl),
        n_ev, sm, events=events)
    torch.cuda.synchronize()
    assert len(events) == len(STAGES) + 1
    want_out, want_ids, want_t, want_l = O.evict_quantize_decode(
        q, k, v, rec, freq, att, val, bt, sl, n_ev, sm)
    assert np.array_equal(ids.cpu().numpy(), want_ids)
    assert np.array_equal(tables.cpu().numpy(), want_t)
    assert np.array_equal(lens.cpu().numpy(), want_l)
    kq, ks = O.quantize_kv_per_block(k.astype(np.float32))
    vq, vs = O.quantize_kv_per_block(v.astype(np.float32))
    assert_attention_close(out, c_oracle.paged_attention(q, kq, ks, vq, vs, want_t, want_l, sm))
    if n_ev == nb:
        assert (lens.cpu().numpy() == 0).all() and (out.cpu().numpy() == 0).all()


@pytest.mark.parametrize("heads,dtype", [(8, torch.float16), (2, torch.bfloat16),
                                         (4, torch.float32), (9, torch.float16)])
def test_quantize_bulk_and_register_paths_agree(cuda, monkeypatch, heads, dtype):
    """The bulk-staged kernel (whole blocks through shared memory) and the
    register kernel give the same codes and scales, with and without a skip
    mask, and both match the oracle."""
    rng = np.random.default_rng(heads)
    x = torch.from_numpy(rng.standard_normal((301, 16, heads, 128), dtype=np.float32))
    x[5, 3, 0, 7] = 1e4  # an outlier block-head
    x = x.to(dtype).cuda()
    skip = dev((rng.random(301) < 0.2).astype(np.uint8))
    res = []
    for register in (False, True):
        if register:
            monkeypatch.setenv("PKV_QUANTIZE_REGISTER", "1")
        q0, s0 = cuda.quantize_kv_per_block(x)
        q1 = torch.zeros_like(q0)
        s1 = torch.zeros_like(s0)
        cuda.quantize_kv_per_block_except(x, skip, q1, s1)
        res.append((q0.cpu(), s0.cpu(), q1.cpu(), s1.cpu()))
    for a, b in zip(res[0], res[1]):
        assert torch.equal(a, b)
    wq, ws = O.quantize_kv_per_block(x.float().cpu().numpy())
    assert np.array_equal(res[0][0].numpy(), wq)
    assert np.array_equal(res[0][1].numpy().view(np.uint32), ws.view(np.uint32))


def _half_integer_block(rng, amax, heads):
    """A [1, 16, heads, 128] block whose values sit at, and a few ulps around,
    (k + 0.5) * scale for scale = fl(amax / 127): the inputs where rounding
    x / scale to an integer is decided in the last bits."""
    s = np.float32(amax) / np.float32(127)
    vals = []
    for k in range(-127, 127):
        c = np.float32((k + 0.5) * np.float64(s))
        for d in range(-3, 4):
            v = c
            for _ in range(abs(d)):
                v = np.nextafter(v, np.float32(np.inf if d > 0 else -np.inf), dtype=np.float32)
            vals.append(v)
    vals = np.array(vals, dtype=np.float32)
    x = rng.choice(vals, size=(1, 16, heads, 128)).astype(np.float32)
    x = np.clip(x, -np.float32(amax), np.float32(amax))
    x[0, 0, :, 0] = np.float32(amax)  # pins absmax (and so the scale) per head
    return x


@pytest.mark.parametrize("register", [False, True])
def test_quantize_rounding_window_and_special_values(cuda, monkeypatch, register):
    if register:
        monkeypatch.setenv("PKV_QUANTIZE_REGISTER", "1")
    rng = np.random.default_rng(7)
    blocks = [_half_integer_block(rng, a, 4)
              for a in (1.0, 3.7, 1e-3, 250.0, 6.1e4, 1e-38, 3e-39, 1e30)]
    special = rng.standard_normal((3, 16, 4, 128)).astype(np.float32)
    special[0, 2, 1, 5] = np.nan
    special[1, 7, 2, 9] = np.inf
    special[2, 0, 3, :] = -0.0
    x = np.concatenate(blocks + [special])
    got_q, got_s = cuda.quantize_kv_per_block(dev(x))
    want_q, want_s = O.quantize_kv_per_block(x)
    fin = np.isfinite(x).reshape(x.shape[0], -1, 4, 128).all(axis=(1, 3))  # per block-head
    gq = got_q.cpu().numpy()
    for b in range(x.shape[0]):
        for h in range(4):
            if fin[b, h]:
                assert np.array_equal(gq[b, :, h], want_q[b, :, h]), (b, h)
    assert np.array_equal(got_s.cpu().numpy().view(np.uint32), want_s.view(np.uint32))


def test_report_sections(cuda, tmp_path):
    """The memory / quality / speed report runs on the native kernels and
    emits the reference driver's keys; INT8 error against fp32 attention is
    what per-block INT8 K/V costs (well under the output spread)."""
    from pagedkv_fusion import report
    out = tmp_path / "r.json"
    assert report.main(["--out", str(out), "--speed-iters", "2"]) == 0
    import json
    rep = json.loads(out.read_text())
    assert set(rep) == {"memory", "quality", "speed"}
    for row in rep["quality"]:
        assert set(row) == {"distribution", "rmse", "max_abs", "out_std"}
        assert row["rmse"] < 0.05 * row["out_std"]
    for row in rep["speed"]:
        assert {"num_seqs", "seq_len", "int8_kernel_p50_ms", "fp16_sdpa_gathered_p50_ms"} <= set(row)


@pytest.mark.parametrize("dtype,bs,heads,warp_path", [
    # bulk-streamed path (blocks <= 32 KB, KV heads dividing 8)
    (torch.float16, 16, 8, False), (torch.float32, 16, 4, False), (torch.bfloat16, 16, 2, False),
    (torch.float16, 32, 4, False), (torch.float16, 16, 1, False),
    # one warp per (block, head) from global memory: other shapes, or forced
    (torch.float16, 16, 8, True), (torch.float32, 16, 3, False), (torch.bfloat16, 32, 8, False),
    (torch.float16, 32, 40, False)])
def test_attention_stats_match_oracle(cuda, monkeypatch, dtype, bs, heads, warp_path):
    """Key-derived attention statistics (the eviction score's attention
    input) against the float64 restatement; then fed to the fused scorer."""
    if warp_path:
        monkeypatch.setenv("PKV_ATTN_STATS_WARP", "1")
    rng = np.random.default_rng(heads + bs)
    nb = 777
    k = torch.from_numpy(rng.standard_normal((nb, bs, heads, 128), dtype=np.float32)).to(dtype)
    q = rng.standard_normal((heads, 128)).astype(np.float32)
    got = cuda.attention_stats(k.cuda(), dev(q), 1 / np.sqrt(128)).cpu().numpy()
    want = O.attention_stats(k.float().numpy(), q, 1 / np.sqrt(128))
    np.testing.assert_allclose(got, want, rtol=2e-5, atol=1e-7)
    assert (got > 0).all() and (got <= 1).all()
    # the statistics are a valid input to the bit-exact eviction scorer
    rec = rng.random(nb, dtype=np.float32)
    freq = rng.random(nb, dtype=np.float32)
    valid = np.ones((nb, bs), bool)
    scores = cuda.eviction_scores(dev(rec), dev(freq), dev(got), dev(valid)).cpu().numpy()
    assert np.array_equal(scores.view(np.uint32),
                          O.eviction_scores(rec, freq, got, valid).view(np.uint32))
