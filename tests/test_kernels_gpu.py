"""CUDA kernels against the oracle on the same seeded inputs.

Restates the reference's GPU gate (tests/test_kernels_gpu.py: same shapes,
rtol/atol 2e-4 for attention) and adds the stricter contract of this build:

* eviction scores and int8 codes / scales bit-exact (compared as bits);
* eviction indices equal to the oracle's, order included, with forced ties,
  NaN / -0.0 / inf, every k from 0 to beyond n;
* attention within 1e-3 of max|ref| (max relative error) and within the
  reference's elementwise rtol/atol 2e-4, on both kernel paths;
* bitwise determinism across runs.

Every test calls through pagedkv_fusion._C / ops, i.e. the C ABI of
libpagedkv_sm100.so.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from conftest import load_golden, sha
from oracle import c_oracle
from oracle import oracle as O
from pagedkv_fusion import problems

pytestmark = pytest.mark.gpu

ATTN_RTOL = 2e-4   # reference gate, tests/test_kernels_gpu.py:84
ATTN_ATOL = 2e-4
ATTN_MAXREL = 1e-3  # max |got - ref| / max |ref|


def bits(a):
    a = a.cpu().numpy() if isinstance(a, torch.Tensor) else a
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def assert_attention_close(got, want):
    got = got.cpu().numpy() if isinstance(got, torch.Tensor) else got
    np.testing.assert_allclose(got, want, rtol=ATTN_RTOL, atol=ATTN_ATOL)
    scale = max(float(np.abs(want).max()), 1e-30)
    assert float(np.abs(got - want).max()) / scale <= ATTN_MAXREL


@pytest.fixture
def rng():
    return np.random.default_rng(42)


# ---------------------------------------------------------------------------
# eviction scores
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("num_blocks,block_size", [(1, 16), (64, 16), (517, 32), (2048, 16)])
def test_eviction_scores_match_reference(cuda, rng, num_blocks, block_size):
    from pagedkv_fusion import ops
    recency = rng.random(num_blocks, dtype=np.float32)
    frequency = rng.random(num_blocks, dtype=np.float32)
    attn = rng.random((num_blocks, block_size), dtype=np.float32)
    mask = rng.random((num_blocks, block_size)) > 0.2
    want = O.eviction_scores(recency, frequency, attn, mask)
    got = ops.eviction_scores(dev(recency), dev(frequency), dev(attn), dev(mask))
    assert got.is_cuda and ops.backend_in_use() == "cuda"
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-5, atol=1e-6)  # reference gate
    np.testing.assert_array_equal(bits(got), bits(want))                      # this build


def test_eviction_scores_golden_block_sizes(cuda):
    ev = load_golden("eviction")
    for bs in (1, 3, 7, 8, 9, 16, 17, 32, 33, 100, 128, 129, 200):
        args = [dev(ev[f"bs{bs}_{n}"]) for n in ("rec", "freq", "attn", "mask")]
        np.testing.assert_array_equal(bits(cuda.eviction_scores(*args)), bits(ev[f"bs{bs}_scores"]))
        np.testing.assert_array_equal(bits(cuda.eviction_scores(*args, 0.7, 0.2, 0.1)),
                                      bits(ev[f"bs{bs}_scores_w"]))


def test_eviction_fully_invalid_blocks(cuda):
    mask = torch.zeros(8, 16, dtype=torch.bool, device="cuda")
    rec, freq = torch.rand(8, device="cuda"), torch.rand(8, device="cuda")
    got = cuda.eviction_scores(rec, freq, torch.rand(8, 16, device="cuda"), mask)
    assert torch.isfinite(got).all()
    want = O.eviction_scores(rec.cpu().numpy(), freq.cpu().numpy(), np.zeros((8, 16), np.float32),
                             np.zeros((8, 16), bool))
    np.testing.assert_array_equal(bits(got), bits(want))


@pytest.mark.parametrize("tag,kw", [("w16k", dict(mask="all")), ("w16k_mask", dict(mask="random")),
                                    ("w16k_ties", dict(mask="all", ties=True))])
def test_eviction_16k_scores_and_selection(cuda, tag, kw):
    ev = load_golden("eviction")
    rec, freq, att, msk = problems.eviction_problem(seed=0, **kw)
    assert sha(rec, freq, att, msk) == str(ev[f"{tag}_digest"])
    d = [dev(rec), dev(freq), dev(att), dev(msk)]
    scores = cuda.eviction_scores(*d)
    np.testing.assert_array_equal(bits(scores), bits(ev[f"{tag}_scores"]))
    for k in (1, 2458, 8192):
        np.testing.assert_array_equal(cuda.eviction_select(scores, k).cpu().numpy(),
                                      ev[f"{tag}_idx_k{k}"])
        s2, idx = cuda.eviction_scores_select(*d, k)
        np.testing.assert_array_equal(bits(s2), bits(ev[f"{tag}_scores"]))
        np.testing.assert_array_equal(idx.cpu().numpy(), ev[f"{tag}_idx_k{k}"])


# ---------------------------------------------------------------------------
# selection
# ---------------------------------------------------------------------------

def test_select_known_answers(cuda):
    ev = load_golden("eviction")
    np.testing.assert_array_equal(cuda.eviction_select(dev(ev["kat_scores"]), 3).cpu().numpy(),
                                  [1, 2, 3])
    sp = dev(ev["special_scores"])
    np.testing.assert_array_equal(cuda.eviction_select(sp, sp.numel()).cpu().numpy(),
                                  ev["special_idx"])
    np.testing.assert_array_equal(cuda.eviction_select(sp, 5).cpu().numpy(), ev["special_idx_k5"])


@pytest.mark.parametrize("n", [1, 2, 3, 5, 100, 2047, 2048, 2049, 4096, 4097, 16384, 70001])
def test_select_sizes_with_ties(cuda, n):
    r = np.random.default_rng(n)
    s = (np.floor(r.random(n) * 37) / 37).astype(np.float32)  # many exact ties
    s[r.random(n) < 0.01] = -0.0
    for k in sorted({0, 1, n // 7, n // 2, n, n + 5}):
        got = cuda.eviction_select(dev(s), k).cpu().numpy()
        np.testing.assert_array_equal(got, O.select_eviction_candidates(s, k))


@pytest.mark.parametrize("dist", ["equal", "two_values", "nan_heavy", "neg_zero", "spread",
                                  "clustered"])
@pytest.mark.parametrize("n", [1, 977, 16384])
def test_select_adversarial_distributions_both_paths(cuda, monkeypatch, dist, n):
    """Single-launch cluster path (n <= 16384) and the multi-kernel sort on
    distributions that defeat key-range bucketing (all keys in one bin)."""
    r = np.random.default_rng(n + len(dist))
    if dist == "equal":
        s = np.full(n, 0.25, np.float32)
    elif dist == "two_values":
        s = np.where(r.random(n) < 0.5, 0.1, 0.7).astype(np.float32)
    elif dist == "nan_heavy":
        s = r.random(n).astype(np.float32)
        s[r.random(n) < 0.6] = np.nan
    elif dist == "neg_zero":
        s = np.where(r.random(n) < 0.5, -0.0, 0.0).astype(np.float32)
    elif dist == "spread":
        s = (r.standard_normal(n) * 1e30).astype(np.float32)
        s[::7] = np.inf
        s[::11] = -np.inf
    else:
        s = (0.5 + r.random(n) * 1e-6).astype(np.float32)
    for k in sorted({1, max(1, n // 7), n}):
        want = O.select_eviction_candidates(s, k)
        np.testing.assert_array_equal(cuda.eviction_select(dev(s), k).cpu().numpy(), want)
        monkeypatch.setenv("PKV_EVICTION_MULTI_KERNEL", "1")
        np.testing.assert_array_equal(cuda.eviction_select(dev(s), k).cpu().numpy(), want)
        monkeypatch.delenv("PKV_EVICTION_MULTI_KERNEL")


def test_fused_eviction_unaligned_rows_and_odd_block_size(cuda):
    """Rows that are not 16-byte aligned take the generic scorer."""
    r = np.random.default_rng(5)
    n, bs = 3000, 16
    big = r.random((n * bs + 1), dtype=np.float32)
    att_d = dev(big)[1:].view(n, bs)          # 4-byte offset: unaligned rows
    att = big[1:].reshape(n, bs)
    msk = r.random((n, bs)) > 0.3
    rec, freq = r.random(n, dtype=np.float32), r.random(n, dtype=np.float32)
    want_s = O.eviction_scores(rec, freq, att, msk)
    s, idx = cuda.eviction_scores_select(dev(rec), dev(freq), att_d, dev(msk), 450)
    np.testing.assert_array_equal(bits(s), bits(want_s))
    np.testing.assert_array_equal(idx.cpu().numpy(), O.select_eviction_candidates(want_s, 450))
    for bs in (7, 33):
        att = r.random((n, bs), dtype=np.float32)
        msk = r.random((n, bs)) > 0.3
        want_s = O.eviction_scores(rec, freq, att, msk)
        s, idx = cuda.eviction_scores_select(dev(rec), dev(freq), dev(att), dev(msk), 999)
        np.testing.assert_array_equal(bits(s), bits(want_s))
        np.testing.assert_array_equal(idx.cpu().numpy(), O.select_eviction_candidates(want_s, 999))


def test_select_rejects_negative_k(cuda):
    with pytest.raises(RuntimeError, match="non-negative"):
        cuda.eviction_select(torch.zeros(4, device="cuda"), -1)


def test_sharded_candidates_merge_to_global_selection(cuda):
    ev = load_golden("eviction")
    s = ev["w16k_ties_scores"]
    k = 2458
    bounds = [0, 4096, 4097, 9000, 16384]
    keys = [cuda.eviction_local_candidates(dev(s[lo:hi]), k, lo)
            for lo, hi in zip(bounds[:-1], bounds[1:])]
    want_keys = [O.pack_candidate_keys(s[lo:hi], np.arange(lo, hi))
                 for lo, hi in zip(bounds[:-1], bounds[1:])]
    for got, want in zip(keys, want_keys):
        np.testing.assert_array_equal(got.cpu().numpy().view(np.uint64), np.sort(want)[:k])
    merged = cuda.eviction_merge(torch.cat(keys), k).cpu().numpy()
    np.testing.assert_array_equal(merged, ev["w16k_ties_idx_k2458"])


# ---------------------------------------------------------------------------
# quantization
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("case", ["rand", "edge", "tie", "f16"])
def test_quantize_golden_bit_exact(cuda, case):
    qz = load_golden("quantize")
    q, s = cuda.quantize_kv_per_block(dev(qz[f"{case}_kv"]))
    np.testing.assert_array_equal(q.cpu().numpy(), qz[f"{case}_q"])
    np.testing.assert_array_equal(bits(s), bits(qz[f"{case}_scale"]))


@pytest.mark.parametrize("shape", [(1, 16, 1, 32), (7, 16, 8, 128), (3, 32, 40, 128),
                                   (5, 16, 3, 100), (2, 8, 2, 3), (257, 16, 8, 128)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_quantize_shapes_and_dtypes(cuda, shape, dtype):
    g = torch.Generator().manual_seed(sum(shape))
    kv = (torch.randn(shape, generator=g) * 4).to(dtype)
    q, s = cuda.quantize_kv_per_block(kv.cuda())
    wq, ws = O.quantize_kv_per_block(kv.float().numpy())
    np.testing.assert_array_equal(q.cpu().numpy(), wq)
    np.testing.assert_array_equal(bits(s), bits(ws))


def test_quantize_heavy_tail_workload_full(cuda):
    # the whole 8,192-block heavy-tailed K cache (134M values), bit for bit
    q, k, v, bt, sl, sm = problems.decode_heavy_tail_problem(0)
    qk, sk = cuda.quantize_kv_per_block(dev(k))
    wq, ws = O.quantize_kv_per_block(k)
    np.testing.assert_array_equal(qk.cpu().numpy(), wq)
    np.testing.assert_array_equal(bits(sk), bits(ws))


def test_quantize_module_mirror(cuda):
    from pagedkv_fusion.quantize import dequantize_kv_per_block, quantize_kv_per_block
    kv = torch.randn(6, 16, 4, 64)
    q, s = quantize_kv_per_block(kv)        # host tensor in, host tensor out
    assert q.device.type == "cpu"
    wq, ws = O.quantize_kv_per_block(kv.numpy())
    np.testing.assert_array_equal(q.numpy(), wq)
    np.testing.assert_allclose(dequantize_kv_per_block(q, s).numpy(),
                               O.dequantize_kv_per_block(wq, ws), rtol=1e-6)


# ---------------------------------------------------------------------------
# paged attention
# ---------------------------------------------------------------------------

def quantized_problem(q, k, v, bt, sl, sm):
    kq, ks = O.quantize_kv_per_block(k)
    vq, vs = O.quantize_kv_per_block(v)
    return q, kq, ks, vq, vs, bt, sl, sm


def run_attention(args):
    from pagedkv_fusion import ops
    q, kq, ks, vq, vs, bt, sl, sm = args
    return ops.quant_paged_attention(dev(q), dev(kq), dev(ks), dev(vq), dev(vs), dev(bt), dev(sl),
                                     sm)


@pytest.mark.parametrize("i", [0, 1, 2, 3])
def test_attention_reference_shapes(cuda, i):
    """The reference gate's four shapes, against the reference's own output."""
    at = load_golden("attention")
    S, H, Hkv, D, bs, L = (int(x) for x in at[f"gpu{i}_shape"])
    prob = problems.make_paged_kv_problem(np.random.default_rng(42), S, H, Hkv, D, bs, L)
    args = quantized_problem(*prob)
    got = run_attention(args)
    assert_attention_close(got, at[f"gpu{i}_out"])
    assert_attention_close(got, c_oracle.paged_attention(*args))


CASES = [
    # (S, H, Hkv, D, bs, max_len, kv_scale)  -- fast path shapes
    (4, 8, 8, 128, 16, 600, 1.0),
    (5, 32, 8, 128, 16, 700, 1.0),    # G=4
    (3, 16, 2, 128, 16, 1500, 1.0),   # G=8, HG=2
    (2, 8, 1, 128, 16, 900, 1.0),     # HG=1, G=8
    (3, 4, 4, 128, 32, 2000, 1.0),    # bs 32
    (6, 40, 40, 128, 16, 1200, 1.0),  # 40 heads (5 groups of 8)
    (4, 24, 12, 128, 16, 777, 3.0),   # G=2, HG=4 of 12
    (3, 6, 6, 128, 16, 300, 0.01),    # tiny values
    # generic path shapes
    (4, 8, 8, 64, 16, 200, 1.0),
    (3, 8, 2, 96, 8, 333, 1.0),
    (2, 4, 4, 256, 16, 700, 1.0),
    (2, 6, 3, 128, 64, 300, 1.0),
    (2, 6, 2, 32, 24, 100, 1.0),      # group 3 (not a power of two)
]


@pytest.mark.parametrize("S,H,Hkv,D,bs,L,scale", CASES)
def test_attention_cases(cuda, S, H, Hkv, D, bs, L, scale):
    prob = problems.make_paged_kv_problem(np.random.default_rng(S * 1000 + H + D + bs), S, H,
                                          Hkv, D, bs, L, kv_scale=scale)
    args = quantized_problem(*prob)
    assert_attention_close(run_attention(args), c_oracle.paged_attention(*args))


def test_attention_forced_generic_path_agrees(cuda, monkeypatch):
    prob = problems.make_paged_kv_problem(np.random.default_rng(9), 4, 8, 8, 128, 16, 900)
    args = quantized_problem(*prob)
    fast = run_attention(args)
    monkeypatch.setenv("PKV_DECODE_GENERIC", "1")
    slow = run_attention(args)
    want = c_oracle.paged_attention(*args)
    assert_attention_close(fast, want)
    assert_attention_close(slow, want)


@pytest.mark.parametrize("ctas", ["1", "3", "7", "64", "500"])
def test_attention_stream_grid_sizes(cuda, monkeypatch, ctas):
    """Persistent stream kernel with few and many CTAs: units straddling
    CTAs, several chunks and several units per CTA, idle CTAs."""
    monkeypatch.setenv("PKV_DECODE_CTAS", ctas)
    for seed, shape in ((11, (5, 8, 8, 128, 16, 1100)), (12, (9, 32, 8, 128, 16, 2500)),
                        (13, (4, 4, 1, 128, 32, 3000))):
        prob = problems.make_paged_kv_problem(np.random.default_rng(seed), *shape)
        args = quantized_problem(*prob)
        assert_attention_close(run_attention(args), c_oracle.paged_attention(*args))


def test_attention_stream_one_sequence_over_all_ctas(cuda):
    """One 12,288-token sequence: every CTA of the persistent grid holds a
    slice of the same units, so the CTA completing a unit merges hundreds of
    partials.  The merge runs in page order whichever CTA arrives last, so
    repeated calls agree bit for bit."""
    prob = problems.make_paged_kv_problem(np.random.default_rng(21), 1, 16, 8, 128, 16, 12288)
    args = quantized_problem(*prob)
    want = c_oracle.paged_attention(*args)
    outs = [run_attention(args) for _ in range(3)]
    assert_attention_close(outs[0], want)
    for o in outs[1:]:
        assert torch.equal(o, outs[0])


def _tc_form(monkeypatch, form):
    """persistent: one KV head per unit, three or four CTAs per SM walking the units
    (the default); split: one CTA per split (both followed by the combine
    kernel); page: whole pages per copy, all KV heads of a sequence in one
    CTA, the stream kernel's scheduling (on request; one launch)."""
    if form == "split":
        monkeypatch.setenv("PKV_DECODE_TC_SPLIT", "1")
    elif form == "page":
        monkeypatch.setenv("PKV_DECODE_TC_PAGES", "1")


@pytest.mark.parametrize("form", ["page", "persistent", "split"])
@pytest.mark.parametrize("group", [2, 4, 8])
@pytest.mark.parametrize("pages", ["auto", "8", "16", "32"])
def test_attention_tensor_core_gqa(cuda, monkeypatch, form, group, pages):
    """GQA groups of 2/4/8 query heads per KV head run on the tcgen05 kernel
    (q.K and p.V as int8 MMAs into tensor memory); ragged lengths, partial
    128-token tiles, one to four tiles per split, several splits; the
    page, persistent and split forms."""
    if pages != "auto":
        monkeypatch.setenv("PKV_DECODE_SPLIT_PAGES", pages)
    _tc_form(monkeypatch, form)
    from pagedkv_fusion import _C
    for seed, S, hkv, L in ((31, 7, 4, 1500), (32, 3, 2, 130), (33, 12, 8, 700), (34, 2, 1, 17)):
        # the page form needs Hkv x (8 / 16 / 24 columns for groups of 2 / 4 / 8)
        # <= 128 accumulator columns; 8 KV heads x groups of 8 stay per head
        cols = hkv * {2: 8, 4: 16, 8: 24}[group]
        want_launches = 1 if form == "page" and cols <= 128 else 2
        assert _C.quant_paged_attention_kernel_launches(S, group * hkv, hkv, 128, 16, 94) == \
            want_launches
        prob = problems.make_paged_kv_problem(np.random.default_rng(seed), S, group * hkv, hkv,
                                              128, 16, L)
        args = quantized_problem(*prob)
        assert_attention_close(run_attention(args), c_oracle.paged_attention(*args))


@pytest.mark.parametrize("form", ["page", "persistent"])
@pytest.mark.parametrize("group", [2, 4, 8])
def test_tensor_core_persistent_merge_edges(cuda, monkeypatch, form, group):
    """The tensor-core path with its combine: sequences without pages (zero
    output) and of one page, a long sequence with many splits whose units
    wrap around the persistent grid, repeated calls bit for bit, and a
    workspace of random bytes."""
    _tc_form(monkeypatch, form)
    r = np.random.default_rng(70 + group)
    hkv = 2
    q, k, v, bt, sl, sm = problems.make_paged_kv_problem(r, 6, group * hkv, hkv, 128, 16, 40000)
    sl[1] = 0
    sl[3] = min(int(sl[3]), 9)
    args = quantized_problem(q, k, v, bt, sl, sm)
    want = c_oracle.paged_attention(*args)
    cuda.read_device_error(reset=True)
    got = run_attention(args)
    assert_attention_close(got, want)
    assert float(got[1].abs().max()) == 0.0
    assert torch.equal(got, run_attention(args))
    S, H = q.shape[0], q.shape[1]
    nbytes = cuda._attn_ws(S, H, hkv, 128, 16, bt.shape[1])
    dargs = [dev(a) for a in args[:7]]
    out = torch.empty_like(dargs[0])
    ws = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device="cuda")
    rc = cuda._attn(*(t.data_ptr() for t in dargs[:7]), out.data_ptr(), S, H, hkv, 128, 16,
                    dargs[1].shape[0], bt.shape[1], float(sm), ws.data_ptr(), ws.numel(),
                    torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    assert torch.equal(out, got)
    assert cuda.read_device_error(reset=True) == 0


@pytest.mark.parametrize("group", [2, 4, 8])
def test_tensor_core_forms_agree_bitwise(cuda, monkeypatch, group):
    """The persistent and split forms run the same arithmetic per unit (same
    MMAs, same epilogue): bit-identical outputs, on a batch that gives every
    persistent CTA several units; the page form within the oracle tolerance."""
    prob = problems.make_paged_kv_problem(np.random.default_rng(90 + group), 40, group * 8, 8,
                                          128, 16, 2000)
    args = quantized_problem(*prob)
    want = c_oracle.paged_attention(*args)
    outs = {}
    for form in ("page", "persistent", "split"):
        with monkeypatch.context() as mp:
            _tc_form(mp, form)
            outs[form] = run_attention(args)
    assert_attention_close(outs["persistent"], want)
    assert torch.equal(outs["persistent"], outs["split"])
    # the page form normalizes per 128-token chunk and merges the chunks
    # online: the same oracle tolerance, not the same bits
    assert_attention_close(outs["page"], want)


def test_attention_tensor_core_matches_cuda_core_path(cuda, monkeypatch):
    """The tensor-core and CUDA-core kernels use the same integer formats:
    their outputs agree to fp32 rounding."""
    prob = problems.make_paged_kv_problem(np.random.default_rng(35), 9, 32, 8, 128, 16, 2100)
    args = quantized_problem(*prob)
    tc = run_attention(args)
    monkeypatch.setenv("PKV_DECODE_TC", "0")
    cc = run_attention(args)
    scale = float(cc.abs().max())
    assert float((tc - cc).abs().max()) / scale < 2e-6


@pytest.mark.parametrize("pages", ["1", "2", "8", "32"])
def test_attention_split_sizes(cuda, monkeypatch, pages):
    monkeypatch.setenv("PKV_DECODE_SPLIT", "1")
    monkeypatch.setenv("PKV_DECODE_SPLIT_PAGES", pages)
    prob = problems.make_paged_kv_problem(np.random.default_rng(11), 5, 8, 8, 128, 16, 1100)
    args = quantized_problem(*prob)
    assert_attention_close(run_attention(args), c_oracle.paged_attention(*args))


def fixed_length_problem(seed, S, H, Hkv, D, bs, L):
    """S sequences of exactly L tokens over shuffled blocks (3 spare)."""
    rng = np.random.default_rng(seed)
    pages = (L + bs - 1) // bs
    perm = rng.permutation(S * pages + 3).astype(np.int32)
    bt = perm[:S * pages].reshape(S, pages)
    q = rng.standard_normal((S, H, D), dtype=np.float32)
    k = rng.standard_normal((S * pages + 3, bs, Hkv, D), dtype=np.float32)
    v = rng.standard_normal((S * pages + 3, bs, Hkv, D), dtype=np.float32)
    return q, k, v, bt, np.full(S, L, np.int32), 1.0 / math.sqrt(D)


def test_attention_edge_lengths(cuda):
    at = load_golden("attention")
    for L in (1, 15, 16, 17):
        rng = np.random.default_rng(int(at[f"edge{L}_seed"]))
        q, k, v, bt, sl, sm = problems.make_paged_kv_problem(rng, 1, 8, 4, 64, 16, L)
        sl[:] = L
        got = run_attention(quantized_problem(q, k, v, bt, sl, sm))
        assert_attention_close(got, at[f"edge{L}_out"])
    # fast path around page and split boundaries
    for L in (1, 15, 16, 17, 511, 512, 513, 4096):
        args = quantized_problem(*fixed_length_problem(L, 2, 8, 8, 128, 16, L))
        assert_attention_close(run_attention(args), c_oracle.paged_attention(*args))


def test_attention_seq_len_beyond_table_is_clamped_and_reported(cuda):
    """seq_len asks for more pages than the table row holds: only the
    covered tokens are attended and PKV_DEVERR_SEQ_TOO_LONG is recorded."""
    for D in (128, 64):  # fast and generic paths
        q, k, v, bt, sl, sm = fixed_length_problem(3, 3, 8, 8, D, 16, 700)
        sl[2] = 5000  # the table covers 704 tokens
        args = quantized_problem(q, k, v, bt, sl, sm)
        cuda.read_device_error(reset=True)
        got = run_attention(args)
        assert cuda.read_device_error(reset=True) == 4
        assert_attention_close(got, O.paged_attention(*args))


def test_attention_zero_length_sequence_gives_zeros(cuda):
    q, k, v, bt, sl, sm = problems.make_paged_kv_problem(np.random.default_rng(5), 3, 8, 8, 128,
                                                         16, 300)
    sl[1] = 0
    args = quantized_problem(q, k, v, bt, sl, sm)
    got = run_attention(args).cpu().numpy()
    assert (got[1] == 0).all()
    assert_attention_close(got, O.paged_attention(*args))


def test_attention_small_decode_workload(cuda):
    at = load_golden("attention")
    prob = problems.decode_small_problem(0)
    args = quantized_problem(*prob)
    assert_attention_close(run_attention(args), at["small_out"])


def test_attention_host_inputs_roundtrip(cuda):
    from pagedkv_fusion import ops
    at = load_golden("attention")
    args = quantized_problem(*problems.decode_small_problem(0))
    got = ops.quant_paged_attention(*args)  # NumPy in, NumPy out, computed on the GPU
    assert isinstance(got, np.ndarray)
    assert_attention_close(got, at["small_out"])


def test_attention_deterministic(cuda):
    args = quantized_problem(*problems.make_paged_kv_problem(np.random.default_rng(42)))
    a, b = run_attention(args), run_attention(args)
    assert torch.equal(a, b)
    args = quantized_problem(*problems.decode_small_problem(0))
    assert torch.equal(run_attention(args), run_attention(args))


@pytest.mark.parametrize("unit_cost,min_pages", [(0, 1), (0, 4), (3, 4), (7, 1), (2, 16), (40, 2)])
@pytest.mark.parametrize("shape", [(37, 1000, 8), (2, 9000, 8), (5, 300, 2)])
def test_stream_share_parameters_match_oracle(cuda, monkeypatch, unit_cost, min_pages, shape):
    """The stream kernel's page shares (a unit's fixed cost counted in pages,
    the fewest pages per CTA) move the CTA boundaries and so the partials
    and merges; every setting stays within the attention tolerance, on
    ragged lengths with empty sequences."""
    S, L, hkv = shape
    r = np.random.default_rng(S * 131 + L)
    q, k, v, bt, sl, sm = problems.make_paged_kv_problem(r, S, hkv, hkv, 128, 16, L)
    sl[::4] = 0                      # sequences without pages
    sl[1::5] = np.minimum(sl[1::5], 16)  # one page or less
    args = quantized_problem(q, k, v, bt, sl, sm)
    want = c_oracle.paged_attention(*args)
    monkeypatch.setenv("PKV_STREAM_UNIT_COST", str(unit_cost))
    monkeypatch.setenv("PKV_STREAM_MIN_PAGES", str(min_pages))
    assert cuda.quant_paged_attention_kernel_launches(S, hkv, hkv, 128, 16, bt.shape[1]) == 1
    cuda.read_device_error(reset=True)
    got = run_attention(args)
    assert_attention_close(got, want)
    assert torch.equal(got, run_attention(args))  # deterministic for a fixed setting
    assert cuda.read_device_error(reset=True) == 0


@pytest.mark.parametrize("ctas", [0, 16, 17, 33, 200])
def test_stream_long_sequence_two_level_merge(cuda, monkeypatch, ctas):
    """One long sequence (778 pages) over many CTAs: more than 16 partials
    per unit merge in two levels (groups of 16, then the groups); grids of
    17 / 33 CTAs leave a group of one.  0 = the default grid."""
    r = np.random.default_rng(321)
    q, k, v, bt, sl, sm = problems.make_paged_kv_problem(r, 1, 8, 8, 128, 16, 32768)
    sl[:] = bt.shape[1] * 16 - 5  # the table's every page, the last one partial
    assert bt.shape[1] > 16 * 16  # enough pages for every grid tried here
    args = quantized_problem(q, k, v, bt, sl, sm)
    want = c_oracle.paged_attention(*args)
    if ctas:
        monkeypatch.setenv("PKV_DECODE_CTAS", str(ctas))
    monkeypatch.setenv("PKV_STREAM_MIN_PAGES", "1")
    cuda.read_device_error(reset=True)
    got = run_attention(args)
    assert_attention_close(got, want)
    assert torch.equal(got, run_attention(args))
    assert cuda.read_device_error(reset=True) == 0


@pytest.mark.parametrize("shape", [(8, 512, 8), (37, 1000, 8), (3, 5000, 4)])
def test_stream_workspace_needs_no_initialisation(cuda, shape):
    """The stream kernel's arrival counters carry a per-launch tag: a
    workspace holding random bytes, or the counters a previous launch left,
    gives the same output, bit for bit, as a fresh one."""
    S, L, hkv = shape
    r = np.random.default_rng(S)
    q, k, v, bt, sl, sm = problems.make_paged_kv_problem(r, S, hkv, hkv, 128, 16, L)
    args = [dev(a) if isinstance(a, np.ndarray) else a for a in quantized_problem(q, k, v, bt, sl, sm)]
    qd, kq, ks, vq, vs, btd, sld, smf = args
    assert cuda.quant_paged_attention_kernel_launches(S, hkv, hkv, 128, 16, bt.shape[1]) == 1
    nbytes = cuda._attn_ws(S, hkv, hkv, 128, 16, bt.shape[1])
    cuda.read_device_error(reset=True)
    want = cuda.quant_paged_attention(*args)

    def call(ws):
        out = torch.empty_like(qd)
        rc = cuda._attn(qd.data_ptr(), kq.data_ptr(), ks.data_ptr(), vq.data_ptr(), vs.data_ptr(),
                        btd.data_ptr(), sld.data_ptr(), out.data_ptr(), S, hkv, hkv, 128, 16,
                        kq.shape[0], bt.shape[1], float(smf), ws.data_ptr(), ws.numel(),
                        torch.cuda.current_stream().cuda_stream)
        assert rc == 0
        return out

    garbage = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, device="cuda")
    assert torch.equal(call(garbage), want)
    ones = torch.full((nbytes,), 0xFF, dtype=torch.uint8, device="cuda")
    assert torch.equal(call(ones), want)
    reused = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    for _ in range(3):  # counters left by the previous launch
        assert torch.equal(call(reused), want)
    assert cuda.read_device_error(reset=True) == 0


def test_attention_bad_block_id_is_reported(cuda):
    q, k, v, bt, sl, sm = problems.make_paged_kv_problem(np.random.default_rng(8), 2, 8, 8, 128,
                                                         16, 64)
    sl[:] = 64
    bt = np.full((2, 4), 0, np.int32)
    bt[1, 2] = 10_000_000  # far outside the cache
    args = quantized_problem(q, k, v, bt, sl, sm)
    cuda.read_device_error(reset=True)
    got = run_attention(args)
    torch.cuda.synchronize()
    assert cuda.read_device_error(reset=True) == 1
    assert torch.isfinite(got).all()
    assert cuda.read_device_error(reset=True) == 0


def test_attention_heavy_tail_workload_sample(cuda):
    """The 64 x 2048 heavy-tailed workload at full size on the GPU, checked
    against the double-precision oracle on all 64 sequences."""
    q, k, v, bt, sl, sm = problems.decode_heavy_tail_problem(0)
    kq_d, ks_d = cuda.quantize_kv_per_block(dev(k))
    vq_d, vs_d = cuda.quantize_kv_per_block(dev(v))
    from pagedkv_fusion import ops
    got = ops.quant_paged_attention(dev(q), kq_d, ks_d, vq_d, vs_d, dev(bt), dev(sl), sm)
    pick = np.arange(64)
    sub_bt = bt[pick]
    used = np.unique(sub_bt)
    remap = np.full(bt.max() + 1, -1, np.int64)
    remap[used] = np.arange(used.size)
    kq, ks = kq_d.cpu().numpy()[used], ks_d.cpu().numpy()[used]
    vq, vs = vq_d.cpu().numpy()[used], vs_d.cpu().numpy()[used]
    want = c_oracle.paged_attention(q[pick], kq, ks, vq, vs, remap[sub_bt].astype(np.int32),
                                    sl[pick], sm)
    assert_attention_close(got.cpu().numpy()[pick], want)
    assert math.isclose(sm, 1 / math.sqrt(128))


def test_write_to_cache_matches_oracle(cuda):
    r = np.random.default_rng(77)
    nb, bs, hkv, hd = 12, 16, 4, 128
    cache = r.integers(-127, 128, (2, nb, bs, hkv, hd)).astype(np.int8)
    scales = r.random((2, nb, hkv)).astype(np.float32)
    key = r.standard_normal((9, hkv, hd)).astype(np.float32)
    val = r.standard_normal((9, hkv, hd)).astype(np.float32)
    slots = np.array([5, 6, 33, 100, 101, 102, 150, 7, 191])
    want_c, want_s = cache.copy(), scales.copy()
    O.write_to_cache(key, val, want_c, want_s, slots, bs)
    dc, ds = dev(cache), dev(scales)
    cuda.write_to_cache(dev(key), dev(val), dc, ds, dev(slots), bs)
    np.testing.assert_array_equal(dc.cpu().numpy(), want_c)
    np.testing.assert_array_equal(bits(ds), bits(want_s))


def test_eviction_plan_replays_match_eager(cuda):
    """The captured score + select replays on updated statistics buffers and
    returns what the eager call returns for the same values."""
    from pagedkv_fusion import ops
    rec, freq, att, msk = problems.eviction_problem(seed=3)
    d = [dev(a) for a in (rec, freq, att, msk)]
    plan = ops.EvictionPlan(*d, 2458)
    for seed in (3, 4, 5):
        new = problems.eviction_problem(seed=seed, mask="random")
        for buf, a in zip(d, new):
            buf.copy_(dev(a))
        scores, idx = plan.run()
        want = O.select_eviction_candidates(O.eviction_scores(*new), 2458)
        assert np.array_equal(idx.cpu().numpy(), want)
        assert np.array_equal(bits(scores), bits(O.eviction_scores(*new)))


def test_eviction_8_cta_cluster_variant(cuda):
    """The one-launch selection pinned to its 8-CTA cluster variant (the
    cluster size is chosen once per process, so this runs in a fresh one):
    scores and indices equal to the golden vectors at 16,384 blocks."""
    import os
    import subprocess
    import sys
    from conftest import PKG, ROOT
    code = r'''
import numpy as np, torch
from conftest import load_golden, sha
from pagedkv_fusion import _C, problems
ev = load_golden("eviction")
for tag, kw in (("w16k", dict(mask="all")), ("w16k_ties", dict(mask="all", ties=True))):
    rec, freq, att, msk = problems.eviction_problem(seed=0, **kw)
    assert sha(rec, freq, att, msk) == str(ev[f"{tag}_digest"])
    d = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (rec, freq, att, msk)]
    for k in (1, 2458, 8192):
        s, idx = _C.eviction_scores_select(*d, k)
        assert np.array_equal(s.cpu().numpy().view(np.uint32), ev[f"{tag}_scores"].view(np.uint32))
        assert np.array_equal(idx.cpu().numpy(), ev[f"{tag}_idx_k{k}"]), (tag, k)
print("ok")
'''
    env = dict(os.environ, PKV_EVICTION_CLUSTER="8")
    env["PYTHONPATH"] = os.pathsep.join([str(ROOT / "tests"), str(PKG), str(ROOT),
                                         env.get("PYTHONPATH", "")])
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr


@pytest.mark.parametrize("dist", ["random", "grid_ties", "equal", "nan_neg_zero"])
@pytest.mark.parametrize("n", [20000, 70001, 1_200_000])
def test_select_large_radix_prefilter(cuda, dist, n):
    """Selections above 16,384 blocks with k well below n take the radix
    prefilter (the k-th key's prefix over up to four 16-bit digits, then only
    the keys at or below it sorted): indices equal to the oracle's, order
    included, through the scores path, the fused path and the merge path."""
    r = np.random.default_rng(n + len(dist))
    if dist == "random":
        s = r.random(n).astype(np.float32)
    elif dist == "grid_ties":
        s = (np.floor(r.random(n) * 64) / 64).astype(np.float32)
    elif dist == "equal":  # one key value: the prefix is found down to the block ids
        s = np.full(n, 0.5, np.float32)
    else:
        s = r.standard_normal(n).astype(np.float32)
        s[r.random(n) < 0.3] = np.nan
        s[r.random(n) < 0.2] = -0.0
        s[r.random(n) < 0.2] = 0.0
    for k in sorted({1, 1000, n // 7, min(n // 5, 177_000), n // 2}):
        want = O.select_eviction_candidates(s, k)
        np.testing.assert_array_equal(cuda.eviction_select(dev(s), k).cpu().numpy(), want)
    k = n // 7
    want = O.select_eviction_candidates(s, k)
    keys = (O.orderable_keys(s).astype(np.uint64) << np.uint64(32)) | np.arange(n, dtype=np.uint64)
    np.testing.assert_array_equal(cuda.eviction_merge(dev(keys.view(np.int64)), k).cpu().numpy(),
                                  want)
    if dist == "random":  # fused scores + select on the same sizes
        rec = r.random(n, dtype=np.float32)
        freq = r.random(n, dtype=np.float32)
        att = r.random((n, 16), dtype=np.float32)
        msk = r.random((n, 16)) > 0.2
        sc = O.eviction_scores(rec, freq, att, msk)
        s2, idx = cuda.eviction_scores_select(dev(rec), dev(freq), dev(att), dev(msk), k)
        np.testing.assert_array_equal(bits(s2), bits(sc))
        np.testing.assert_array_equal(idx.cpu().numpy(), O.select_eviction_candidates(sc, k))


def test_select_without_radix_prefilter(cuda):
    """PKV_EVICTION_RADIX=0 (read once per process, so in a fresh one):
    selections above 16,384 blocks sort every key instead; indices equal
    to the oracle's, scores and merge paths."""
    import os
    import subprocess
    import sys
    from conftest import PKG, ROOT
    code = r'''
import numpy as np, torch
from oracle import oracle as O
from pagedkv_fusion import _C
r = np.random.default_rng(3)
n = 140001
s = (np.floor(r.random(n) * 256) / 256).astype(np.float32)
s[r.random(n) < 0.1] = np.nan
d = torch.from_numpy(s).cuda()
assert _C._select_ws(n, 1000) == (1 << 18) * 8  # the sort keys only
for k in (1, 1000, 20000):
    assert np.array_equal(_C.eviction_select(d, k).cpu().numpy(), O.select_eviction_candidates(s, k)), k
keys = (O.orderable_keys(s).astype(np.uint64) << np.uint64(32)) | np.arange(n, dtype=np.uint64)
got = _C.eviction_merge(torch.from_numpy(keys.view(np.int64)).cuda(), 20000).cpu().numpy()
assert np.array_equal(got, O.select_eviction_candidates(s, 20000))
print("ok")
'''
    env = dict(os.environ, PKV_EVICTION_RADIX="0")
    env["PYTHONPATH"] = os.pathsep.join([str(ROOT / "tests"), str(PKG), str(ROOT),
                                         env.get("PYTHONPATH", "")])
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stdout + r.stderr
