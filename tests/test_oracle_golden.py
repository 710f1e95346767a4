"""The oracle (NumPy and C restatements) pinned against golden vectors that
were produced by running the reference package itself
(tests/golden/make_golden.py).  CPU only."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import load_golden, sha
from oracle import c_oracle
from oracle import oracle as O
from pagedkv_fusion import problems

EV = load_golden("eviction")
QZ = load_golden("quantize")
AT = load_golden("attention")
BS_CASES = (1, 3, 7, 8, 9, 16, 17, 32, 33, 100, 128, 129, 200)


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


# ---------------------------------------------------------------------------
# eviction scores
# ---------------------------------------------------------------------------

def test_scores_reference_random_problem():
    args = (EV["rand64_rec"], EV["rand64_freq"], EV["rand64_attn"], EV["rand64_mask"])
    np.testing.assert_array_equal(bits(O.eviction_scores(*args)), bits(EV["rand64_scores"]))
    np.testing.assert_array_equal(bits(c_oracle.eviction_scores(*args)),
                                  bits(EV["rand64_scores"]))


@pytest.mark.parametrize("bs", BS_CASES)
def test_scores_all_block_sizes_bit_exact(bs):
    args = tuple(EV[f"bs{bs}_{n}"] for n in ("rec", "freq", "attn", "mask"))
    want, want_w = EV[f"bs{bs}_scores"], EV[f"bs{bs}_scores_w"]
    np.testing.assert_array_equal(bits(O.eviction_scores(*args)), bits(want))
    np.testing.assert_array_equal(bits(c_oracle.eviction_scores(*args)), bits(want))
    np.testing.assert_array_equal(bits(O.eviction_scores(*args, 0.7, 0.2, 0.1)), bits(want_w))
    np.testing.assert_array_equal(bits(c_oracle.eviction_scores(*args, 0.7, 0.2, 0.1)),
                                  bits(want_w))


@pytest.mark.parametrize("tag,kw", [("w16k", dict(mask="all")), ("w16k_mask", dict(mask="random")),
                                    ("w16k_ties", dict(mask="all", ties=True))])
def test_scores_16k_workload(tag, kw):
    rec, freq, att, msk = problems.eviction_problem(seed=0, **kw)
    assert sha(rec, freq, att, msk) == str(EV[f"{tag}_digest"]), "generator drifted"
    np.testing.assert_array_equal(bits(O.eviction_scores(rec, freq, att, msk)),
                                  bits(EV[f"{tag}_scores"]))
    np.testing.assert_array_equal(bits(c_oracle.eviction_scores(rec, freq, att, msk)),
                                  bits(EV[f"{tag}_scores"]))


@pytest.mark.parametrize("n", [1, 2, 7, 8, 9, 15, 16, 17, 64, 100, 128, 129, 256, 300, 1000])
def test_pairwise_order_matches_numpy(n):
    x = np.random.default_rng(n).standard_normal((50, n)).astype(np.float32)
    want = x.sum(axis=1)
    got = np.array([np.float32(0.0) + O.pairwise_sum(r) for r in x], np.float32)
    np.testing.assert_array_equal(bits(got), bits(want))


def test_all_negative_zero_row_sums_to_positive_zero():
    att = np.full((2, 16), -0.0, np.float32)
    msk = np.ones((2, 16), bool)
    rec = np.zeros(2, np.float32)
    s1 = O.eviction_scores(rec, rec, att, msk)
    s2 = c_oracle.eviction_scores(rec, rec, att, msk)
    np.testing.assert_array_equal(bits(s1), bits(s2))


# ---------------------------------------------------------------------------
# selection
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("tag", ["w16k", "w16k_mask", "w16k_ties"])
@pytest.mark.parametrize("k", [1, 2458, 8192])
def test_select_16k_workload(tag, k):
    sc = EV[f"{tag}_scores"]
    np.testing.assert_array_equal(O.select_eviction_candidates(sc, k), EV[f"{tag}_idx_k{k}"])
    np.testing.assert_array_equal(c_oracle.select(sc, k), EV[f"{tag}_idx_k{k}"])


def test_select_tie_break_known_answer():
    np.testing.assert_array_equal(O.select_eviction_candidates(EV["kat_scores"], 3), [1, 2, 3])
    np.testing.assert_array_equal(EV["kat_idx"], [1, 2, 3])
    np.testing.assert_array_equal(c_oracle.select(EV["kat_scores"], 3), [1, 2, 3])


def test_select_special_values():
    sc = EV["special_scores"]
    np.testing.assert_array_equal(O.select_eviction_candidates(sc, sc.size), EV["special_idx"])
    np.testing.assert_array_equal(O.select_eviction_candidates(sc, 5), EV["special_idx_k5"])
    np.testing.assert_array_equal(c_oracle.select(sc, sc.size), EV["special_idx"])


def test_ties_exist_in_tie_workload():
    sc = EV["w16k_ties_scores"]
    assert np.unique(sc).size < sc.size // 2  # thousands of exact ties


def test_select_k_beyond_n_and_zero():
    sc = np.array([0.2, 0.1], np.float32)
    np.testing.assert_array_equal(O.select_eviction_candidates(sc, 5), [1, 0])
    assert O.select_eviction_candidates(sc, 0).size == 0


def test_merge_of_shards_equals_global_selection():
    sc = EV["w16k_ties_scores"]
    k = 2458
    keys = []
    for lo, hi in ((0, 5000), (5000, 5001), (5001, 16384)):
        local = O.select_eviction_candidates(sc[lo:hi], k)
        keys.append(O.pack_candidate_keys(sc[lo:hi][local], local + lo))
    np.testing.assert_array_equal(O.merge_candidate_keys(np.concatenate(keys), k),
                                  EV["w16k_ties_idx_k2458"])


# ---------------------------------------------------------------------------
# quantization
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("case", ["rand", "edge", "tie", "f16"])
def test_quantize_bit_exact(case):
    kv = QZ[f"{case}_kv"]
    q, s = O.quantize_kv_per_block(kv)
    np.testing.assert_array_equal(q, QZ[f"{case}_q"])
    np.testing.assert_array_equal(bits(s), bits(QZ[f"{case}_scale"]))
    qc, sc = c_oracle.quantize(kv.astype(np.float32))
    np.testing.assert_array_equal(qc, QZ[f"{case}_q"])
    np.testing.assert_array_equal(bits(sc), bits(QZ[f"{case}_scale"]))


def test_quantize_torch_twin_agrees():
    np.testing.assert_array_equal(QZ["rand_q_torch"], QZ["rand_q"])
    np.testing.assert_array_equal(bits(QZ["rand_scale_torch"]), bits(QZ["rand_scale"]))


def test_quantize_properties(rng):
    kv = rng.standard_normal((8, 16, 4, 64)).astype(np.float32) * 3.0
    q, scale = O.quantize_kv_per_block(kv)
    err = np.abs(kv - O.dequantize_kv_per_block(q, scale))
    assert (err <= scale[:, None, :, None] / 2.0 + 1e-7).all()
    assert q.max() <= 127 and q.min() >= -127
    z, zs = O.quantize_kv_per_block(np.zeros((2, 16, 2, 32), np.float32))
    assert (z == 0).all() and (zs == 1.0).all()


# ---------------------------------------------------------------------------
# paged attention
# ---------------------------------------------------------------------------

def _regen(i):
    S, H, Hkv, D, bs, L = (int(x) for x in AT[f"gpu{i}_shape"])
    q, k, v, bt, sl, sm = problems.make_paged_kv_problem(np.random.default_rng(42), S, H, Hkv, D,
                                                         bs, L)
    assert sha(q, k, v, bt, sl) == str(AT[f"gpu{i}_digest"]), "generator drifted"
    return q, k, v, bt, sl, sm


@pytest.mark.parametrize("i", [0, 1, 2, 3])
def test_attention_reference_gpu_shapes(i):
    q, k, v, bt, sl, sm = _regen(i)
    kq, ks = O.quantize_kv_per_block(k)
    vq, vs = O.quantize_kv_per_block(v)
    assert sha(kq, vq) == str(AT[f"gpu{i}_kq_digest"])
    want = AT[f"gpu{i}_out"]
    np.testing.assert_allclose(O.paged_attention(q, kq, ks, vq, vs, bt, sl, sm), want,
                               rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(c_oracle.paged_attention(q, kq, ks, vq, vs, bt, sl, sm), want,
                               rtol=1e-5, atol=1e-6)


def test_attention_default_and_edges():
    q, k, v, bt, sl, sm = problems.make_paged_kv_problem(np.random.default_rng(1234))
    assert sha(q, k, v, bt, sl) == str(AT["default_digest"])
    kq, ks = O.quantize_kv_per_block(k)
    vq, vs = O.quantize_kv_per_block(v)
    np.testing.assert_allclose(O.paged_attention(q, kq, ks, vq, vs, bt, sl, sm),
                               AT["default_out"], rtol=1e-5, atol=1e-6)
    for L in (1, 15, 16, 17):
        rng = np.random.default_rng(int(AT[f"edge{L}_seed"]))
        q, k, v, bt, sl, sm = problems.make_paged_kv_problem(rng, 1, 8, 4, 64, 16, L)
        sl[:] = L
        assert sha(q, k, v, bt, sl) == str(AT[f"edge{L}_digest"])
        kq, ks = O.quantize_kv_per_block(k)
        vq, vs = O.quantize_kv_per_block(v)
        np.testing.assert_allclose(c_oracle.paged_attention(q, kq, ks, vq, vs, bt, sl, sm),
                                   AT[f"edge{L}_out"], rtol=1e-5, atol=1e-6)


def test_attention_small_decode_workload():
    q, k, v, bt, sl, sm = problems.decode_small_problem(0)
    assert sha(q, k, v, bt, sl) == str(AT["small_digest"])
    kq, ks = O.quantize_kv_per_block(k)
    vq, vs = O.quantize_kv_per_block(v)
    assert sha(kq, ks, vq, vs) == str(AT["small_codes_digest"])
    np.testing.assert_allclose(O.paged_attention(q, kq, ks, vq, vs, bt, sl, sm), AT["small_out"],
                               rtol=1e-5, atol=1e-6)


def test_write_to_cache_oracle_semantics(rng):
    nb, bs, hkv, hd = 6, 16, 2, 32
    cache = np.zeros((2, nb, bs, hkv, hd), np.int8)
    scales = np.ones((2, nb, hkv), np.float32)
    key = rng.standard_normal((5, hkv, hd)).astype(np.float32)
    val = rng.standard_normal((5, hkv, hd)).astype(np.float32)
    slots = np.array([3, 17, 4, 40, 18])
    O.write_to_cache(key, val, cache, scales, slots, bs)
    # block 0 holds tokens 0 and 2: one shared scale per head
    _, s0 = O.quantize_kv_per_block(key[[0, 2]][None])
    np.testing.assert_array_equal(scales[0, 0], s0[0])
    assert (cache[:, 5] == 0).all()
