"""The vLLM-shaped backend (pagedkv_fusion.backend) in a small serving loop:
prefill writes, then decode steps that each append one token per sequence
through ``write_to_cache`` and run ``decode_forward`` -- eagerly and as a
captured ``DecodePlan`` -- against the oracle on a host mirror of the cache
(reference integration/vllm/pagedkv_fusion_backend.py:63-118)."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import c_oracle
from oracle import oracle as O

pytestmark = pytest.mark.gpu

ATTN_RTOL = ATTN_ATOL = 2e-4
ATTN_MAXREL = 1e-3


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def assert_attention_close(got, want):
    got = got.cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=ATTN_RTOL, atol=ATTN_ATOL)
    assert float(np.abs(got - want).max()) / max(float(np.abs(want).max()), 1e-30) <= ATTN_MAXREL


def slots_for(tables, seq, positions, bs):
    return np.array([tables[seq, p // bs] * bs + p % bs for p in positions], np.int64)


@pytest.mark.parametrize("heads,kv_heads,dtype", [(32, 8, torch.float32), (8, 8, torch.float16),
                                                  (16, 2, torch.bfloat16)])
def test_serving_loop_matches_oracle(heads, kv_heads, dtype):
    from pagedkv_fusion.backend import PagedKVFusionBackend, PagedKVFusionMetadata
    r = np.random.default_rng(11)
    S, bs, D, nb, width = 4, 16, 128, 96, 20
    tables = np.full((S, width), -1, np.int32)
    perm = r.permutation(nb).astype(np.int32)
    for s in range(S):
        tables[s] = perm[s * width:(s + 1) * width]
    lens = np.array([37, 64, 1, 150], np.int32)

    cache_h = np.zeros((2, nb, bs, kv_heads, D), np.int8)
    scale_h = np.ones((2, nb, kv_heads), np.float32)
    cache, scale = dev(cache_h), dev(scale_h)
    be = PagedKVFusionBackend(fallback_backend=None)
    tdt = {torch.float32: np.float32, torch.float16: np.float16, torch.bfloat16: np.float32}

    def write(positions_per_seq):
        seqs = [s for s, ps in enumerate(positions_per_seq) for _ in ps]
        slots = np.concatenate([slots_for(tables, s, ps, bs)
                                for s, ps in enumerate(positions_per_seq)])
        n = len(seqs)
        k = torch.from_numpy(r.standard_normal((n, kv_heads, D)).astype(tdt[dtype])).to(dtype)
        v = torch.from_numpy(r.standard_normal((n, kv_heads, D)).astype(tdt[dtype])).to(dtype)
        be.write_to_cache(k.cuda(), v.cuda(), cache, scale, dev(slots), bs)
        O.write_to_cache(k.float().numpy(), v.float().numpy(), cache_h, scale_h, slots, bs)

    # prefill: each sequence's first lens[s] tokens, block by block
    for s in range(S):
        for b0 in range(0, int(lens[s]), bs):
            pos = [[] for _ in range(S)]
            pos[s] = list(range(b0, min(b0 + bs, int(lens[s]))))
            write(pos)

    q = torch.zeros((S, heads, D), dtype=torch.float32, device="cuda")
    sl = dev(lens.copy())
    meta = PagedKVFusionMetadata(block_tables=dev(tables), seq_lens=sl, k_scale=scale[0],
                                 v_scale=scale[1])
    sm = 1.0 / math.sqrt(D)
    plan = be.capture_decode(q, cache, scale, meta, sm)
    for step in range(5):
        write([[int(lens[s])] for s in range(S)])  # the new token of each sequence
        lens += 1
        qh = r.standard_normal((S, heads, D)).astype(np.float32)
        q.copy_(dev(qh))
        sl.copy_(dev(lens))
        eager = be.decode_forward(q, cache, scale, meta, sm)
        replay = plan.run().clone()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(cache.cpu().numpy(), cache_h)
        np.testing.assert_array_equal(scale.cpu().numpy().view(np.uint32), scale_h.view(np.uint32))
        want = c_oracle.paged_attention(qh, cache_h[0], scale_h[0], cache_h[1], scale_h[1],
                                        tables, lens, sm)
        assert_attention_close(eager, want)
        assert torch.equal(eager, replay), f"graph replay differs at step {step}"


def test_forward_routes_decode_and_prefill():
    from pagedkv_fusion.backend import PagedKVFusionBackend, PagedKVFusionMetadata

    class Fallback:
        calls = 0

        def forward(self, *args, **kwargs):
            Fallback.calls += 1
            return "fallback"

    r = np.random.default_rng(5)
    be = PagedKVFusionBackend(Fallback())
    cache = dev(r.integers(-127, 128, (2, 8, 16, 2, 64)).astype(np.int8))
    scale = dev(r.random((2, 8, 2)).astype(np.float32))
    tables = dev(np.arange(8, dtype=np.int32).reshape(2, 4))
    lens = dev(np.array([64, 17], np.int32))
    q = dev(r.standard_normal((2, 4, 64)).astype(np.float32))
    meta = PagedKVFusionMetadata(tables, lens, scale[0], scale[1])
    assert be.forward(q, cache, scale, meta, 0.125, is_prefill=True) == "fallback"
    out = be.forward(q, cache, scale, meta, 0.125, is_prefill=False)
    assert Fallback.calls == 1 and isinstance(out, torch.Tensor)
    want = c_oracle.paged_attention(q.cpu().numpy(), *(t.cpu().numpy() for t in
                                    (cache[0], scale[0], cache[1], scale[1], tables, lens)), 0.125)
    assert_attention_close(out, want)
