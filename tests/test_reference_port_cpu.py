"""The CPU baseline's port against the reference's own ``paged_attention_ref``.

The bench's CPU legs time ``oracle.paged_attention`` (the NumPy port) rather
than the reference module, which cannot travel to a GPU host.  This test
times both on this host, single-threaded BLAS, on one sequence of the
large-head workload's shape (40 query / 40 KV heads, D 128, bs 16, 4,096
tokens), checks that they agree, and that the port is not slower than the
reference (a slower port would flatter every GPU/CPU ratio).  Skips where
the reference package is not installed under ``baseline/_ref``.
"""

from __future__ import annotations

import importlib.util
import time

import numpy as np
import pytest

from oracle import oracle as O
from reference_tree import locate


def _load_reference():
    ref = locate()
    if ref is None:
        pytest.skip("the reference package is not installed under baseline/_ref")
    spec = importlib.util.spec_from_file_location("pkv_reference_module",
                                                  ref / "pagedkv_fusion" / "reference.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _best_of(fn, n):
    best = float("inf")
    for _ in range(n):
        t0 = time.perf_counter()
        fn()
        best = min(best, time.perf_counter() - t0)
    return best


def test_port_costs_what_the_reference_costs():
    refmod = _load_reference()
    threadpoolctl = pytest.importorskip("threadpoolctl")
    rng = np.random.default_rng(5)
    L, H, D, bs = 4096, 40, 128, 16
    n = L // bs
    kq = rng.integers(-127, 128, size=(n, bs, H, D), dtype=np.int8)
    vq = rng.integers(-127, 128, size=(n, bs, H, D), dtype=np.int8)
    ks = (rng.random((n, H), dtype=np.float32) * 0.02 + 0.01).astype(np.float32)
    vs = (rng.random((n, H), dtype=np.float32) * 0.02 + 0.01).astype(np.float32)
    q = rng.standard_normal((1, H, D)).astype(np.float32)
    bt = rng.permutation(n).astype(np.int32)[None]
    sl = np.array([L], np.int32)
    sm = 1.0 / np.sqrt(D)
    with threadpoolctl.threadpool_limits(1):
        want = refmod.paged_attention_ref(q, kq, ks, vq, vs, bt, sl, sm)
        got = O.paged_attention(q, kq, ks, vq, vs, bt, sl, sm)
        np.testing.assert_allclose(got, want, rtol=2e-4, atol=2e-5)
        t_ref = _best_of(lambda: refmod.paged_attention_ref(q, kq, ks, vq, vs, bt, sl, sm), 5)
        t_port = _best_of(lambda: O.paged_attention(q, kq, ks, vq, vs, bt, sl, sm), 5)
    print(f"paged_attention_ref {t_ref * 1e3:.1f} ms, port {t_port * 1e3:.1f} ms, "
          f"port/ref {t_port / t_ref:.2f}")
    assert t_port <= 1.25 * t_ref, (t_port, t_ref)
