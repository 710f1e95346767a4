"""The allocation-free decode entry point, called through the C ABI.

pkv_quant_paged_attention_noalloc serves callers that cannot allocate
device memory (a plugin given only input/output pointers by a framework
that owns all device memory, or a serving path that must not pay
cudaMalloc's synchronization): its split-K scratch is a fixed array inside
the library, shared by every call on a device and never cleared.

Both kernel families that keep state in that array are exercised, each on
two problems of different shapes called back to back, so every call starts
on the scratch contents the previous one left:

* groups of 2 and 4 query heads per KV head take the tensor-core kernel,
  whose split partials are merged by a second kernel; on request
  (PKV_DECODE_TC_PAGES=1) the whole-page tensor-core kernel, one launch,
  whose arrival counters and partials live in the scratch;
* one query head per KV head takes the persistent stream kernel (one
  launch per call, asserted), whose launch-tagged arrival counters live in
  the scratch and are not reset between calls.

Each output is compared bit for bit with the allocating entry point (same
plan, same kernels, deterministic merges) and with the double-precision C
oracle within the attention tolerance used everywhere (rtol/atol 2e-4, max
relative error 1e-3).  A call too large for the scratch is rejected.  The
file sorts last so a stop-at-first-failure run has already run every other
test; it also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes as ct
import math

import numpy as np
import pytest
import torch

from conftest import ensure_native_built
from oracle import c_oracle
from oracle import oracle as O
from pagedkv_fusion import problems

pytestmark = pytest.mark.gpu

ATTN_RTOL = ATTN_ATOL = 2e-4
ATTN_MAXREL = 1e-3


def _lib():
    lib = ct.CDLL(str(ensure_native_built()))
    f = lib.pkv_quant_paged_attention_noalloc
    f.argtypes = [ct.c_void_p] * 8 + [ct.c_int32] * 5 + [ct.c_int64, ct.c_int32, ct.c_float,
                                                          ct.c_void_p]
    f.restype = ct.c_int
    lib.pkv_noalloc_scratch_bytes.restype = ct.c_size_t
    lib.pkv_last_error_string.restype = ct.c_char_p
    n = lib.pkv_quant_paged_attention_kernel_launches
    n.argtypes = [ct.c_int32] * 6
    n.restype = ct.c_int
    return lib


def _call_noalloc(lib, q, kq, ks, vq, vs, bt, sl, sm):
    S, H, D = q.shape
    NB, bs, Hkv, _ = kq.shape
    out = torch.full_like(q, float("nan"))
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.pkv_quant_paged_attention_noalloc(
        q.data_ptr(), kq.data_ptr(), ks.data_ptr(), vq.data_ptr(), vs.data_ptr(), bt.data_ptr(),
        sl.data_ptr(), out.data_ptr(), S, H, Hkv, D, bs, NB, bt.shape[1], sm, stream)
    return rc, out


def _problem(seed, S, H, Hkv, L):
    q, k, v, bt, sl, sm = problems.make_paged_kv_problem(np.random.default_rng(seed), S, H, Hkv,
                                                         128, 16, L)
    kq, ks = O.quantize_kv_per_block(k)
    vq, vs = O.quantize_kv_per_block(v)
    host = (q, kq, ks, vq, vs, bt, sl)
    d = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in host]
    return host, d, sm


def _check_twice(lib, cases, launches):
    from pagedkv_fusion import _C
    for seed, (S, H, Hkv, L) in cases:
        host, d, sm = _problem(seed, S, H, Hkv, L)
        assert lib.pkv_quant_paged_attention_kernel_launches(
            S, H, Hkv, 128, 16, host[5].shape[1]) == launches
        want = _C.quant_paged_attention(*d, sm).cpu().numpy()
        ref = c_oracle.paged_attention(*host, sm)
        np.testing.assert_allclose(want, ref, rtol=ATTN_RTOL, atol=ATTN_ATOL)
        for _ in range(2):
            rc, got = _call_noalloc(lib, *d, sm)
            assert rc == 0, lib.pkv_last_error_string().decode()
            torch.cuda.synchronize()
            got = got.cpu().numpy()
            np.testing.assert_array_equal(got, want)
            np.testing.assert_allclose(got, ref, rtol=ATTN_RTOL, atol=ATTN_ATOL)
            assert float(np.abs(got - ref).max()) / float(np.abs(ref).max()) <= ATTN_MAXREL


def test_noalloc_tensor_core_path_twice():
    """Groups of 2 and 4 (tensor-core kernel + combine): the second problem
    overwrites the first's partials in the shared scratch."""
    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a visible CUDA device")
    _check_twice(_lib(), ((1, (12, 16, 8, 3000)), (2, (5, 32, 8, 1700))), launches=2)


def test_noalloc_page_kernel_twice(monkeypatch):
    """Groups of 2 and 4 on the whole-page tensor-core kernel (one launch):
    the second problem starts on the counters and partials the first left
    in the shared scratch."""
    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a visible CUDA device")
    monkeypatch.setenv("PKV_DECODE_TC_PAGES", "1")
    _check_twice(_lib(), ((1, (12, 16, 8, 3000)), (2, (5, 32, 8, 1700))), launches=1)


def test_noalloc_stream_kernel_reuses_its_counters():
    """One query head per KV head (persistent stream kernel, one launch):
    the first problem has 37 x 8 units, the second 5 x 4, so the second
    call's units map to arrival counters the first call left behind, and
    each problem has units split over several CTAs (counters in use)."""
    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a visible CUDA device")
    _check_twice(_lib(), ((3, (37, 8, 8, 1000)), (4, (5, 4, 4, 9000)), (3, (37, 8, 8, 1000))),
                 launches=1)


def test_noalloc_rejects_work_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a visible CUDA device")
    lib = _lib()
    cap = lib.pkv_noalloc_scratch_bytes()
    assert cap == 32 << 20
    # 2,048 sequences x 40 heads of 8,192 tokens: hundreds of MB of split-K
    # partials; rejected on the host before any kernel is launched
    S, H, D, bs, M = 2048, 40, 128, 16, 512
    q = torch.zeros(S, H, D, device="cuda")
    kq = torch.zeros(4, bs, H, D, dtype=torch.int8, device="cuda")
    ks = torch.ones(4, H, device="cuda")
    bt = torch.zeros(S, M, dtype=torch.int32, device="cuda")
    sl = torch.full((S,), M * bs, dtype=torch.int32, device="cuda")
    rc, _ = _call_noalloc(lib, q, kq, ks, kq, ks, bt, sl, 1 / math.sqrt(D))
    assert rc == 2
    assert "scratch" in lib.pkv_last_error_string().decode()
