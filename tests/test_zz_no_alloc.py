"""The allocation-free decode entry point, called through the C ABI.

pkv_quant_paged_attention_noalloc serves callers that cannot allocate
device memory (a plugin given only input/output pointers by a framework
that owns all device memory, or a serving path that must not pay
cudaMalloc's synchronization): its split-K scratch is a fixed array inside
the library.  This test calls it twice in a row on the same inputs, with no
workspace, and checks both outputs against the allocating entry point's
(same kernels, so equal within the attention tolerance used everywhere:
rtol/atol 2e-4).  It also checks that a call too large for the scratch is
rejected.  The file sorts last so a stop-at-first-failure run has already
run every other test; it also passes alone in a fresh process.
"""

from __future__ import annotations

import ctypes as ct
import math

import numpy as np
import pytest
import torch

from conftest import ensure_native_built
from oracle import oracle as O
from pagedkv_fusion import problems

pytestmark = pytest.mark.gpu


def _lib():
    lib = ct.CDLL(str(ensure_native_built()))
    f = lib.pkv_quant_paged_attention_noalloc
    f.argtypes = [ct.c_void_p] * 8 + [ct.c_int32] * 5 + [ct.c_int64, ct.c_int32, ct.c_float,
                                                          ct.c_void_p]
    f.restype = ct.c_int
    lib.pkv_noalloc_scratch_bytes.restype = ct.c_size_t
    lib.pkv_last_error_string.restype = ct.c_char_p
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


def _device_problem(seed, S, H, Hkv, L):
    q, k, v, bt, sl, sm = problems.make_paged_kv_problem(np.random.default_rng(seed), S, H, Hkv,
                                                         128, 16, L)
    kq, ks = O.quantize_kv_per_block(k)
    vq, vs = O.quantize_kv_per_block(v)
    d = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (q, kq, ks, vq, vs, bt, sl)]
    return d, sm


def test_noalloc_matches_allocating_entry_point_twice():
    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a visible CUDA device")
    lib = _lib()
    from pagedkv_fusion import _C
    # two different problems, so the second call must overwrite the first's
    # partials in the shared scratch
    for seed, (S, H, Hkv, L) in ((1, (12, 16, 8, 3000)), (2, (5, 32, 8, 1700))):
        d, sm = _device_problem(seed, S, H, Hkv, L)
        want = _C.quant_paged_attention(*d, sm)
        for _ in range(2):
            rc, got = _call_noalloc(lib, *d, sm)
            assert rc == 0, lib.pkv_last_error_string().decode()
            torch.cuda.synchronize()
            np.testing.assert_allclose(got.cpu().numpy(), want.cpu().numpy(), rtol=2e-4,
                                       atol=2e-4)


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
