"""The C-ABI library: it loads without a GPU, exports every symbol that
include/pagedkv_fusion.h declares, and rejects bad arguments before touching
the device.  CPU only: no call here launches a kernel."""

from __future__ import annotations

import ctypes as ct
import re

import numpy as np
import pytest

from conftest import ROOT, ensure_native_built

HEADER = ROOT / "include" / "pagedkv_fusion.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(pkv_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    return ct.CDLL(str(ensure_native_built()))


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("pkv_eviction_scores", "pkv_eviction_select", "pkv_quant_paged_attention",
                     "pkv_quantize_kv_per_block", "pkv_eviction_merge",
                     "pkv_eviction_local_candidates", "pkv_write_to_cache",
                     "pkv_last_error_string", "pkv_read_device_error"):
        assert required in names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"


def test_version_and_error_string(lib):
    lib.pkv_version.restype = ct.c_int
    assert lib.pkv_version() == 10000
    lib.pkv_last_error_string.restype = ct.c_char_p
    assert isinstance(lib.pkv_last_error_string(), bytes)


def _err(lib):
    lib.pkv_last_error_string.restype = ct.c_char_p
    return lib.pkv_last_error_string().decode()


def test_select_rejects_negative_k(lib):
    f = lib.pkv_eviction_select
    f.argtypes = [ct.c_void_p, ct.c_int64, ct.c_int64, ct.c_void_p, ct.c_void_p, ct.c_size_t,
                  ct.c_void_p]
    assert f(None, 10, -1, None, None, 0, None) == 1
    assert "non-negative" in _err(lib)


def test_select_with_nothing_to_do_is_ok(lib):
    f = lib.pkv_eviction_select
    f.argtypes = [ct.c_void_p, ct.c_int64, ct.c_int64, ct.c_void_p, ct.c_void_p, ct.c_size_t,
                  ct.c_void_p]
    assert f(None, 0, 5, None, None, 0, None) == 0


def _attn(lib):
    f = lib.pkv_quant_paged_attention
    f.argtypes = [ct.c_void_p] * 8 + [ct.c_int32] * 5 + [ct.c_int64, ct.c_int32, ct.c_float,
                                                          ct.c_void_p, ct.c_size_t, ct.c_void_p]
    return f


@pytest.mark.parametrize("shape,msg", [
    ((4, 8, 8, 48, 16, 100), "head_dim % 32 == 0"),
    ((4, 8, 8, 288, 16, 100), "head_dim % 32 == 0"),
    ((4, 8, 8, 128, 128, 100), "block_size <= 64"),
    ((4, 8, 3, 128, 16, 100), "num_heads % num_kv_heads"),
])
def test_decode_rejects_reference_envelope_violations(lib, shape, msg):
    S, H, Hkv, D, bs, NB = shape
    assert _attn(lib)(*([None] * 8), S, H, Hkv, D, bs, NB, 4, 0.1, None, 0, None) == 1
    assert msg in _err(lib)


def test_decode_rejects_null_pointers(lib):
    assert _attn(lib)(*([None] * 8), 2, 8, 8, 128, 16, 10, 4, 0.1, None, 0, None) == 1
    assert "null" in _err(lib)


def test_decode_workspace_size(lib):
    f = lib.pkv_quant_paged_attention_workspace_size
    f.argtypes = [ct.c_int32] * 6
    f.restype = ct.c_size_t
    # 64 sequences of 128 pages: split-K partials for 8 heads x 128 dims
    ws = f(64, 8, 8, 128, 16, 128)
    assert ws > 64 * 8 * 128 * 4
    assert f(0, 8, 8, 128, 16, 128) == 0


def test_decode_kernel_launches_per_call(lib, monkeypatch):
    f = lib.pkv_quant_paged_attention_kernel_launches
    f.argtypes = [ct.c_int32] * 6
    f.restype = ct.c_int
    monkeypatch.delenv("PKV_DECODE_SPLIT", raising=False)
    monkeypatch.delenv("PKV_DECODE_GENERIC", raising=False)
    assert f(64, 8, 8, 128, 16, 128) == 1      # persistent stream kernel
    assert f(512, 32, 8, 128, 16, 512) == 2    # GQA group of 4: per-head tensor-core + combine
    assert f(512, 24, 8, 128, 16, 512) == 2    # group of 3: generic kernel + combine
    assert f(512, 32, 8, 128, 32, 256) == 1    # group of 4, block_size 32: stream kernel
    assert f(2048, 8, 8, 128, 16, 128) == 2    # > 1,024 sequences: split-K + combine
    assert f(8, 8, 8, 64, 16, 32) == 2         # head_dim 64: generic kernel + combine
    assert f(0, 8, 8, 128, 16, 128) == 0
    monkeypatch.setenv("PKV_DECODE_TC_PAGES", "1")
    assert f(512, 32, 8, 128, 16, 512) == 1    # whole-page tensor-core kernel
    assert f(512, 64, 8, 128, 16, 512) == 2    # group of 8 x 8 KV heads: stays per head
    monkeypatch.setenv("PKV_DECODE_TC", "0")
    assert f(512, 32, 8, 128, 16, 512) == 1    # tensor-core path off: stream kernel
    monkeypatch.setenv("PKV_DECODE_SPLIT", "1")
    assert f(64, 8, 8, 128, 16, 128) == 2


def test_quantize_rejects_bad_dtype(lib):
    f = lib.pkv_quantize_kv_per_block
    f.argtypes = [ct.c_void_p, ct.c_int32, ct.c_void_p, ct.c_void_p, ct.c_int64, ct.c_int32,
                  ct.c_int32, ct.c_int32, ct.c_void_p]
    assert f(None, 7, None, None, 4, 16, 8, 128, None) == 1
    assert "float32" in _err(lib)


def test_select_workspace_is_padded_key_array(lib):
    f = lib.pkv_eviction_select_workspace_size
    f.argtypes = [ct.c_int64, ct.c_int64]
    f.restype = ct.c_size_t
    assert f(16384, 2458) == 16384 * 8
    assert f(16385, 8000) == 32768 * 8  # no radix prefilter: k too large


def test_select_workspace_adds_radix_prefilter_above_16k(lib):
    """Above 16,384 blocks, when next_pow2(k + 1024) candidates are at most
    an eighth of the padded keys (a quarter above 2^16 padded keys, half
    from 2^20 on), the workspace adds 16 bytes of alignment slack, the candidate buffer, a
    65,536-bin histogram and a 256-byte state; otherwise it stays the padded
    key array."""
    import os
    f = lib.pkv_eviction_select_workspace_size
    f.argtypes = [ct.c_int64, ct.c_int64]
    f.restype = ct.c_size_t
    keys = (1 << 21) * 8  # 1.2 M keys padded to 2^21
    if os.environ.get("PKV_EVICTION_RADIX", "1").startswith("0"):
        pytest.skip("radix prefilter switched off in this environment")
    assert f(1_200_000, 1000) == keys + 16 + 2048 * 8 + 65536 * 4 + 256
    assert f(1_200_000, 177_000) == keys + 16 + (1 << 18) * 8 + 65536 * 4 + 256
    # half of the padded keys: prefiltered from 2^20 padded keys on
    assert f(1_200_000, 600_000) == keys + 16 + (1 << 20) * 8 + 65536 * 4 + 256
    assert f(354_000, 177_000) == (1 << 19) * 8
    assert f(1_200_000, 1_100_000) == keys  # candidates = all the padded keys
    assert f(70001, 10000) == (1 << 17) * 8 + 16 + 16384 * 8 + 65536 * 4 + 256
    assert f(20000, 1000) == (1 << 15) * 8 + 16 + 2048 * 8 + 65536 * 4 + 256
    assert f(20000, 8000) == (1 << 15) * 8  # 16,384 candidates: half the keys
    assert f(40000, 12000) == (1 << 16) * 8  # a quarter, at 2^16 padded keys
    assert f(300_000, 100_000) == (1 << 19) * 8 + 16 + (1 << 17) * 8 + 65536 * 4 + 256
    assert f(16384, 1) == 16384 * 8  # the one-launch cluster range


def test_shim_imports_and_rejects_host_tensors():
    torch = pytest.importorskip("torch")
    from pagedkv_fusion import _C
    x = torch.zeros(4)
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.eviction_scores(x, x, torch.zeros(4, 16), torch.ones(4, 16, dtype=torch.bool))
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.quant_paged_attention(torch.zeros(1, 1, 32), *([x] * 6), 0.1)


def test_ops_fails_loudly_without_a_device():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a device is visible")
    from pagedkv_fusion import ops
    assert ops.backend_in_use() == "cuda"
    with pytest.raises(RuntimeError, match="CUDA device"):
        ops.eviction_scores(np.zeros(2, np.float32), np.zeros(2, np.float32),
                            np.zeros((2, 16), np.float32), np.ones((2, 16), bool))


def test_fastcall_module_reaches_the_same_library():
    """The METH_FASTCALL module the eviction calls use: built beside the
    library, argument count checked, and the library's own status codes
    returned (invalid sizes are rejected before any CUDA call)."""
    ensure_native_built()
    from pagedkv_fusion import _C
    fast = _C._fast
    with pytest.raises(TypeError):
        fast.eviction_select(None, 4, 2)
    assert fast.eviction_select(None, 4, -1, None, None, 0, None) == 1
    assert fast.eviction_scores(None, None, None, None, None, -1, 16, 0.4, 0.3, 0.3, None) == 1
    assert fast.eviction_scores_select(None, None, None, None, None, 8, 16, 0.4, 0.3, 0.3, -2,
                                       None, None, 0, None) == 1
    assert "k" in _C._last_error().decode()
