"""Host logic of the vLLM-shaped backend (pagedkv_fusion.backend): shape
envelope, prefill routing, and loud failure of decode without a device.
CPU only."""

from __future__ import annotations

import pytest
import torch

from pagedkv_fusion.backend import PagedKVFusionBackend, PagedKVFusionMetadata


class Fallback:
    def __init__(self):
        self.calls = []

    def forward(self, *args, **kwargs):
        self.calls.append((args, kwargs))
        return "fallback"


def test_class_surface_matches_reference_adapter():
    assert PagedKVFusionBackend.supports_prefill is False
    assert PagedKVFusionBackend.supports_decode is True
    fields = [f.name for f in PagedKVFusionMetadata.__dataclass_fields__.values()]
    assert fields == ["block_tables", "seq_lens", "k_scale", "v_scale"]
    for name in ("write_to_cache", "decode_forward", "forward"):
        assert callable(getattr(PagedKVFusionBackend, name))


@pytest.mark.parametrize("q_shape,cache_shape,qdt,ok", [
    ((4, 32, 128), (2, 10, 16, 8, 128), torch.float32, True),
    ((4, 8, 64), (2, 10, 32, 8, 64), torch.float32, True),
    ((4, 8, 256), (2, 10, 64, 8, 256), torch.float32, True),
    ((4, 8, 128), (2, 10, 16, 8, 128), torch.float16, False),   # q is float32 (v1)
    ((4, 8, 48), (2, 10, 16, 8, 48), torch.float32, False),     # D % 32
    ((4, 8, 288), (2, 10, 16, 8, 288), torch.float32, False),   # D <= 256
    ((4, 8, 128), (2, 10, 128, 8, 128), torch.float32, False),  # bs <= 64
    ((4, 12, 128), (2, 10, 16, 8, 128), torch.float32, False),  # H % Hkv
    ((4, 8, 128), (10, 16, 8, 128), torch.float32, False),      # not [2, ...]
])
def test_supports_is_the_kernel_envelope(q_shape, cache_shape, qdt, ok):
    q = torch.zeros(q_shape, dtype=qdt)
    cache = torch.zeros(cache_shape, dtype=torch.int8)
    assert PagedKVFusionBackend.supports(q, cache) is ok


def test_prefill_goes_to_fallback_without_touching_a_device():
    fb = Fallback()
    be = PagedKVFusionBackend(fb)
    assert be.forward("x", 1, key="y", is_prefill=True) == "fallback"
    assert fb.calls == [(("x", 1), {"key": "y"})]


def test_decode_without_a_device_fails_loudly():
    if torch.cuda.is_available():
        pytest.skip("a device is visible")
    be = PagedKVFusionBackend(Fallback())
    q = torch.zeros((1, 8, 128))
    cache = torch.zeros((2, 4, 16, 8, 128), dtype=torch.int8)
    scale = torch.ones((2, 4, 8))
    meta = PagedKVFusionMetadata(torch.zeros((1, 4), dtype=torch.int32),
                                 torch.ones(1, dtype=torch.int32), scale[0], scale[1])
    with pytest.raises(RuntimeError, match="CUDA device"):
        be.forward(q, cache, scale, meta, 0.1, is_prefill=False)
    with pytest.raises(RuntimeError, match="CUDA device"):
        be.write_to_cache(q[0], q[0], cache, scale, torch.zeros(8, dtype=torch.int64), 16)
