"""Runs the reference's own callers, unchanged, on this build's ``_C``.

Usage: ``python reference_dropin_run.py <reference tree> <package dir>``
(run in a process of its own: it imports the reference's ``pagedkv_fusion``
package, which shares its name with this build's).

The reference package is first on ``sys.path``.  This build's ctypes module
``pagedkv_fusion/_C.py`` is registered as ``pagedkv_fusion._C``, the module
the reference's dispatch layer imports (pagedkv_fusion/ops.py:32-37) and
its compiled extension would provide (csrc/bindings.cpp:14-26).  Then:

1. the reference's kernel gate ``tests/test_kernels_gpu.py`` runs unchanged
   under pytest (eviction scores rtol 1e-5 / atol 1e-6, attention rtol and
   atol 2e-4, bitwise determinism; tests/test_kernels_gpu.py:34-98);
2. the reference's vLLM adapter (integration/vllm/pagedkv_fusion_backend.py)
   fills an INT8 cache through its own ``write_to_cache`` loop (:63-95, the
   reference's torch quantizer on the GPU), including partial blocks, and
   decodes through ``decode_forward`` -> ``ops`` -> ``_C`` (:97-118).  The
   decode is checked against ``reference.paged_attention_ref`` on the
   adapter's cache (rtol/atol 2e-4).  This build's native
   ``_C.write_to_cache``, given the same tokens, must equal the oracle's
   restatement of the adapter (NumPy semantics of reference.py) bit for
   bit, and the adapter's own cache to within what the reference's torch
   quantizer rounds differently on a GPU: torch divides by the Python
   scalar 127.0 as a multiply by fl(1/127) there (quantize.py:28), so a
   few percent of its scales sit one ulp from reference.py's IEEE quotient
   (reference.py:100-103) and a code next to a rounding boundary may move
   by one (reported: the share of equal scales, the largest differences).

Prints one JSON line: the gate's pass/fail/skip counts and the adapter
checks.  Exit code 0 only when everything passed and nothing was skipped.
"""

from __future__ import annotations

import importlib.util
import json
import math
import sys
from pathlib import Path


def _install_c(ref: Path, pkg: Path):
    sys.path.insert(0, str(ref))
    import pagedkv_fusion  # the reference package

    if Path(pagedkv_fusion.__file__).resolve().parent != (ref / "pagedkv_fusion").resolve():
        raise RuntimeError(f"imported {pagedkv_fusion.__file__}, not the reference package")
    spec = importlib.util.spec_from_file_location("pagedkv_fusion._C",
                                                  pkg / "pagedkv_fusion" / "_C.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["pagedkv_fusion._C"] = mod
    spec.loader.exec_module(mod)
    pagedkv_fusion._C = mod
    return mod


class _Counts:
    def __init__(self):
        self.passed = self.failed = self.skipped = 0
        self.failures: list[str] = []

    def pytest_runtest_logreport(self, report):
        if report.when == "call" and report.passed:
            self.passed += 1
        elif report.failed:
            self.failed += 1
            self.failures.append(report.nodeid)
        elif report.skipped:
            self.skipped += 1

    def pytest_collectreport(self, report):
        if report.failed:
            self.failed += 1
            self.failures.append(f"collect {report.nodeid}")
        elif report.skipped:  # a module-level skip, e.g. no _C
            self.skipped += 1


def run_gate(ref: Path) -> dict:
    import pytest

    counts = _Counts()
    rc = pytest.main(["-q", "-p", "no:cacheprovider", "-o", "addopts=", "--rootdir", str(ref),
                      "--confcutdir", str(ref / "tests"), str(ref / "tests" / "test_kernels_gpu.py")],
                     plugins=[counts])
    return {"rc": int(rc), "passed": counts.passed, "failed": counts.failed,
            "skipped": counts.skipped, "failures": counts.failures}


def run_adapter(ref: Path, C, root: Path) -> dict:
    import numpy as np
    import torch

    from pagedkv_fusion import ops, reference

    sys.path.append(str(root))  # after the reference package: oracle only
    from oracle import oracle as O

    spec = importlib.util.spec_from_file_location(
        "pagedkv_fusion_backend", ref / "integration" / "vllm" / "pagedkv_fusion_backend.py")
    be_mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(be_mod)

    rng = np.random.default_rng(2024)
    S, H, Hkv, D, bs, width = 6, 32, 8, 128, 16, 24
    nb = S * width + 5
    tables = rng.permutation(nb)[:S * width].reshape(S, width).astype(np.int32)
    lens = np.array([1, 15, 16, 17, 200, 381], np.int32)
    dev = torch.device("cuda")
    cache = torch.zeros((2, nb, bs, Hkv, D), dtype=torch.int8, device=dev)
    scale = torch.ones((2, nb, Hkv), dtype=torch.float32, device=dev)
    cache_n, scale_n = cache.clone(), scale.clone()
    cache_h, scale_h = cache.cpu().numpy(), scale.cpu().numpy()
    backend = be_mod.PagedKVFusionBackend(fallback_backend=None)

    # prefill in chunks of 11 tokens (chunks straddle block boundaries, so
    # blocks are written partially and then rewritten), then 3 decode steps
    # of one token per sequence
    writes = []
    for s in range(S):
        for p0 in range(0, max(int(lens[s]) - 3, 0), 11):
            writes.append([(s, p) for p in range(p0, min(p0 + 11, int(lens[s]) - 3))])
    for t in (3, 2, 1):
        writes.append([(s, int(lens[s]) - t) for s in range(S) if lens[s] >= t])
    for w in writes:
        slots_h = np.array([int(tables[s, p // bs]) * bs + p % bs for s, p in w], np.int64)
        k_h = rng.standard_normal((len(w), Hkv, D)).astype(np.float32)
        v_h = rng.standard_normal((len(w), Hkv, D)).astype(np.float32)
        k, v, slots = (torch.from_numpy(a).to(dev) for a in (k_h, v_h, slots_h))
        backend.write_to_cache(k, v, cache, scale, slots, bs)
        C.write_to_cache(k, v, cache_n, scale_n, slots, bs)
        O.write_to_cache(k_h, v_h, cache_h, scale_h, slots_h, bs)
    torch.cuda.synchronize()
    a_c, a_s = cache.cpu().numpy(), scale.cpu().numpy()
    n_c, n_s = cache_n.cpu().numpy(), scale_n.cpu().numpy()
    native_is_oracle = bool(np.array_equal(n_c, cache_h)
                            and np.array_equal(n_s.view(np.uint32), scale_h.view(np.uint32)))
    ulp = np.abs(a_s.view(np.int32).astype(np.int64) - n_s.view(np.int32).astype(np.int64))
    same_scale = ulp == 0  # [2, nb, Hkv]
    code_diff = np.abs(a_c.astype(np.int16) - n_c.astype(np.int16))  # [2, nb, bs, Hkv, D]
    adapter_vs_native = {"scales_equal_frac": float(same_scale.mean()),
                         "codes_equal_frac": float((code_diff == 0).mean()),
                         "max_scale_ulp": int(ulp.max()), "max_code_diff": int(code_diff.max())}
    adapter_close = ulp.max() <= 1 and code_diff.max() <= 1

    q = torch.from_numpy(rng.standard_normal((S, H, D)).astype(np.float32)).to(dev)
    meta = be_mod.PagedKVFusionMetadata(block_tables=torch.from_numpy(tables).to(dev),
                                        seq_lens=torch.from_numpy(lens).to(dev),
                                        k_scale=scale[0], v_scale=scale[1])
    sm = 1.0 / math.sqrt(D)
    got = backend.decode_forward(q, cache, scale, meta, sm).cpu().numpy()
    want = reference.paged_attention_ref(q.cpu().numpy(), a_c[0], a_s[0], a_c[1], a_s[1], tables,
                                         lens, sm)
    close = bool(np.allclose(got, want, rtol=2e-4, atol=2e-4))
    max_rel = float(np.abs(got - want).max() / np.abs(want).max())
    return {"backend_in_use": ops.backend_in_use(), "writes": len(writes),
            "native_equals_oracle": native_is_oracle, "adapter_vs_native": adapter_vs_native,
            "decode_allclose_2e-4": close, "decode_max_rel_err": max_rel,
            "ok": bool(ops.backend_in_use() == "cuda" and native_is_oracle and adapter_close
                       and close)}


def main() -> int:
    ref, pkg = Path(sys.argv[1]).resolve(), Path(sys.argv[2]).resolve()
    root = Path(__file__).resolve().parent.parent
    C = _install_c(ref, pkg)
    from pagedkv_fusion import ops

    result = {"c_module": C.__file__, "library": C.LIBRARY_PATH,
              "ops_module": ops.__file__, "ops_backend": ops.backend_in_use()}
    result["gate"] = run_gate(ref)
    result["adapter"] = run_adapter(ref, C, root)
    g = result["gate"]
    ok = (g["rc"] == 0 and g["failed"] == 0 and g["skipped"] == 0 and g["passed"] > 0
          and result["adapter"]["ok"] and result["ops_backend"] == "cuda")
    result["ok"] = ok
    print("DROPIN " + json.dumps(result), flush=True)
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
