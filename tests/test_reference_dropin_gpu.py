"""The reference's own callers on this build's ``_C`` (the drop-in claim).

Runs ``tests/reference_dropin_run.py`` in a process of its own: the
reference package, installed unchanged under ``baseline/_ref`` (see
``tests/reference_tree.py``), imports this build's ctypes module as its
``pagedkv_fusion._C``; its kernel gate ``tests/test_kernels_gpu.py`` must
pass in full (none skipped), and its vLLM adapter must write and decode a
cache through ``ops`` -> ``_C`` within the gate's tolerance.  Skips where the
reference tree is not installed.
"""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from conftest import PKG, ensure_native_built
from reference_tree import locate

pytestmark = pytest.mark.gpu


def test_reference_gate_and_adapter_on_this_c_module():
    if not torch.cuda.is_available():
        pytest.fail("gpu test run without a visible CUDA device")
    ref = locate()
    if ref is None:
        pytest.skip("the reference package is not installed under baseline/_ref")
    ensure_native_built()
    runner = Path(__file__).resolve().parent / "reference_dropin_run.py"
    r = subprocess.run([sys.executable, str(runner), str(ref), str(PKG)], capture_output=True,
                       text=True, timeout=600)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("DROPIN ")]
    assert lines, f"runner printed no result (rc {r.returncode}):\n{r.stdout[-3000:]}\n{r.stderr[-3000:]}"
    res = json.loads(lines[-1][len("DROPIN "):])
    print(json.dumps(res, indent=1))
    assert res["ops_backend"] == "cuda"
    assert Path(res["library"]).resolve().is_relative_to(PKG.resolve())
    gate = res["gate"]
    assert gate["failed"] == 0 and gate["skipped"] == 0 and gate["passed"] >= 10, gate
    ad = res["adapter"]
    assert ad["native_equals_oracle"], ad
    assert ad["decode_allclose_2e-4"] and ad["decode_max_rel_err"] <= 1e-3, ad
    assert ad["adapter_vs_native"]["max_scale_ulp"] <= 1, ad
    assert ad["adapter_vs_native"]["max_code_diff"] <= 1, ad
    assert res["ok"] and r.returncode == 0
