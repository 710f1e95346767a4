"""Generate golden vectors by running the reference package itself.

Run in a container where the reference is mounted (read-only) at
/root/reference:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py

It imports ``pagedkv_fusion.reference`` / ``quantize`` / ``testing_utils``
from the reference tree, evaluates them on seeded inputs and writes
``golden_*.npz`` next to this file.  Large inputs are not stored: the
fixture keeps the seed and a SHA-256 of the input bytes, and the tests
regenerate the inputs with the package's own seeded generators and check
the digest first (which also pins those generators to the reference's).
Nothing on the GPU path reads the reference at run time; only these
fixtures travel.
"""

from __future__ import annotations

import hashlib
import json
import math
import sys
from pathlib import Path

import numpy as np

REF = Path("/root/reference")
HERE = Path(__file__).resolve().parent
PKG = HERE.parent.parent / (
    "pagedkv-fusion-custom-cuda-kernels-for-kv-cache-eviction-quantized-paged-attention_b200")


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def load_reference():
    sys.path.insert(0, str(REF))
    import importlib
    ref = importlib.import_module("pagedkv_fusion.reference")
    tu = importlib.import_module("pagedkv_fusion.testing_utils")
    qz = importlib.import_module("pagedkv_fusion.quantize")
    sys.path.pop(0)
    return ref, tu, qz


def main():
    ref, tu, qz = load_reference()
    import torch

    # the package's own generators, loaded by path (the reference package
    # has the same top-level name)
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "pkv_problems", PKG / "pagedkv_fusion" / "problems.py")
    problems = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(problems)

    meta = {"numpy": np.__version__, "torch": torch.__version__,
            "reference": "pagedkv-fusion 0.1.1"}

    # ---------------- eviction -------------------------------------------
    ev = {}
    # (a) the reference test's random problem (tests/test_eviction.py:11-16)
    rng = np.random.default_rng(1234)
    rec = rng.random(64, dtype=np.float32)
    freq = rng.random(64, dtype=np.float32)
    att = rng.random((64, 16), dtype=np.float32)
    msk = rng.random((64, 16)) > 0.2
    ev["rand64_rec"], ev["rand64_freq"], ev["rand64_attn"], ev["rand64_mask"] = rec, freq, att, msk
    ev["rand64_scores"] = ref.eviction_scores_ref(rec, freq, att, msk, 0.4, 0.3, 0.3)
    # (b) many block sizes, random masks, some fully invalid blocks, -0.0
    for bs in (1, 3, 7, 8, 9, 16, 17, 32, 33, 100, 128, 129, 200):
        rng = np.random.default_rng(100 + bs)
        nb = 37
        rec = rng.random(nb, dtype=np.float32)
        freq = rng.random(nb, dtype=np.float32)
        att = (rng.standard_normal((nb, bs)) * 3).astype(np.float32)
        att[0, 0] = -0.0
        msk = rng.random((nb, bs)) > 0.3
        msk[1] = False
        msk[2] = True
        ev[f"bs{bs}_rec"], ev[f"bs{bs}_freq"], ev[f"bs{bs}_attn"], ev[f"bs{bs}_mask"] = (
            rec, freq, att, msk)
        ev[f"bs{bs}_scores"] = ref.eviction_scores_ref(rec, freq, att, msk)
        ev[f"bs{bs}_scores_w"] = ref.eviction_scores_ref(rec, freq, att, msk, 0.7, 0.2, 0.1)
    # (c) the 16K-block eviction workload (all valid), inputs by digest
    for tag, kw in (("w16k", dict(mask="all")), ("w16k_mask", dict(mask="random")),
                    ("w16k_ties", dict(mask="all", ties=True))):
        rec, freq, att, msk = problems.eviction_problem(seed=0, **kw)
        sc = ref.eviction_scores_ref(rec, freq, att, msk)
        ev[f"{tag}_digest"] = np.array(sha(rec, freq, att, msk))
        ev[f"{tag}_scores"] = sc
        for k in (1, 2458, 8192):
            ev[f"{tag}_idx_k{k}"] = ref.select_eviction_candidates_ref(sc, k)
    # (d) selection known-answer tests
    ev["kat_scores"] = np.array([0.3, 0.1, 0.1, 0.2], np.float32)
    ev["kat_idx"] = ref.select_eviction_candidates_ref(ev["kat_scores"], 3)
    special = np.array([0.5, np.nan, -0.0, 0.0, np.inf, -np.inf, 0.5, -1.0, np.nan,
                        1e-45, -1e-45, 0.0, -0.0, 3.0], np.float32)
    ev["special_scores"] = special
    ev["special_idx"] = ref.select_eviction_candidates_ref(special, special.shape[0])
    ev["special_idx_k5"] = ref.select_eviction_candidates_ref(special, 5)
    np.savez_compressed(HERE / "golden_eviction.npz", **ev)

    # ---------------- quantization ----------------------------------------
    qd = {}
    rng = np.random.default_rng(1234)
    kv = rng.standard_normal((6, 16, 4, 64)).astype(np.float32)
    qd["rand_kv"] = kv
    qd["rand_q"], qd["rand_scale"] = ref.quantize_kv_per_block_ref(kv)
    kv = (np.random.default_rng(7).standard_normal((2, 16, 2, 32)) * 50).astype(np.float32)
    kv[1, :, 1, :] = 0.0                         # zero (block, head)
    kv[0, :, 0, :] *= 100.0                      # blown-up (block, head)
    qd["edge_kv"] = kv
    qd["edge_q"], qd["edge_scale"] = ref.quantize_kv_per_block_ref(kv)
    # exact half-way points: absmax 127 gives scale 1, so x.5 values tie
    kv = np.zeros((1, 4, 1, 32), np.float32)
    kv[0, 0, 0, :] = np.arange(32) - 15.5
    kv[0, 1, 0, :] = np.arange(32) * 0.5 - 8.0
    kv[0, 2, 0, 0] = 127.0
    kv[0, 3, 0, :] = -np.arange(32) * 0.25
    qd["tie_kv"] = kv
    qd["tie_q"], qd["tie_scale"] = ref.quantize_kv_per_block_ref(kv)
    kv16 = np.random.default_rng(11).standard_normal((5, 16, 3, 128)).astype(np.float16)
    qd["f16_kv"] = kv16
    qd["f16_q"], qd["f16_scale"] = ref.quantize_kv_per_block_ref(kv16)
    # torch twin of the reference on the same data (quantize.py:15-31)
    qt, st = qz.quantize_kv_per_block(torch.from_numpy(qd["rand_kv"]))
    qd["rand_q_torch"], qd["rand_scale_torch"] = qt.numpy(), st.numpy()
    np.savez_compressed(HERE / "golden_quantize.npz", **qd)

    # ---------------- paged attention --------------------------------------
    at = {}
    shapes = [(1, 1, 1, 32, 16, 1), (4, 8, 8, 64, 16, 200), (4, 8, 2, 128, 16, 300),
              (16, 32, 8, 128, 32, 1024)]
    for i, (S, H, Hkv, D, bs, L) in enumerate(shapes):
        # same construction as the reference GPU test (tests/test_kernels_gpu.py:61-86)
        rng = np.random.default_rng(42)
        q, k, v, bt, sl, sm = tu.make_paged_kv_problem(rng, S, H, Hkv, D, bs, L)
        rng2 = np.random.default_rng(42)
        mine = problems.make_paged_kv_problem(rng2, S, H, Hkv, D, bs, L)
        assert all(np.array_equal(a, b) for a, b in zip(mine[:5], (q, k, v, bt, sl)))
        kq, ks = qz.quantize_kv_per_block(torch.from_numpy(k))
        vq, vs = qz.quantize_kv_per_block(torch.from_numpy(v))
        out = ref.paged_attention_ref(q, kq.numpy(), ks.numpy(), vq.numpy(), vs.numpy(),
                                      bt, sl, sm)
        at[f"gpu{i}_shape"] = np.array([S, H, Hkv, D, bs, L])
        at[f"gpu{i}_digest"] = np.array(sha(q, k, v, bt, sl))
        at[f"gpu{i}_out"] = out
        at[f"gpu{i}_kscale"] = ks.numpy()
        at[f"gpu{i}_kq_digest"] = np.array(sha(kq.numpy(), vq.numpy()))
    # default-sized reference problem (make_paged_kv_problem defaults, seed 1234)
    rng = np.random.default_rng(1234)
    q, k, v, bt, sl, sm = tu.make_paged_kv_problem(rng)
    kq, ks = ref.quantize_kv_per_block_ref(k)
    vq, vs = ref.quantize_kv_per_block_ref(v)
    at["default_digest"] = np.array(sha(q, k, v, bt, sl))
    at["default_out"] = ref.paged_attention_ref(q, kq, ks, vq, vs, bt, sl, sm)
    # edge lengths around the block boundary (tests/test_paged_attention.py:74-87)
    for L in (1, 15, 16, 17):
        # first seed whose random length needs as many pages as L, so the
        # table covers L once seq_len is forced to L
        seed = 500 + L
        while True:
            rng = np.random.default_rng(seed)
            q, k, v, bt, sl, sm = tu.make_paged_kv_problem(rng, 1, 8, 4, 64, 16, L)
            if (int(sl[0]) + 15) // 16 == (L + 15) // 16:
                break
            seed += 1000
        sl[:] = L
        at[f"edge{L}_seed"] = np.array(seed)
        kq, ks = ref.quantize_kv_per_block_ref(k)
        vq, vs = ref.quantize_kv_per_block_ref(v)
        at[f"edge{L}_digest"] = np.array(sha(q, k, v, bt, sl))
        at[f"edge{L}_out"] = ref.paged_attention_ref(q, kq, ks, vq, vs, bt, sl, sm)
    # the 8 x 512 CPU-runnable decode workload
    q, k, v, bt, sl, sm = problems.decode_small_problem(0)
    kq, ks = ref.quantize_kv_per_block_ref(k)
    vq, vs = ref.quantize_kv_per_block_ref(v)
    at["small_digest"] = np.array(sha(q, k, v, bt, sl))
    at["small_codes_digest"] = np.array(sha(kq, ks, vq, vs))
    at["small_out"] = ref.paged_attention_ref(q, kq, ks, vq, vs, bt, sl, sm)
    assert math.isclose(sm, 1 / math.sqrt(128))
    np.savez_compressed(HERE / "golden_attention.npz", **at)

    (HERE / "golden_meta.json").write_text(json.dumps(meta, indent=1) + "\n")
    for f in sorted(HERE.glob("golden_*")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
