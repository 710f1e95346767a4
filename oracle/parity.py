"""Sampled decode parity for device-resident workloads (TEST INFRASTRUCTURE ONLY).

A decode step over a cache of tens of GB cannot be restated on the CPU in
full, but every sequence's output depends only on its own pages.  This
checker copies the pages of a few sequences of a device-resident paged
cache to the host, renumbers them, evaluates ``paged_attention_ref``
(reference ``pagedkv_fusion/reference.py:140-173``) in double precision
with the C oracle, and compares those sequences' rows of the kernel's
output.  Used by the tests and by the benchmark after its timed region.
"""

from __future__ import annotations

import numpy as np

from . import c_oracle

ATTN_RTOL = 2e-4   # reference gate, tests/test_kernels_gpu.py:84
ATTN_ATOL = 2e-4
ATTN_MAXREL = 1e-3  # max |got - ref| / max |ref|


def sample_sequences(seq_lens, n: int) -> np.ndarray:
    """Up to ``n`` sequence indices: the shortest, the longest and the rest
    evenly spaced in index order."""
    lens = np.asarray(seq_lens)
    S = len(lens)
    if S == 0:
        return np.zeros(0, np.int64)
    pick = set(np.linspace(0, S - 1, max(1, min(n, S) - 2)).astype(int).tolist())
    pick.add(int(np.argmin(lens)))
    pick.add(int(np.argmax(lens)))
    return np.array(sorted(pick), dtype=np.int64)


def sampled_decode_parity(q, k_cache, k_scale, v_cache, v_scale, block_tables, seq_lens,
                          sm_scale: float, out, picks) -> dict:
    """Oracle check of ``out`` (the kernel's ``[S, H, D]`` result, any
    device) on the sequences ``picks``.  ``q`` and the caches are torch
    tensors (device or host), ``block_tables`` / ``seq_lens`` host arrays or
    tensors.  Returns ``{"sampled_seqs", "sampled_tokens", "max_rel_err",
    "max_abs_err", "allclose", "ok"}``; ``ok`` means within the attention
    tolerance (elementwise rtol/atol 2e-4 and max relative error 1e-3)."""
    import torch

    bt = block_tables.cpu().numpy() if isinstance(block_tables, torch.Tensor) else \
        np.asarray(block_tables)
    sl = seq_lens.cpu().numpy() if isinstance(seq_lens, torch.Tensor) else np.asarray(seq_lens)
    picks = np.asarray(picks, dtype=np.int64)
    bs = int(k_cache.shape[1])
    M = bt.shape[1]
    sub_len = np.clip(sl[picks].astype(np.int64), 0, M * bs)
    sub_pages = (sub_len + bs - 1) // bs
    width = max(1, int(sub_pages.max()) if len(picks) else 1)
    sub_bt = np.full((len(picks), width), -1, dtype=np.int32)
    used = []
    for i, s in enumerate(picks):
        used.append(bt[s, :sub_pages[i]].astype(np.int64))
    flat = np.concatenate(used) if used else np.zeros(0, np.int64)
    uniq, inv = np.unique(flat, return_inverse=True)
    pos = 0
    for i in range(len(picks)):
        n = int(sub_pages[i])
        sub_bt[i, :n] = inv[pos:pos + n]
        pos += n
    idx = torch.from_numpy(uniq).to(k_cache.device)
    kq = k_cache.index_select(0, idx).cpu().numpy()
    vq = v_cache.index_select(0, idx).cpu().numpy()
    ks = k_scale.index_select(0, idx).cpu().numpy()
    vs = v_scale.index_select(0, idx).cpu().numpy()
    qp = q.index_select(0, torch.from_numpy(picks).to(q.device)).cpu().numpy()
    want = c_oracle.paged_attention(qp, kq, ks, vq, vs, sub_bt, sub_len.astype(np.int32),
                                    sm_scale)
    got = out.index_select(0, torch.from_numpy(picks).to(out.device)).cpu().numpy()
    abs_err = float(np.abs(got - want).max()) if got.size else 0.0
    rel = abs_err / max(float(np.abs(want).max()) if want.size else 0.0, 1e-30)
    close = bool(np.allclose(got, want, rtol=ATTN_RTOL, atol=ATTN_ATOL))
    return {"sampled_seqs": int(len(picks)), "sampled_tokens": int(sub_len.sum()),
            "max_rel_err": rel, "max_abs_err": abs_err, "allclose": close,
            "ok": bool(close and rel <= ATTN_MAXREL and np.isfinite(got).all())}
