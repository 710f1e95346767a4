"""ctypes loader for the C oracle (TEST INFRASTRUCTURE ONLY)."""

from __future__ import annotations

import ctypes as ct

import numpy as np

from .build import build

_lib = None


def _load():
    global _lib
    if _lib is None:
        _lib = ct.CDLL(str(build()))
        P = ct.c_void_p
        I64 = ct.c_int64
        _lib.pkv_oracle_eviction_scores.argtypes = [P, P, P, P, P, I64, I64,
                                                    ct.c_float, ct.c_float, ct.c_float]
        _lib.pkv_oracle_eviction_scores.restype = None
        _lib.pkv_oracle_select.argtypes = [P, I64, I64, P]
        _lib.pkv_oracle_select.restype = I64
        _lib.pkv_oracle_quantize.argtypes = [P, P, P, I64, I64, I64, I64]
        _lib.pkv_oracle_quantize.restype = None
        _lib.pkv_oracle_paged_attention.argtypes = [P, P, P, P, P, P, P, P] + [I64] * 7 + [
            ct.c_double]
        _lib.pkv_oracle_paged_attention.restype = I64
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ct.c_void_p)


def eviction_scores(recency, frequency, attn, valid, w_r=0.4, w_f=0.3, w_a=0.3):
    lib = _load()
    rec = np.ascontiguousarray(recency, np.float32)
    freq = np.ascontiguousarray(frequency, np.float32)
    att = np.ascontiguousarray(attn, np.float32)
    val = np.ascontiguousarray(valid, dtype=bool).view(np.uint8)
    out = np.empty(att.shape[0], np.float32)
    lib.pkv_oracle_eviction_scores(_p(rec), _p(freq), _p(att), _p(val), _p(out),
                                   att.shape[0], att.shape[1], np.float32(w_r),
                                   np.float32(w_f), np.float32(w_a))
    return out


def select(scores, k):
    lib = _load()
    s = np.ascontiguousarray(scores, np.float32)
    out = np.empty(max(0, min(k, s.shape[0])), np.int64)
    n = lib.pkv_oracle_select(_p(s), s.shape[0], k, _p(out))
    return out[:n]


def quantize(kv):
    lib = _load()
    x = np.ascontiguousarray(kv, np.float32)
    nb, bs, nkv, hd = x.shape
    q = np.empty(x.shape, np.int8)
    sc = np.empty((nb, nkv), np.float32)
    lib.pkv_oracle_quantize(_p(x), _p(q), _p(sc), nb, bs, nkv, hd)
    return q, sc


def paged_attention(q, kq, ks, vq, vs, block_tables, seq_lens, sm_scale):
    lib = _load()
    q = np.ascontiguousarray(q, np.float32)
    kq = np.ascontiguousarray(kq, np.int8)
    vq = np.ascontiguousarray(vq, np.int8)
    ks = np.ascontiguousarray(ks, np.float32)
    vs = np.ascontiguousarray(vs, np.float32)
    bt = np.ascontiguousarray(block_tables, np.int32)
    sl = np.ascontiguousarray(seq_lens, np.int32)
    out = np.empty_like(q)
    S, H, D = q.shape
    NB, bs, Hkv, _ = kq.shape
    rc = lib.pkv_oracle_paged_attention(_p(q), _p(kq), _p(ks), _p(vq), _p(vs), _p(bt),
                                        _p(sl), _p(out), S, H, Hkv, D, bs, NB,
                                        bt.shape[1], float(sm_scale))
    if rc != 0:
        raise IndexError(f"sequence {-rc - 1}: block id out of range")
    return out
