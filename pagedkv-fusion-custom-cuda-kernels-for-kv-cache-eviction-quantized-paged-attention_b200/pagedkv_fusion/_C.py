"""``pagedkv_fusion._C`` -- the native boundary, bound with ctypes.

Drop-in for the reference's pybind11 module (csrc/bindings.cpp:14-26): the
same two functions with the same argument names, defaults and error type
(``RuntimeError`` where the reference's ``TORCH_CHECK`` raises), plus the
entry points this build adds (native quantizer, deterministic selection,
sharded-eviction candidates and merge, cache writer).  Every function takes
CUDA tensors, allocates its outputs with torch's caching allocator on the
input's device, and enqueues work on that device's current stream without
synchronizing -- as the reference launcher does (quant_paged_attention.cu:
207-223).  The arithmetic happens in ``lib/libpagedkv_sm100.so``; importing
this module fails with ``ImportError`` when that library has not been built.
"""

from __future__ import annotations

import ctypes as ct
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent / "lib" / "libpagedkv_sm100.so"
if not _LIB_PATH.exists():
    raise ImportError(f"{_LIB_PATH} is not built (run build.py in the package root)")
_lib = ct.CDLL(str(_LIB_PATH))


def _load_pycall():
    """The METH_FASTCALL module over the same library (csrc/pkv_pycall.c):
    the eviction calls' arguments cost ~0.2 us there against ~2.2 us as
    ctypes conversions, on a path whose GPU time is ~13 us."""
    import importlib.machinery
    import importlib.util
    import sysconfig
    path = _LIB_PATH.parent / ("_pkv_pycall" + sysconfig.get_config_var("EXT_SUFFIX"))
    if not path.exists():
        raise ImportError(f"{path} is not built (run build.py in the package root)")
    loader = importlib.machinery.ExtensionFileLoader("_pkv_pycall", str(path))
    spec = importlib.util.spec_from_file_location("_pkv_pycall", str(path), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


_fast = _load_pycall()

_P, _I32, _I64, _F, _SZ = ct.c_void_p, ct.c_int32, ct.c_int64, ct.c_float, ct.c_size_t


def _sig(name, args, res=ct.c_int):
    fn = getattr(_lib, name)
    fn.argtypes = args
    fn.restype = res
    return fn


_last_error = _sig("pkv_last_error_string", [], ct.c_char_p)
_version = _sig("pkv_version", [])
_read_err = _sig("pkv_read_device_error", [_P, ct.c_int])
_scores = _sig("pkv_eviction_scores", [_P, _P, _P, _P, _P, _I64, _I32, _F, _F, _F, _P])
_select_ws = _sig("pkv_eviction_select_workspace_size", [_I64, _I64], _SZ)
_select = _sig("pkv_eviction_select", [_P, _I64, _I64, _P, _P, _SZ, _P])
_fused_ws = _sig("pkv_eviction_scores_select_workspace_size", [_I64, _I64], _SZ)
_fused = _sig("pkv_eviction_scores_select",
              [_P, _P, _P, _P, _P, _I64, _I32, _F, _F, _F, _I64, _P, _P, _SZ, _P])
_local = _sig("pkv_eviction_local_candidates", [_P, _I64, _I64, _I64, _P, _P, _SZ, _P])
_merge_ws = _sig("pkv_eviction_merge_workspace_size", [_I64, _I64], _SZ)
_merge = _sig("pkv_eviction_merge", [_P, _I64, _I64, _P, _P, _SZ, _P])
_quant = _sig("pkv_quantize_kv_per_block", [_P, _I32, _P, _P, _I64, _I32, _I32, _I32, _P])
_attn_ws = _sig("pkv_quant_paged_attention_workspace_size", [_I32] * 6, _SZ)
_attn_launches = _sig("pkv_quant_paged_attention_kernel_launches", [_I32] * 6, ct.c_int)
_quant_except = _sig("pkv_quantize_kv_per_block_except",
                     [_P, _I32, _P, _P, _P, _I64, _I32, _I32, _I32, _P])
_mark = _sig("pkv_mark_blocks", [_P, _I64, _I64, _I64, _P, _P])
_stats_ws = _sig("pkv_attention_stats_workspace_size", [_I64, _I32, _I32], _SZ)
_stats = _sig("pkv_attention_stats", [_P, _I32, _P, _P, _I64, _I32, _I32, _I32, _F, _P, _SZ, _P])
_compact = _sig("pkv_compact_block_tables", [_P, _P, _P, _P, _P, _I32, _I32, _I32, _I64, _P])
_attn = _sig("pkv_quant_paged_attention",
             [_P] * 8 + [_I32] * 5 + [_I64, _I32, _F, _P, _SZ, _P])
_wtc_ws = _sig("pkv_write_to_cache_workspace_size", [_I64, _I32], _SZ)
_wtc = _sig("pkv_write_to_cache",
            [_P, _P, _I32, _P, _P, _P, _I64, _I64, _I32, _I32, _I32, _P, _SZ, _P])

LIBRARY_PATH = str(_LIB_PATH)
_DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


# Workspace bytes per (num_blocks, k, device).  The size depends on the
# selection path, which PKV_EVICTION_MULTI_KERNEL can change between calls;
# a call that finds its cached size too small (PKV_ERR_WORKSPACE) asks the
# library again and retries once, so the environment is not read per call.
_FUSED_WS_CACHE: dict = {}
_SELECT_WS_CACHE: dict = {}
_ERR_WORKSPACE = 3


def _check(rc: int):
    if rc != 0:
        raise RuntimeError(_last_error().decode() or f"pagedkv_fusion error {rc}")


def _require(cond: bool, msg: str):
    if not cond:
        raise RuntimeError(msg)


def _stream(t: torch.Tensor) -> int:
    """Raw cudaStream_t of the current stream on ``t``'s device."""
    return torch._C._cuda_getCurrentRawStream(t.device.index)


def _workspace(nbytes: int, device) -> tuple[torch.Tensor | None, int]:
    if nbytes == 0:
        return None, 0
    ws = torch.empty(nbytes, dtype=torch.uint8, device=device)
    return ws, ws.data_ptr()


def version() -> int:
    return _version()


def read_device_error(reset: bool = True) -> int:
    """Synchronizes the current device and returns (and by default clears)
    the error code kernels recorded there (0 = none)."""
    code = ct.c_int32(0)
    rc = _read_err(ct.byref(code), 1 if reset else 0)
    if rc not in (0, 5):
        _check(rc)
    return int(code.value)


# ---------------------------------------------------------------------------
# Reference-module functions (csrc/bindings.cpp:16-25)
# ---------------------------------------------------------------------------

_F32, _BOOL = torch.float32, torch.bool


def eviction_scores(recency, frequency, attn_weights, valid_mask, w_recency=0.4,
                    w_frequency=0.3, w_attention=0.3):
    """Fused eviction score per block; see reference.py:38-71."""
    if not (recency.is_cuda and frequency.is_cuda and attn_weights.is_cuda
            and valid_mask.is_cuda):
        raise RuntimeError("all inputs must be CUDA tensors")
    if recency.dtype is not _F32:
        raise RuntimeError("recency must be float32")
    if attn_weights.dim() != 2:
        raise RuntimeError("attn_weights must be [num_blocks, block_size]")
    if valid_mask.dtype is not _BOOL:
        raise RuntimeError("valid_mask must be bool")
    if frequency.dtype is not _F32 or attn_weights.dtype is not _F32:
        raise RuntimeError("frequency and attn_weights must be float32")
    nb, bs = attn_weights.shape
    if valid_mask.shape != attn_weights.shape or recency.numel() != nb or frequency.numel() != nb:
        raise RuntimeError("valid_mask must match attn_weights; recency/frequency need "
                           "num_blocks entries")
    rec = recency if recency.is_contiguous() else recency.contiguous()
    freq = frequency if frequency.is_contiguous() else frequency.contiguous()
    att = attn_weights if attn_weights.is_contiguous() else attn_weights.contiguous()
    msk = valid_mask if valid_mask.is_contiguous() else valid_mask.contiguous()
    out = torch.empty(nb, dtype=_F32, device=rec.device)
    rc = _fast.eviction_scores(rec.data_ptr(), freq.data_ptr(), att.data_ptr(), msk.data_ptr(),
                               out.data_ptr(), nb, bs, float(w_recency), float(w_frequency),
                               float(w_attention),
                               torch._C._cuda_getCurrentRawStream(rec.device.index))
    if rc:
        _check(rc)
    return out


def quant_paged_attention(q, k_cache_q, k_scale, v_cache_q, v_scale, block_tables, seq_lens,
                          sm_scale):
    """INT8 paged decode attention; see reference.py:140-173."""
    _require(q.is_cuda, "q must be a CUDA tensor")
    _require(all(t.is_cuda for t in (k_cache_q, k_scale, v_cache_q, v_scale, block_tables,
                                     seq_lens)), "all inputs must be CUDA tensors")
    _require(q.dtype == torch.float32, "q must be float32 (v1)")
    _require(k_cache_q.dtype == torch.int8, "k_cache_q must be int8")
    _require(v_cache_q.dtype == torch.int8, "v_cache_q must be int8")
    _require(k_scale.dtype == torch.float32 and v_scale.dtype == torch.float32,
             "k_scale/v_scale must be float32")
    _require(block_tables.dtype == torch.int32, "block_tables must be int32")
    _require(q.dim() == 3 and k_cache_q.dim() == 4 and block_tables.dim() == 2,
             "expected q [S, H, D], caches [NB, bs, Hkv, D], block_tables [S, M]")
    S, H, D = q.shape
    NB, bs, Hkv, Dk = k_cache_q.shape
    _require(Dk == D and tuple(v_cache_q.shape) == tuple(k_cache_q.shape),
             "cache head_dim must match q")
    _require(tuple(k_scale.shape) == (NB, Hkv) and tuple(v_scale.shape) == (NB, Hkv),
             "scales must be [num_blocks, num_kv_heads]")
    _require(block_tables.shape[0] == S and seq_lens.numel() == S,
             "block_tables/seq_lens must have num_seqs rows")
    qc, kc, ks = q.contiguous(), k_cache_q.contiguous(), k_scale.contiguous()
    vc, vs, bt = v_cache_q.contiguous(), v_scale.contiguous(), block_tables.contiguous()
    sl = seq_lens.to(torch.int32).contiguous()
    out = torch.empty_like(qc)
    M = bt.shape[1]
    ws, wp = _workspace(_attn_ws(S, H, Hkv, D, bs, M), qc.device)
    _check(_attn(qc.data_ptr(), kc.data_ptr(), ks.data_ptr(), vc.data_ptr(), vs.data_ptr(),
                 bt.data_ptr(), sl.data_ptr(), out.data_ptr(), S, H, Hkv, D, bs, NB, M,
                 float(sm_scale), wp, 0 if ws is None else ws.numel(), _stream(qc)))
    return out


# ---------------------------------------------------------------------------
# Entry points added by this build
# ---------------------------------------------------------------------------

def quant_paged_attention_kernel_launches(num_seqs, num_heads, num_kv_heads, head_dim, block_size,
                                          max_blocks_per_seq):
    """Kernels one quant_paged_attention call of these shapes launches."""
    return int(_attn_launches(num_seqs, num_heads, num_kv_heads, head_dim, block_size,
                              max_blocks_per_seq))


def quantize_kv_per_block(kv, out_q=None, out_scale=None):
    """Native per-(block, head) INT8 quantization; see reference.py:88-105.

    ``out_q`` / ``out_scale`` (contiguous int8 / float32 CUDA tensors of the
    result shapes, e.g. slices of a paged cache) receive the result in place
    when given.
    """
    _require(kv.is_cuda, "kv must be a CUDA tensor")
    if kv.dim() != 4:
        raise ValueError(f"expected 4D [nb, bs, nkv, hd], got {tuple(kv.shape)}")
    _require(kv.dtype in _DTYPE_CODE, "kv must be float32, float16 or bfloat16")
    x = kv.contiguous()
    nb, bs, nkv, hd = x.shape
    if out_q is None:
        q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    else:
        _require(out_q.dtype == torch.int8 and tuple(out_q.shape) == tuple(x.shape)
                 and out_q.is_contiguous() and out_q.device == x.device,
                 "out_q must be a contiguous int8 tensor shaped like kv")
        q = out_q
    if out_scale is None:
        scale = torch.empty((nb, nkv), dtype=torch.float32, device=x.device)
    else:
        _require(out_scale.dtype == torch.float32 and tuple(out_scale.shape) == (nb, nkv)
                 and out_scale.is_contiguous() and out_scale.device == x.device,
                 "out_scale must be a contiguous float32 [num_blocks, num_kv_heads] tensor")
        scale = out_scale
    _check(_quant(x.data_ptr(), _DTYPE_CODE[x.dtype], q.data_ptr(), scale.data_ptr(), nb, bs,
                  nkv, hd, _stream(x)))
    return q, scale


def quantize_kv_per_block_except(kv, skip, out_q, out_scale):
    """quantize_kv_per_block into ``out_q`` / ``out_scale`` for the blocks
    whose ``skip`` byte is zero; blocks with a nonzero byte are left as they
    are (the survivors of an eviction are quantized, the evicted ones not)."""
    _require(kv.is_cuda and skip.is_cuda, "kv and skip must be CUDA tensors")
    if kv.dim() != 4:
        raise ValueError(f"expected 4D [nb, bs, nkv, hd], got {tuple(kv.shape)}")
    _require(kv.dtype in _DTYPE_CODE, "kv must be float32, float16 or bfloat16")
    x = kv.contiguous()
    nb, bs, nkv, hd = x.shape
    _require(skip.dtype in (torch.uint8, torch.bool) and skip.numel() == nb and skip.is_contiguous(),
             "skip must be a contiguous uint8/bool [num_blocks] tensor")
    _require(out_q.dtype == torch.int8 and tuple(out_q.shape) == tuple(x.shape)
             and out_q.is_contiguous() and out_q.device == x.device,
             "out_q must be a contiguous int8 tensor shaped like kv")
    _require(out_scale.dtype == torch.float32 and tuple(out_scale.shape) == (nb, nkv)
             and out_scale.is_contiguous() and out_scale.device == x.device,
             "out_scale must be a contiguous float32 [num_blocks, num_kv_heads] tensor")
    _check(_quant_except(x.data_ptr(), _DTYPE_CODE[x.dtype], skip.data_ptr(), out_q.data_ptr(),
                         out_scale.data_ptr(), nb, bs, nkv, hd, _stream(x)))
    return out_q, out_scale


def attention_stats(k, q, sm_scale: float):
    """Per-token attention weights ``[num_blocks, block_size]`` derived from the
    key pool ``k`` ``[nb, bs, Hkv, 128]`` and one query per KV head ``q``
    ``[Hkv, 128]``: mean over heads of exp(s - max s), s = sm_scale * q.k."""
    _require(k.is_cuda and q.is_cuda, "k and q must be CUDA tensors")
    _require(k.dim() == 4 and k.dtype in _DTYPE_CODE, "k must be [nb, bs, nkv, hd] float32/16/bf16")
    nb, bs, nkv, hd = k.shape
    _require(q.dtype == torch.float32 and tuple(q.shape) == (nkv, hd), "q must be float32 [nkv, hd]")
    kc, qc = k.contiguous(), q.contiguous()
    attn = torch.empty((nb, bs), dtype=torch.float32, device=kc.device)
    ws, wp = _workspace(_stats_ws(nb, bs, nkv), kc.device)
    _check(_stats(kc.data_ptr(), _DTYPE_CODE[kc.dtype], qc.data_ptr(), attn.data_ptr(), nb, bs,
                  nkv, hd, float(sm_scale), wp, 0 if ws is None else ws.numel(), _stream(kc)))
    return attn


def mark_blocks(ids, id_offset: int, num_blocks: int):
    """uint8 [num_blocks] mask with 1 at ``id - id_offset`` for each id of
    ``ids`` (int64, global block ids) that falls in this range."""
    _require(ids.is_cuda, "ids must be a CUDA tensor")
    _require(ids.dtype == torch.int64 and ids.dim() == 1, "ids must be int64 [n]")
    i = ids.contiguous()
    mask = torch.empty(int(num_blocks), dtype=torch.uint8, device=i.device)
    _check(_mark(i.data_ptr(), i.numel(), int(id_offset), int(num_blocks), mask.data_ptr(),
                 _stream(i)))
    return mask


def compact_block_tables(block_tables, seq_lens, evicted, num_blocks: int, block_size: int):
    """Block tables without the evicted blocks and the tokens each sequence
    keeps: ``(tables, lens)``, int32, a valid input to quant_paged_attention."""
    _require(block_tables.is_cuda and seq_lens.is_cuda and evicted.is_cuda,
             "all inputs must be CUDA tensors")
    _require(block_tables.dtype == torch.int32 and block_tables.dim() == 2,
             "block_tables must be int32 [S, M]")
    _require(evicted.dtype in (torch.uint8, torch.bool) and evicted.numel() == int(num_blocks),
             "evicted must be a uint8/bool [num_blocks] mask")
    bt = block_tables.contiguous()
    S, M = bt.shape
    sl = seq_lens.to(torch.int32).contiguous()
    _require(sl.numel() == S, "seq_lens must have num_seqs entries")
    ev = evicted.contiguous()
    out_bt = torch.empty_like(bt)
    out_sl = torch.empty_like(sl)
    _check(_compact(bt.data_ptr(), sl.data_ptr(), ev.data_ptr(), out_bt.data_ptr(),
                    out_sl.data_ptr(), S, M, int(block_size), int(num_blocks), _stream(bt)))
    return out_bt, out_sl


def eviction_select(scores, k: int):
    """Indices of the k lowest scores, ascending by (score, id); int64."""
    if not scores.is_cuda:
        raise RuntimeError("scores must be a CUDA tensor")
    if scores.dtype is not _F32 or scores.dim() != 1:
        raise RuntimeError("scores must be float32 [n]")
    k = int(k)
    if k < 0:
        raise RuntimeError("k must be non-negative")
    s = scores if scores.is_contiguous() else scores.contiguous()
    n = s.numel()
    kk = k if k < n else n
    out = torch.empty(kk, dtype=torch.int64, device=s.device)
    if kk == 0:
        return out
    dev = s.device.index
    key = (n, kk, dev)
    nbytes = _SELECT_WS_CACHE.get(key)
    if nbytes is None:
        nbytes = _SELECT_WS_CACHE[key] = _select_ws(n, kk)
    stream = torch._C._cuda_getCurrentRawStream(dev)
    for attempt in (0, 1):
        ws = torch.empty(nbytes, dtype=torch.uint8, device=s.device) if nbytes else None
        rc = _fast.eviction_select(s.data_ptr(), n, kk, out.data_ptr(),
                                   None if ws is None else ws.data_ptr(), nbytes, stream)
        if rc != _ERR_WORKSPACE or attempt:
            break
        nbytes = _SELECT_WS_CACHE[key] = _select_ws(n, kk)
    if rc:
        _check(rc)
    return out


def eviction_scores_select(recency, frequency, attn_weights, valid_mask, k: int,
                           w_recency=0.4, w_frequency=0.3, w_attention=0.3):
    """Scores and the k selected block ids from one call: ``(scores, idx)``.

    Checks are plain attribute tests, the workspace size is cached per
    (num_blocks, k, device) and the call goes through the METH_FASTCALL
    module: this call sits on the eviction latency path, where a few
    microseconds of host time are a large share of the total.
    """
    if not (recency.is_cuda and frequency.is_cuda and attn_weights.is_cuda
            and valid_mask.is_cuda):
        raise RuntimeError("all inputs must be CUDA tensors")
    if recency.dtype is not _F32 or frequency.dtype is not _F32 or attn_weights.dtype is not _F32:
        raise RuntimeError("recency/frequency/attn must be float32")
    if attn_weights.dim() != 2:
        raise RuntimeError("attn_weights must be [num_blocks, block_size]")
    if valid_mask.dtype is not _BOOL:
        raise RuntimeError("valid_mask must be bool")
    k = int(k)
    if k < 0:
        raise RuntimeError("k must be non-negative")
    nb, bs = attn_weights.shape
    if valid_mask.shape != attn_weights.shape:
        raise RuntimeError("valid_mask must match attn_weights")
    rec = recency if recency.is_contiguous() else recency.contiguous()
    freq = frequency if frequency.is_contiguous() else frequency.contiguous()
    att = attn_weights if attn_weights.is_contiguous() else attn_weights.contiguous()
    msk = valid_mask if valid_mask.is_contiguous() else valid_mask.contiguous()
    dev = rec.device
    scores = torch.empty(nb, dtype=_F32, device=dev)
    kk = k if k < nb else nb
    idx = torch.empty(kk, dtype=torch.int64, device=dev)
    key = (nb, kk, dev.index)
    nbytes = _FUSED_WS_CACHE.get(key)
    if nbytes is None:
        nbytes = _FUSED_WS_CACHE[key] = _fused_ws(nb, kk) if kk else 0
    stream = torch._C._cuda_getCurrentRawStream(dev.index)
    for attempt in (0, 1):
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev) if nbytes else None
        rc = _fast.eviction_scores_select(
            rec.data_ptr(), freq.data_ptr(), att.data_ptr(), msk.data_ptr(), scores.data_ptr(), nb,
            bs, float(w_recency), float(w_frequency), float(w_attention), kk, idx.data_ptr(),
            None if ws is None else ws.data_ptr(), nbytes, stream)
        if rc != _ERR_WORKSPACE or attempt:
            break
        nbytes = _FUSED_WS_CACHE[key] = _fused_ws(nb, kk) if kk else 0
    if rc:
        _check(rc)
    return scores, idx


def eviction_local_candidates(scores, k: int, id_offset: int = 0):
    """This rank's min(k, n) smallest candidate keys (uint64 bit patterns
    in an int64 tensor): orderable(score) << 32 | (id_offset + i)."""
    _require(scores.is_cuda and scores.dtype == torch.float32, "scores must be CUDA float32")
    s = scores.contiguous()
    n = s.numel()
    kk = min(int(k), n)
    out = torch.empty(kk, dtype=torch.int64, device=s.device)
    if kk == 0:
        return out
    ws, wp = _workspace(_merge_ws(n, kk), s.device)
    _check(_local(s.data_ptr(), n, kk, int(id_offset), out.data_ptr(), wp, ws.numel(),
                  _stream(s)))
    return out


def eviction_merge(keys, k: int):
    """Block ids of the k smallest gathered candidate keys, ascending."""
    _require(keys.is_cuda and keys.dtype == torch.int64, "keys must be a CUDA int64 tensor")
    c = keys.contiguous()
    n = c.numel()
    kk = min(int(k), n)
    out = torch.empty(kk, dtype=torch.int64, device=c.device)
    if kk == 0:
        return out
    ws, wp = _workspace(_merge_ws(n, kk), c.device)
    _check(_merge(c.data_ptr(), n, kk, out.data_ptr(), wp, ws.numel(), _stream(c)))
    return out


def write_to_cache(key, value, kv_cache_int8, scale_cache, slot_mapping, block_size: int):
    """Quantize + scatter new tokens into the [2, NB, bs, Hkv, D] cache
    (integration/vllm/pagedkv_fusion_backend.py:63-95 semantics)."""
    _require(all(t.is_cuda for t in (key, value, kv_cache_int8, scale_cache, slot_mapping)),
             "all inputs must be CUDA tensors")
    _require(key.dtype in _DTYPE_CODE and value.dtype == key.dtype,
             "key/value must share a float32/float16/bfloat16 dtype")
    _require(kv_cache_int8.dtype == torch.int8 and kv_cache_int8.dim() == 5
             and kv_cache_int8.shape[0] == 2, "kv_cache_int8 must be int8 [2, NB, bs, Hkv, D]")
    _require(kv_cache_int8.is_contiguous() and scale_cache.is_contiguous(),
             "caches must be contiguous (they are written in place)")
    _, NB, bs, Hkv, D = kv_cache_int8.shape
    _require(int(block_size) == bs, "block_size must match the cache")
    _require(scale_cache.dtype == torch.float32 and tuple(scale_cache.shape) == (2, NB, Hkv),
             "scale_cache must be float32 [2, NB, Hkv]")
    kc, vc = key.contiguous(), value.contiguous()
    _require(tuple(kc.shape[1:]) == (Hkv, D) and kc.shape == vc.shape,
             "key/value must be [num_tokens, Hkv, D]")
    sm = slot_mapping.to(torch.int64).contiguous()
    nt = kc.shape[0]
    ws, wp = _workspace(_wtc_ws(nt, Hkv), kc.device)
    _check(_wtc(kc.data_ptr(), vc.data_ptr(), _DTYPE_CODE[kc.dtype], kv_cache_int8.data_ptr(),
                scale_cache.data_ptr(), sm.data_ptr(), nt, NB, bs, Hkv, D, wp,
                0 if ws is None else ws.numel(), _stream(kc)))
