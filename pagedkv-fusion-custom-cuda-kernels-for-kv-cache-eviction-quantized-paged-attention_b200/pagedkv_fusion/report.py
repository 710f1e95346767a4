"""Memory / quality / speed report of the INT8 paged decode, with the
sections and JSON keys of the reference's benchmarks/bench_quant_attention.py
(``{"memory": [...], "quality": [...], "speed": [...]}``), measured on this
package's kernels.

* memory  -- KV-cache bytes, INT8 + fp32 scales vs fp16 (exact arithmetic),
             for the reference's three cache configurations.
* quality -- output RMSE / max |error| of the INT8 decode (native quantize +
             native decode) against fp32 attention on the unquantized K/V,
             for N(0,1) and heavy-tailed (x8 scale, 0.1 % of K x10) caches,
             on the reference's 8 x 512 problem recipe.
* speed   -- decode-step latency of the INT8 kernel (one ``ops`` call +
             synchronize, p50 wall) and of fp16 ``scaled_dot_product_attention``
             over the same K/V gathered dense (the reference's baseline),
             at its shapes: 32 query / 8 KV heads, D 128, bs 16.

Usage: ``python -m pagedkv_fusion.report --out results/quant_bench.json``
"""

from __future__ import annotations

import argparse
import json
import statistics
import time
from pathlib import Path

import numpy as np
import torch

from . import ops, problems
from .quantize import quantize_kv_per_block


def kv_bytes_fp16(num_blocks, block_size, num_kv_heads, head_dim):
    return 2 * num_blocks * block_size * num_kv_heads * head_dim * 2


def kv_bytes_int8(num_blocks, block_size, num_kv_heads, head_dim):
    return 2 * num_blocks * block_size * num_kv_heads * head_dim + 2 * num_blocks * num_kv_heads * 4


def measure_memory(cfgs):
    rows = []
    for c in cfgs:
        fp16, int8 = kv_bytes_fp16(**c), kv_bytes_int8(**c)
        rows.append(c | {"fp16_MiB": fp16 / 2**20, "int8_MiB": int8 / 2**20,
                         "savings_pct": 100 * (1 - int8 / fp16)})
    return rows


def _fp32_paged_attention(q, k, v, block_tables, seq_lens, sm_scale):
    """fp32 attention over the unquantized pages (GQA: kv head = h // group)."""
    out = torch.empty_like(q)
    bs, hkv = k.shape[1], k.shape[2]
    group = q.shape[1] // hkv
    for s in range(q.shape[0]):
        L = int(seq_lens[s])
        blocks = block_tables[s, :(L + bs - 1) // bs].long()
        ks = k[blocks].reshape(-1, hkv, k.shape[3])[:L].repeat_interleave(group, dim=1)
        vs = v[blocks].reshape(-1, hkv, v.shape[3])[:L].repeat_interleave(group, dim=1)
        logits = torch.einsum("hd,thd->ht", q[s], ks) * sm_scale
        out[s] = torch.einsum("ht,thd->hd", torch.softmax(logits, dim=-1), vs)
    return out


def measure_quality(seed=0):
    rows = []
    dev = torch.device("cuda", torch.cuda.current_device())
    for name, kv_scale in (("gaussian_unit", 1.0), ("heavy_tail_x8", 8.0)):
        rng = np.random.default_rng(seed)
        q, k, v, bt, sl, sm = problems.make_paged_kv_problem(rng, num_seqs=8, max_seq_len=512,
                                                             kv_scale=kv_scale)
        if name == "heavy_tail_x8":
            spike = rng.random(k.shape) < 0.001
            k = np.where(spike, k * 10, k).astype(np.float32)
        qd, kd, vd = (torch.from_numpy(a).to(dev) for a in (q, k, v))
        btd, sld = torch.from_numpy(bt).to(dev), torch.from_numpy(sl).to(dev)
        kq, ks = quantize_kv_per_block(kd)
        vq, vs = quantize_kv_per_block(vd)
        out_q = ops.quant_paged_attention(qd, kq, ks, vq, vs, btd, sld, sm)
        out_fp = _fp32_paged_attention(qd, kd, vd, btd, sld, sm)
        err = (out_q - out_fp).double()
        rows.append({"distribution": name,
                     "rmse": float(err.pow(2).mean().sqrt()),
                     "max_abs": float(err.abs().max()),
                     "out_std": float(out_fp.double().std())})
    return rows


def _sdpa_gathered(qf, kf, vf, num_seqs, seq_len, num_heads, num_kv_heads, head_dim):
    kg = kf.reshape(num_seqs, seq_len, num_kv_heads, head_dim)
    vg = vf.reshape(num_seqs, seq_len, num_kv_heads, head_dim)
    kg = kg.repeat_interleave(num_heads // num_kv_heads, dim=2)
    vg = vg.repeat_interleave(num_heads // num_kv_heads, dim=2)
    return torch.nn.functional.scaled_dot_product_attention(
        qf[:, :, None, :].transpose(1, 2), kg.transpose(1, 2), vg.transpose(1, 2))


def _p50_ms(fn, iters):
    ts = []
    for _ in range(iters):
        t0 = time.perf_counter()
        fn()
        torch.cuda.synchronize()
        ts.append((time.perf_counter() - t0) * 1e3)
    return statistics.median(ts)


def measure_speed(iters=20):
    rows = []
    dev = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    for num_seqs, seq_len in ((8, 512), (32, 1024), (64, 2048)):
        num_heads, num_kv_heads, head_dim, bs = 32, 8, 128, 16
        n_blk = num_seqs * ((seq_len + bs - 1) // bs)
        k = torch.randn((n_blk, bs, num_kv_heads, head_dim), generator=g, device=dev)
        v = torch.randn((n_blk, bs, num_kv_heads, head_dim), generator=g, device=dev)
        kq, ksc = quantize_kv_per_block(k)
        vq, vsc = quantize_kv_per_block(v)
        bt = torch.arange(n_blk, dtype=torch.int32, device=dev).reshape(num_seqs, -1)
        sl = torch.full((num_seqs,), seq_len, dtype=torch.int32, device=dev)
        q = torch.randn((num_seqs, num_heads, head_dim), generator=g, device=dev)
        args = (q, kq, ksc, vq, vsc, bt, sl, head_dim ** -0.5)
        for _ in range(3):
            ops.quant_paged_attention(*args)
        torch.cuda.synchronize()
        int8_ms = _p50_ms(lambda: ops.quant_paged_attention(*args), iters)
        sargs = (q.half(), k.half(), v.half(), num_seqs, seq_len, num_heads, num_kv_heads, head_dim)
        _sdpa_gathered(*sargs)
        torch.cuda.synchronize()
        sdpa_ms = _p50_ms(lambda: _sdpa_gathered(*sargs), iters)
        rows.append({"num_seqs": num_seqs, "seq_len": seq_len,
                     "int8_kernel_p50_ms": int8_ms, "fp16_sdpa_gathered_p50_ms": sdpa_ms,
                     "iters": iters, "sdpa_iters": iters})
    return rows


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--out", type=Path, default=Path("results/quant_bench.json"))
    ap.add_argument("--speed-iters", type=int, default=20)
    args = ap.parse_args(argv)
    mem_cfgs = [dict(num_blocks=4096, block_size=16, num_kv_heads=8, head_dim=128),
                dict(num_blocks=16384, block_size=16, num_kv_heads=8, head_dim=128),
                dict(num_blocks=16384, block_size=16, num_kv_heads=40, head_dim=128)]
    report = {"memory": measure_memory(mem_cfgs), "quality": measure_quality(),
              "speed": measure_speed(iters=args.speed_iters)}
    args.out.parent.mkdir(parents=True, exist_ok=True)
    args.out.write_text(json.dumps(report, indent=2))
    print(json.dumps(report, indent=2))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
