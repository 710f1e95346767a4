"""Profiling workloads for the kernels, and an Nsight Compute wrapper.

The counterpart of the reference's ``scripts/profile_kernels.py`` (targets
``eviction`` and ``attention``, the same defaults), plus ``quantize`` and
``stats`` (attention statistics from an fp16 key pool).
Without ``--ncu`` it only runs the workload: a few warm-up calls, then the
calls to profile.  With ``--ncu`` it first runs the same workload without
the profiler and, only if that exits cleanly, once more under ``ncu`` with a
capture that ends by itself: one kernel (``-k``), one launch after the
warm-up (``-s``/``-c``), ``--clock-control none`` (the GPU's clocks are left
as they are).  Keep the workload small (a few GB on the device) when using
``--set full``.

    python -m pagedkv_fusion.profile_kernels attention --num-seqs 64 --seq-len 2048
    python -m pagedkv_fusion.profile_kernels quantize --blocks 60000 --ncu --out prof_q
    python -m pagedkv_fusion.profile_kernels eviction --num-blocks 16384
    python -m pagedkv_fusion.profile_kernels stats --blocks 16384 --kv-heads 8 --ncu --out prof_s
    python -m pagedkv_fusion.profile_kernels eviction --num-blocks 1200000 --ncu \
        --kernel regex:bitonic_global --per-call 12

Above 16,384 blocks the eviction call runs the multi-kernel selection
(radix prefilter, tile sorts, global merge passes) instead of the one-launch
cluster kernel; ``--ncu`` then needs ``--kernel`` (the kernel to capture)
and ``--per-call`` (how many launches matching it one call makes, so the
capture skips the warm-up calls' launches).
"""

from __future__ import annotations

import argparse
import math
import os
import shutil
import subprocess
import sys

# kernel-name pattern and launches per call of each target's calls
KERNELS = {
    "eviction": ("regex:evict_cluster", 1),  # the one-launch path (<= 16,384 blocks)
    "attention": ("regex:decode_(stream|tc_stream|tcp|tc|fast|generic)_kernel", 1),
    "quantize": ("regex:quantize_bulk", 1),
    "stats": ("regex:attn_logits", 1),
}


def _eviction(args, torch):
    from pagedkv_fusion import ops
    g = torch.Generator(device="cuda").manual_seed(0)
    n, bs = args.num_blocks, args.block_size
    rec = torch.rand(n, device="cuda", generator=g)
    freq = torch.rand(n, device="cuda", generator=g)
    attn = torch.rand(n, bs, device="cuda", generator=g)
    mask = torch.ones(n, bs, dtype=torch.bool, device="cuda")
    k = int(n * 0.15)
    return lambda: ops.eviction_scores_and_candidates(rec, freq, attn, mask, k)


def _attention(args, torch):
    from pagedkv_fusion import _C, ops
    g = torch.Generator(device="cuda").manual_seed(0)
    S, L, H, Hkv, bs, D = (args.num_seqs, args.seq_len, args.heads, args.kv_heads,
                           args.block_size, 128)
    pages = (L + bs - 1) // bs
    nb = S * pages
    kq = torch.empty((nb, bs, Hkv, D), dtype=torch.int8, device="cuda")
    vq = torch.empty_like(kq)
    ks = torch.empty((nb, Hkv), dtype=torch.float32, device="cuda")
    vs = torch.empty_like(ks)
    step = max(1, (1 << 28) // (bs * Hkv * D * 4))  # build the cache in 256 MB slices
    for b0 in range(0, nb, step):
        b1 = min(nb, b0 + step)
        for out_q, out_s in ((kq, ks), (vq, vs)):
            x = torch.randn((b1 - b0, bs, Hkv, D), device="cuda", generator=g)
            _C.quantize_kv_per_block(x, out_q=out_q[b0:b1], out_scale=out_s[b0:b1])
    bt = torch.randperm(nb, device="cuda", generator=g).to(torch.int32).reshape(S, pages)
    sl = torch.full((S,), L, dtype=torch.int32, device="cuda")
    q = torch.randn((S, H, D), device="cuda", generator=g)
    a = (q, kq, ks, vq, vs, bt.contiguous(), sl, 1.0 / math.sqrt(D))
    return lambda: ops.quant_paged_attention(*a)


def _quantize(args, torch):
    from pagedkv_fusion import _C
    g = torch.Generator(device="cuda").manual_seed(0)
    nb, Hkv = args.blocks, args.kv_heads
    x = torch.randn((nb, 16, Hkv, 128), device="cuda", dtype=torch.float16, generator=g)
    skip = (torch.rand(nb, device="cuda", generator=g) < args.skip_fraction).to(torch.uint8)
    q = torch.empty(x.shape, dtype=torch.int8, device="cuda")
    s = torch.empty((nb, Hkv), dtype=torch.float32, device="cuda")
    return lambda: _C.quantize_kv_per_block_except(x, skip, q, s)


def _stats(args, torch):
    from pagedkv_fusion import _C
    g = torch.Generator(device="cuda").manual_seed(5)
    nb, Hkv = args.blocks, args.kv_heads
    k = torch.randn((nb, args.block_size, Hkv, 128), device="cuda", generator=g).half()
    q = torch.randn((Hkv, 128), device="cuda", generator=g)
    return lambda: _C.attention_stats(k, q, 1 / math.sqrt(128))


def run_workload(args) -> None:
    import torch
    if not torch.cuda.is_available():
        sys.exit("ERROR: no CUDA device visible")
    call = {"eviction": _eviction, "attention": _attention, "quantize": _quantize,
            "stats": _stats}[args.target](args, torch)
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    for _ in range(args.iters):
        call()
    torch.cuda.synchronize()


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("target", choices=sorted(KERNELS))
    ap.add_argument("--num-blocks", type=int, default=16384, help="eviction: blocks")
    ap.add_argument("--block-size", type=int, default=16)
    ap.add_argument("--num-seqs", type=int, default=32, help="attention: sequences")
    ap.add_argument("--seq-len", type=int, default=2048, help="attention: tokens per sequence")
    ap.add_argument("--heads", type=int, default=32, help="attention: query heads")
    ap.add_argument("--kv-heads", type=int, default=8, help="attention / quantize: KV heads")
    ap.add_argument("--blocks", type=int, default=60000,
                    help="quantize / stats: fp16 blocks")
    ap.add_argument("--skip-fraction", type=float, default=0.15, help="quantize: blocks skipped")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--ncu", action="store_true",
                    help="run once plainly, then capture one launch under ncu")
    ap.add_argument("--out", default="prof", help="ncu report path (without .ncu-rep)")
    ap.add_argument("--kernel", default=None,
                    help="ncu -k pattern overriding the target's (e.g. regex:bitonic_global)")
    ap.add_argument("--per-call", type=int, default=None,
                    help="launches matching --kernel per call (default: the target's)")
    args = ap.parse_args(argv)
    if args.ncu and args.target == "eviction" and args.num_blocks > 16384 and args.kernel is None:
        ap.error("above 16,384 blocks eviction runs the multi-kernel selection: pass --kernel "
                 "(and --per-call) to name the kernel to capture")
    if not args.ncu:
        run_workload(args)
        return 0
    ncu = shutil.which("ncu")
    if ncu is None:
        sys.exit("ERROR: ncu not found on PATH")
    raw = list(argv if argv is not None else sys.argv[1:])
    plain = [sys.executable, "-m", "pagedkv_fusion.profile_kernels"]
    skip = False
    for a in raw:  # the plain run takes the workload arguments only
        if skip:
            skip = False
            continue
        if a == "--ncu":
            continue
        if a in ("--kernel", "--per-call", "--out"):
            skip = True
            continue
        if a.startswith(("--kernel=", "--per-call=", "--out=")):
            continue
        plain.append(a)
    env = dict(os.environ)
    rc = subprocess.run(plain, env=env).returncode
    if rc != 0:
        print(f"plain run exited {rc}: not profiled", file=sys.stderr)
        return rc
    pattern, per_call = KERNELS[args.target]
    if args.kernel is not None:
        pattern = args.kernel
    if args.per_call is not None:
        per_call = args.per_call
    cmd = [ncu, "--set", "full", "--clock-control", "none", "-k", pattern,
           "-s", str(args.warmup * per_call), "-c", "1", "-o", args.out, "--force-overwrite"] + plain
    print("running:", " ".join(cmd), flush=True)
    return subprocess.run(cmd, env=env).returncode


if __name__ == "__main__":
    sys.exit(main())
