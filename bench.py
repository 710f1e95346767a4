#!/usr/bin/env python3
"""Benchmark: INT8 paged decode throughput (and eviction top-k latency).

Workload (default ``--workload large-head``): one decode step over 512
sequences with lengths uniform in [1024, 8192] (multiples of 16), 40 query /
40 KV heads, head_dim 128, block_size 16 -- about 155K physical blocks,
24 GB of INT8 K+V with per-(block, head) fp32 scales from N(0,1) data.  With
``--gpus N`` (one process per GPU, launched by torch.distributed.run) the
work is partitioned by ``distributed.plan_decode_shards``: by sequence
(balanced by tokens), and by KV head where one sequence dominates (strong
scaling); each rank holds only its shard's blocks and heads and no
collective touches the data path.  ``--workload heavy-tail`` runs the
64 x 2048, 8-head decode with 0.1 % of K entries x10 instead, and
``--workload long-context`` four sequences of 32K-256K tokens at 40 heads
(the longest holds 53 % of the tokens, so ranks split it by head).

One step = one ``pagedkv_fusion._C.quant_paged_attention`` call (one
persistent decode kernel for these shapes) over device-resident inputs; K
steps are timed with CUDA events between barriers and device
synchronizations, the max over ranks is reported.  The KV working set
(24 GB, 268 MB for the heavy-tail workload) is larger than the 126 MB L2, so
no flush is needed.  After the timed region every rank checks a sample of
its sequences' outputs against the double-precision C oracle (``parity``);
the run exits non-zero when that check fails.

Printed JSON (rank 0, one line): ``value`` = decode tokens/s (sequences
decoded per second, all ranks); ``roofline`` = algorithmic HBM bytes of one
step / measured step time against the measured copy bandwidth;
``e2e`` = the same metric through ``ops.quant_paged_attention`` with q,
block tables and seq_lens in pinned host memory and the output read back
every step; ``cpu_baseline`` = the NumPy port of the reference decode on a
sample of the workload's sequences on this host, scaled to the workload's
tokens; ``eviction`` = fused score + top-k over 16,384 blocks (k = 2,458)
p50 device and wall latency; ``extras`` = the heavy-tailed 64 x 2048 decode
and the reference benchmark's 32/8-head GQA shape, each timed, against the
roofline and checked against the oracle on every sequence.

``--impl reference`` times the reference's CPU implementation of the path
(the NumPy port under oracle/, all host cores) on bounded samples of the
same workload and prints the same line with ``"impl": "reference"``.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "pagedkv-fusion-custom-cuda-kernels-for-kv-cache-eviction-quantized-paged-attention_b200"
sys.path.insert(0, str(PKG))
sys.path.insert(0, str(ROOT))

from pagedkv_fusion import problems  # noqa: E402

METRIC = "int8_paged_decode_tokens_per_s"
UNIT = "tokens/s"
BLOCK = 16
HEAD_DIM = 128

WORKLOADS = {
    "large-head": dict(name="decode_large_head_512seq_L1024-8192_h40_d128_bs16", heads=40,
                       kv_heads=40, parity_seqs=12),
    "heavy-tail": dict(name="decode_heavy_tail_64seq_L2048_h8_d128_bs16", heads=8, kv_heads=8,
                       parity_seqs=64),
    "long-context": dict(name="decode_long_context_4seq_L32K-256K_h40_d128_bs16", heads=40,
                         kv_heads=40, parity_seqs=2),
    "composition": dict(name="evict15_quantize_decode_1024seq_L4096-32768_h8_d128_bs16_fp16",
                        heads=8),
}
EVICT_FRACTION = 0.15
CPU_MAX_TOKENS = 16384  # longest sequence prefix a CPU-leg process decodes


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="large-head")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-eviction", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extras", action="store_true")
    ap.add_argument("--no-parity", action="store_true")
    return ap.parse_args()


def workload_seq_lens(workload: str) -> np.ndarray:
    if workload == "large-head":
        return problems.large_head_seq_lens(seed=0)
    if workload == "composition":
        return problems.composition_seq_lens(seed=0)
    if workload == "long-context":
        return problems.long_context_seq_lens()
    return np.full(64, 2048, dtype=np.int32)


def workload_config(wl: dict, lens: np.ndarray) -> dict:
    """The workload's identity: the same dict on both arms of the bench."""
    return {"workload": wl["name"], "num_seqs": int(len(lens)),
            "total_kv_tokens": int(lens.sum()), "heads": wl["heads"],
            "kv_heads": wl["kv_heads"], "head_dim": HEAD_DIM, "block_size": BLOCK,
            "l2": "inputs larger than L2 (no flush)"}


def cpu_sample(lens: np.ndarray, workers: int) -> np.ndarray:
    """Sequence indices the CPU legs decode: ``workers`` evenly spaced over
    the workload (one per process)."""
    return np.unique(np.linspace(0, len(lens) - 1, min(workers, len(lens))).astype(int))


def algorithmic_bytes(lens: np.ndarray, heads: int, kv_heads: int) -> int:
    """HBM bytes one decode step must move: INT8 K and V of every token,
    one fp32 K and V scale per (page, kv head), q and out, the block-table
    entries used and seq_lens."""
    lens = np.asarray(lens, dtype=np.int64)
    pages = (lens + BLOCK - 1) // BLOCK
    kv = int(lens.sum()) * kv_heads * HEAD_DIM * 2
    scales = int(pages.sum()) * kv_heads * 4 * 2
    qo = len(lens) * heads * HEAD_DIM * 4 * 2
    tables = int(pages.sum()) * 4 + len(lens) * 4
    return kv + scales + qo + tables


# ---------------------------------------------------------------------------
# CPU reference decode (NumPy port of the reference, all host cores)
# ---------------------------------------------------------------------------

_WORKER_CACHE: dict = {}


def _cpu_decode_one(job):
    """Decode one sequence with the NumPy port (inside a worker process);
    the sequence's arrays are memory-mapped from the staging directory."""
    from oracle import oracle as O
    root, i = job
    if (root, i) not in _WORKER_CACHE:
        _WORKER_CACHE[(root, i)] = [np.load(os.path.join(root, f"{i}_{n}.npy"), mmap_mode="r")
                                    for n in ("q", "kq", "ks", "vq", "vs", "L")]
    q, kq, ks, vq, vs, L = _WORKER_CACHE[(root, i)]
    n = kq.shape[0]
    bt = np.arange(n, dtype=np.int32)[None]
    sl = np.array([int(L)], dtype=np.int32)
    O.paged_attention(np.asarray(q)[None], kq, ks, vq, vs, bt, sl, 1.0 / math.sqrt(HEAD_DIM))
    return int(L)


class CpuDecodePool:
    """One spawned worker process per host core (capped), each decoding one
    sequence per step with the NumPy port, BLAS single-threaded so the
    processes do not oversubscribe the cores.  Sequences are staged once as
    .npy files (tmpfs when available) and memory-mapped by the workers."""

    def __init__(self, tasks):
        import multiprocessing as mp
        import tempfile
        base = "/dev/shm" if os.path.isdir("/dev/shm") else None
        self.root = tempfile.mkdtemp(prefix="pkv_cpu_", dir=base)
        for i, t in enumerate(tasks):
            for name, arr in zip(("q", "kq", "ks", "vq", "vs", "L"), t):
                np.save(os.path.join(self.root, f"{i}_{name}.npy"), np.asarray(arr))
        self.jobs = [(self.root, i) for i in range(len(tasks))]
        saved = {k: os.environ.get(k) for k in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS",
                                                 "MKL_NUM_THREADS")}
        for k in saved:
            os.environ[k] = "1"
        try:
            self.pool = mp.get_context("spawn").Pool(len(tasks))
        finally:
            for k, v in saved.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v

    def step(self):
        t0 = time.perf_counter()
        self.pool.map(_cpu_decode_one, self.jobs, chunksize=1)
        return time.perf_counter() - t0

    def close(self):
        import shutil
        self.pool.terminate()
        self.pool.join()
        shutil.rmtree(self.root, ignore_errors=True)


def synthetic_host_sequence(rng, L: int, heads: int, heavy: bool):
    """One sequence of the workload built on the host: N(0,1) K/V (K spiked
    for the heavy-tail workload) quantized with the oracle quantizer."""
    from oracle import oracle as O
    n = (L + BLOCK - 1) // BLOCK
    k = rng.standard_normal((n, BLOCK, heads, HEAD_DIM), dtype=np.float32)
    v = rng.standard_normal((n, BLOCK, heads, HEAD_DIM), dtype=np.float32)
    if heavy:
        spike = rng.random(k.shape) < 0.001
        k[spike] *= np.float32(10)
    kq, ks = O.quantize_kv_per_block(k)
    vq, vs = O.quantize_kv_per_block(v)
    q = rng.standard_normal((heads, HEAD_DIM), dtype=np.float32)
    return (q, kq, ks, vq, vs, int(L))


def cores_available() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    wl = WORKLOADS[args.workload]
    lens = workload_seq_lens(args.workload)
    workers = max(1, min(cores_available(), 32))
    idx = cpu_sample(lens, workers)
    rng = np.random.default_rng(0)
    tasks = [synthetic_host_sequence(rng, min(int(lens[i]), CPU_MAX_TOKENS), wl["heads"],
                                     args.workload == "heavy-tail") for i in idx]
    pool = CpuDecodePool(tasks)
    try:
        for _ in range(args.warmup):
            pool.step()
        times = [pool.step() for _ in range(args.steps)]
    finally:
        pool.close()
    t = statistics.fmean(times)
    value, sample = cpu_rate(lens, idx, sum(x[5] for x in tasks), t, wl["heads"])
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": len(lens) / value * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(wl, lens), "parallelism": f"cpu x{len(idx)} processes",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": len(idx), "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def cpu_rate(lens: np.ndarray, idx: np.ndarray, sample_tokens: int, t: float,
             heads: int) -> tuple[float, str]:
    """Whole-workload decode tokens/s from a CPU step over the sampled
    sequences ``idx`` (``sample_tokens`` tokens decoded; sequences longer
    than CPU_MAX_TOKENS are decoded over their first CPU_MAX_TOKENS) that
    took ``t`` seconds: the workload's sequences per second at the
    sample's tokens per second (decode time is linear in tokens)."""
    step_s = t * float(lens.sum()) / sample_tokens
    return len(lens) / step_s, (
        f"{len(idx)} of the {len(lens)} sequences (evenly spaced, {sample_tokens} tokens, "
        f"{heads} heads), one sequence per single-threaded process, {t:.3f} s per sample "
        f"step, scaled by the workload's {int(lens.sum())} tokens")


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, mx, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "power_w_max": max(power) if power else None,
                "samples": len(sm), "reasons": sorted(reasons)}


def eviction_bench(torch, C, ops, iters: int = 200):
    from oracle import oracle as O
    rec, freq, att, msk = problems.eviction_problem(seed=0)
    k = 2458
    d = [torch.from_numpy(a).cuda() for a in (rec, freq, att, msk)]
    want = O.select_eviction_candidates(O.eviction_scores(rec, freq, att, msk), k)
    _, idx = C.eviction_scores_select(*d, k)
    exact = bool(np.array_equal(idx.cpu().numpy(), want))
    stream = torch.cuda.current_stream()
    for _ in range(20):
        C.eviction_scores_select(*d, k)
    dev_us = []
    for _ in range(iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        # keep the GPU busy while the host enqueues, so the events bracket
        # device execution only (not Python launch latency)
        torch.cuda._sleep(100_000)
        e0.record(stream)
        C.eviction_scores_select(*d, k)
        e1.record(stream)
        e1.synchronize()
        dev_us.append(e0.elapsed_time(e1) * 1e3)
    fused_wall = []
    for _ in range(iters):  # one fused call + sync
        t0 = time.perf_counter()
        ops.eviction_scores_and_candidates(*d, k)
        torch.cuda.synchronize()
        fused_wall.append((time.perf_counter() - t0) * 1e6)
    plan = ops.EvictionPlan(*d, k)
    plan.run()
    torch.cuda.synchronize()
    exact = exact and bool(np.array_equal(plan.indices.cpu().numpy(), want))
    graph_wall = []
    for _ in range(iters):  # the serving loop's measure: one graph replay + sync
        t0 = time.perf_counter()
        plan.run()
        torch.cuda.synchronize()
        graph_wall.append((time.perf_counter() - t0) * 1e6)
    wall = []
    for _ in range(iters):  # the reference's measure: two ops calls + sync
        t0 = time.perf_counter()
        s = ops.eviction_scores(*d)
        ops.select_eviction_candidates(s, k)
        torch.cuda.synchronize()
        wall.append((time.perf_counter() - t0) * 1e6)
    # attention statistics derived from an fp16 K pool of the same shape
    # (16,384 blocks x 16 tokens x 8 KV heads x 128): the HBM-bound producer
    # of the attention term
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    kpool = torch.randn((16384, 16, 8, 128), generator=g, device="cuda").half()
    qh = torch.randn((8, 128), generator=g, device="cuda")
    for _ in range(5):
        C.attention_stats(kpool, qh, 1 / math.sqrt(128))
    torch.cuda.synchronize()
    st_us = []
    for _ in range(50):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(100_000)  # the events bracket device execution, not the enqueue
        e0.record(stream)
        C.attention_stats(kpool, qh, 1 / math.sqrt(128))
        e1.record(stream)
        e1.synchronize()
        st_us.append(e0.elapsed_time(e1) * 1e3)
    stats_bytes = kpool.numel() * 2 + 16384 * 16 * 8 * 4 * 2 + 16384 * 16 * 4
    del kpool
    cpu = []
    for _ in range(50):
        t0 = time.perf_counter()
        O.select_eviction_candidates(O.eviction_scores(rec, freq, att, msk), k)
        cpu.append((time.perf_counter() - t0) * 1e6)
    return {"config": "16384 blocks x 16 tokens, k=2458", "exact": exact,
            "device_p50_us": statistics.median(dev_us),
            "device_p90_us": statistics.quantiles(dev_us, n=10)[8],
            "fused_wall_p50_us": statistics.median(fused_wall),
            "graph_wall_p50_us": statistics.median(graph_wall),
            "wall_p50_us": statistics.median(wall),
            "wall_p90_us": statistics.quantiles(wall, n=10)[8],
            "cpu_port_p50_us": statistics.median(cpu),
            "attention_stats_from_fp16_k": {
                "device_p50_us": statistics.median(st_us),
                "gb_s": stats_bytes / (statistics.median(st_us) / 1e6) / 1e9,
                "bytes": stats_bytes}}


def read_peak() -> tuple[float, str]:
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        return float(json.loads(pk.read_text())["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs"
    return 6650.0, "fallback 6650 GB/s"


def time_back_to_back(torch, fn, steps: int, warmup: int) -> float:
    """Mean ms per call of ``fn`` over ``steps`` back-to-back calls between
    one CUDA-event pair on the current stream (after ``warmup`` calls)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def decode_extra(torch, C, name: str, lens: np.ndarray, heads: int, kv_heads: int, heavy: bool,
                 device, peak: float, peak_source: str) -> dict:
    """A further decode configuration on one GPU: timed (200 back-to-back
    calls), against the roofline, and checked against the oracle on every
    sequence."""
    from oracle.parity import sampled_decode_parity
    q, kc, ks, vc, vs, bt_np, nb = problems.device_paged_cache(lens, kv_heads, heads, device,
                                                               seed=7, heavy=heavy)
    bt = torch.from_numpy(bt_np).to(device)
    sl = torch.from_numpy(lens.astype(np.int32)).to(device)
    sm = 1.0 / math.sqrt(HEAD_DIM)
    a = (q, kc, ks, vc, vs, bt, sl, sm)
    ms = time_back_to_back(torch, lambda: C.quant_paged_attention(*a), 200, 10)
    out = C.quant_paged_attention(*a)
    parity = sampled_decode_parity(q, kc, ks, vc, vs, bt_np, lens, sm, out,
                                   np.arange(len(lens)))
    byts = algorithmic_bytes(lens, heads, kv_heads)
    launches = C.quant_paged_attention_kernel_launches(len(lens), heads, kv_heads, HEAD_DIM,
                                                       BLOCK, bt_np.shape[1])
    gbs = byts / (ms / 1e3) / 1e9
    return {"workload": name, "num_seqs": int(len(lens)), "total_kv_tokens": int(lens.sum()),
            "heads": heads, "kv_heads": kv_heads, "us_per_call": ms * 1e3,
            "kernel_launches_per_call": launches,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                         "frac": gbs / peak, "bytes_per_call": byts,
                         "basis": "algorithmic bytes / mean CUDA-event time of one call "
                                  "(200 back-to-back calls)", "peak_source": peak_source},
            "parity": parity}


def run_gpu_arm(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)

    from pagedkv_fusion import _C as C
    from pagedkv_fusion import ops
    from pagedkv_fusion.distributed import plan_decode_shards

    wl = WORKLOADS[args.workload]
    all_lens = workload_seq_lens(args.workload)
    shards = plan_decode_shards(all_lens, wl["heads"], wl["kv_heads"], world)
    shard = shards[rank]
    lens = all_lens[shard.seqs]
    heads = shard.heads[1] - shard.heads[0]
    kv_heads = shard.kv_heads
    q, kc, ks, vc, vs, bt_np, nb = problems.device_paged_cache(
        lens, kv_heads, heads, device, seed=1000 + rank, heavy=args.workload == "heavy-tail")
    bt = torch.from_numpy(bt_np).to(device)
    sl = torch.from_numpy(lens.astype(np.int32)).to(device)
    sm = 1.0 / math.sqrt(HEAD_DIM)
    step_args = (q, kc, ks, vc, vs, bt, sl, sm)
    my_bytes = algorithmic_bytes(lens, heads, kv_heads)
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    stream = torch.cuda.current_stream()
    sampler = ClockSampler(local) if rank == 0 else None
    for _ in range(args.warmup):
        C.quant_paged_attention(*step_args)
    barrier()
    if sampler:
        sampler.start()
        time.sleep(0.3)  # let the sampler attach before the timed region
    barrier()
    # one event pair around the K back-to-back calls: per-step events would
    # add their own gaps to the stream.  Each call is one kernel launch (the
    # stream kernel needs no counter reset), so total / K is also the mean
    # launch duration, inter-launch gaps included.
    t_begin = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    out = None
    t_begin.record(stream)
    for i in range(args.steps):
        out = C.quant_paged_attention(*step_args)
    t_end.record(stream)
    barrier()
    clocks = sampler.stop() if sampler else None
    total_ms = t_begin.elapsed_time(t_end)
    mean_launch_ms = total_ms / args.steps
    t = torch.tensor([total_ms], dtype=torch.float64, device=device)
    per_rank = None
    if world > 1:
        # every rank's step time and share, for the imbalance of the plan
        mine = torch.tensor([total_ms / args.steps, float(lens.sum()), float(len(lens)),
                             float(kv_heads)], dtype=torch.float64, device=device)
        gathered = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(gathered, mine)
        rows = [g.cpu().tolist() for g in gathered]
        ms = [r[0] for r in rows]
        per_rank = {"ms_per_step": ms, "kv_tokens": [int(r[1]) for r in rows],
                    "seqs": [int(r[2]) for r in rows], "kv_heads": [int(r[3]) for r in rows],
                    "max_over_mean_ms": max(ms) / (sum(ms) / len(ms))}
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t.item()) / args.steps
    value = len(all_lens) / (ms_per_step / 1e3)

    # parity of the timed step's output on a sample of this rank's sequences
    # (outside the timed region), reduced over ranks
    parity = None
    if not args.no_parity and args.steps > 0:
        from oracle.parity import sample_sequences, sampled_decode_parity
        picks = sample_sequences(lens, wl["parity_seqs"])
        p = sampled_decode_parity(q, kc, ks, vc, vs, bt_np, lens, sm, out, picks)
        red = torch.tensor([p["max_rel_err"], p["max_abs_err"], 0.0 if p["ok"] else 1.0,
                            p["sampled_seqs"], p["sampled_tokens"]], dtype=torch.float64,
                           device=device)
        if world > 1:
            mx = red[:3].clone()
            sm_ = red[3:].clone()
            dist.all_reduce(mx, op=dist.ReduceOp.MAX)
            dist.all_reduce(sm_, op=dist.ReduceOp.SUM)
            red = torch.cat([mx, sm_])
        r = red.cpu().tolist()
        parity = {"ok": r[2] == 0.0, "max_rel_err": r[0], "max_abs_err": r[1],
                  "sampled_seqs": int(r[3]), "sampled_tokens": int(r[4]),
                  "tolerance": "max rel err 1e-3 and allclose(rtol=2e-4, atol=2e-4)",
                  "oracle": "double-precision C restatement of paged_attention_ref on the "
                            "sampled sequences' pages copied from the timed cache"}

    # end-to-end: host (pinned) q / tables / lengths in, host output back
    e2e = None
    if not args.no_e2e:
        q_h = q.cpu().pin_memory()
        bt_h = torch.from_numpy(bt_np).pin_memory()
        sl_h = torch.from_numpy(lens.astype(np.int32)).pin_memory()
        n_e2e = max(1, min(args.steps, 50))
        for _ in range(3):
            ops.quant_paged_attention(q_h, kc, ks, vc, vs, bt_h, sl_h, sm)
        barrier()
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            out_h = ops.quant_paged_attention(q_h, kc, ks, vc, vs, bt_h, sl_h, sm)
        elapsed = time.perf_counter() - t0
        assert out_h.device.type == "cpu"
        te = torch.tensor([elapsed / n_e2e], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        e2e = {"value": len(all_lens) / float(te.item()), "unit": UNIT,
               "h2d_bytes_per_step": int(q_h.numel() * 4 + bt_h.numel() * 4 + sl_h.numel() * 4),
               "d2h_bytes_per_step": int(q_h.numel() * 4),
               "note": "KV cache device-resident (serving state); per-step inputs and output "
                       "cross PCIe; wall clock per step, max over ranks"}

    # DRAM traffic per launch (dram__bytes_read.sum + dram__bytes_write.sum)
    # from ncu captures of decode_stream_kernel<16, 8, 1>.  Heavy-tail
    # workload: 272,910,336 B for 269,517,056 algorithmic bytes.  A
    # large-head launch (24 GB resident) is too large to capture; a 40/40-head
    # case of 32 sequences x 4,608 tokens (the same instantiation, five head
    # groups per sequence) read 1,513,802,752 B and wrote 3,766,272 B for
    # 1,514,246,272 algorithmic bytes, so the large-head traffic is that ratio
    # times its own algorithmic bytes (traffic grows with the pages streamed).
    if args.workload == "heavy-tail":
        traffic = my_bytes * (272910336 / 269517056)
        traffic_basis = "ncu capture of this workload"
    else:
        traffic = my_bytes * ((1513802752 + 3766272) / 1514246272)
        traffic_basis = ("ncu capture of a 40/40-head 32 x 4,608-token case of the same kernel: "
                         "its traffic/algorithmic ratio x this workload's algorithmic bytes")
    launches_per_step = C.quant_paged_attention_kernel_launches(
        len(lens), heads, kv_heads, HEAD_DIM, BLOCK, bt_np.shape[1])
    plan_name = ("persistent decode_stream_kernel" if launches_per_step == 1
                 else "split-K decode kernel + combine")
    peak, peak_source = read_peak()
    result = None
    if rank == 0:
        achieved = my_bytes / (mean_launch_ms / 1e3) / 1e9
        result = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "s8/f32", "data": "synthetic",
            "config": workload_config(wl, all_lens),
            "parallelism": (f"{world // shard.head_split} sequence group(s) x "
                            f"{shard.head_split} KV-head slice(s)"),
            "rank0": {"seqs": int(len(lens)), "kv_heads": kv_heads, "blocks": nb,
                      "kv_tokens": int(lens.sum())},
            "ranks": per_rank,
            "kv_tokens_per_s": float(all_lens.sum()) / (ms_per_step / 1e3),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "traffic_unit": "bytes per launch", "traffic_basis": traffic_basis,
                         "basis": f"{my_bytes} algorithmic bytes per step on rank 0 / mean "
                                  "CUDA-event time of one quant_paged_attention call over the "
                                  "timed region (events around the back-to-back calls, "
                                  f"{launches_per_step} kernel launch(es) per call: {plan_name})",
                         "peak_source": peak_source},
            "parity": parity, "clocks": clocks, "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps,
        }
    # CPU baseline, eviction latency and the extra decode shapes on rank 0 at N = 1
    if rank == 0 and world == 1:
        if not args.no_eviction:
            result["eviction"] = eviction_bench(torch, C, ops)
        if not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_baseline_from_device(
                torch, args, lens, step_args, bt_np, heads)
        if not args.no_extras:
            del step_args, q, kc, ks, vc, vs, out
            torch.cuda.empty_cache()
            result["extras"] = {
                "heavy_tail": decode_extra(torch, C, WORKLOADS["heavy-tail"]["name"],
                                           workload_seq_lens("heavy-tail"), 8, 8, True, device,
                                           peak, peak_source),
                "gqa_32_8": decode_extra(torch, C, "decode_gqa_64seq_L2048_h32_kv8_d128_bs16",
                                         np.full(64, 2048, dtype=np.int32), 32, 8, False, device,
                                         peak, peak_source),
            }
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if result is not None:
        print(json.dumps(result), flush=True)
    ok = parity is None or parity["ok"]
    if result is not None and "extras" in result:
        ok = ok and all(x["parity"]["ok"] for x in result["extras"].values())
    return 0 if ok else 1


def cpu_baseline_from_device(torch, args, lens, step_args, bt_np, heads):
    """The NumPy port of the reference decode on a sample of this run's own
    sequences (their pages copied to the host), one process per core, scaled
    to the workload's tokens."""
    q, kc, ks, vc, vs, _, _, _ = step_args
    workers = max(1, min(cores_available(), 32))
    idx = cpu_sample(lens, workers)
    tasks = []
    for s in idx:
        L = min(int(lens[s]), CPU_MAX_TOKENS)
        pages = bt_np[s, :(L + BLOCK - 1) // BLOCK].astype(np.int64)
        p = torch.from_numpy(pages).to(kc.device)
        tasks.append((q[s].cpu().numpy(), kc[p].cpu().numpy(), ks[p].cpu().numpy(),
                      vc[p].cpu().numpy(), vs[p].cpu().numpy(), L))
    pool = CpuDecodePool(tasks)
    try:
        pool.step()
        times = [pool.step() for _ in range(5)]
    finally:
        pool.close()
    t = statistics.median(times)
    value, sample = cpu_rate(lens, idx, sum(x[5] for x in tasks), t, heads)
    return {"value": value, "unit": UNIT, "cores": len(idx), "kind": "port",
            "sample": sample + ", median of 5 steps"}


# ---------------------------------------------------------------------------
# Evict -> quantize -> decode composition (one serving step)
# ---------------------------------------------------------------------------

def composition_stage_bytes(nb: int, n_evict_local: int, lens_after: np.ndarray, num_seqs: int,
                            max_pages: int, heads: int) -> dict:
    """Algorithmic HBM bytes of each stage of one composed step on a rank."""
    blk = BLOCK * heads * HEAD_DIM
    surv = nb - n_evict_local
    return {
        "score": nb * (4 + 4 + BLOCK * 4 + BLOCK) + nb * 4,
        "select": nb * 4 + n_evict_local * 8 + nb,
        "quantize": 2 * surv * (blk * 2 + blk + heads * 4) + 2 * nb,
        "compact": num_seqs * max_pages * 4 * 2 + num_seqs * 8 + nb,
        "decode": algorithmic_bytes(lens_after, heads, heads),
    }


def run_composition(args):
    """The composed serving step over 1,024 sequences of 4K-32K tokens: score
    all blocks, evict the lowest 15 % globally (sharded
    top-k + all-gather at N > 1), quantize the survivors from fp16, decode
    over the compacted tables.  Sequences are sharded by tokens; each rank
    holds its sequences' fp16 blocks and INT8 cache."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    from pagedkv_fusion import _C as C
    from pagedkv_fusion.compose import STAGES, evict_quantize_decode

    heads = WORKLOADS["composition"]["heads"]
    all_lens = workload_seq_lens("composition")
    shards = problems.balanced_shards(all_lens, world)
    pages_of = lambda idx: int(((all_lens[idx].astype(np.int64) + BLOCK - 1) // BLOCK).sum())
    shard_blocks = [pages_of(sh) for sh in shards]
    offset = int(sum(shard_blocks[:rank]))
    total_blocks = int(sum(shard_blocks))
    n_evict = int(EVICT_FRACTION * total_blocks)
    lens = all_lens[shards[rank]]
    pages = (lens.astype(np.int64) + BLOCK - 1) // BLOCK
    nb = int(pages.sum())

    g = torch.Generator(device=device)
    g.manual_seed(2000 + rank)
    shape = (nb, BLOCK, heads, HEAD_DIM)
    k_src = torch.empty(shape, dtype=torch.float16, device=device)
    v_src = torch.empty_like(k_src)
    chunk = max(1, (1 << 28) // (BLOCK * heads * HEAD_DIM))
    for dst in (k_src, v_src):
        for lo in range(0, nb, chunk):
            hi = min(nb, lo + chunk)
            dst[lo:hi] = torch.randn((hi - lo,) + shape[1:], generator=g, device=device).half()
    rec = torch.rand(nb, generator=g, device=device)
    freq = torch.rand(nb, generator=g, device=device)
    att = torch.rand((nb, BLOCK), generator=g, device=device)
    val = torch.ones((nb, BLOCK), dtype=torch.bool, device=device)
    k_cache = torch.empty(shape, dtype=torch.int8, device=device)
    v_cache = torch.empty_like(k_cache)
    k_scale = torch.empty((nb, heads), dtype=torch.float32, device=device)
    v_scale = torch.empty_like(k_scale)
    perm = np.random.default_rng(rank).permutation(nb).astype(np.int32)
    bt_np = np.full((len(lens), int(pages.max())), -1, dtype=np.int32)
    starts = np.concatenate([[0], np.cumsum(pages)])
    for i in range(len(lens)):
        bt_np[i, :pages[i]] = perm[starts[i]:starts[i + 1]]
    bt = torch.from_numpy(bt_np).to(device)
    sl = torch.from_numpy(lens.astype(np.int32)).to(device)
    q = torch.randn((len(lens), heads, HEAD_DIM), generator=g, device=device)
    sm = 1.0 / math.sqrt(HEAD_DIM)

    def step(events=None):
        return evict_quantize_decode(
            q, k_src, v_src, rec, freq, att, val, bt, sl, n_evict, sm, k_cache=k_cache,
            k_scale=k_scale, v_cache=v_cache, v_scale=v_scale, block_offset=offset,
            total_blocks=total_blocks if world > 1 else None, events=events)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        out, ids, tables, lens_after = step()
    barrier()
    sampler = ClockSampler(local) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier()
    ev = [[] for _ in range(args.steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.steps):
        out, ids, tables, lens_after = step(ev[i])
    t1.record()
    barrier()
    clocks = sampler.stop() if sampler else None
    stage_ms = {name: statistics.fmean(e[j].elapsed_time(e[j + 1]) for e in ev)
                for j, name in enumerate(STAGES)}
    t = torch.tensor([t0.elapsed_time(t1) / args.steps], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t.item())
    ids_np = ids.cpu().numpy()
    n_ev_local = int(((ids_np >= offset) & (ids_np < offset + nb)).sum())
    byts = composition_stage_bytes(nb, n_ev_local, lens_after.cpu().numpy(), len(lens),
                                   bt_np.shape[1], heads)
    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    peak = float(peaks.get("hbm_gbs", 6650.0))
    stages = {n: {"ms": stage_ms[n], "bytes": byts[n],
                  "gb_s": byts[n] / (stage_ms[n] / 1e3) / 1e9} for n in STAGES}
    if rank == 0:
        total_bytes = sum(byts.values())
        print(json.dumps({
            "metric": "evict_quantize_decode_step_tokens_per_s", "unit": "tokens/s",
            "value": len(all_lens) / (ms_per_step / 1e3), "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16->s8/f32", "data": "synthetic",
            "config": {"workload": WORKLOADS["composition"]["name"],
                       "num_seqs": int(len(all_lens)), "total_kv_tokens": int(all_lens.sum()),
                       "blocks_total": total_blocks, "evicted": n_evict, "heads": heads,
                       "kv_heads": heads, "head_dim": HEAD_DIM, "block_size": BLOCK,
                       "blocks_rank0": nb, "parallelism": f"sequence-sharded x{world}",
                       "l2": "inputs larger than L2 (no flush)"},
            "stages_rank0": stages,
            "roofline": {"bound": "hbm", "achieved": total_bytes / (ms_per_step / 1e3) / 1e9,
                         "peak": peak, "unit": "GB/s",
                         "frac": total_bytes / (ms_per_step / 1e3) / 1e9 / peak,
                         "basis": "sum of the stages' algorithmic bytes on rank 0 / step time"},
            "clocks": clocks,
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    args = parse_args()
    if args.workload == "composition":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable":
                              "the reference has no evict -> quantize -> decode step; its "
                              "demo quantizes every block and decodes unchanged tables"}))
            return 0
        return run_composition(args)
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_gpu_arm(args)


if __name__ == "__main__":
    sys.exit(main())
