"""Benchmark: sparse-attention forward+backward tokens/s at 32K (configuration 4).

One step = one training pass of the sparse attention stage over one batch of
synthetic configuration-4 input: ``m3_sparse_attention`` forward, then its
backward (dQ, dK, dV, including the k2q CSR build), on a selection produced by
this library's own ``m3_index_score`` + ``m3_topk`` before the timed region.

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference]

``--gpus N`` (torchrun, one process per GPU): one sequence (the default
configuration 4, or ``--config 5``) is split by query ranges with context
parallelism (K/V all-gathered, dK/dV reduce-scattered inside every step), and a
packed batch (``--config 3``) by whole sequences (LPT on their cost, no
collective); both are strong scaling, the job's tokens over the slowest rank's
time. ``--impl reference`` times the reference algorithm's CPU
restatement (oracle/msa_oracle.py, float64 numpy; the reference itself is pure
Python and cannot run configuration 4) on a bounded sample, on rank 0 only.

Prints one JSON line (rank 0).
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

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "sparse-attn fwd+bwd tokens/s @32K on 1/2/4/8 B200; TFLOP/s vs BF16 peak"
UNIT = "tokens/s"

# Tensor-core attention kernels timed inside the step, with the share of the selected
# FLOPs each one performs: forward 4*D per (row, key); the fused backward all 8*D (S^T
# recomputation not counted). The separate dK/dV (6*D) and dQ (2*D) kernels run only when
# just one of the two gradients is requested.
KERNEL_SHARE = {"attn_fwd_tc": ("fwd", 1.0), "attn_bwd_tc": ("bwd", 1.0),
                "attn_dkdv_tc": ("bwd", 0.75), "attn_dq_tc": ("bwd", 0.25)}

# DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of the fused backward
# at configuration 4 on one GPU: one ncu capture of the configuration-4 shapes at T = 8192
# (bench.py --tokens 8192), scaled to T = 32768 by the selected (query, key) pairs, x 4.413;
# its traffic grows in proportion (its dQ accumulator exceeds L2 at both sizes). Summary and
# command in profiles/attn_tc_kernels_cfg4shapes_t8192.md. The forward's does not scale (its
# accumulator slice stays in L2 at 8K tokens), so it has no entry.
NCU_TRAFFIC: dict = {
    ("cfg4_32k_headline", "attn_bwd_tc"): 33.78e9,
}


def parse():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=4, help="workload (default: configuration 4, the headline)")
    ap.add_argument("--cpu-sample-tokens", type=int, default=64,
                    help="query tokens in the CPU baseline sample, evenly spaced (about 25 s of float64 numpy on "
                         "16 cores)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tokens", type=int, default=0,
                    help="profiling only: one sequence of this many tokens with the workload's heads and K")
    ap.add_argument("--inputs", choices=["unit", "rms4", "outlier"], default="unit",
                    help="input scale: unit RMS per head (default); q and k at RMS 2 each (logits 4x); or unit RMS "
                         "with one key row of group 0 at 8x the norm, in the middle of the first sequence")
    return ap.parse_args()


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], d.get("bf16_tflops_sustained"), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def workload(args):
    import dataclasses

    from msa_triton_b200.workloads import CONFIGS

    w = CONFIGS[args.config]
    if args.tokens:
        w = dataclasses.replace(w, name=f"{w.name}@{args.tokens}", lengths=(args.tokens,))
    return w


def scale_inputs(host, kind):
    """The input sets of --inputs (bf16 scaling by powers of two is exact)."""
    if kind == "rms4":
        host["q"] = host["q"] * 2
        host["k"] = host["k"] * 2
    elif kind == "outlier":
        k = host["k"].clone()
        k[int(host["cu_seqlens"][1]) // 2, 0] *= 8
        host["k"] = k
    return host


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self.skip = 0

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "10",
                 "-i", str(self.gpu_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        # nvidia-smi takes a moment to start: wait for its first sample so that a short
        # timed region is still sampled, and keep only the samples taken after this point
        deadline = time.time() + 5.0
        while self.proc is not None and not self.lines and self.proc.poll() is None and time.time() < deadline:
            time.sleep(0.005)
        self.skip = len(self.lines)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        # a timed region shorter than the sampling period (multi-GPU steps of a few ms) may see
        # no sample: then wait (at most 0.5 s) for the first one after it, and say so
        self.after = 0
        if self.proc is not None and len(self.lines) <= self.skip:
            deadline = time.time() + 0.5
            while len(self.lines) <= self.skip and self.proc.poll() is None and time.time() < deadline:
                time.sleep(0.002)
            self.after = min(1, len(self.lines) - self.skip)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)

    def summary(self):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines[self.skip:]:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        out = {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}
        if getattr(self, "after", 0):
            out["note"] = "timed region shorter than the sampling period: first sample after it"
        return out


# ----------------------------------------------------------------------------- distributed
def dist_setup(n):
    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    import torch
    import torch.distributed as dist

    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(x, world):
    import torch
    import torch.distributed as dist

    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- CPU baseline
_CPU_ARRAYS: dict = {}


def _cpu_init(folder):
    """Pool worker start-up: map the workload arrays (shared through the page cache)."""
    import numpy as np

    sys.path.insert(0, str(REPO))
    for name in ("q", "k", "v", "go", "ids", "cu"):
        _CPU_ARRAYS[name] = np.load(os.path.join(folder, name + ".npy"), mmap_mode="r")


def _cpu_chunk(args):
    """Oracle fwd+bwd for a chunk of query tokens (runs in a spawned worker)."""
    import numpy as np

    from oracle import msa_oracle as O

    block, scale, tokens = args
    q, k, v, go, ids, cu = (_CPU_ARRAYS[n] for n in ("q", "k", "v", "go", "ids", "cu"))
    _, start, pos = O.token_positions(np.asarray(cu))
    hq, groups = q.shape[1], k.shape[1]
    ratio = hq // groups
    dk = {}
    dv = {}
    for t in tokens:
        for g in range(groups):
            keys = O.selected_keys(np.asarray(ids[t, g]), start[t], pos[t], block)
            if keys.size == 0:
                continue
            hs = slice(g * ratio, (g + 1) * ratio)
            kk = k[keys, g].astype(np.float64)
            vv = v[keys, g].astype(np.float64)
            qt = q[t, hs].astype(np.float64)
            gt = go[t, hs].astype(np.float64)
            logits = qt @ kk.T * scale
            p = np.exp(logits - logits.max(axis=1, keepdims=True))
            p /= p.sum(axis=1, keepdims=True)
            _out = p @ vv
            dp = gt @ vv.T
            ds = p * (dp - (p * dp).sum(axis=1, keepdims=True)) * scale
            _dq = ds @ kk
            dk[g] = dk.get(g, 0) + (ds.T @ qt).sum()
            dv[g] = dv.get(g, 0) + (p.T @ gt).sum()
    return len(tokens)


def sample_tokens_of(w, n):
    """n query tokens spread evenly over the packed batch (every position class of the causal
    work: early tokens see fewer keys than the (K blocks) plateau)."""
    import numpy as np

    return sorted({int(x) for x in np.linspace(0, w.total_tokens - 1, n).round()})


def cpu_baseline(w, inputs, ids, tokens):
    """The reference algorithm's float64 CPU restatement (oracle) on the query tokens `tokens`:
    attention forward + backward of every head of each token over its selected blocks (`ids`,
    the same selection as the GPU run), all host cores. The workload arrays reach the workers
    as memory-mapped files; only the compute is timed."""
    import multiprocessing as mp
    import tempfile

    import numpy as np

    cores = os.cpu_count() or 1
    with tempfile.TemporaryDirectory() as folder:
        for name, t in (("q", inputs["q"]), ("k", inputs["k"]), ("v", inputs["v"]), ("go", inputs["grad_out"])):
            np.save(os.path.join(folder, name + ".npy"), t.float().numpy())
        np.save(os.path.join(folder, "ids.npy"), np.asarray(ids))
        np.save(os.path.join(folder, "cu.npy"), inputs["cu_seqlens"].numpy())
        parts = [tokens[i::cores] for i in range(cores)]
        tasks = [(w.block_size, w.dim ** -0.5, part) for part in parts if part]
        ctx = mp.get_context("spawn")
        with ctx.Pool(len(tasks), initializer=_cpu_init, initargs=(folder,)) as pool:
            pool.map(_cpu_chunk, [(w.block_size, w.dim ** -0.5, tokens[:1])] * len(tasks))  # warm the workers
            start = time.perf_counter()
            done = sum(pool.map(_cpu_chunk, tasks))
            elapsed = time.perf_counter() - start
    return {"value": done / elapsed, "unit": UNIT, "cores": len(tasks), "kind": "port",
            "sample": f"{done} query tokens evenly spaced over {w.name} (all {w.q_heads} heads, their top-"
                      f"{w.topk_blocks} blocks), attention fwd+bwd, float64 numpy restatement of the reference "
                      f"algorithm, {elapsed:.1f}s"}


def cpu_selection_rows(w, inputs, tokens):
    """The reference algorithm's selection for `tokens` on the CPU (float64 index-score rows and
    the top-k rule of triton/topk.py), in a full-size ids array (other rows -1)."""
    import numpy as np

    from oracle import msa_oracle as O

    cu = inputs["cu_seqlens"].numpy()
    _, _, pos = O.token_positions(cu)
    rows = O.index_score_rows(inputs["index_q"].float().numpy(), inputs["index_k"].float().numpy(), cu,
                              w.max_seqlen, tokens, block_size=w.block_size)
    ids = np.full((w.total_tokens, w.groups, w.topk_blocks), -1, dtype=np.int32)
    ids[tokens] = O.topk_at_positions(rows.astype(np.float32), pos[tokens], block_size=w.block_size,
                                      topk_blocks=w.topk_blocks, local_blocks=w.local_blocks)
    return ids


def eager_baseline():
    """The reference's native-dtype eager attention (oracle restatement, pinned bit-exactly to it)
    on configuration 1, forward + backward, all host cores; configurations 4 and 5 cannot run on
    it (dense masks)."""
    import torch

    from msa_triton_b200.workloads import CONFIGS, make_inputs, random_selection
    from oracle import msa_oracle as O

    w1 = CONFIGS[1]
    x = make_inputs(w1)
    ids = random_selection(list(w1.lengths), w1.groups, w1.block_size, w1.topk_blocks, seed=0,
                           local_blocks=w1.local_blocks).numpy()
    args = (x["q"], x["k"], x["v"], ids, x["cu_seqlens"].numpy(), w1.max_seqlen, x["grad_out"])
    O.sparse_attention_eager(*args, block_size=w1.block_size)  # warm
    start = time.perf_counter()
    O.sparse_attention_eager(*args, block_size=w1.block_size)
    elapsed = time.perf_counter() - start
    return {"cfg1_attention_fwd_bwd_s": round(elapsed, 3),
            "cfg1_tokens_per_s": round(w1.total_tokens / elapsed, 1),
            "nproc": os.cpu_count(), "torch_threads": torch.get_num_threads(),
            "cfg4": "not run: the dense [1,64,32768,32768] mask and logits exceed host RAM (69 GB bool, 275 GB fp32)",
            "cfg5": "not run: the dense [1,64,131072,131072] logits need about 4.4 TB"}


def bench_config(w, world, mode, global_seqs, inputs):
    """The `config` object both arms print (the driver compares them). mode: "single",
    "shards" (packed batch split by whole sequences) or "cp" (context parallel)."""
    return {"workload": w.name, "model": "MiniMax-M3 sparse attention layer", "seq_len": w.max_seqlen,
            "global_batch": global_seqs, "q_heads": w.q_heads, "kv_groups": w.groups, "head_dim": w.dim,
            "block_size": w.block_size, "topk_blocks": w.topk_blocks, "local_blocks": w.local_blocks,
            "parallelism": {"single": "single", "shards": f"whole-sequence shards x{world}",
                            "cp": f"context parallel (query ranges, NCCL all-gather / reduce-scatter) x{world}"}[mode],
            "l2_policy": "inputs larger than L2 (q, dO 537 MB each)", "inputs": inputs,
            "selection": "this path's index score + top-k (seeded synthetic inputs)",
            "metadata": "prepare_batch(cu_seqlens) once per batch: no per-call device read"}


# ----------------------------------------------------------------------------- our arm
def run_ours(args):
    import torch

    from msa_triton_b200 import _lib, m3_index_score, m3_sparse_attention, m3_topk, prepare_batch
    from msa_triton_b200.workloads import attention_flops, make_inputs

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    w = workload(args)
    hbm_peak, bf16_peak, bf16_sustained, peak_kind = peaks()
    host = scale_inputs(make_inputs(w), args.inputs)
    # a packed batch on several GPUs: each rank takes whole sequences (LPT on their cost),
    # no collective; the job's throughput is the whole batch over the slowest rank's time
    global_tokens, global_seqs, w_global = w.total_tokens, len(w.lengths), w
    sharded = world > 1 and len(w.lengths) > 1
    # one long sequence on several GPUs: context parallelism (equal query ranges; K/V
    # all-gathered, dK/dV reduce-scattered inside each step)
    cp = world > 1 and len(w.lengths) == 1
    if cp:
        from msa_triton_b200.distributed import context_parallel_range, cp_select_blocks, cp_sparse_attention

        lo_cp, hi_cp = context_parallel_range(w.total_tokens, world, rank)
        host = {n: t if n == "cu_seqlens" else t[lo_cp:hi_cp].contiguous() for n, t in host.items()}
    if sharded:
        import dataclasses

        from msa_triton_b200.distributed import shard_packed_batch, take_tokens

        shard = shard_packed_batch(host["cu_seqlens"], world, rank, q_heads=w.q_heads, groups=w.groups, dim=w.dim,
                                   index_dim=w.index_dim, block_size=w.block_size, topk_blocks=w.topk_blocks)
        host = {n: shard.cu_seqlens if n == "cu_seqlens" else take_tokens(t, shard) for n, t in host.items()}
        bounds = shard.cu_seqlens.tolist()
        w = dataclasses.replace(w, lengths=tuple(b - a for a, b in zip(bounds[:-1], bounds[1:])))
    cu_h = host["cu_seqlens"]
    x = {n: t.to(dev) for n, t in host.items()}
    cu = x["cu_seqlens"]
    with torch.no_grad():
        if cp:
            ids = cp_select_blocks(x["index_q"], x["index_k"], global_tokens, block_size=w.block_size,
                                   topk_blocks=w.topk_blocks, local_blocks=w.local_blocks)
        else:
            scores = m3_index_score(x["index_q"], x["index_k"], cu, w.max_seqlen, block_size=w.block_size)
            ids = m3_topk(scores, cu, block_size=w.block_size, topk_blocks=w.topk_blocks,
                          local_blocks=w.local_blocks)
            del scores
    q = x["q"].requires_grad_()
    k = x["k"].requires_grad_()
    v = x["v"].requires_grad_()
    go = x["grad_out"]

    # the boundaries are read to the host once per batch (as a training loop does for all
    # its layers), so a step issues no device-to-host synchronisation
    prepared = prepare_batch(cu)

    def attend(qd, kd, vd, idsd, cud, prep):
        if cp:
            return cp_sparse_attention(qd, kd, vd, idsd, global_tokens, block_size=w.block_size)
        return m3_sparse_attention(qd, kd, vd, idsd, cud, w.max_seqlen, block_size=w.block_size, prepared=prep)

    def step():
        q.grad = k.grad = v.grad = None
        out = attend(q, k, v, ids, cu, prepared)
        out.backward(go)
        return out

    for _ in range(args.warmup):
        step()
    barrier(world)
    _lib.timing_enable(True)  # event pairs around the tensor-core attention kernels (same stream)
    for name in KERNEL_SHARE:
        _lib.kernel_time(name)  # drop anything recorded before the timed region
    launches0 = _lib.kernel_launches()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier(world)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        barrier(world)
    ms = e0.elapsed_time(e1) / args.steps
    launches = (_lib.kernel_launches() - launches0) // args.steps
    kernel_ms = {}
    for name in KERNEL_SHARE:
        total, n = _lib.kernel_time(name)
        if n:
            kernel_ms[name] = max_over_ranks(total / n, world)
    _lib.timing_enable(False)
    ms = max_over_ranks(ms, world)
    flops = attention_flops(w)
    if cp:  # this rank's queries only (the kernels' roofline is rank 0's)
        p = torch.arange(lo_cp, hi_cp, dtype=torch.int64)
        kb = torch.clamp(p // w.block_size + 1, max=w.topk_blocks)
        nsel = int(((p % w.block_size) + 1 + w.block_size * (kb - 1)).sum()) * w.q_heads
        flops = {"fwd": 4 * w.dim * nsel, "bwd": 8 * w.dim * nsel, "fwd_bwd": 12 * w.dim * nsel}

    # forward rows re-run on the tensor cores (row bound too far above the logits) and rows
    # left to the float64 row kernel, on this input set (outside the timed region)
    reruns = None
    if not cp:
        import ctypes

        from msa_triton_b200 import _dispatch

        with _dispatch.keep_fwd_workspace():
            attend(q.detach(), k.detach(), v.detach(), ids, cu, prepared)
            if _dispatch.last_fwd_workspace is not None:
                ws_, tot_, hq_, nr_ = _dispatch.last_fwd_workspace
                a_, b_ = ctypes.c_int32(0), ctypes.c_int32(0)
                _lib.call("msa_attn_fwd_tc_rerun_counts", _lib.ptr(ws_), tot_, hq_, nr_, ctypes.byref(a_),
                          ctypes.byref(b_))
                reruns = {"tc_rerun_rows": a_.value, "f64_rows": b_.value}
                _dispatch.last_fwd_workspace = None

    # per-stage device times (instrumented pass, outside the timed region)
    stage = {}
    # forward and backward separately: median of 3 device-timed runs
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    fwd_t, bwd_t = [], []
    for _ in range(3):
        q.grad = k.grad = v.grad = None
        torch.cuda.synchronize()
        a.record(stream)
        out = attend(q, k, v, ids, cu, prepared)
        b.record(stream)
        torch.cuda.synchronize()
        fwd_t.append(a.elapsed_time(b))
        a.record(stream)
        out.backward(go)
        b.record(stream)
        torch.cuda.synchronize()
        bwd_t.append(a.elapsed_time(b))
    stage["forward"], stage["backward"] = statistics.median(fwd_t), statistics.median(bwd_t)
    if cp:  # the rank's selection: index score of its query range + top-k (index_k all-gathered)
        with torch.no_grad():
            a.record(stream)
            cp_select_blocks(x["index_q"], x["index_k"], global_tokens, block_size=w.block_size,
                             topk_blocks=w.topk_blocks, local_blocks=w.local_blocks)
            b.record(stream)
            torch.cuda.synchronize()
            stage["cp_select_blocks"] = a.elapsed_time(b)
    if not cp:
        with torch.no_grad():
            a.record(stream)
            sc = m3_index_score(x["index_q"], x["index_k"], cu, w.max_seqlen, block_size=w.block_size)
            b.record(stream)
            torch.cuda.synchronize()
            stage["index_score"] = a.elapsed_time(b)
            a.record(stream)
            m3_topk(sc, cu, block_size=w.block_size, topk_blocks=w.topk_blocks, local_blocks=w.local_blocks)
            b.record(stream)
            torch.cuda.synchronize()
            stage["topk"] = a.elapsed_time(b)
            del sc
        # the whole three-stage pipeline as the reference's stage timer runs it (benchmark.py:88-102):
        # index score -> top-k -> attention forward + backward, median of 5 device-timed runs
        def pipeline():
            with torch.no_grad():
                sc_ = m3_index_score(x["index_q"], x["index_k"], cu, w.max_seqlen, block_size=w.block_size,
                                     prepared=prepared)
                sel_ = m3_topk(sc_, cu, block_size=w.block_size, topk_blocks=w.topk_blocks,
                               local_blocks=w.local_blocks, prepared=prepared)
            q.grad = k.grad = v.grad = None
            attend(q, k, v, sel_, cu, prepared).backward(go)

        times = []
        for rep in range(6):
            torch.cuda.synchronize()
            a.record(stream)
            pipeline()
            b.record(stream)
            torch.cuda.synchronize()
            if rep:
                times.append(a.elapsed_time(b))
        stage["pipeline"] = statistics.median(times)
        # the indexer's KL loss (teacher: this step's attention LSE), forward + backward, warm then timed
        from msa_triton_b200 import m3_index_kl_loss

        with torch.no_grad():
            _, lse_t = m3_sparse_attention(q, k, v, ids, cu, w.max_seqlen, block_size=w.block_size,
                                           return_lse=True, prepared=prepared)
        iq_t = x["index_q"].detach().clone().requires_grad_()
        ik_t = x["index_k"].detach().clone().requires_grad_()
        kl_times = []
        for rep in range(4):  # one warm-up call, then the median of three
            torch.cuda.synchronize()
            a.record(stream)
            kl = m3_index_kl_loss(iq_t, ik_t, q.detach(), k.detach(), ids, cu, w.max_seqlen, block_size=w.block_size,
                                  lse=lse_t, prepared=prepared)
            kl.backward()
            b.record(stream)
            torch.cuda.synchronize()
            if rep:
                kl_times.append(a.elapsed_time(b))
            iq_t.grad = ik_t.grad = None
        stage["index_kl_fwd_bwd"] = statistics.median(kl_times)
        del iq_t, ik_t, lse_t
        # the index score when the indexer trains (gradients w.r.t. index_q / index_k), warm then timed
        iq_t = x["index_q"].detach().clone().requires_grad_()
        ik_t = x["index_k"].detach().clone().requires_grad_()
        up = torch.randn(w.total_tokens, w.groups, (w.max_seqlen + w.block_size - 1) // w.block_size, device=dev)
        train_fwd, train_bwd = [], []
        for rep in range(4):  # one warm-up call, then the median of three
            c = torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            a.record(stream)
            sc = m3_index_score(iq_t, ik_t, cu, w.max_seqlen, block_size=w.block_size)
            b.record(stream)
            sc.backward(up)
            c.record(stream)
            torch.cuda.synchronize()
            if rep:
                train_fwd.append(a.elapsed_time(b))
                train_bwd.append(b.elapsed_time(c))
            iq_t.grad = ik_t.grad = None
            del sc
        stage["index_score_train_fwd"] = statistics.median(train_fwd)
        stage["index_score_train_bwd"] = statistics.median(train_bwd)
        del iq_t, ik_t, up

    # dominant kernel: the tensor-core attention kernel with the largest device time per step,
    # timed by CUDA event pairs on its own stream inside the timed region. Its algorithmic
    # FLOPs per launch are its share of the selected FLOPs (recompute not counted).
    dom = max(kernel_ms, key=kernel_ms.get)
    dom_flops = KERNEL_SHARE[dom][1] * flops[KERNEL_SHARE[dom][0]]
    achieved = dom_flops / (kernel_ms[dom] * 1e-3) / 1e12
    peak = bf16_sustained or bf16_peak  # kernels timed inside a long step: the sustained figure
    traffic = NCU_TRAFFIC.get((w.name, dom)) if world == 1 else None  # per-rank launches do less work
    roofline = {"bound": "tensor", "kernel": dom, "achieved": round(achieved, 3), "peak": peak, "unit": "TFLOP/s",
                "frac": round(achieved / peak, 5), "peak_kind": f"{peak_kind} bf16 sustained",
                "kernel_ms": round(kernel_ms[dom], 4), "algorithmic_tflop_per_launch": round(dom_flops / 1e12, 4),
                "traffic": traffic}

    # End to end through the public API: every step copies its inputs from pinned host
    # memory and its results (out, dq, dk, dv) back to pinned host memory. Steps are
    # pipelined over two input/output buffer sets: the host->device copy of step s+1 and
    # the device->host copy of step s-1 run on their own streams while step s computes.
    pin = {n: host[n].pin_memory() for n in ("q", "k", "v", "grad_out")}
    ids_h = ids.cpu().pin_memory()
    cu_pin = cu_h.pin_memory()
    out_names = (("out", "q"), ("dq", "q"), ("dk", "k"), ("dv", "v"))
    outs_h = [{n: torch.empty(host[m].shape, dtype=host[m].dtype).pin_memory() for n, m in out_names}
              for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in pin.values()) + ids_h.numel() * 4 + cu_h.numel() * 4
    d2h = sum(t.numel() * t.element_size() for t in outs_h[0].values())
    bufs = [{"q": torch.empty_like(x["q"]), "k": torch.empty_like(x["k"]), "v": torch.empty_like(x["v"]),
             "grad_out": torch.empty_like(go), "ids": torch.empty_like(ids), "cu": torch.empty_like(cu)}
            for _ in range(2)]
    # each buffer set's cu_seqlens receives the same host values every step: prepared from them
    preps = [prepare_batch(bufs[j]["cu"], bounds=cu_h.tolist()) for j in range(2)]
    h2d_stream, d2h_stream = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    in_free = [torch.cuda.Event() for _ in range(2)]
    out_ready = [torch.cuda.Event() for _ in range(2)]
    out_free = [torch.cuda.Event() for _ in range(2)]
    for e in in_free + out_free:
        e.record(stream)
    results = [None, None]

    def upload(step):
        j = step % 2
        with torch.cuda.stream(h2d_stream):
            h2d_stream.wait_event(in_free[j])
            for n in ("q", "k", "v", "grad_out"):
                bufs[j][n].copy_(pin[n], non_blocking=True)
            bufs[j]["ids"].copy_(ids_h, non_blocking=True)
            bufs[j]["cu"].copy_(cu_pin, non_blocking=True)
            in_ready[j].record(h2d_stream)

    def compute(step):
        j = step % 2
        # bounded run-ahead (two buffer sets): the host waits until the download that
        # last used this set is done, as a pipelined loader with a queue of two would
        out_free[j].synchronize()
        stream.wait_event(in_ready[j])
        stream.wait_event(out_free[j])  # the previous device->host copy from this set is done
        qd, kd, vd = (bufs[j][n].detach().requires_grad_() for n in ("q", "k", "v"))
        o = attend(qd, kd, vd, bufs[j]["ids"], bufs[j]["cu"], preps[j])
        o.backward(bufs[j]["grad_out"])
        in_free[j].record(stream)
        results[j] = (o.detach(), qd.grad, kd.grad, vd.grad)
        out_ready[j].record(stream)

    def download(step):
        j = step % 2
        with torch.cuda.stream(d2h_stream):
            d2h_stream.wait_event(out_ready[j])
            for (n, _), t in zip(out_names, results[j]):
                outs_h[j][n].copy_(t, non_blocking=True)
                t.record_stream(d2h_stream)
            out_free[j].record(d2h_stream)

    def e2e_run(n_steps):
        h2d_stream.wait_stream(stream)  # copies start inside the timed region
        upload(0)
        for step in range(n_steps):
            if step + 1 < n_steps:
                upload(step + 1)
            compute(step)
            download(step)
        stream.wait_stream(d2h_stream)

    e2e_run(3)
    barrier(world)
    # steady-state throughput: the first upload and the last download (one step's
    # copies each, not overlapped with anything) are spread over at least 16 steps
    e2e_steps = max(16, args.steps)
    a.record(stream)
    e2e_run(e2e_steps)
    b.record(stream)
    barrier(world)
    e2e_ms = max_over_ranks(a.elapsed_time(b) / e2e_steps, world)
    # the results of the last step really arrived: compare its output with the device copy
    last = outs_h[(e2e_steps - 1) % 2]["out"]
    if not torch.equal(last, results[(e2e_steps - 1) % 2][0].cpu()):
        raise SystemExit("end-to-end: host copy of the output does not match the device result")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(w, host, ids.cpu().numpy(), sample_tokens_of(w, args.cpu_sample_tokens))
        cpu["eager"] = eager_baseline()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    tokens = global_tokens if (sharded or cp) else w.total_tokens * world
    # selected FLOPs of the whole job (all ranks)
    job_flops = attention_flops(w_global)["fwd_bwd"] if (sharded or cp) else flops["fwd_bwd"] * world
    line = {
        "metric": METRIC, "value": round(tokens / (ms * 1e-3), 1), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
        "scaling": "strong" if (sharded or cp) else "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1), unit RMS per head)",
        "config": bench_config(w_global, world, "shards" if sharded else "cp" if cp else "single", global_seqs,
                               args.inputs),
        "tflops": round(job_flops / (ms * 1e-3) / 1e12, 3),
        "frac_of_bf16_peak": round(job_flops / (ms * 1e-3) / 1e12 / (bf16_peak * world), 5),
        "stage_ms": {k2: round(v2, 4) for k2, v2 in stage.items()},
        "kernel_ms": {k2: round(v2, 4) for k2, v2 in kernel_ms.items()},
        "roofline": roofline,
        "e2e": {"value": round(tokens / (e2e_ms * 1e-3), 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3)},
        "gpu_launches": int(launches),
        "forward_reruns": reruns,
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------- reference arm
def run_reference(args):
    """The reference arm: the reference algorithm's CPU restatement on this arm's workload and
    selection rule, rank 0 only. Each step is a bounded sample: attention fwd+bwd of query tokens
    spread evenly over the batch, with the reference's own selection for them (float64 index
    score rows + top-k, computed before the timed steps)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # rank 0 alone times the CPU reference
    import torch

    from msa_triton_b200.workloads import make_inputs

    w = workload(args)
    host = scale_inputs(make_inputs(w), args.inputs)
    sample = max(8, args.cpu_sample_tokens // 4)  # one bounded sample per step: the whole run stays within minutes
    tokens = sample_tokens_of(w, sample)
    ids = cpu_selection_rows(w, host, tokens)
    values = []
    for i in range(args.warmup + args.steps):
        r = cpu_baseline(w, host, ids, tokens)
        if i >= args.warmup:
            values.append(r["value"])
    value = statistics.median(values)
    sample_desc = r["sample"].split(", float64")[0] + ", selection by the reference algorithm (float64 index " \
        "score rows + top-k), float64 numpy restatement; one sample per step"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(w.total_tokens / value * 1e3, 1),
        "ms_per_step_note": "extrapolated: the whole workload's tokens at the sampled tokens' rate",
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded N(0,1), unit RMS per head)",
        "config": bench_config(w, args.gpus, "single" if args.gpus == 1 else "shards" if len(w.lengths) > 1 else "cp",
                               len(w.lengths), args.inputs),
        "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": r["cores"], "kind": "port",
                         "sample": sample_desc, "torch_threads": torch.get_num_threads()},
        "eager": eager_baseline(),
        "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
