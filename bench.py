#!/usr/bin/env python
"""Benchmark of the B200 packed attention backend (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Headline workload (config 3 of the benchmark plan, the document batch): 512 documents per
GPU, lengths log-normal (median 600, sigma 0.8) clipped to [64, 8192], 16 heads x 64, bf16
q/k/v ~ N(0,1); ONE STEP = the attention of a 28-layer ModernBERT-large stack, global
attention every 3rd layer (10 global) and a +-64 sliding window elsewhere (18 local).
Metric: useful-pair TFLOP/s = 4 * allowed (query, key) pairs * H * D / time, summed over all
ranks' sequences / the slowest rank's time (weak scaling: the global batch is N x 512
documents, token-balanced over the ranks by LPT sequence partition, no collective on the
hot path).

``--impl reference`` times the reference's own CPU path for the same workload on the
host's cores (a bounded sample of the documents per step): its x86 C kernel
``pe_local_attention`` (packed_encoders/cpu/local_attention_x86.c, compiled from the
reference tree into oracle/_ref) for local layers and its per-sequence fp32 SDPA policy
for global layers longer than 128 tokens (packed_encoders/cpu/attention.py:400-403,
442-457).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

# dram__bytes_read.sum + dram__bytes_write.sum of one full-size attn_fwd_kernel launch (config 3
# global layer, all 512 documents), from a one-pass ncu capture of
# `python bench.py --case config3-global --iters 2`: 3.698 GB read + 0.899 GB written.
NCU_TRAFFIC_GLOBAL = 3.698e9 + 0.899e9


def _env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def _peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data["bf16_tflops"]),
                "bf16_tflops_sustained": float(data.get("bf16_tflops_sustained", data["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"pe_b200_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.fh, stderr=subprocess.DEVNULL)
            time.sleep(0.25)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(parts)
                float(parts[1])
            except ValueError:
                rows.pop()
        try:
            self.path.unlink()
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        loaded = [x for x in sm if x > 0.5 * max(sm)] or sm
        names = {5: "hw_slowdown", 6: "hw_thermal_slowdown", 7: "sw_thermal_slowdown", 8: "sw_power_cap"}
        reasons = sorted({names[i] for r in rows for i in names if r[i].lower() == "active"})
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace('.', '', 1).isdigit())
                if any(r[3].replace('.', '', 1).isdigit() for r in rows) else None}


# ----------------------------------------------------------------------------------------- CPU
CPU_SAMPLE_EVERY = 32  # one document per 32-document stratum of the length-sorted batch


def cpu_sample(lengths, every=CPU_SAMPLE_EVERY):
    """Length-stratified sample: sort the batch, cut it into strata of `every` documents, take the
    document at a fixed rank inside each stratum (the rank whose sample best matches the batch's
    mean, token-weighted and pair-weighted lengths). Returns [(length, stratum lengths)]."""
    order = sorted(lengths)
    strata = [order[i:i + every] for i in range(0, len(order), every)]

    def moments(ls):
        return [sum(x ** (p + 1) for x in ls) / sum(x ** p for x in ls) for p in (0, 1, 2)]

    target = moments(order)
    best = None
    for rank in range(every):
        pick = [st[min(rank, len(st) - 1)] for st in strata]
        dev = max(abs(a / b - 1) for a, b in zip(moments(pick), target))
        if best is None or dev < best[0]:
            best = (dev, [(st[min(rank, len(st) - 1)], st) for st in strata])
    return best[1]


class ReferenceCPU:
    """The reference's own CPU attention path, timed on this host's cores: CPUAttention.local
    (its x86 C kernel pe_local_attention, packed_encoders/cpu/local_attention_x86.c:192-235) and
    CPUAttention.global_ (per-sequence fp32 SDPA past 128 tokens, packed_encoders/cpu/
    attention.py:394-403,442-457). When the reference package is not importable, the same
    arithmetic runs through oracle/_ref (the reference's C file compiled from its source) and a
    per-sequence fp32 SDPA loop."""

    def __init__(self, heads, threads):
        import tempfile

        self.heads, self.threads = heads, threads
        torch.set_num_threads(threads)
        self.engine = None
        if _reference_importable():
            os.environ.setdefault("PACKED_ENCODERS_CPU_CACHE_DIR", tempfile.mkdtemp(prefix="pe_ref_cpu_"))
            try:
                from packed_encoders.cpu.attention import CPUAttention

                self.engine = CPUAttention("native", 64, 64, threads)
            except Exception as exc:  # noqa: BLE001
                self.engine_error = f"{type(exc).__name__}: {str(exc)[:80]}"
        self.kind = "reference package CPUAttention (native x86 kernel + per-sequence SDPA)" if self.engine \
            else "oracle/_ref pe_local_attention + per-sequence fp32 SDPA"

    def inputs(self, lengths, seed=5):
        gen = torch.Generator().manual_seed(seed)
        total = sum(lengths)
        return [torch.randn(1, self.heads, total, 64, generator=gen) for _ in range(3)]

    def local(self, q, k, v, lengths):
        boundaries = torch.tensor(lengths, dtype=torch.int32)
        if self.engine is not None:
            return self.engine.local(q, k, v, lengths, boundaries)
        import oracle

        return oracle.reference_local_attention(q[0], k[0], v[0], lengths, 64, threads=self.threads)

    def global_(self, q, k, v, lengths):
        boundaries = torch.tensor(lengths, dtype=torch.int32)
        if self.engine is not None:
            return self.engine.global_(q, k, v, lengths, boundaries)
        import torch.nn.functional as F

        off = 0
        for n in lengths:
            F.scaled_dot_product_attention(q[:, :, off:off + n], k[:, :, off:off + n], v[:, :, off:off + n])
            off += n


def cpu_reference_measure(lengths, heads, layers, *, threads, passes=1):
    """Estimated reference-CPU throughput on the whole batch from a stratified sample.

    Local layers: the sample in one call (its throughput; local work is linear in length).
    Global layers: each sampled document alone, its efficiency weighted by the useful FLOPs of
    its stratum, so the estimate has the batch's length mix (global work is quadratic in length).
    Returns a dict with the per-kind and the layer-mix figures."""
    from packed_encoders_b200.workloads import useful_flops

    started = time.perf_counter()
    cpu = ReferenceCPU(heads, threads)
    sample = cpu_sample(lengths)
    picks = [n for n, _ in sample]
    kinds = sorted(set(layers))
    res = {"kind": cpu.kind, "threads": threads, "sample_docs": len(picks), "sample_tokens": sum(picks)}
    est_s = {}
    with torch.inference_mode():
        q, k, v = cpu.inputs(picks)
        for window, causal in kinds:
            if window == (-1, -1):
                t_docs = [0.0] * len(picks)
                for _ in range(passes):
                    off = 0
                    for j, n in enumerate(picks):
                        sl = slice(off, off + n)
                        t0 = time.perf_counter()
                        cpu.global_(q[:, :, sl], k[:, :, sl], v[:, :, sl], [n])
                        t_docs[j] += (time.perf_counter() - t0) / passes
                        off += n
                est = 0.0
                for (n, stratum), t in zip(sample, t_docs):
                    eff = useful_flops([n], heads, 64, window, causal) / t
                    est += useful_flops(stratum, heads, 64, window, causal) / eff
                res["global_sample_s"] = round(sum(t_docs), 4)
            else:
                t = 0.0
                for _ in range(passes):
                    t0 = time.perf_counter()
                    cpu.local(q, k, v, picks)
                    t += (time.perf_counter() - t0) / passes
                est = useful_flops(lengths, heads, 64, window, causal) / (useful_flops(picks, heads, 64, window, causal) / t)
                res["local_sample_s"] = round(t, 4)
            name = "global" if window == (-1, -1) else "local"
            est_s[(window, causal)] = est
            res[f"{name}_tflops"] = round(useful_flops(lengths, heads, 64, window, causal) / est / 1e12, 4)
    total_flops = sum(useful_flops(lengths, heads, 64, w, c) for w, c in layers)
    total_s = sum(est_s[kind] for kind in layers)
    res["mix_tflops"] = round(total_flops / total_s / 1e12, 4)
    res["mix_s_estimated"] = round(total_s, 3)
    res["elapsed_s"] = round(time.perf_counter() - started, 3)  # wall time of this measurement
    return res


# ----------------------------------------------------------------------------------------- GPU
def make_step(pe, q, k, v, cu, max_len, layers, *, record_kernel=None):
    """One step = the attention of every layer in `layers`: one tile schedule per attention
    kind (built on device each step), then one kernel launch per layer. When `record` is a
    list, CUDA events bracket each launch of kind `record_kernel` on the launching stream."""
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream()
    scale = q.shape[2] ** -0.5

    def one_step(record=None):
        plans = {kind: pe.ops.plan_attention(q, k, cu, max_len, window=kind[0], causal=kind[1])
                 for kind in sorted(set(layers))}
        for window, causal in layers:
            ev = None
            if record is not None and (window, causal) == record_kernel:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record(stream)
            pe.packed_attention(q, k, v, cu, max_len, scale=scale, window=window, causal=causal, out=out,
                                plan=plans[(window, causal)])
            if ev is not None:
                ev[1].record(stream)
                record.append(ev)
        return out

    return one_step, out


def run_b200(args):
    import torch.distributed as dist

    import packed_encoders_b200 as pe
    from packed_encoders_b200 import shard as shard_mod
    from packed_encoders_b200 import workloads as wl

    world = _env_int("WORLD_SIZE", 1)
    rank = _env_int("RANK", 0)
    local_rank = _env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta
        # NCCL prints its version banner on stdout at communicator creation (when NCCL_DEBUG asks
        # for it): send fd 1 to stderr meanwhile, so rank 0's stdout carries only the JSON line.
        sys.stdout.flush()
        saved_fd = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
            dist.barrier()
        finally:
            import ctypes
            ctypes.CDLL(None).fflush(None)
            os.dup2(saved_fd, 1)
            os.close(saved_fd)

    layers = wl.config3("mix").layers
    lengths_all = wl.config3_lengths(512 * world, seed=0)
    costs = [shard_mod.pattern_cost(n, (wl.GLOBAL, wl.LOCAL64), alpha=64.0) for n in lengths_all]
    shards = shard_mod.partition(lengths_all, world, costs)
    my = shards[rank]
    heads, dim = 16, 64
    q, k, v = wl.make_qkv(my.lengths, heads, heads, dim, seed=1 + rank, device=device)
    cu = my.cu_seqlens(device)
    max_len = max(my.lengths)
    flops_by_kind = {kind: wl.useful_flops(my.lengths, heads, dim, *kind) for kind in set(layers)}
    step_flops = sum(flops_by_kind[kind] for kind in layers)

    one_step, out = make_step(pe, q, k, v, cu, max_len, layers, record_kernel=wl.GLOBAL)
    for _ in range(args.warmup):
        one_step(None)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    stream = torch.cuda.current_stream()
    launches0 = pe.ops.LAUNCHES["kernels"]
    kernel_events = []
    with ClockSampler(local_rank) as clocks:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for _ in range(args.steps):
            one_step(kernel_events)
        end.record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    launches = pe.ops.LAUNCHES["kernels"] - launches0
    elapsed_ms = start.elapsed_time(end)
    kernel_ms = [a.elapsed_time(b) for a, b in kernel_events]
    err = pe.device_error_word()

    # e2e: the same step through the public API from pinned host buffers, H2D + D2H timed.
    # Double-buffered like a serving loop: step s computes on device buffer s % 2 while the inputs
    # of step s + 1 arrive in the other buffer on an H2D stream and the output of step s - 1
    # leaves on a D2H stream. Every step copies all of its inputs and its output; the timed
    # region runs from the first H2D to the end of the last D2H.
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    hcu = cu.cpu().pin_memory()
    houts = [torch.empty(out.shape, dtype=out.dtype).pin_memory() for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in (hq, hk, hv, hcu))
    d2h = houts[0].numel() * houts[0].element_size()
    e2e_steps = max(2, min(2 * args.steps, 10))
    dev_sets = [(q, k, v, cu), tuple(t.clone() for t in (q, k, v, cu))]
    step_fns = [one_step, make_step(pe, *dev_sets[1], max_len, layers)[0]]
    step_fns[1](None)  # warm-up of the second buffer's step (allocations outside the timed region)
    h2d_stream, d2h_stream = torch.cuda.Stream(device), torch.cuda.Stream(device)
    copied = [torch.cuda.Event() for _ in range(2)]
    computed = [torch.cuda.Event() for _ in range(2)]
    drained = [torch.cuda.Event() for _ in range(2)]

    def upload(b):
        for dst, src in zip(dev_sets[b], (hq, hk, hv, hcu)):
            dst.copy_(src, non_blocking=True)
        copied[b].record(h2d_stream)

    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(stream)
    h2d_stream.wait_event(e_start)
    with torch.cuda.stream(h2d_stream):
        upload(0)
    for s_ in range(e2e_steps):
        b = s_ % 2
        if s_ + 1 < e2e_steps:  # next step's inputs, once the step that last read that buffer is done
            if s_ >= 1:
                h2d_stream.wait_event(computed[1 - b])
            with torch.cuda.stream(h2d_stream):
                upload(1 - b)
        stream.wait_event(copied[b])
        if s_ >= 2:
            stream.wait_event(drained[b])  # this buffer's previous output has left
        res = step_fns[b](None)
        computed[b].record(stream)
        d2h_stream.wait_event(computed[b])
        with torch.cuda.stream(d2h_stream):
            houts[b].copy_(res, non_blocking=True)
            drained[b].record(d2h_stream)
    stream.wait_stream(h2d_stream)
    stream.wait_stream(d2h_stream)
    e_end.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e_start.elapsed_time(e_end)

    strong = strong_scaling(pe, wl, shard_mod, args, world, rank, device) if world > 1 else None

    totals = torch.tensor([elapsed_ms, e2e_ms, float(step_flops), float(my.tokens), float(h2d), float(d2h)],
                          dtype=torch.float64, device=device)
    if world > 1:
        tmax = totals[:2].clone()
        dist.all_reduce(tmax, op=dist.ReduceOp.MAX)
        tsum = totals[2:].clone()
        dist.all_reduce(tsum, op=dist.ReduceOp.SUM)
        elapsed_ms, e2e_ms = tmax.tolist()
        step_flops_all, tokens_all, h2d_all, d2h_all = tsum.tolist()
    else:
        step_flops_all, tokens_all, h2d_all, d2h_all = float(step_flops), float(my.tokens), float(h2d), float(d2h)

    if rank != 0:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return

    peaks = _peaks()
    ms_per_step = elapsed_ms / args.steps
    value = step_flops_all * args.steps / (elapsed_ms / 1e3) / 1e12
    e2e_value = step_flops_all * e2e_steps / (e2e_ms / 1e3) / 1e12
    avg_kernel_ms = statistics.mean(kernel_ms) if kernel_ms else None
    achieved = flops_by_kind[wl.GLOBAL] / (avg_kernel_ms / 1e3) / 1e12 if avg_kernel_ms else None
    traffic = None
    if NCU_TRAFFIC_GLOBAL is not None:
        traffic = NCU_TRAFFIC_GLOBAL
    record = {
        "metric": "useful-pair attention TFLOP/s, 28-layer ModernBERT-large document batch (10 global + 18 local)",
        "value": round(value, 3),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_per_step, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "config": {
            "workload": "config3-document-batch: 512 docs/GPU, lognormal(median 600, sigma 0.8) in [64,8192], "
                        "16 heads x 64, 28 layers (global every 3rd, else window +-64)",
            "heads": heads, "head_dim": dim, "n_seq_per_gpu": 512, "tokens_rank0": my.tokens,
            "tokens_all_ranks": int(tokens_all), "global_batch_seqs": 512 * world,
            "parallelism": f"dp{world} (LPT token-balanced sequence partition, no collective)",
            "l2": "inputs larger than L2 (q,k,v,out = %.2f GB per layer)" % (
                (q.numel() + k.numel() + v.numel() + out.numel()) * 2 / 1e9),
        },
        "tokens_per_s": round(tokens_all * args.steps / (elapsed_ms / 1e3), 1),
        "roofline": {
            "kernel": "attn_fwd_kernel (global layer, config 3)",
            "bound": "tensor",
            "achieved": round(achieved, 3) if achieved else None,
            "peak": peaks["bf16_tflops"],
            "unit": "TFLOP/s",
            "frac": round(achieved / peaks["bf16_tflops"], 4) if achieved else None,
            "frac_of_sustained": round(achieved / peaks["bf16_tflops_sustained"], 4) if achieved else None,
            "peak_source": f"{peaks['source']} (MEASURED_PEAKS.json bf16_tflops burst)",
            "traffic": traffic,
            "traffic_unit": "bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum, full-size launch)",
            "algorithmic_bytes": wl.algorithmic_bytes(my.tokens, my.tokens, heads, heads, dim),
            "avg_launch_ms": round(avg_kernel_ms, 4) if avg_kernel_ms else None,
            "launches": len(kernel_ms),
        },
        "e2e": {
            "value": round(e2e_value, 3), "unit": "TFLOP/s",
            "h2d_bytes_per_step": int(h2d_all), "d2h_bytes_per_step": int(d2h_all),
            "steps": e2e_steps,
            "note": "per step: pinned H2D of q,k,v,cu_seqlens, the 28-layer attention through "
                    "packed_encoders_b200.packed_attention, D2H of the output; double-buffered: the H2D of "
                    "step s+1 and the D2H of step s-1 run on copy streams during step s; timed from the "
                    "first H2D to the end of the last D2H",
        },
        "clocks": clocks.summary(),
        "gpu_launches": launches,
        "device_error_word": err,
    }
    if strong is not None:
        record["strong_scaling"] = strong
    if world == 1 and not args.no_cpu_baseline:
        record["cpu_baseline"] = cpu_baseline_record(args)
    if world == 1 and not args.no_extra:
        record["workloads"] = extra_workloads(pe, wl, peaks)
        try:
            record["comparators"] = comparators(pe, wl, record["workloads"])
        except Exception as exc:  # noqa: BLE001
            record["comparators"] = {"failed": f"{type(exc).__name__}: {str(exc)[:120]}"}
        try:
            record["config5_output_gate"] = gate_fusion(pe, wl)
        except Exception as exc:  # noqa: BLE001
            record["config5_output_gate"] = {"failed": f"{type(exc).__name__}: {str(exc)[:120]}"}
        try:
            record["config3_rope"] = rope_fusion(pe, wl)
        except Exception as exc:  # noqa: BLE001
            record["config3_rope"] = {"failed": f"{type(exc).__name__}: {str(exc)[:120]}"}
        try:
            record["config3_backward"] = backward_layers(pe, wl)
        except Exception as exc:  # noqa: BLE001
            record["config3_backward"] = {"failed": f"{type(exc).__name__}: {str(exc)[:120]}"}
        try:
            record["config4_full_forward"] = config4_forward(pe)
        except Exception as exc:  # noqa: BLE001
            record["config4_full_forward"] = {"failed": f"{type(exc).__name__}: {str(exc)[:120]}"}
    print(json.dumps(record), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def strong_scaling(pe, wl, shard_mod, args, world, rank, device):
    """The fixed 512-document config-3 batch split over `world` ranks (LPT on the 28-layer cost,
    the same partition as the headline's), each rank timing its share for the same number of steps;
    the job's time is the slowest rank's. Reported beside the weak-scaling headline, so the
    1 -> N curve shows what the partition's imbalance costs. Every rank takes the same collectives."""
    import torch.distributed as dist

    layers = wl.config3("mix").layers
    lengths = wl.config3_lengths(512, seed=0)
    costs = [shard_mod.pattern_cost(n, (wl.GLOBAL, wl.LOCAL64), alpha=64.0) for n in lengths]
    shards = shard_mod.partition(lengths, world, costs)
    mine = shards[rank]
    heads, dim = 16, 64
    q, k, v = wl.make_qkv(mine.lengths, heads, heads, dim, seed=1 + rank, device=device)
    cu = mine.cu_seqlens(device)
    one_step, _ = make_step(pe, q, k, v, cu, max(mine.lengths), layers)
    for _ in range(args.warmup):
        one_step(None)
    torch.cuda.synchronize()
    dist.barrier()
    stream = torch.cuda.current_stream()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(args.steps):
        one_step(None)
    b.record(stream)
    torch.cuda.synchronize()
    dist.barrier()
    ms = torch.tensor([a.elapsed_time(b) / args.steps], dtype=torch.float64, device=device)
    all_ms = [torch.zeros_like(ms) for _ in range(world)]
    dist.all_gather(all_ms, ms)
    rank_ms = [float(t.item()) for t in all_ms]
    flops = sum(wl.useful_flops(lengths, heads, dim, *kind) for kind in layers)
    loads = [sh.load for sh in shards]
    del q, k, v, cu
    return {"global_batch_seqs": 512, "tokens": sum(lengths), "ms_per_step": round(max(rank_ms), 4),
            "value": round(flops / (max(rank_ms) / 1e3) / 1e12, 3), "unit": "TFLOP/s",
            "rank_ms_per_step": [round(x, 4) for x in rank_ms],
            "load_max_over_mean": round(max(loads) / (sum(loads) / len(loads)), 4),
            "time_max_over_mean": round(max(rank_ms) / (sum(rank_ms) / len(rank_ms)), 4),
            "partition": "LPT on cost 64*L + pairs(L) over one global and one local layer"}


def cpu_baseline_record(args):
    from packed_encoders_b200 import workloads as wl

    threads = max(1, len(os.sched_getaffinity(0)))
    w = wl.config3("mix")
    runs = cpu_reference_runs(w, threads, warmup=3, steps=5)
    m = runs["median"]
    return {"value": m["mix_tflops"], "unit": "TFLOP/s", "cores": threads, "kind": "reference",
            "local_tflops": m["local_tflops"], "global_tflops": m["global_tflops"],
            "runs_mix_tflops": runs["mix_tflops"],
            "sample": f"{m['sample_docs']} of 512 documents ({m['sample_tokens']} tokens), one per 32-document "
                      f"stratum of the length-sorted batch; global layers timed per document and weighted by "
                      f"their stratum's FLOPs, local layers timed as one call; 28-layer mix = 10 global + 18 "
                      f"local; {m['kind']}; median of 5 estimates after 3 warm-up ones, the same function "
                      f"and counts as bench.py --impl reference --steps 5 --warmup 3"}


def cpu_reference_runs(w, threads, *, warmup, steps):
    """`warmup` untimed and `steps` timed stratified estimates (cpu_reference_measure); the median
    estimate (by its 28-layer time) and every run's layer-mix throughput."""
    for _ in range(warmup):
        cpu_reference_measure(w.lengths, w.heads, w.layers, threads=threads)
    runs = [cpu_reference_measure(w.lengths, w.heads, w.layers, threads=threads) for _ in range(max(1, steps))]
    median = sorted(runs, key=lambda r: r["mix_s_estimated"])[len(runs) // 2]
    return {"median": median, "mix_tflops": [r["mix_tflops"] for r in runs], "elapsed_s": [r["elapsed_s"] for r in runs]}


def extra_workloads(pe, wl, peaks, iters=10):
    """Per-configuration single-launch numbers (L2 flushed between timed launches)."""
    res = {}
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    cases = [
        ("config1-global", wl.config1("global")), ("config1-local", wl.config1("local")),
        ("config2-query-batch", wl.config2()),
        ("config3-global", wl.config3("global")), ("config3-local", wl.config3("local")),
        ("config5-gqa-causal", wl.config5()),
    ]
    for name, w in cases:
        q, k, v = wl.make_qkv(w.lengths, w.heads, w.kv_heads, w.head_dim, seed=1)
        cu = w.cu_seqlens().cuda()
        (window, causal), = set(w.layers)
        out = torch.empty_like(q)
        plan = pe.ops.plan_attention(q, k, cu, max(w.lengths), window=window, causal=causal)
        times = []
        for i in range(iters + 3):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            pe.packed_attention(q, k, v, cu, max(w.lengths), scale=w.scale, window=window, causal=causal,
                                out=out, plan=plan)
            b.record()
            torch.cuda.synchronize()
            if i >= 3:
                times.append(a.elapsed_time(b))
        ms = statistics.median(times)
        flops = wl.useful_flops(w.lengths, w.heads, w.head_dim, window, causal)
        nbytes = wl.algorithmic_bytes(w.tokens, w.tokens, w.heads, w.kv_heads, w.head_dim)
        tflops = flops / (ms / 1e3) / 1e12
        gbs = nbytes / (ms / 1e3) / 1e9
        res[name] = {"ms": round(ms, 4), "tflops": round(tflops, 2), "tokens_per_s": round(w.tokens / (ms / 1e3), 1),
                     "hbm_gbs": round(gbs, 1), "tensor_frac": round(tflops / peaks["bf16_tflops"], 4),
                     "hbm_frac": round(gbs / peaks["hbm_gbs"], 4), "tokens": w.tokens}
        del q, k, v, out, plan
    return res


def _reference_importable():
    """The reference package from its git-ignored install under baseline/_ref."""
    from oracle.reference_tree import add_reference_to_path

    if not add_reference_to_path():
        return False
    try:
        import packed_encoders  # noqa: F401
        return True
    except Exception:  # noqa: BLE001
        return False


def _time_call(fn, iters=10, flush=None):
    times = []
    for i in range(iters + 3):
        if flush is not None:
            flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        if i >= 3:
            times.append(a.elapsed_time(b))
    return statistics.median(times)


def comparators(pe, wl, ours):
    """The reference's own GPU kernels on the same box and inputs: FlashAttention-2 varlen (the
    compiled-FA path of packed_encoders/ops.py:364-371, imported from the image whether or not
    the reference package is) and, inside its envelope (H=12, D=64, Smax<=128, no causal: config
    2), the reference's Triton packed-short kernel (_kernels/triton_packed_attention.py:45-143).
    FA4 4.0.0b16, the reference's preferred sm_100 kernel (runtime/attention.py:192-196), is not
    installable in this image."""
    out = {"fa4": "unavailable: flash-attn-4 4.0.0b16 is not installed in this image"}
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    try:
        from flash_attn import flash_attn_varlen_func
    except Exception as exc:  # noqa: BLE001
        flash_attn_varlen_func = None
        out["fa2"] = f"unavailable: {type(exc).__name__}"
    triton_short = None
    if _reference_importable():
        try:
            from packed_encoders._kernels.triton_packed_attention import packed_short_attention as triton_short
        except Exception as exc:  # noqa: BLE001
            out["triton"] = f"unavailable: {type(exc).__name__}: {str(exc)[:80]}"
    else:
        out["triton"] = "unavailable: reference package not importable (baseline/_ref missing)"

    cases = [("config1-global", wl.config1("global")), ("config1-local", wl.config1("local")),
             ("config2-query-batch", wl.config2()), ("config3-global", wl.config3("global")),
             ("config3-local", wl.config3("local")), ("config5-gqa-causal", wl.config5())]
    for name, w in cases:
        q, k, v = wl.make_qkv(w.lengths, w.heads, w.kv_heads, w.head_dim, seed=1)
        cu = w.cu_seqlens().cuda()
        (window, causal), = set(w.layers)
        flops = wl.useful_flops(w.lengths, w.heads, w.head_dim, window, causal)
        entry = {}
        if flash_attn_varlen_func is not None:
            try:
                fn = lambda: flash_attn_varlen_func(q, k, v, cu, cu, max(w.lengths), max(w.lengths), dropout_p=0.0,
                                                    softmax_scale=w.scale, causal=causal, window_size=window)
                ms = _time_call(fn, flush=flush)
                entry["fa2_ms"] = round(ms, 4)
                entry["fa2_tflops"] = round(flops / (ms / 1e3) / 1e12, 2)
            except Exception as exc:  # noqa: BLE001
                entry["fa2"] = f"failed: {type(exc).__name__}: {str(exc)[:80]}"
        if triton_short is not None and w.heads == 12 and w.head_dim == 64 and max(w.lengths) <= 128 and not causal:
            half = None if window == (-1, -1) else window[0]
            try:
                with torch.no_grad():
                    fn = lambda: triton_short(q, k, v, cu, max(w.lengths), half_window=half, softmax_scale=w.scale)
                    ms = _time_call(fn, flush=flush)
                entry["triton_ms"] = round(ms, 4)
                entry["triton_tflops"] = round(flops / (ms / 1e3) / 1e12, 2)
            except Exception as exc:  # noqa: BLE001
                entry["triton"] = f"failed: {type(exc).__name__}: {str(exc)[:80]}"
        if name in ours:
            entry["b200_ms"] = ours[name]["ms"]
            ref_ms = [x for x in (entry.get("fa2_ms"), entry.get("triton_ms")) if x is not None]
            if ref_ms:
                entry["speedup_vs_best_reference_kernel"] = round(min(ref_ms) / ours[name]["ms"], 3)
        out[name] = entry
        del q, k, v
    return out


def gate_fusion(pe, wl, iters=10):
    """Config 5 with the Qwen3.5 output gate through packed_attention(..., gate=g) (attention, then
    this library's gate pass), against attention followed by the reference's own gate kernel
    (_kernels/hybrid.py:208-219, Triton). The fused-epilogue form (PE_B200_GATE=fused) is chosen
    once per process, so it is not timed here."""
    w = wl.config5()
    q, k, v = wl.make_qkv(w.lengths, w.heads, w.kv_heads, w.head_dim, seed=1)
    gate = torch.randn(q.shape, device="cuda", generator=torch.Generator("cuda").manual_seed(7)).to(torch.bfloat16)
    cu = w.cu_seqlens().cuda()
    (window, causal), = set(w.layers)
    plan = pe.ops.plan_attention(q, k, cu, max(w.lengths), window=window, causal=causal)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    kw = dict(scale=w.scale, window=window, causal=causal, plan=plan)
    res = {}
    ref_gate = None
    if _reference_importable():
        try:
            from packed_encoders._kernels.hybrid import sigmoid_gate as ref_gate
        except Exception as exc:  # noqa: BLE001
            res["reference_gate_kernel"] = f"unavailable: {type(exc).__name__}: {str(exc)[:80]}"
    else:
        res["reference_gate_kernel"] = "unavailable: reference package not importable"
    if ref_gate is None:  # no stand-in: the comparison is against the reference's own kernel or nothing
        return res

    def gated():
        pe.packed_attention(q, k, v, cu, max(w.lengths), gate=gate, **kw)

    def unfused():
        o = pe.packed_attention(q, k, v, cu, max(w.lengths), **kw)
        ref_gate(o, gate)

    times = {"gated_call_ms": [], "attention_then_reference_gate_ms": []}
    for _ in range(3):  # interleaved: the power-capped clock drifts between measurements
        times["gated_call_ms"].append(_time_call(gated, iters, flush))
        times["attention_then_reference_gate_ms"].append(_time_call(unfused, iters, flush))
    for key, vals in times.items():
        res[key] = round(statistics.median(vals), 4)
    res["speedup_vs_reference_gate"] = round(res["attention_then_reference_gate_ms"] / res["gated_call_ms"], 3)
    del q, k, v, gate, plan
    return res


def rope_fusion(pe, wl, iters=10):
    """Config 3 layers with RoPE (ModernBERT's BSHD path, forward.py:197-205): q/k/v are views of
    one packed qkv [T, 3*H*D] and the rotary tables are per token [T, 64] (gathered from position
    tables, forward.py:493-510). This library's call (packed_attention(..., rope=): its rope pass,
    then attention), the same attention without rotation (the floor), and the reference's
    apply_rope_bshd pass (_kernels/rope.py:302-345, CuteDSL) followed by the same attention."""
    w = wl.config3("mix")
    lengths = w.lengths
    q, k, v = wl.make_qkv(lengths, w.heads, w.kv_heads, w.head_dim, seed=1)
    tq, h, d = q.shape
    qkv = torch.stack((q, k, v), 1).reshape(tq, 3 * h * d)
    del q, k, v
    view = qkv.view(tq, 3, h, d)
    cu = w.cu_seqlens().cuda()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    ref_rope = None
    res = {}
    if _reference_importable():
        try:
            from packed_encoders._kernels.rope import apply_rope_bshd as ref_rope
        except Exception as exc:  # noqa: BLE001
            res["reference_rope_kernel"] = f"unavailable: {type(exc).__name__}: {str(exc)[:80]}"
    else:
        res["reference_rope_kernel"] = "unavailable: reference package not importable"
    pos_all = torch.cat([torch.arange(n, device="cuda") for n in lengths])
    for kind, (window, causal), theta in (("local", wl.LOCAL64, 10000.0), ("global", wl.GLOBAL, 160000.0)):
        inv = 1.0 / theta ** (torch.arange(0, d, 2, dtype=torch.float32, device="cuda") / d)
        pos = torch.arange(max(lengths), dtype=torch.float32, device="cuda")
        emb = torch.cat((pos[:, None] * inv, pos[:, None] * inv), -1)
        cos_p, sin_p = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)  # position tables [S, 64]
        cos, sin = cos_p[pos_all], sin_p[pos_all]  # per-token gather (packed_forward, forward.py:506-507)
        kw = dict(scale=w.scale, window=window, causal=causal)  # all build their schedule per call

        def rope_pass():
            pe.packed_attention(view[:, 0], view[:, 1], view[:, 2], cu, max(lengths), rope=(cos, sin), **kw)

        def attention_only():  # the same attention on q/k that need no rotation (the floor)
            pe.packed_attention(view[:, 0], view[:, 1], view[:, 2], cu, max(lengths), **kw)

        def separate():
            rq, rk = ref_rope(qkv, h, d, cos, sin)
            pe.packed_attention(rq, rk, view[:, 2], cu, max(lengths), **kw)

        times = {"rope_call_ms": [], "attention_only_ms": []}
        if ref_rope is not None:  # no stand-in: the reference's own kernel or no comparison
            times["reference_rope_then_attention_ms"] = []
        for _ in range(3):
            times["rope_call_ms"].append(_time_call(rope_pass, iters, flush))
            times["attention_only_ms"].append(_time_call(attention_only, iters, flush))
            if ref_rope is not None:
                times["reference_rope_then_attention_ms"].append(_time_call(separate, iters, flush))
        r = {key: round(statistics.median(val), 4) for key, val in times.items()}
        r["rope_call_over_attention_only"] = round(r["rope_call_ms"] / r["attention_only_ms"], 3)
        if ref_rope is not None:
            r["speedup_vs_reference"] = round(r["reference_rope_then_attention_ms"] / r["rope_call_ms"], 3)
        res[kind] = r
        del cos, sin, cos_p, sin_p
    del qkv, view
    return res


def backward_layers(pe, wl, iters=5):
    """Config 3 layers (512 documents, 16 x 64, global and +-64) backward: this library's
    packed_attention_backward against FlashAttention-2's varlen backward on the same inputs and
    dout. FLOP = 2.5 x the useful forward FLOP (five matmuls of the recomputing backward against
    two of the forward); L2 flushed between calls."""
    res = {}
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    w = wl.config3("mix")
    q, k, v = wl.make_qkv(w.lengths, w.heads, w.kv_heads, w.head_dim, seed=1)
    dout = torch.randn(q.shape, device="cuda", generator=torch.Generator("cuda").manual_seed(3)).to(torch.bfloat16)
    cu = w.cu_seqlens().cuda()
    try:
        from flash_attn import flash_attn_varlen_func
    except Exception as exc:  # noqa: BLE001
        flash_attn_varlen_func = None
        res["fa2"] = f"unavailable: {type(exc).__name__}"
    for kind, (window, causal) in (("global", wl.GLOBAL), ("local", wl.LOCAL64)):
        out, lse = pe.packed_attention(q, k, v, cu, max(w.lengths), scale=w.scale, window=window, causal=causal,
                                       return_lse=True)
        fn = lambda: pe.packed_attention_backward(dout, q, k, v, out, lse, cu, max(w.lengths), scale=w.scale,
                                                  window=window, causal=causal)
        ms = _time_call(fn, iters, flush)
        flops = 2.5 * wl.useful_flops(w.lengths, w.heads, w.head_dim, window, causal)
        r = {"ms": round(ms, 4), "tflops": round(flops / (ms / 1e3) / 1e12, 2)}
        if flash_attn_varlen_func is not None:
            try:
                qg, kg, vg = (t.detach().clone().requires_grad_() for t in (q, k, v))
                o = flash_attn_varlen_func(qg, kg, vg, cu, cu, max(w.lengths), max(w.lengths), softmax_scale=w.scale,
                                           causal=causal, window_size=window)
                fa = lambda: torch.autograd.grad(o, (qg, kg, vg), dout, retain_graph=True)
                fms = _time_call(fa, iters, flush)
                r["fa2_ms"] = round(fms, 4)
                r["speedup_vs_fa2"] = round(fms / ms, 3)
                del qg, kg, vg, o
            except Exception as exc:  # noqa: BLE001
                r["fa2"] = f"failed: {type(exc).__name__}: {str(exc)[:80]}"
        res[kind] = r
        del out, lse
    del q, k, v, dout
    return res


def config4_forward(pe):
    """Config 4: a random-init ModernBERT-base packed_forward (22 layers, hidden 768, 12 heads,
    GeGLU 1152, global every 3rd layer, RoPE theta 160000 / 10000) in bf16 on 256 queries
    U[16,48] + 64 documents U[256,8192], through the reference's own forward with the b200
    attention backend installed, against the same forward on its FlashAttention-2 path."""
    if not _reference_importable():
        return {"unavailable": "reference package not importable (baseline/_ref missing)"}
    import packed_encoders as pe_ref
    from packed_encoders import forward
    from packed_encoders.arch.modernbert import ModernBert
    from packed_encoders.config import ModernBertParams
    from transformers import ModernBertConfig, ModernBertModel

    from packed_encoders_b200 import install

    install.install()
    torch.manual_seed(0)
    cfg = ModernBertConfig()
    cfg._attn_implementation = "sdpa"
    model = ModernBertModel(cfg).to("cuda", torch.bfloat16).eval()
    pe_ref.pack(model, engine=ModernBert(pieces=install.b200_pieces()), attention_backend="b200", validate=False)
    params = ModernBertParams.from_hf_config(model.config)
    g = torch.Generator().manual_seed(0)
    lengths = [int(x) for x in torch.randint(16, 49, (256,), generator=g)] + \
              [int(x) for x in torch.randint(256, 8193, (64,), generator=g)]
    cu = torch.tensor([0, *torch.tensor(lengths).cumsum(0).tolist()], dtype=torch.int32, device="cuda")
    ids = torch.randint(1, cfg.vocab_size, (sum(lengths),), device="cuda", generator=torch.Generator(device="cuda").manual_seed(1))
    pos = torch.cat([torch.arange(n, device="cuda") for n in lengths])
    res = {"tokens": sum(lengths), "sequences": len(lengths)}
    from packed_encoders.arch.modernbert_pieces import default_execution

    for backend in ("b200", "flash"):
        # the FA2 run uses the reference's own pieces (its BSHD attention piece calls FA)
        execution = None if backend == "b200" else default_execution()
        try:
            with torch.inference_mode():
                fn = lambda: forward.packed_forward(model, params, ids, cu, max(lengths), pos, backend=backend,
                                                    execution=execution)
                ms = _time_call(fn, iters=5)
            res[f"{backend}_ms"] = round(ms, 3)
            res[f"{backend}_tokens_per_s"] = round(sum(lengths) / (ms / 1e3), 1)
        except Exception as exc:  # noqa: BLE001
            res[backend] = f"failed: {type(exc).__name__}: {str(exc)[:100]}"
    if "b200_ms" in res and "flash_ms" in res:
        res["speedup_vs_reference_fa2_forward"] = round(res["flash_ms"] / res["b200_ms"], 3)
    del model
    return res


def run_reference(args):
    """The reference arm: the reference's own CPU path for the same workload, metric and unit, on
    this host's cores (rank 0 only under torchrun). One step = one stratified estimate of the
    28-layer step of the 512-document batch (cpu_reference_measure)."""
    world = _env_int("WORLD_SIZE", 1)
    rank = _env_int("RANK", 0)
    if rank != 0:
        return
    from packed_encoders_b200 import workloads as wl

    threads = max(1, len(os.sched_getaffinity(0)))
    w = wl.config3("mix")
    runs = cpu_reference_runs(w, threads, warmup=args.warmup, steps=args.steps)
    last = runs["median"]
    value = last["mix_tflops"]
    record = {
        "impl": "reference",
        "metric": "useful-pair attention TFLOP/s, 28-layer ModernBERT-large document batch (10 global + 18 local)",
        "value": round(value, 4), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(statistics.mean(runs["elapsed_s"]) * 1e3, 2), "higher_is_better": True,
        "scaling": "weak", "estimated_full_step_ms": round(last["mix_s_estimated"] * 1e3, 1), "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config3-document-batch: 512 docs, lognormal(median 600, sigma 0.8) in [64,8192], "
                               "16 heads x 64, 28 layers (global every 3rd, else window +-64)",
                   "heads": w.heads, "head_dim": 64, "estimate": "stratified sample, see cpu_baseline.sample"},
        "local_tflops": last["local_tflops"], "global_tflops": last["global_tflops"],
        "runs_mix_tflops": runs["mix_tflops"],
        "cpu_baseline": {"value": round(value, 4), "unit": "TFLOP/s", "cores": threads, "kind": "reference",
                         "sample": f"{last['sample_docs']} of 512 documents per step, one per 32-document stratum of "
                                   f"the length-sorted batch, stratum-weighted; value = the median step; "
                                   f"{last['kind']}"},
        "e2e": {"value": round(value, 4), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(record), flush=True)


def run_case(args):
    """Profiling helper: ``--case NAME --iters N [--seqs S] [--rope] [--gate] [--backward]`` launches
    one configuration N times (no timing output), e.g. for an ncu capture of a small case of the same
    kernel. ``--rope``: q/k/v are views of one packed qkv and the call applies RoPE (head_dim 64);
    ``--gate``: the call applies the output gate; ``--backward``: one forward with LSE, then N
    backward calls on it."""
    import packed_encoders_b200 as pe
    from packed_encoders_b200 import workloads as wl

    makers = {"config1-global": lambda: wl.config1("global"), "config1-local": lambda: wl.config1("local"),
              "config2": wl.config2, "config3-global": lambda: wl.config3("global"),
              "config3-local": lambda: wl.config3("local"), "config5": wl.config5}
    w = makers[args.case]()
    lengths = list(w.lengths[: args.seqs]) if args.seqs else list(w.lengths)
    q, k, v = wl.make_qkv(lengths, w.heads, w.kv_heads, w.head_dim, seed=1)
    cu = torch.zeros(len(lengths) + 1, dtype=torch.int32)
    cu[1:] = torch.tensor(lengths).cumsum(0)
    cu = cu.cuda()
    (window, causal), = set(w.layers)
    extra = {}
    if args.rope:
        qkv = torch.stack((q, k, v), 1)
        q, k, v = qkv[:, 0], qkv[:, 1], qkv[:, 2]
        inv = 1.0 / 10000.0 ** (torch.arange(0, 64, 2, dtype=torch.float32, device="cuda") / 64)
        pos = torch.cat([torch.arange(n, dtype=torch.float32, device="cuda") for n in lengths])
        emb = torch.cat((pos[:, None] * inv, pos[:, None] * inv), -1)
        extra["rope"] = (emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16))
    if args.gate:
        extra["gate"] = torch.randn(q.shape, device="cuda").to(torch.bfloat16)
    out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
    if args.backward:
        out, lse = pe.packed_attention(q, k, v, cu, max(lengths), scale=w.scale, window=window, causal=causal,
                                       return_lse=True)
        dout = torch.randn(q.shape, device="cuda", generator=torch.Generator("cuda").manual_seed(3)).to(q.dtype)
        for _ in range(args.iters):
            pe.packed_attention_backward(dout, q, k, v, out, lse, cu, max(lengths), scale=w.scale, window=window,
                                         causal=causal)
    else:
        for _ in range(args.iters):
            pe.packed_attention(q, k, v, cu, max(lengths), scale=w.scale, window=window, causal=causal, out=out,
                                **extra)
    torch.cuda.synchronize()
    print(json.dumps({"case": args.case, "tokens": sum(lengths), "seqs": len(lengths), "iters": args.iters,
                      "device_error_word": pe.device_error_word()}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default=None, help="profiling helper: run one configuration --iters times")
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--seqs", type=int, default=0, help="with --case: use only the first SEQS sequences")
    ap.add_argument("--rope", action="store_true", help="with --case: q/k/v views of one qkv, RoPE in the call")
    ap.add_argument("--gate", action="store_true", help="with --case: output gate in the call")
    ap.add_argument("--backward", action="store_true", help="with --case: one forward, then --iters backward calls")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.case:
        run_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
