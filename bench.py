#!/usr/bin/env python
"""Benchmark: sparse FP8 MLA decode step on B200 (BASELINE.json metric
"sparse-decode us/step & % roofline").

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 1|2|4] [--mode batch|head|replicate]

A step is one pass of the hot path over one batch: the decode kernel (K1)
plus the split combine (K3), on the schedule that get_mla_metadata (K2)
computed once for the batch (FlashMLA's protocol: metadata once per batch,
reused by every layer; its own time is reported as sched_meta_us).
Default workload: BASELINE config 1 (b 32, s_q 1, h_q 64, top-k 2048,
128K-token context per request, page 256, random block tables, V32 FP8
cache), synthetic seeded data.  L2 is flushed (256 MiB write) before every
timed step; the gathered KV (43 MB) is below L2 size, so without the flush
the rows would be L2-resident across steps.

N > 1 (torchrun, one rank per GPU).  "batch" mode (default) shards the
requests of one global batch: rank r builds only requests
partition.batch_range(B, r, N) and their cache pages (each request is
generated from its own seed, so the shards are exactly the unsharded
batch's requests) and decodes them; no collective in the data path.
Configs 1-3 are one GPU's batch, so B = b x N (weak scaling); config 4 is
the whole-box batch, B = 256 over all ranks (strong scaling).  "head" mode
splits h_q over the ranks with a replicated cache.  After the timed region
(batch and head) the shards are all-gathered with NCCL and rank 0 compares
sampled rows with an unsharded decode of the same requests
("partition_check").  "replicate" runs an independent config-sized batch
per rank.  Timing: CUDA events on the launching stream, max over ranks.

The default run (config 1, no overrides) also carries, at N = 1, configs 2
and 4 ("other_configs") and the writer / indexer next to the decode
("next_rows"); at N > 1, config 4 batch- and head-sharded
("partition_config4").

--impl reference times the CPU oracle port (oracle/, a numpy restatement
of the reference's tests/reference.py) on this host's cores on the same
workload (the global batch of the mode); rank 0 only.  It imports only
host-side modules of the package, so libdsv4b.so is not loaded.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "deepseek-v4-flash-sm120_b200"))

FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
FLUSH_BYTES = 256 << 20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=1, choices=[1, 2, 3, 4],
                    help="BASELINE config; 3 = the CUDA-graph batch x context sweep")
    ap.add_argument("--mode", choices=["batch", "head", "replicate"], default="batch",
                    help="N > 1: batch = shard the requests of one global batch; head = shard h_q over "
                         "a replicated cache; replicate = an independent batch per rank")
    ap.add_argument("--batch", type=int, default=None, help="override b (per rank)")
    ap.add_argument("--ctx", type=int, default=None,
                    help="override the per-request context (cache size); same per-step work "
                         "(b, h_q, top-k) on a smaller cache, for profiler captures")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-next-rows", action="store_true",
                    help="skip the writer / indexer summaries in the config-1 line")
    ap.add_argument("--json-out", default=None)
    ap.add_argument("--op", choices=["decode", "kv_write", "mqa_logits", "prefill", "mma_rates", "gather_rates"],
                    default="decode",
                    help="kv_write: the KV-cache writer (quantise + scatter); mqa_logits: the indexer "
                         "logits (fp8_paged_mqa_logits) over config 1's contexts; mma_rates: cycles per "
                         "tcgen05.mma of the decode kernel's operand shapes (resident operands); "
                         "gather_rates: random whole-row gathers per load mechanism")
    ap.add_argument("--next-n", type=int, default=1, help="mqa_logits: query rows per request")
    ap.add_argument("--page-order", choices=["random", "sequential"], default="random",
                    help="mqa_logits: physical order of each request's pages (block table)")
    ap.add_argument("--kv-layout", choices=["v32", "model1"], default="v32")
    ap.add_argument("--tokens", type=int, default=131072, help="kv_write: tokens written per step")
    ap.add_argument("--pages", type=int, default=16384, help="kv_write: cache pages of 256 tokens")
    ap.add_argument("--slots", choices=["paged", "random"], default="paged",
                    help="kv_write: 'paged' = consecutive slots inside randomly placed pages (a prefill "
                         "chunk through a block table); 'random' = every token at a random slot")
    return ap.parse_args()


# ------------------------------------------------------------------ peaks / clocks
def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(path))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, local_rank: int):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [x.strip() for x in vis.split(",") if x.strip()]
        self.gpu = ids[local_rank] if local_rank < len(ids) else str(local_rank)
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-i", self.gpu, "-lms", "50"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        time.sleep(0.06)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), f[3], f[5:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[3]) if v.lower() == "active"})
        return {
            "sm_mhz": statistics.median([r[0] for r in rows]) if rows else None,
            "sm_max_mhz": max(r[1] for r in rows) if rows else None,
            "reasons": reasons,
            "samples": len(rows),
        }


def bind_to_gpu_numa_node(device_index: int):
    """Pin this process's CPU affinity to the NUMA node of the GPU's PCIe
    root before pinned host buffers are allocated, so that host <-> device
    copies do not cross sockets.  Returns the node, or None where the
    topology is not visible (nothing is changed then)."""
    try:
        import torch
        props = torch.cuda.get_device_properties(device_index)
        bus = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        node = int(open(f"/sys/bus/pci/devices/{bus}/numa_node").read().strip())
        if node < 0:
            return None
        cpus = set()
        for part in open(f"/sys/devices/system/node/node{node}/cpulist").read().strip().split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return node
    except Exception:
        return None


# ------------------------------------------------------------------ workload
# Config 4 is the whole-box batch (b = 256 requests over all ranks, strong
# scaling); the other configurations are one GPU's batch, so in batch mode
# the global batch is b x N requests (weak scaling: per-GPU work fixed).
WHOLE_BOX_CONFIGS = (4,)


def workload(cfg: int, batch_override, ctx_override=None):
    """The configuration's BatchSpec (b = the per-GPU batch, or for config
    4 the whole-box batch)."""
    from deepseek_v4_kernel import kvcache
    spec = kvcache.sweep_spec(32, 131072) if cfg == 3 else kvcache.CONFIGS[cfg]
    spec = kvcache.BatchSpec(**{**spec.__dict__, "seed": 1000})
    if batch_override:
        spec.b = batch_override
    if ctx_override:
        spec.ctx, spec.cache_ctx = ctx_override, None
    return spec


def global_batch(cfg: int, spec, mode: str, world: int):
    """(global BatchSpec, requests per step over all ranks) for a mode."""
    from deepseek_v4_kernel import kvcache
    if mode == "batch" and cfg not in WHOLE_BOX_CONFIGS:
        return kvcache.BatchSpec(**{**spec.__dict__, "b": spec.b * world}), spec.b * world
    if mode == "replicate":
        return spec, spec.b * world
    return spec, spec.b


def scaling_kind(cfg: int, mode: str) -> str:
    if mode == "head" or (mode == "batch" and cfg in WHOLE_BOX_CONFIGS):
        return "strong"
    return "weak"


def build_inputs(spec_g, mode: str, rank: int, world: int, device):
    """This rank's batch.  batch: requests batch_range(b, rank, N) of the
    global batch, built by this rank alone; head: the whole batch on every
    rank (replicated cache; the rank decodes its head slice); replicate:
    an independent config-sized batch per rank (seed 1000 + rank)."""
    from deepseek_v4_kernel import kvcache, partition
    if mode == "batch":
        lo, hi = partition.batch_range(spec_g.b, rank, world)
        return kvcache.make_batch_shard(spec_g, lo, hi, device=device), (lo, hi)
    if mode == "head":
        return kvcache.make_batch_shard(spec_g, 0, spec_g.b, device=device), (0, spec_g.b)
    s = kvcache.BatchSpec(**{**spec_g.__dict__, "seed": 1000 + rank})
    return kvcache.make_batch(s, device=device), (0, s.b)


def algorithmic(spec, h_q_local=None):
    h = h_q_local or spec.h_q
    bpt = 656 if spec.layout == "v32" else 584
    d_qk = 576 if spec.layout == "v32" else 512
    rows = spec.b * spec.s_q * spec.topk
    kv_bytes = rows * bpt
    flops = 2.0 * spec.b * spec.s_q * h * spec.topk * (d_qk + 512)
    return kv_bytes, flops


def workload_name(spec, mode, world, b_global=None):
    return (f"b{b_global or spec.b} s_q{spec.s_q} h_q{spec.h_q} "
            f"topk{spec.topk} ctx{spec.ctx} page{spec.page_block} {spec.layout.upper()} fp8 KV"
            + (f", {mode}-sharded x{world}" if world > 1 else ""))


# ------------------------------------------------------------------ reference arm (CPU oracle)
def run_reference(args, spec, world, rank):
    """The reference's CPU path (the numpy port of tests/reference.py) on
    this host's cores, for the same workload as our arm: the global batch of
    the run's mode, a bounded sample of whole query rows per step, times
    scaled to the full global batch."""
    if rank != 0:
        return
    import torch
    from threadpoolctl import threadpool_limits
    from concurrent.futures import ThreadPoolExecutor

    from deepseek_v4_kernel import kvcache  # host-only module: does not map libdsv4b.so
    from oracle import sparse_decode_oracle as O

    spec_g, reqs = global_batch(args.config, spec, args.mode, world)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    threads = os.cpu_count() or 1

    def load(lo, hi):
        bt = kvcache.make_batch_shard(spec_g, lo, hi, device=dev)
        return (bt.q.float().cpu().numpy(), bt.kv.cpu().numpy(), bt.indices.cpu().numpy(),
                bt.attn_sink.cpu().numpy() if bt.attn_sink is not None else None, bt.sm_scale)

    def one(data, rows):
        q, kv, idx, sink, scale = data
        return O.sparse_decode_reference(q[rows], kv, idx[rows], None, sink, scale, spec.page_block,
                                         layout=spec.layout)

    # bounded sample: as many whole requests as fit in ~2 s per step
    first = load(0, 1)
    t0 = time.perf_counter()
    with threadpool_limits(1):
        one(first, [0])
    per_row = max(time.perf_counter() - t0, 1e-4)
    n_rows = int(min(reqs, spec_g.b, max(1, threads * 2.0 / per_row)))
    data = load(0, n_rows) if n_rows > 1 else first
    chunks = [list(range(i, n_rows, threads)) for i in range(min(threads, n_rows))]
    times = []
    with threadpool_limits(1), ThreadPoolExecutor(threads) as ex:
        for i in range(args.warmup + args.steps):
            t = time.perf_counter()
            list(ex.map(lambda c: one(data, c), chunks))
            dt = time.perf_counter() - t
            if i >= args.warmup:
                times.append(dt * reqs / n_rows)       # scaled to the full global batch
    us = statistics.median(times) * 1e6
    sample = (f"{n_rows} of {reqs} requests per step (times scaled to the full batch of the run), "
              f"numpy port of tests/reference.py, gather of the top-k rows only")
    line = {
        "metric": "sparse_decode_us_per_step", "value": round(us, 1), "unit": "us/step",
        "impl": "reference", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(us / 1e3, 3), "higher_is_better": False,
        "scaling": scaling_kind(args.config, args.mode),
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"config{args.config}: " + workload_name(spec, args.mode, world, reqs),
                   "cpu_threads": threads},
        "cpu_baseline": {"value": round(us, 1), "unit": "us/step", "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(us, 1), "unit": "us/step", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline_quick(spec, bt, budget_s=12.0):
    """Oracle port timed on this host's cores on a bounded sample of the
    workload (whole query rows), scaled to the full batch."""
    import numpy as np
    from threadpoolctl import threadpool_limits
    from concurrent.futures import ThreadPoolExecutor
    from oracle import sparse_decode_oracle as O

    q = bt.q.float().cpu().numpy()
    kv = bt.kv.cpu().numpy()
    idx = bt.indices.cpu().numpy()
    sink = bt.attn_sink.cpu().numpy() if bt.attn_sink is not None else None
    threads = os.cpu_count() or 1

    def one(rows):
        return O.sparse_decode_reference(q[rows], kv, idx[rows], None, sink, bt.sm_scale,
                                         spec.page_block, layout=spec.layout)

    with threadpool_limits(1):
        t0 = time.perf_counter()
        one([0])
        per_row = max(time.perf_counter() - t0, 1e-4)
    n_rows = int(min(spec.b, max(threads, threads * (budget_s / 3) / per_row)))
    n_rows = max(1, min(n_rows, spec.b))
    chunks = [list(range(i, n_rows, threads)) for i in range(min(threads, n_rows))]
    reps = []
    with threadpool_limits(1), ThreadPoolExecutor(threads) as ex:
        for _ in range(3):
            t = time.perf_counter()
            list(ex.map(one, chunks))
            reps.append((time.perf_counter() - t) * spec.b / n_rows)
    return {"value": round(statistics.median(reps) * 1e6, 1), "unit": "us/step", "cores": threads,
            "kind": "port",
            "sample": f"{n_rows} of {spec.b} query rows, 3 reps, median, scaled to the full batch; "
                      f"numpy port of tests/reference.py (gathers only the top-k rows)"}


# ------------------------------------------------------------------ our arm
def verify_partition(args, spec_g, out, lse, h_range, world, rank, device):
    """Outside the timed region: reassemble the shards with NCCL and compare
    sampled rows with an unsharded decode of the same requests (our public
    op on one GPU).  Returns a summary on rank 0, None elsewhere."""
    import torch
    from deepseek_v4_kernel import kvcache, ops, partition
    if args.mode == "batch":
        out_all = partition.all_gather_batch(out, spec_g.b, world)
        lse_all = partition.all_gather_batch(lse, spec_g.b, world)
        if rank != 0:
            return None
        b = spec_g.b
        picks = sorted({0, b // 3, (2 * b) // 3, b - 1})
        errs = []
        for r in picks:
            one = kvcache.make_batch_shard(spec_g, r, r + 1, device=device)
            o, l, _, _ = ops.sparse_decode_fwd(one.q, one.kv, one.indices, None, one.attn_sink, None, None,
                                               None, None, None, 512, one.sm_scale)
            errs.append(((out_all[r].float() - o[0].float()).abs().max().item(),
                         (lse_all[r] - l[0]).abs().max().item()))
        what = f"requests {picks} of the all-gathered batch vs each request decoded alone"
    else:  # head
        full = partition.all_gather_heads(out, world)
        if rank != 0:
            return None
        bt, _ = build_inputs(spec_g, "head", 0, 1, device)
        o, l, _, _ = ops.sparse_decode_fwd(bt.q, bt.kv, bt.indices, None, bt.attn_sink, None, None,
                                           None, None, None, 512, bt.sm_scale)
        errs = [((full.float() - o.float()).abs().max().item(), 0.0)]
        what = "all-gathered head shards vs the unsharded decode (all heads, one GPU)"
    max_out = max(e[0] for e in errs)
    max_lse = max(e[1] for e in errs)
    return {"checked": what, "max_abs_err_out": max_out, "max_abs_err_lse": max_lse,
            "ok": bool(max_out <= 2e-2 and max_lse <= 1e-3)}


def run_ours(args, spec, world, rank, local_rank):
    """Times the decode step of this rank's shard; returns the JSON line on
    rank 0 (None on the other ranks)."""
    import torch
    import torch.distributed as dist

    import deepseek_v4_kernel as dk
    from deepseek_v4_kernel import _lib, ops, partition

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    lib = _lib.lib
    assert lib.dsv4b_check_device(local_rank) == 0, "not an sm_100 GPU"

    spec_g, reqs = global_batch(args.config, spec, args.mode, world)
    bt, (r_lo, r_hi) = build_inputs(spec_g, args.mode, rank, world, device)
    h_lo, h_hi = 0, spec.h_q
    if args.mode == "head" and world > 1:
        h_lo, h_hi = partition.head_range(spec.h_q, rank, world)
    q = bt.q[:, :, h_lo:h_hi].contiguous()
    sink = bt.attn_sink[h_lo:h_hi].contiguous() if bt.attn_sink is not None else None
    b, s_q, h_q, d_qk = q.shape
    out = torch.empty(b, s_q, h_q, 512, dtype=torch.bfloat16, device=device)
    lse = torch.empty(b, h_q, s_q, dtype=torch.float32, device=device)
    p = ops.build_params(q, bt.kv, bt.indices, None, sink, None, None, None, 512, bt.sm_scale, out, lse)
    stream = torch.cuda.current_stream(device)
    sh = stream.cuda_stream

    # K2 once per batch (timed separately)
    ev_s0, ev_s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tsm, ns = ops.get_mla_metadata_tensors(p, device)  # first call: one-time set-up
    torch.cuda.synchronize()
    # K2's device time: 20 scheduler calls captured in one CUDA graph (the
    # host-side cost of each Python call is not part of it)
    g_s = torch.cuda.CUDAGraph()
    side_s = torch.cuda.Stream(device)
    side_s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side_s), torch.cuda.graph(g_s, stream=side_s):
        for _ in range(20):
            ops.get_mla_metadata_tensors(p, device)
    torch.cuda.current_stream(device).wait_stream(side_s)
    g_s.replay()
    torch.cuda.synchronize()
    ev_s0.record()
    g_s.replay()
    ev_s1.record()
    torch.cuda.synchronize()
    del g_s
    sched_us = ev_s0.elapsed_time(ev_s1) * 1e3 / 20
    parts = tsm.size(0)
    cluster = ops.plan_cluster_size(p, parts)
    launches_per_step = 1 if cluster > 1 else 2  # decode (+ combine unless the clusters merged)
    nbytes = lib.dsv4b_workspace_bytes(b, s_q, h_q, parts)
    ws = ops.workspace(device, nbytes)
    pp = ctypes.byref(p)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=device)

    def step(evs=None):
        # The public entry point: the decode kernel, plus (when the plan
        # splits rows outside clusters) the combine launched as its
        # programmatic dependent -- nothing may be enqueued between them.
        rc = lib.dsv4b_sparse_decode(pp, tsm.data_ptr(), ns.data_ptr(), parts, ws.data_ptr(), ws.numel(), sh)
        if evs is not None:
            evs[1].record(stream)
        if rc:
            raise RuntimeError(f"decode failed: {rc}")

    for _ in range(args.warmup):
        flush.zero_()
        step()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    sampler = ClockSampler(local_rank)
    sampler.start()
    time.sleep(0.15)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    for i in range(args.steps):
        flush.zero_()
        evs[i][0].record(stream)
        step(evs[i])
        evs[i][2].record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = sampler.stop()
    dec_ms = [e[0].elapsed_time(e[1]) for e in evs]
    t_step = statistics.median(dec_ms)  # evs[1] follows the step's last launch directly
    assert dk.read_kernel_status(device) == 0, "kernel wait timeout"

    verify = None
    if world > 1 and args.mode in ("batch", "head"):
        verify = verify_partition(args, spec_g, out, lse, (h_lo, h_hi), world, rank, device)

    # max over ranks
    if world > 1:
        t = torch.tensor([t_step], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_step = t.item()

    # e2e through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        numa_node = bind_to_gpu_numa_node(local_rank)
        q_host = q.cpu().pin_memory()
        idx_host = bt.indices.cpu().pin_memory()
        q_dev = torch.empty_like(q)
        idx_dev = torch.empty_like(bt.indices)
        out_host = torch.empty(out.shape, dtype=out.dtype).pin_memory()
        lse_host = torch.empty(lse.shape, dtype=lse.dtype).pin_memory()
        meta, _ = dk.get_mla_metadata()
        n_e2e = max(1, min(args.steps, 200))

        def e2e_step():
            q_dev.copy_(q_host, non_blocking=True)
            idx_dev.copy_(idx_host, non_blocking=True)
            o, l = dk.flash_mla_with_kvcache(q_dev, bt.kv, None, None, 512, meta, softmax_scale=bt.sm_scale,
                                             is_fp8_kvcache=True, indices=idx_dev, attn_sink=sink)
            out_host.copy_(o, non_blocking=True)
            lse_host.copy_(l, non_blocking=True)

        for _ in range(3):
            flush.zero_()
            e2e_step()
        torch.cuda.synchronize()
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(n_e2e)]
        for i in range(n_e2e):
            flush.zero_()
            ev[i][0].record(stream)
            e2e_step()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        t_e2e = statistics.median([a.elapsed_time(b_) for a, b_ in ev])
        # host wall clock: n back-to-back steps, no flush between them, one
        # synchronise at the end (exposes the host-side enqueue cost)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            e2e_step()
        torch.cuda.synchronize()
        t_wall = (time.perf_counter() - t0) / n_e2e * 1e3
        if world > 1:
            t = torch.tensor([t_e2e, t_wall], dtype=torch.float64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_e2e, t_wall = t.tolist()
        h2d = q_host.numel() * q_host.element_size() + idx_host.numel() * idx_host.element_size()
        d2h = out_host.numel() * out_host.element_size() + lse_host.numel() * lse_host.element_size()
        e2e = {"value": round(t_e2e * 1e3, 2), "unit": "us/step", "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": d2h,
               "wall_us": round(t_wall * 1e3, 2),
               "path": "deepseek_v4_kernel.flash_mla_with_kvcache (FlashMLASchedMeta reused), "
                       "pinned host q/indices -> device, out/lse -> pinned host",
               "timing": "value: CUDA events around each step (L2 flushed before it); wall_us: host "
                         f"perf_counter over {n_e2e} back-to-back steps with no flush, one sync at the end",
               "host_numa_node": numa_node}

    if rank != 0:
        return None
    hbm_peak, tc_peak, peak_src = measured_peaks()
    kv_bytes, flops = algorithmic(bt.spec, h_q)
    achieved_gbs = kv_bytes / (t_step * 1e-3) / 1e9
    achieved_tf = flops / (t_step * 1e-3) / 1e12
    bound = "hbm" if kv_bytes / hbm_peak / 1e9 >= flops / tc_peak / 1e12 else "tensor"
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath) and world == 1:
        try:
            traffic = json.load(open(tpath)).get(f"config{args.config}")
        except Exception:
            traffic = None
    if bound == "hbm":
        roof = {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": hbm_peak, "unit": "GB/s",
                "frac": round(achieved_gbs / hbm_peak, 4), "traffic": traffic}
    else:
        roof = {"bound": "tensor", "achieved": round(achieved_tf, 1), "peak": tc_peak, "unit": "TFLOP/s",
                "frac": round(achieved_tf / tc_peak, 4), "traffic": traffic}
    roof["peak_source"] = peak_src
    roof["kernel"] = "sparse_decode_kernel (K1)" + (" + combine_kernel (K3)" if launches_per_step > 1 else "")
    roof["per"] = "rank 0's shard" if world > 1 else "the whole batch"
    roof["algorithmic_bytes_per_launch"] = kv_bytes
    roof["algorithmic_flops_per_launch"] = flops
    roof["tensor_frac"] = round(achieved_tf / tc_peak, 4)
    roof["hbm_frac"] = round(achieved_gbs / hbm_peak, 4)
    t_roof_us = max(kv_bytes / hbm_peak / 1e3, flops / tc_peak / 1e6)
    tokens = reqs * spec.s_q
    line = {
        "metric": "sparse_decode_us_per_step",
        "value": round(t_step * 1e3, 2),
        "unit": "us/step",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_step, 5),
        "higher_is_better": False,
        "scaling": scaling_kind(args.config, args.mode),
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q / latent / RoPE, random page tables, distinct top-k)",
        "config": {"workload": f"config{args.config}: " + workload_name(spec, args.mode, world, reqs),
                   "l2": "flushed before every step (256 MiB write)",
                   "parallelism": f"{args.mode}-shard x{world}" if world > 1 else "single GPU",
                   "rank0_requests": [r_lo, r_hi], "rank0_heads": [h_lo, h_hi],
                   "num_sm_parts": parts, "cluster_size": cluster},
        "decode_kernel_us": round(t_step * 1e3, 2),
        "combine_launched": launches_per_step > 1,
        "sched_meta_us": round(sched_us, 2),
        "roofline_time_us": round(t_roof_us, 2),
        "step_roofline_frac": round(t_roof_us / (t_step * 1e3), 4),
        "tokens_per_s": round(tokens / (t_step * 1e-3), 1),
        "roofline": roof,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
    }
    if verify is not None:
        line["partition_check"] = verify
    if e2e:
        line["e2e"] = e2e
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_quick(bt.spec, bt)
    return line


def summary_of(line):
    """The fields of a sub-run's line carried under another line's key."""
    keep = ("value", "unit", "n_gpus", "scaling", "decode_kernel_us", "combine_launched", "tokens_per_s",
            "roofline_time_us", "step_roofline_frac", "gpu_launches", "clocks", "partition_check")
    d = {k: line[k] for k in keep if k in line}
    d["workload"] = line["config"]["workload"]
    d["parallelism"] = line["config"]["parallelism"]
    r = line["roofline"]
    d["roofline"] = {k: r[k] for k in ("bound", "achieved", "peak", "unit", "frac", "hbm_frac", "tensor_frac")}
    return d


def sub_runs(args, world, rank, local_rank):
    """Extra workloads carried by the default line: at N = 1 configs 2 and
    4 on one GPU; at N > 1 config 4's whole-box batch, batch-sharded and
    head-sharded.  20 timed steps each, no e2e / CPU baseline."""
    import copy
    import torch
    plan = ([(2, "batch"), (4, "batch")] if world == 1 else [(4, "batch"), (4, "head")])
    out = {}
    for cfg, mode in plan:
        a = copy.copy(args)
        a.config, a.mode, a.steps, a.warmup = cfg, mode, 20, 5
        a.no_e2e, a.no_cpu_baseline, a.batch, a.ctx = True, True, None, None
        key = f"config{cfg}" + ("" if world == 1 else f"_{mode}")
        try:
            line = run_ours(a, workload(cfg, None), world, rank, local_rank)
            if line is not None:
                out[key] = summary_of(line)
        except Exception as e:  # reported in the line, the headline stands
            out[key] = {"error": f"{type(e).__name__}: {e}"[:300]}
        torch.cuda.empty_cache()
    return out


def next_rows(args):
    """The two steps either side of the decode in a serving step (the cache
    write before it, the indexer that picks its top-k), measured
    with their own bench modes and summarised in the headline line: the
    KV-cache writer (131,072 tokens, V32 and MODEL1) and the indexer logits
    (config 1's contexts).  A failure here is reported, not raised."""
    import copy
    import torch
    out = {}
    for name, fn, kw in (("kv_write_v32", run_kv_write, {"kv_layout": "v32"}),
                         ("kv_write_model1", run_kv_write, {"kv_layout": "model1"}),
                         ("mqa_logits", run_mqa_logits, {})):
        a = copy.copy(args)
        a.steps, a.warmup, a.tokens, a.pages, a.slots = 20, 3, 131072, 16384, "paged"
        a.next_n, a.page_order, a.batch, a.ctx = 1, "random", None, None
        for k, v in kw.items():
            setattr(a, k, v)
        try:
            d = fn(a)
            out[name] = {"metric": d["metric"], "value": d["value"], "unit": d["unit"],
                         "workload": d["config"]["workload"], "roofline": d["roofline"],
                         "cpu_baseline": d["cpu_baseline"], "gpu_launches": d["gpu_launches"]}
        except Exception as e:  # reported in the line, the headline stands
            out[name] = {"error": f"{type(e).__name__}: {e}"[:300]}
        torch.cuda.empty_cache()
    return out


def run_kv_write(args):
    """One step = one dsv4b_kv_cache_write of --tokens bf16 tokens (a
    prefill chunk) into BASELINE config 1's cache geometry (16,384 pages of
    256 tokens) at random distinct slots.  Per step the kernel reads
    1,152 (V32) / 1,024 (MODEL1) B of bf16 per token plus an 8-B slot and
    writes 656 / 584 B, more than L2 holds, so no flush is needed."""
    import numpy as np
    import torch

    from deepseek_v4_kernel import _lib, cache_ops
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    n, page, nb = args.tokens, 256, args.pages
    v32 = args.kv_layout == "v32"
    g = torch.Generator(device=device).manual_seed(0)
    nope = torch.randn(n, 512 if v32 else 448, generator=g, device=device).to(torch.bfloat16)
    rope = torch.randn(n, 64, generator=g, device=device).to(torch.bfloat16)
    if args.slots == "random":
        slots = torch.randperm(nb * page, generator=g, device=device)[:n].contiguous()
    else:
        pages = torch.randperm(nb, generator=g, device=device)[: -(-n // page)]
        t = torch.arange(n, device=device)
        slots = (pages[t // page] * page + t % page).contiguous()
    if v32:
        cache = torch.zeros(nb, page, 1, 656, dtype=torch.uint8, device=device)
        layout, bs = _lib.LAYOUT_V32, None
    else:
        cache = torch.zeros(nb, page * 584, dtype=torch.uint8, device=device)
        layout, bs = _lib.LAYOUT_MODEL1, page
    per_tok_read = (1024 if v32 else 896) + 128 + 8
    per_tok_write = 656 if v32 else 584
    alg = n * (per_tok_read + per_tok_write)

    def step():
        cache_ops.kv_cache_write(layout, nope, rope, slots, cache, block_size=bs)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    # The K timed launches are one CUDA graph, so they run back to back on
    # the device whatever the host-side cost of a Python call.
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(device)
    cap.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(cap):
        with torch.cuda.graph(graph, stream=cap):
            for _ in range(args.steps):
                step()
    torch.cuda.current_stream(device).wait_stream(cap)
    graph.replay()          # warm replay
    torch.cuda.synchronize()
    clk = ClockSampler(0)
    clk.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record()
    graph.replay()
    t1.record()
    torch.cuda.synchronize()
    clocks = clk.stop()
    t_step_ms = t0.elapsed_time(t1) / args.steps
    t_kernel_ms = t_step_ms
    hbm_peak, _, peak_src = measured_peaks()
    ach = alg / (t_kernel_ms * 1e-3) / 1e9

    # CPU baseline: the oracle on a bounded sample of the same tokens
    from oracle import kv_writer_oracle as KW
    sample = min(n, 16384)
    nb_s = -(-sample // page)
    arena = np.zeros((nb_s, page * (656 if v32 else 584)), np.uint8)
    nb_bits = nope[:sample].cpu().view(torch.int16).numpy().view(np.uint16)
    rp_bits = rope[:sample].cpu().view(torch.int16).numpy().view(np.uint16)
    sl = np.arange(sample)
    c0 = time.perf_counter()
    KW.kv_cache_write(args.kv_layout, arena, page, nb_bits, rp_bits, sl)
    cpu_s = time.perf_counter() - c0
    line = {
        "metric": "kv_cache_write_us_per_step",
        "value": round(t_step_ms * 1e3, 2),
        "unit": "us/step",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_step_ms, 5),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u8",
        "data": "synthetic (seeded N(0,1) bf16 tokens, %s slots)" % (
            "random distinct" if args.slots == "random" else "page-consecutive, random physical pages"),
        "config": {"workload": f"kv_write {args.kv_layout} ({args.slots} slots): {n} tokens into {nb} pages x 256"
                               + (" (config 1 cache geometry)" if nb == 16384 else ""),
                   "l2": f"no flush: {alg / 1e6:.0f} MB moved per step, above L2 size"},
        "kernel_us": round(t_kernel_ms * 1e3, 2),
        "timing": "one CUDA graph of `steps` writer launches, CUDA events around its replay",
        "tokens_per_s": round(n / (t_step_ms * 1e-3), 1),
        "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(ach / hbm_peak, 4), "traffic": None, "peak_source": peak_src,
                     "kernel": "kv_write_%s_kernel" % args.kv_layout,
                     "algorithmic_bytes_per_launch": alg},
        "gpu_launches": args.steps,
        "clocks": clocks,
        "cpu_baseline": {"value": round(cpu_s / sample * n * 1e6, 1), "unit": "us/step", "cores": 1,
                         "kind": "port", "sample": f"oracle/kv_writer_oracle.py on {sample} of the {n} "
                                                   f"tokens, scaled to {n}"},
    }
    return line


def run_mqa_logits(args):
    """One step = one fp8_paged_mqa_logits call over b requests x ctx
    positions (default BASELINE config 1: b 32, 131,072 positions, 64
    heads x 128, pages of 64), K launches in one CUDA graph.  Per position
    the kernel reads 128 e4m3 values + a 4-B scale and writes next_n 4-B
    logits; the 554 MB cache is above L2 size, so no flush is needed."""
    import numpy as np
    import torch

    from deepseek_v4_kernel import indexer
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    B = args.batch or 32
    ctx_len = args.ctx or 131072
    H, P, nn = 64, 64, args.next_n
    pages = -(-ctx_len // P)
    nb = B * pages
    g = torch.Generator(device=device).manual_seed(0)
    arena = torch.empty(nb, P * 132, dtype=torch.uint8, device=device)
    arena[:, :P * 128] = torch.randn(nb, P * 128, generator=g, device=device).to(torch.float8_e4m3fn).view(torch.uint8)
    arena[:, P * 128:] = (torch.rand(nb, P, generator=g, device=device) * 0.1).view(torch.uint8).view(nb, P * 4)
    kv = arena.view(nb, P, 1, 132)
    q = torch.randn(B, nn, H, 128, generator=g, device=device).to(torch.float8_e4m3fn)
    w = torch.randn(B * nn, H, generator=g, device=device)
    ctx = torch.full((B,), ctx_len, dtype=torch.int32, device=device)
    if args.page_order == "random":
        bt = torch.randperm(nb, generator=g, device=device).view(B, pages).int()
    else:
        bt = torch.arange(nb, device=device, dtype=torch.int32).view(B, pages)
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    sched = indexer.get_paged_mqa_logits_metadata(ctx, P, sms)
    out = torch.empty(B * nn, ctx_len, dtype=torch.float32, device=device)

    def step():
        indexer.fp8_paged_mqa_logits(q, kv, w, ctx, bt, sched, ctx_len, True, out=out)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(device)
    cap.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(cap):
        with torch.cuda.graph(graph, stream=cap):
            for _ in range(args.steps):
                step()
    torch.cuda.current_stream(device).wait_stream(cap)
    graph.replay()
    torch.cuda.synchronize()
    clk = ClockSampler(0)
    clk.start()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0.record()
    graph.replay()
    t1.record()
    torch.cuda.synchronize()
    clocks = clk.stop()
    t_ms = t0.elapsed_time(t1) / args.steps
    positions = B * ctx_len
    alg = positions * 132 + positions * nn * 4 + q.numel() + w.numel() * 4 + bt.numel() * 4
    flops = 2.0 * nn * H * 128 * positions
    hbm_peak, tc_peak, peak_src = measured_peaks()
    ach = alg / (t_ms * 1e-3) / 1e9

    from oracle import mqa_logits_oracle as M
    c0 = time.perf_counter()
    M.fp8_paged_mqa_logits(q[:1].view(torch.uint8).cpu().numpy(), arena[bt[0].long()].cpu().numpy(),
                           w[:nn].cpu().numpy(), np.array([ctx_len]), np.arange(pages)[None, :], P, ctx_len)
    cpu_s = time.perf_counter() - c0
    line = {
        "metric": "mqa_logits_us_per_step",
        "value": round(t_ms * 1e3, 2),
        "unit": "us/step",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_ms, 5),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp8-e4m3 (fp32 accumulate)",
        "data": "synthetic (seeded N(0,1) e4m3 q and cache, uniform scales, %s page tables)" % args.page_order,
        "config": {"workload": f"mqa_logits: b{B} next_n{nn} h{H} d128 ctx{ctx_len} page{P} (config 1 contexts)",
                   "l2": f"no flush: {alg / 1e6:.0f} MB per step, above L2 size"},
        "timing": "one CUDA graph of `steps` launches, CUDA events around its replay",
        "positions_per_s": round(positions / (t_ms * 1e-3), 1),
        "roofline": {"bound": "hbm", "achieved": round(ach, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(ach / hbm_peak, 4), "traffic": None, "peak_source": peak_src,
                     "kernel": "mqa_logits_kernel", "algorithmic_bytes_per_launch": alg,
                     "algorithmic_flops_per_launch": flops,
                     "tensor_frac_of_bf16_peak": round(flops / (t_ms * 1e-3) / 1e12 / tc_peak, 4)},
        "gpu_launches": args.steps,
        "clocks": clocks,
        "cpu_baseline": {"value": round(cpu_s * B * 1e6, 1), "unit": "us/step", "cores": 1, "kind": "port",
                         "sample": f"oracle/mqa_logits_oracle.py (float64 numpy) on 1 of the {B} requests, "
                                   f"scaled to {B}"},
    }
    return line


def run_gather_rates(args):
    """Random whole-row gathers (656-B V32 records, config 1's cache
    geometry: 16,384 pages x 256 rows, 2.75 GB) into all 148 SMs with
    nothing else running, per mechanism (dsv4b_gather_rate_probe: 16-byte
    register loads, or one bulk copy per row): config 1's 65,536 rows per
    launch and a 4x larger gather; L2 flushed before every launch, CUDA
    events, median of --steps launches."""
    import statistics as st

    import torch

    from deepseek_v4_kernel import _lib
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    lib = _lib.lib
    row_bytes, nrows_cache = 656, 16384 * 256
    kv = torch.empty(nrows_cache * row_bytes, dtype=torch.uint8, device=device)
    scratch = torch.zeros(148 * 256 + 4, dtype=torch.int32, device=device)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=device)
    g = torch.Generator(device="cpu").manual_seed(7)
    hbm, _, peak_src = measured_peaks()
    stream = torch.cuda.current_stream()
    out = []
    clocks = ClockSampler(0)
    clocks.start()
    for n in (65536, 262144):
        rows = torch.randint(0, nrows_cache, (n,), generator=g, dtype=torch.int32).to(device)
        for mech, name in ((0, "register_16B_loads"), (1, "bulk_copy_per_row")):
            ts = []
            for it in range(args.warmup + args.steps):
                flush.zero_()
                a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                rc = lib.dsv4b_gather_rate_probe(mech, kv.data_ptr(), row_bytes, row_bytes, rows.data_ptr(), n,
                                                 scratch.data_ptr(), scratch.numel() * 4, stream.cuda_stream)
                e.record()
                if rc != 0:
                    raise RuntimeError(_lib.STATUS.get(rc, rc))
                torch.cuda.synchronize()
                if it >= args.warmup:
                    ts.append(a.elapsed_time(e) * 1e3)
            if int(scratch[-4].item()) != 0:
                raise RuntimeError("gather probe: a bounded wait gave up")
            us = st.median(ts)
            gbs = n * row_bytes / us / 1e3
            out.append({"mechanism": name, "rows": n, "bytes": n * row_bytes, "us": round(us, 2),
                        "GB_per_s": round(gbs, 1), "GB_per_s_per_sm": round(gbs / 148, 1),
                        "frac_of_measured_hbm": round(gbs / hbm, 3)})
    clk = clocks.stop()
    return {"metric": "random_row_gather_GBps", "unit": "GB/s", "op": "gather_rates", "row_bytes": row_bytes,
            "cache_bytes": nrows_cache * row_bytes, "hbm_peak_gbs": hbm, "peak_source": peak_src,
            "l2": "flushed before every launch (256 MiB write)", "clocks": clk, "rates": out}


def run_mma_rates(args):
    """Cycles per tcgen05.mma (kind::f16, M 128, K 16) for the decode
    kernel's operand shapes with resident shared-memory operands
    (dsv4b_mma_rate_probe): one CTA alone and one CTA per SM at once; the
    median over CTAs of each CTA's best of six chains.  The dense bf16 peak
    per SM per cycle (measured TFLOP/s / 148 SMs / the sampled clock) is the
    denominator of "frac"."""
    import torch

    from deepseek_v4_kernel import _lib
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    lib = _lib.lib
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    _, bf16_tflops, peak_src = measured_peaks()
    clocks = ClockSampler(0)
    clocks.start()
    shapes = {0: ("qk_n64_kmajor", 64), 1: ("pv_n64_mnmajor", 64), 2: ("qk_a_n128", 128), 3: ("qk_a_n256", 256),
              4: ("qk_n64_kmajor_predesc", 64), 5: ("pv_n64_mnmajor_predesc", 64)}
    out = torch.zeros(2 * sms, dtype=torch.int64, device=device)
    rows = []
    for shape, (name, n) in shapes.items():
        for ctas in (1, sms):
            rc = lib.dsv4b_mma_rate_probe(shape, ctas, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
            if rc != 0:
                raise RuntimeError(_lib.STATUS.get(rc, rc))
            torch.cuda.synchronize()
            v = out[: 2 * ctas].view(ctas, 2).cpu()
            if (v[:, 0] < 0).any():
                raise RuntimeError("mma probe: a bounded wait gave up")
            cyc = float(v[:, 0].double().median())
            mmas = int(v[0, 1])
            rows.append({"shape": name, "n": n, "ctas": ctas, "mmas": mmas, "cycles": cyc,
                         "cycles_per_mma": round(cyc / mmas, 1), "flop_per_cycle": round(2 * 128 * n * 16 * mmas / cyc)})
    clk = clocks.stop()
    # cycles do not depend on the clock; the measured cuBLAS peak is turned
    # into flop per SM cycle at the GPU's maximum SM clock
    mhz = clk.get("sm_max_mhz") or 1965.0
    peak_per_cycle = bf16_tflops * 1e12 / sms / (mhz * 1e6)
    for r in rows:
        r["frac_of_measured_peak"] = round(r["flop_per_cycle"] / peak_per_cycle, 3)
    return {"metric": "tcgen05_mma_cycles", "unit": "SM cycles per MMA", "op": "mma_rates",
            "peak_flop_per_cycle_per_sm": round(peak_per_cycle), "peak_source": peak_src,
            "peak_clock_mhz": mhz, "clocks": clk, "rates": rows}


def run_prefill(args):
    """One step = one flash_mla_sparse_fwd call (sparse prefill, bf16 KV):
    s_q 4096 query tokens x h_q 128 heads, d_qk 512, top-k 2048 over a
    65,536-row KV tensor (tensor-bound: 2.2 TFLOP per step).  --batch sets
    s_q.  The same call of vLLM 0.22's FlashMLA kernel (a compiled library,
    the op the serving engine runs next to the reference's decode) is timed
    beside it when importable, as "library"."""
    import numpy as np
    import torch

    from deepseek_v4_kernel import flash_mla_sparse_fwd
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    s_q, h_q, d, topk, s_kv = args.batch or 4096, 128, 512, 2048, 65536
    g = torch.Generator(device=device).manual_seed(0)
    q = torch.randn(s_q, h_q, d, generator=g, device=device).to(torch.bfloat16)
    kv = torch.randn(s_kv, 1, d, generator=g, device=device).to(torch.bfloat16)
    idx = torch.randint(0, s_kv, (s_q, 1, topk), generator=g, device=device, dtype=torch.int32)
    scale = 1.0 / math.sqrt(d)
    out = torch.empty(s_q, h_q, 512, dtype=torch.bfloat16, device=device)

    def timed(fn):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for a, b in evs:
            a.record()
            fn()
            b.record()
        torch.cuda.synchronize()
        return statistics.median(a.elapsed_time(b) for a, b in evs)

    clk = ClockSampler(0)
    clk.start()
    t_ms = timed(lambda: flash_mla_sparse_fwd(q, kv, idx, scale, 512, out=out))
    clocks = clk.stop()
    lib = None
    try:
        from vllm.third_party.flashmla.flash_mla_interface import flash_mla_sparse_fwd as lib_fwd
        lib_ms = timed(lambda: lib_fwd(q, kv, idx, scale, 512))
        lib = {"value": round(lib_ms * 1e3, 1), "unit": "us/step",
               "what": "vLLM 0.22 FlashMLA flash_mla_sparse_fwd (compiled library), same inputs"}
    except Exception as e:  # not importable on this box
        lib = {"unavailable": f"{type(e).__name__}: {e}"[:200]}
    flops = 2.0 * s_q * h_q * topk * (d + 512)
    hbm_peak, tc_peak, peak_src = measured_peaks()
    ach = flops / (t_ms * 1e-3) / 1e12
    from oracle import sparse_prefill_oracle as SP
    c0 = time.perf_counter()
    SP.sparse_prefill_reference(q[:1].float().cpu().numpy(), kv.float().cpu().numpy(), idx[:1].cpu().numpy(), scale)
    cpu_s = time.perf_counter() - c0
    return {
        "metric": "sparse_prefill_us_per_step",
        "value": round(t_ms * 1e3, 1),
        "unit": "us/step",
        "n_gpus": 1,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_ms, 5),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16 q and KV rows, uniform random top-k rows)",
        "config": {"workload": f"sparse prefill: s_q{s_q} h_q{h_q} d_qk{d} topk{topk} s_kv{s_kv}",
                   "l2": "no flush (the KV tensor, 67 MB, is gathered with reuse across query tokens)"},
        "tokens_per_s": round(s_q / (t_ms * 1e-3), 1),
        "roofline": {"bound": "tensor", "achieved": round(ach, 1), "peak": tc_peak, "unit": "TFLOP/s",
                     "frac": round(ach / tc_peak, 4), "traffic": None, "peak_source": peak_src,
                     "kernel": "sparse_decode_kernel (bf16 prefill layout)", "algorithmic_flops_per_launch": flops},
        "library": lib,
        "gpu_launches": 2 * args.steps,
        "clocks": clocks,
        "cpu_baseline": {"value": round(cpu_s * s_q * 1e6, 1), "unit": "us/step", "cores": 1, "kind": "port",
                         "sample": f"oracle/sparse_prefill_oracle.py (float64 numpy) on 1 of the {s_q} tokens, "
                                   f"scaled to {s_q}"},
    }


def run_sweep(args):
    """b in {1..32} x context in {8K..300K}, h_q 64, top-k
    2048; the whole step (flash_mla_with_kvcache with a reused
    FlashMLASchedMeta) captured in one CUDA graph and replayed, L2 flushed
    before every replay.  Prints one JSON line whose value is the b 32 /
    128K point and whose "sweep" lists every point."""
    import torch

    import deepseek_v4_kernel as dk
    from deepseek_v4_kernel import kvcache, ops

    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    flush = torch.empty(FLUSH_BYTES, dtype=torch.uint8, device=device)
    points = []
    for ctx in (8192, 32768, 131072, 300000):
        for b in (1, 2, 4, 8, 16, 32):
            spec = kvcache.sweep_spec(b, ctx)
            bt = kvcache.make_batch(spec, device=device)
            sched, _ = dk.get_mla_metadata()

            def step():
                return dk.flash_mla_with_kvcache(bt.q, bt.kv, None, None, 512, sched, softmax_scale=bt.sm_scale,
                                                 is_fp8_kvcache=True, indices=bt.indices, attn_sink=bt.attn_sink)

            step()
            torch.cuda.synchronize()
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                step()
            torch.cuda.current_stream().wait_stream(side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                step()
            for _ in range(args.warmup):
                flush.zero_()
                g.replay()
            ts = []
            for _ in range(args.steps):
                flush.zero_()
                a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                g.replay()
                e.record()
                torch.cuda.synchronize()
                ts.append(a.elapsed_time(e) * 1e3)
            # the same step with the scheduler inside the graph: a fresh
            # FlashMLASchedMeta, so the captured first call runs K2 as well
            sched2, _ = dk.get_mla_metadata()

            def step2():
                return dk.flash_mla_with_kvcache(bt.q, bt.kv, None, None, 512, sched2, softmax_scale=bt.sm_scale,
                                                 is_fp8_kvcache=True, indices=bt.indices, attn_sink=bt.attn_sink)

            g2 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g2):
                step2()
            for _ in range(args.warmup):
                flush.zero_()
                g2.replay()
            ts2 = []
            for _ in range(args.steps):
                flush.zero_()
                a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                g2.replay()
                e.record()
                torch.cuda.synchronize()
                ts2.append(a.elapsed_time(e) * 1e3)
            o_ = torch.empty(b, 1, 64, 512, dtype=torch.bfloat16, device=device)
            l_ = torch.empty(b, 64, 1, dtype=torch.float32, device=device)
            p = ops.build_params(bt.q, bt.kv, bt.indices, None, bt.attn_sink, None, None, None, 512, bt.sm_scale,
                                 o_, l_)
            points.append({"b": b, "ctx": ctx, "us_per_step": round(statistics.median(ts), 2),
                           "us_per_step_with_metadata": round(statistics.median(ts2), 2),
                           "cluster_size": ops.plan_cluster_size(p, ops.num_sm_parts(device, 64))})
            del g, g2, bt
            torch.cuda.empty_cache()
    head = next(pt for pt in points if pt["b"] == 32 and pt["ctx"] == 131072)
    assert dk.read_kernel_status(device) == 0, "kernel wait timeout"
    line = {
        "metric": "sparse_decode_us_per_step", "value": head["us_per_step"], "unit": "us/step", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(head["us_per_step"] / 1e3, 5),
        "higher_is_better": False, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) q / latent / RoPE, random page tables, distinct top-k)",
        "config": {"workload": "config3: CUDA-graph sweep, h_q 64, top-k 2048, V32 fp8 KV; value = b32 ctx131072",
                   "l2": "flushed before every replay (256 MiB write)", "parallelism": "single GPU"},
        "sweep": points,
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.op in ("kv_write", "mqa_logits", "prefill", "mma_rates", "gather_rates"):
        if int(os.environ.get("RANK", "0")) == 0 and args.impl == "ours":
            line = {"kv_write": run_kv_write, "mqa_logits": run_mqa_logits, "prefill": run_prefill,
                    "mma_rates": run_mma_rates, "gather_rates": run_gather_rates}[args.op](args)
            print(json.dumps(line), flush=True)
            if args.json_out:
                with open(args.json_out, "w") as f:
                    f.write(json.dumps(line) + "\n")
        return
    if args.config == 3 and args.impl == "ours":
        run_sweep(args)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    spec = workload(args.config, args.batch, args.ctx)
    if args.impl == "reference":
        if rank == 0:
            run_reference(args, spec, world, rank)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    try:
        line = run_ours(args, spec, world, rank, local_rank)
        default_run = args.config == 1 and args.batch is None and args.ctx is None and not args.no_next_rows
        if default_run:
            import torch
            torch.cuda.empty_cache()
            extra = sub_runs(args, world, rank, local_rank)
            if line is not None:
                line["other_configs" if world == 1 else "partition_config4"] = extra
                if world == 1:
                    line["next_rows"] = next_rows(args)
        if line is not None:
            print(json.dumps(line), flush=True)
            if args.json_out:
                with open(args.json_out, "w") as f:
                    f.write(json.dumps(line) + "\n")
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
