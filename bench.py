#!/usr/bin/env python
"""Benchmark of the Origami KV layout hot path on B200.

Headline (N=1): config C2 restore — Llama-3-8B-shaped KV (32 layers, 8 KV heads, head_dim
128, bf16, block 16), one request of 32768 tokens under a seeded block-table permutation.
A step restores every layer (unpack + plane merge + scatter into the paged cache) from
packed chunks resident in HBM; `value` is KV GB/s (bytes of K and V written into the
cache per second, whole job). Weak scaling at N GPUs: N requests, heads sharded by rank
(8/N heads per rank), i.e. the same bytes per GPU and no collective on the data path.

Extra keys: `pack` (the save side over the same layers), `roofline` (the restore
kernel's algorithmic bytes per launch over its CUDA-event duration vs measured HBM
copy bandwidth), `e2e` (the same restore through the public pipeline API from pinned
host chunks, H2D copies inside the timed region), `cpu_baseline` (the CPU oracle
restore on the host cores, rank 0 at N=1), `clocks`, `gpu_launches`.

`--impl reference` times the CPU implementation of the path (the oracle port of the
reference layout: the reference's own CPU packer is a stub) on the host cores.
"""
from __future__ import annotations

import argparse
import datetime
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

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

GB = 1e9


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("origami", "reference"), default="origami")
    ap.add_argument("--planes", default="byte", help="byte | bit | bf16_bits | fp16_bits")
    ap.add_argument("--layers", type=int, default=0,
                    help="layers (default: 32 for C2, as many of 32 as fit one GPU for C3, 8 for C5)")
    ap.add_argument("--config", choices=("C2", "C3", "C5", "CG", "KIVI", "ATTN"), default="C2",
                    help="workload (C2 is the headline; CG / KIVI: quantized restore paths)")
    ap.add_argument("--chunk-bytes", type=int, default=1 << 20, help="codec chunk size (min = target = max)")
    ap.add_argument("--tokens", type=int, default=0, help="C2 only: tokens per request (default 32768)")
    ap.add_argument("--attn-queries", type=int, default=1, help="ATTN only: query tokens per step (default 1)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--bundle-e2e", action="store_true",
                    help="also restore from a bundle_v1 artifact through the host codec (codec-bound)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="bound on the CPU baseline sample")
    ap.add_argument("--no-pipeline", action="store_true", help="skip the C4 exposed-restore measurement")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="C2: skip the reference's own GPU restore (its unpack kernel + index_copy_)")
    ap.add_argument("--pipeline-layers", type=int, default=8, help="C4 layers sampled by the pipeline measurement")
    return ap.parse_args()


# ----------------------------------------------------------------------------------------
# distributed plumbing
# ----------------------------------------------------------------------------------------
def init_dist(backend: str):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if backend == "nccl":
            torch.cuda.set_device(local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local))
        else:
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    elif backend == "nccl":
        torch.cuda.set_device(local)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int, device=None) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def min_over_ranks(x: float, world: int, device=None) -> float:
    return -max_over_ranks(-x, world, device)


def any_over_ranks(flag: bool, world: int, device=None) -> bool:
    return max_over_ranks(1.0 if flag else 0.0, world, device) > 0.5


# A sleep kernel of this many cycles (about 50 ms at the B200's 1965 MHz) runs ahead of
# every timed pass, so that the host has enqueued the pass before the GPU reaches it.
HEAD_START_CYCLES = int(1e8)
HEAD_START_S = 0.04


# ----------------------------------------------------------------------------------------
# clocks during the timed region
# ----------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons, power = [], [], set(), []
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, val in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"),
                                 parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm), "power_w_max": max(power) if power else None}


def measured_hbm_peak():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


# Nominal B200 HBM3e bandwidth (the survey's ~8 TB/s). Every GB/s roofline is reported
# against it as well as against the measured copy peak.
NOMINAL_HBM_GBS = 8000.0


def with_nominal(line: dict) -> dict:
    """Add `nominal_peak` / `nominal_frac` to every HBM roofline block of a result line."""
    def visit(d):
        if isinstance(d, dict):
            r = d.get("roofline")
            if isinstance(r, dict) and r.get("unit") == "GB/s" and isinstance(r.get("achieved"), (int, float)):
                r["nominal_peak"] = NOMINAL_HBM_GBS
                r["nominal_frac"] = round(r["achieved"] / NOMINAL_HBM_GBS, 4)
            for v in d.values():
                visit(v)
    visit(line)
    return line


def profiled_traffic(kernel: str, workload: str, jobs_per_launch: float):
    """DRAM read+write bytes per launch from the committed ncu captures
    (profiles/traffic.txt): lines `kernel workload jobs read write` measured on a launch
    of `jobs` jobs (the bench's own launch where it fits a capture), or older
    `kernel workload bytes_per_job` lines; scaled to the jobs one launch restores or
    packs."""
    p = REPO / "profiles" / "traffic.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if line.startswith("#") or len(parts) < 3 or parts[0] != kernel or parts[1] != workload:
            continue
        if len(parts) >= 5:
            return int(round((int(parts[3]) + int(parts[4])) * jobs_per_launch / int(parts[2])))
        return int(round(int(parts[2]) * jobs_per_launch))
    return None


# ----------------------------------------------------------------------------------------
# workload
# ----------------------------------------------------------------------------------------
class Workload:
    """One rank's share of a benchmark configuration (heads sharded by rank).

    C2  restore, weak scaling: `world` requests of 32768 tokens, 8/N heads per rank.
    C3  restore, strong scaling: 16 ragged requests (T ~ U[4096, 65536]) with interleaved
        block tables in a pool sized for 120 GB (57,220 blocks), 8/N heads per rank.
    C5  save, strong scaling: 64 requests x 8192 tokens of Qwen2-7B KV, 4/N heads per rank.
    """

    def __init__(self, config: str, rank: int, world: int, layers: int, planes_name: str, device,
                 chunk_bytes: int = 1 << 20, tokens_override: int = 0):
        import torch

        from origami_b200 import LayerFormat, plane_spec, workloads
        from origami_b200.layer import pack_layer

        self.config = config
        if config == "C2":
            cfg = workloads.C2
            tokens = [tokens_override or cfg.tokens[0]] * world
            self.scaling = "weak"
        elif config == "C3":
            cfg = workloads.c3_config()
            tokens = list(cfg.tokens)
            self.scaling = "strong"
        elif config == "C5":
            cfg = workloads.C5
            tokens = list(cfg.tokens)
            self.scaling = "strong"
        else:
            raise SystemExit(f"unknown config {config!r}")
        if cfg.heads % world:
            raise SystemExit(f"{cfg.heads} KV heads do not shard over {world} ranks")
        self.cfg = cfg
        self.layers = layers
        self.heads = cfg.heads // world
        self.head0 = rank * self.heads
        self.tokens = tokens
        self.requests = len(tokens)
        self.bs = cfg.block_size
        nbs = [(t + self.bs - 1) // self.bs for t in tokens]
        self.planes = plane_spec(planes_name, cfg.dtype)
        fmts: dict[int, LayerFormat] = {}
        for t in tokens:
            if t not in fmts:
                fmts[t] = LayerFormat(t, self.heads, cfg.head_dim, self.planes, chunk_bytes, chunk_bytes, chunk_bytes)
        self.fmts = [fmts[t] for t in tokens]
        if config == "C2":
            self.NB = sum(nbs)
            pool = workloads.permuted_block_table(self.NB, self.NB, workloads.SEED)
            starts = np.concatenate([[0], np.cumsum(nbs)])
            tables = [pool[int(a):int(b)] for a, b in zip(starts[:-1], starts[1:])]
        else:
            self.NB = workloads.c3_pool_blocks(cfg) if config == "C3" else sum(nbs)
            tables = workloads.interleaved_block_tables(tokens, self.bs, self.NB, workloads.SEED + 5)
        self.block_ids = [t.to(device) for t in tables]
        # Requests with the same token count share a format; each format group keeps its
        # (layer, request) jobs in one packed arena at a uniform 16-byte-multiple stride,
        # so a step is one batched call per group.
        from origami_b200.layer import alloc_jobs_packed, job_stride

        self.groups = []  # (fmt, [(layer, r)], arena)
        by_t: dict[int, list[int]] = {}
        for r, t in enumerate(tokens):
            by_t.setdefault(t, []).append(r)
        self.packed = [[None] * self.requests for _ in range(layers)]
        for t, reqs in by_t.items():
            fmt = fmts[t]
            jobs = [(layer, r) for layer in range(layers) for r in reqs]
            arena = alloc_jobs_packed(fmt, len(jobs), device)
            stride = job_stride(fmt)
            for j, (layer, r) in enumerate(jobs):
                self.packed[layer][r] = arena[j * stride:j * stride + fmt.packed_bytes]
            self.groups.append((fmt, jobs, arena))
        # C3's pool is most of the GPU: instead of a copy of every cache, a restore is checked
        # by packing the restored cache again (pack o restore = identity on the request rows)
        self.keep_orig = config != "C3"
        self.caches, self.orig = [], []
        for layer in range(layers):
            cache = torch.zeros((2, self.NB, self.bs, self.heads, cfg.head_dim), dtype=cfg.dtype, device=device)
            for r in range(self.requests):
                kv = workloads.kv_values(tokens[r], cfg.heads, cfg.head_dim, cfg.dtype,
                                         seed=workloads.SEED + 1000 * layer + r, v_std=cfg.v_std,
                                         device=device)[:, :, self.head0:self.head0 + self.heads]
                workloads.scatter_into_cache(cache, kv.contiguous(), self.block_ids[r])
                pack_layer(cache, self.block_ids[r], self.fmts[r], out=self.packed[layer][r])
            if self.keep_orig:
                self.orig.append(cache.clone())
            self.caches.append(cache)
        torch.cuda.synchronize()

    def kernel_launches(self) -> int:
        """Kernels one batched pass launches (128 jobs per persistent TMA launch; the
        generic tile path launches once per job)."""
        from origami_b200.layer import fused_kernel_name

        n = 0
        for fmt, jobs, _ in self.groups:
            n += len(jobs) if fused_kernel_name(fmt).endswith("tiles") else (len(jobs) + 127) // 128
        return n

    @property
    def units_per_step(self) -> int:
        return self.layers * self.requests

    @property
    def kv_bytes_per_step(self) -> int:
        return self.layers * sum(f.kv_bytes for f in self.fmts)

    @property
    def packed_bytes_per_step(self) -> int:
        return self.layers * sum(f.packed_bytes for f in self.fmts)

    @property
    def max_packed(self) -> int:
        return max(f.packed_bytes for f in self.fmts)

    def verify(self) -> bool:
        import torch

        if self.keep_orig:
            return all(torch.equal(c.view(torch.int16), o.view(torch.int16)) for c, o in zip(self.caches, self.orig))
        from origami_b200.layer import pack_layers

        for fmt, jobs, arena in self.groups:
            again = torch.empty_like(arena)
            pack_layers([self.caches[layer] for layer, _ in jobs], [self.block_ids[r] for _, r in jobs], fmt, again)
            if not torch.equal(again, arena):
                return False
            del again
        return True

    @staticmethod
    def layers_that_fit(config: str, world: int, device) -> int:
        """C3 at as many of its 32 layers as one GPU holds (pool + packed layers, with room
        for the verification buffer and temporaries)."""
        import torch

        from origami_b200 import workloads

        cfg = workloads.c3_config()
        heads = cfg.heads // world
        per_token = 2 * heads * cfg.head_dim * 2
        per_layer = workloads.c3_pool_blocks(cfg) * cfg.block_size * per_token + sum(cfg.tokens) * per_token
        free, _ = torch.cuda.mem_get_info(device)
        return max(1, min(32, int((free - 16 * 2**30) // per_layer)))


def run_origami(args, rank, world, local):
    import torch

    from origami_b200.layer import fused_kernel_name, pack_layers, restore_layers

    device = torch.device("cuda", local)
    layers = args.layers if args.layers else {"C2": 32, "C5": 8}.get(args.config) or Workload.layers_that_fit(
        args.config, world, device)
    if args.config == "C3" and not args.layers:
        layers = int(min_over_ranks(layers, world, device))
    wl = Workload(args.config, rank, world, layers, args.planes, device, args.chunk_bytes, args.tokens)
    stream = torch.cuda.current_stream(device)
    err = torch.zeros(1, dtype=torch.int32, device=device)

    def zero_caches():
        # the originals are kept; zero the caches so the timed restores rebuild them
        for c in wl.caches:
            c.zero_()

    def restore_step(events=None):
        for fmt, jobs, arena in wl.groups:
            if events is not None:
                events.append((torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)))
                events[-1][0].record(stream)
            restore_layers(arena, fmt, [wl.caches[layer] for layer, _ in jobs], [wl.block_ids[r] for _, r in jobs],
                           error_count=err)
            if events is not None:
                events[-1][1].record(stream)

    def pack_step(events=None):
        for fmt, jobs, arena in wl.groups:
            if events is not None:
                events.append((torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)))
                events[-1][0].record(stream)
            pack_layers([wl.caches[layer] for layer, _ in jobs], [wl.block_ids[r] for _, r in jobs], fmt, arena,
                        error_count=err)
            if events is not None:
                events[-1][1].record(stream)

    host_us_per_call = []

    def timed(step_fn):
        """Per-launch CUDA-event durations from an eager pass, then the step time from
        CUDA-graph replays of the same step (no host launch overhead in `value`).

        Both passes start behind a sleep kernel, so the GPU is still busy while the host
        enqueues and the events bracket device work only; a pass whose host enqueue
        outlasted that head start (a stalled host thread, e.g. while nvidia-smi polls the
        driver) is measured again."""
        for _ in range(args.warmup):
            step_fn()
        torch.cuda.synchronize(device)
        for _attempt in range(4):
            launch_events = []
            torch.cuda._sleep(HEAD_START_CYCLES)
            t_host = time.perf_counter()
            step_fn(launch_events)
            host_s = time.perf_counter() - t_host
            torch.cuda.synchronize(device)
            if host_s < HEAD_START_S:
                break
        launch_ms_sum = sum(a.elapsed_time(b) for a, b in launch_events)
        host_us_per_call.append(host_s * 1e6 / max(1, len(launch_events)))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step_fn()
        for _ in range(args.warmup):
            graph.replay()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for _attempt in range(4):
            barrier(world)
            torch.cuda.synchronize(device)
            torch.cuda._sleep(HEAD_START_CYCLES)
            t_host = time.perf_counter()
            t0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            t1.record(stream)
            host_s = time.perf_counter() - t_host
            torch.cuda.synchronize(device)
            # every rank takes the same number of attempts
            if not any_over_ranks(host_s >= HEAD_START_S, world, device):
                break
        barrier(world)
        ms = t0.elapsed_time(t1)
        del graph
        return max_over_ranks(ms, world, device), launch_ms_sum, wl.kernel_launches()

    primary_pack = args.config == "C5"
    clocks = ClockSampler(local)
    clocks.start()
    if primary_pack:
        pack_ms, pack_sum, launches = timed(pack_step)
        clock_info = clocks.stop()
        ok = wl.verify() and int(err.item()) == 0
        zero_caches()
        restore_ms, restore_sum, _ = timed(restore_step)
    else:
        zero_caches()
        restore_ms, restore_sum, launches = timed(restore_step)
        clock_info = clocks.stop()
        ok = wl.verify() and int(err.item()) == 0
        pack_ms, pack_sum, _ = timed(pack_step)
    ok = ok and wl.verify() and int(err.item()) == 0

    steps = args.steps
    peak, peak_kind = measured_hbm_peak()
    alg_step = wl.packed_bytes_per_step + wl.kv_bytes_per_step  # per rank, one pass
    restore_gbs = wl.kv_bytes_per_step * world * steps / (restore_ms / 1e3) / GB
    pack_gbs = wl.kv_bytes_per_step * world * steps / (pack_ms / 1e3) / GB
    achieved_restore = alg_step / (restore_sum / 1e3) / GB
    achieved_pack = alg_step / (pack_sum / 1e3) / GB
    kinds = {fused_kernel_name(f, True) for f in wl.fmts}
    k_restore = "/".join(sorted(kinds))
    k_pack = "/".join(sorted({fused_kernel_name(f, False) for f in wl.fmts}))
    jobs_per_launch = sum(len(jobs) for _, jobs, _ in wl.groups) / launches
    workload_name = (f"C2_restore_T{wl.tokens[0]}_H{wl.heads}_D{wl.cfg.head_dim}_{wl.planes.name}"
                     if args.config == "C2" and args.chunk_bytes == 1 << 20 else None)
    roof_restore = {"kernel": k_restore, "bound": "hbm", "achieved": round(achieved_restore, 1), "peak": peak,
                    "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved_restore / peak, 4),
                    "traffic": profiled_traffic(k_restore, workload_name, jobs_per_launch) if workload_name else None,
                    "algorithmic_bytes_per_launch": alg_step // launches,
                    "launch_ms": round(restore_sum / launches, 5),
                    "host_us_per_call": round(host_us_per_call[0 if not primary_pack else 1], 1)}
    roof_pack = {"kernel": k_pack, "bound": "hbm", "achieved": round(achieved_pack, 1), "peak": peak,
                 "peak_kind": peak_kind, "unit": "GB/s", "frac": round(achieved_pack / peak, 4),
                 "traffic": profiled_traffic(k_pack, workload_name, jobs_per_launch) if workload_name else None,
                 "algorithmic_bytes_per_launch": alg_step // launches,
                 "launch_ms": round(pack_sum / launches, 5)}

    pipeline_info = None
    if not args.no_pipeline and args.config == "C2":
        pipeline_info = run_pipeline_c4(args, device, world)
        ok = ok and pipeline_info.pop("ok")

    barrier(world)  # every rank probes at once: the share of shared host links its copies see
    pcie = measure_pcie(device)
    if pipeline_info is not None:
        pipeline_info["pcie_h2d_frac"] = round(pipeline_info["pcie_h2d_gbs"] / pcie["h2d_gbs"], 3)
    e2e = None
    if not args.no_e2e:
        e2e = run_e2e_save(args, wl, device, world) if primary_pack else run_e2e(args, wl, device, world)
        ok = ok and e2e.pop("ok")
        link = "d2h" if primary_pack else "h2d"
        if f"pcie_{link}_gbs" in e2e:
            e2e[f"pcie_{link}_frac"] = round(e2e[f"pcie_{link}_gbs"] / pcie[f"{link}_gbs"], 3)
    reference_gpu = None
    if args.config == "C2" and not primary_pack and not args.no_reference_gpu and wl.keep_orig:
        reference_gpu = run_reference_gpu_restore(args, wl, device)
    bundle_info = None
    if args.bundle_e2e and not primary_pack:
        bundle_info = run_bundle_e2e(args, wl, device, world)
        ok = ok and bundle_info.pop("ok")

    cfg_desc = {
        "C2": "C2: Llama-3-8B-shaped KV restore, 32768-token request per GPU, seeded block-table permutation",
        "C3": "C3: batched ragged restore, 16 requests T~U[4096,65536], interleaved block tables, 120 GB pool",
        "C5": "C5: save-path stress, Qwen2-7B KV, 64 requests x 8192 tokens, gather+plane split+bitpack",
    }[args.config]
    if primary_pack:
        metric = "KV pack GB/s (gather + plane split + bitpack), whole job"
        value, ms_step, roof = pack_gbs, pack_ms / steps, roof_pack
        secondary = {"restore": {"value": round(restore_gbs, 1), "unit": "GB/s",
                                 "ms_per_step": round(restore_ms / steps, 4), "roofline": roof_restore}}
    else:
        metric = "KV restore GB/s (unpack + plane merge + paged scatter), whole job"
        value, ms_step, roof = restore_gbs, restore_ms / steps, roof_restore
        secondary = {"pack": {"metric": "KV pack GB/s (gather + plane split + bitpack), whole job",
                              "value": round(pack_gbs, 1), "unit": "GB/s", "ms_per_step": round(pack_ms / steps, 4),
                              "roofline": roof_pack}}
    result = {
        "metric": metric,
        "value": round(value, 1),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 4),
        "higher_is_better": True,
        "scaling": wl.scaling,
        "vs_baseline": None,
        "dtype": "u16 (bf16/fp16 bit patterns)",
        "data": "synthetic (seeded N(0,1) x log-uniform channel scales, K outliers x20, V N(0,0.5))",
        "config": {
            "workload": cfg_desc,
            "layers": wl.layers, "requests": wl.requests, "tokens_total": int(sum(wl.tokens)),
            "kv_heads": wl.cfg.heads, "heads_per_rank": wl.heads, "head_dim": wl.cfg.head_dim,
            "block_size": wl.bs, "cache_dtype": str(wl.cfg.dtype).replace("torch.", ""), "planes": wl.planes.name,
            "chunk_bytes": args.chunk_bytes, "parallelism": f"kv-head shard x{world}, no collective",
            "l2": "inputs larger than L2 (%.1f GiB packed + %.1f GiB cache per rank per step)" % (
                wl.packed_bytes_per_step / 2**30, wl.kv_bytes_per_step / 2**30),
        },
        "roofline": roof,
        **secondary,
        "gpu_launches": launches * steps,
        "clocks": clock_info,
        "verified": bool(ok),
    }
    result["pcie"] = pcie
    if e2e is not None:
        result["e2e"] = e2e
    if pipeline_info is not None:
        result["pipeline"] = pipeline_info
    if reference_gpu is not None:
        result["reference_gpu"] = reference_gpu
    if bundle_info is not None:
        result["bundle_e2e"] = bundle_info
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        result["cpu_baseline"], result["cpu_baselines"] = cpu_baseline(args, wl)
        result["host"] = host_cpu()
    if rank == 0:
        print(json.dumps(with_nominal(result)), flush=True)
    return 0 if ok else 1


def measure_pcie(device) -> dict:
    """Pinned host <-> device copy peak of this box, in this run: 256 MiB cudaMemcpyAsync
    each way on one stream, best of 10 after 3 warm-ups (the roofline of the e2e and
    pipeline numbers). With several ranks the caller starts every rank's probe together,
    so the figure is a rank's share of host links the ranks share, as in their e2e copies."""
    import torch

    n = 256 << 20
    host = torch.empty((n,), dtype=torch.uint8, pin_memory=True)
    dev = torch.empty((n,), dtype=torch.uint8, device=device)
    stream = torch.cuda.Stream(device)
    out = {}
    for name, fn in (("h2d_gbs", lambda: dev.copy_(host, non_blocking=True)),
                     ("d2h_gbs", lambda: host.copy_(dev, non_blocking=True))):
        best = float("inf")
        with torch.cuda.stream(stream):
            for i in range(13):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                fn()
                b.record(stream)
                b.synchronize()
                if i >= 3:
                    best = min(best, a.elapsed_time(b))
        out[name] = round(n / (best / 1e3) / GB, 2)
    out["how"] = "pinned cudaMemcpyAsync of 256 MiB, best of 10"
    return out


def run_reference_gpu_restore(args, wl, device) -> dict | None:
    """The reference's own GPU restore of the same layers, inputs resident in HBM: each
    layer's raw-bytes symbols (the gathered blocks, RawBytesTensorAdapter,
    quantization/raw_tensor.py:100-122) in 1 MiB chunks go through the reference's
    unpack_canonical_storage_chunks_cuda (lossless/native_gpu.py:113-146 -> csrc/origami/
    bitpack_layout_cuda.cpp:316-400 -> .cu:91-128, built from the reference's sources into
    oracle/_ref), the dequantize view (raw_tensor.py:125-157) and the index_copy_ block
    scatter of copy_kv_to_hbm (benchmark_utils.py:434-444, 465-532)."""
    import torch

    sys.path.insert(0, str(REPO / "tests" / "golden"))
    try:
        from make_ref_vectors import load_reference_extension

        ext = load_reference_extension()
    except Exception:  # noqa: BLE001
        ext = None
    if ext is None:
        return None
    layers = []
    for layer in range(wl.layers):
        for r in range(wl.requests):
            ids = wl.block_ids[r]
            gathered = torch.index_select(wl.orig[layer], 1, ids)  # the saved layer's blocks
            flat = gathered.reshape(-1).view(torch.uint8).contiguous()
            n = flat.numel()
            bounds = list(range(0, n, 1 << 20)) + [n]
            specs = torch.tensor([[0, 1, a, b, 0, 1] for a, b in zip(bounds[:-1], bounds[1:])], dtype=torch.int64,
                                 device=device)
            layers.append((layer, r, flat, torch.tensor(bounds, dtype=torch.int64, device=device),
                           torch.full((len(bounds) - 1,), 8, dtype=torch.int64, device=device), specs,
                           torch.tensor([1, 1, n], dtype=torch.int64), list(gathered.shape)))
    axes = torch.tensor([0, 1, 2, -1], dtype=torch.int64)
    for c in wl.caches:
        c.zero_()

    def step():
        for layer, r, flat, offs, bits, specs, shape, vshape in layers:
            out = ext.unpack_canonical_storage_chunks_cuda(flat, offs, bits, shape, axes, 1, 1, int(shape[2]), specs)
            value = out.view(wl.cfg.dtype).view(vshape)
            wl.caches[layer].index_copy_(1, wl.block_ids[r], value)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    torch.cuda.synchronize(device)
    ms = t0.elapsed_time(t1)
    ok = all(torch.equal(c.view(torch.int16), o.view(torch.int16)) for c, o in zip(wl.caches, wl.orig))
    del layers
    return {"value": round(wl.kv_bytes_per_step * args.steps / (ms / 1e3) / GB, 1), "unit": "GB/s",
            "ms_per_step": round(ms / args.steps, 3), "verified": ok,
            "path": "reference unpack_canonical_storage_chunks_cuda on each layer's raw-bytes chunks (1 MiB, 8 bits) "
                    "+ dequantize view + index_copy_ block scatter, inputs resident in HBM"}


def run_e2e(args, wl, device, world):
    """Restore from pinned host chunks through RestorePipeline; H2D inside the timed region."""
    import torch

    from origami_b200.pipeline import RestorePipeline

    host = [[torch.empty((wl.fmts[r].packed_bytes,), dtype=torch.uint8, pin_memory=True) for r in range(wl.requests)]
            for _ in range(wl.layers)]
    for layer in range(wl.layers):
        for r in range(wl.requests):
            host[layer][r].copy_(wl.packed[layer][r], non_blocking=True)
    torch.cuda.synchronize(device)
    for c in wl.caches:
        c.zero_()
    pipe = RestorePipeline(device, wl.max_packed, slots=3)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    err_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)

    def step():
        ev = None
        for layer in range(wl.layers):
            for r in range(wl.requests):
                ev = pipe.enqueue(host[layer][r], wl.fmts[r], wl.caches[layer], wl.block_ids[r], error_count=err)
        pipe.restore_stream.wait_event(ev)
        with torch.cuda.stream(pipe.restore_stream):
            err_host.copy_(err, non_blocking=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    barrier(world)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(pipe.copy_stream)
    launches0 = pipe.launches
    for _ in range(args.steps):
        step()
    t1.record(pipe.restore_stream)
    torch.cuda.synchronize(device)
    barrier(world)
    ms = max_over_ranks(t0.elapsed_time(t1), world, device)
    ok = wl.verify() and int(err_host.item()) == 0
    value = wl.kv_bytes_per_step * world * args.steps / (ms / 1e3) / GB
    h2d = wl.packed_bytes_per_step
    return {"value": round(value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
            "ms_per_step": round(ms / args.steps, 3), "pcie_h2d_gbs": round(h2d * args.steps / (ms / 1e3) / GB, 2),
            "gpu_launches": pipe.launches - launches0, "pipeline": "pinned host -> copy stream -> 3-slot ring -> "
            "restore stream, per-layer events", "ok": ok}


def run_bundle_e2e(args, wl, device, world):
    """Restore from a bundle_v1 artifact: the packed layers are deflated once into a bundle
    (native codec, zlib level 1, on every host thread); each step then decodes every
    layer out of the ORIGQZ1 file straight into the pipeline's pinned staging and
    restores it (codec -> H2D -> fused restore). Timed on the restore stream from an
    idle GPU, so the host decode of the first layer is inside the region."""
    import shutil
    import tempfile

    import torch

    from origami_b200.bundle import BundleStore
    from origami_b200.pipeline import RestorePipeline

    root = Path(tempfile.mkdtemp(prefix="origami_bundle_", dir="/dev/shm" if Path("/dev/shm").is_dir() else None))
    try:
        store = BundleStore(root)
        names = {}
        for r in range(wl.requests):
            layers = []
            for layer in range(wl.layers):
                h = torch.empty((wl.fmts[r].packed_bytes,), dtype=torch.uint8, pin_memory=True)
                h.copy_(wl.packed[layer][r])
                names[(layer, r)] = f"model.layers.{layer}.self_attn.attn"
                layers.append((names[(layer, r)], wl.fmts[r], h))
            store.put_packed_layers(cache_key=f"req{r}", request_id=f"req{r}", token_count=wl.tokens[r],
                                    layers=layers, dtype=wl.cfg.dtype)
        bundles = [store.open_qat_bundle(f"req{r}") for r in range(wl.requests)]
        comp = sum(int(b.records["comp_len"].sum()) for b in bundles)
        raw = sum(int(b.raw_bytes) for b in bundles)
        for c in wl.caches:
            c.zero_()
        pipe = RestorePipeline(device, wl.max_packed, slots=3)
        err = torch.zeros(1, dtype=torch.int32, device=device)
        err_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)

        def step():
            ev = None
            for layer in range(wl.layers):
                for r in range(wl.requests):
                    ev = pipe.enqueue_from_bundle(bundles[r], names[(layer, r)], wl.fmts[r], wl.caches[layer],
                                                  wl.block_ids[r], error_count=err)
            pipe.restore_stream.wait_event(ev)
            with torch.cuda.stream(pipe.restore_stream):
                err_host.copy_(err, non_blocking=True)

        steps = max(1, min(args.steps, 3))
        step()
        torch.cuda.synchronize(device)
        barrier(world)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(pipe.restore_stream)
        for _ in range(steps):
            step()
        t1.record(pipe.restore_stream)
        torch.cuda.synchronize(device)
        barrier(world)
        ms = max_over_ranks(t0.elapsed_time(t1), world, device)
        ok = wl.verify() and int(err_host.item()) == 0
        return {"value": round(wl.kv_bytes_per_step * world * steps / (ms / 1e3) / GB, 2), "unit": "GB/s",
                "steps": steps, "ms_per_step": round(ms / steps, 2), "compressed_bytes_per_step": comp,
                "compression_ratio": round(comp / raw, 4), "host_threads": os.cpu_count(),
                "codec": "zlib level 1 raw deflate (native, all host threads)",
                "pipeline": "ORIGQZ1 file (page cache) -> inflate into pinned staging -> copy stream -> "
                            "restore stream", "ok": ok}
    finally:
        shutil.rmtree(root, ignore_errors=True)


def run_e2e_save(args, wl, device, world):
    """Save into pinned host chunks through SavePipeline (pack on a save stream, D2H on a
    copy stream); the block tables go H2D every step; D2H inside the timed region."""
    import torch

    from origami_b200.pipeline import SavePipeline

    host = [[torch.empty((wl.fmts[r].packed_bytes,), dtype=torch.uint8, pin_memory=True) for r in range(wl.requests)]
            for _ in range(wl.layers)]
    ids_host = [t.cpu().pin_memory() for t in wl.block_ids]
    ids_dev = [torch.empty_like(t) for t in wl.block_ids]
    pipe = SavePipeline(device, wl.max_packed, slots=3)
    err = torch.zeros(1, dtype=torch.int32, device=device)

    def step():
        done = None
        with torch.cuda.stream(pipe.save_stream):
            for h, d in zip(ids_host, ids_dev):
                d.copy_(h, non_blocking=True)
        for layer in range(wl.layers):
            for r in range(wl.requests):
                done = pipe.enqueue(wl.caches[layer], ids_dev[r], wl.fmts[r], host[layer][r], error_count=err)
        pipe.copy_stream.wait_event(done)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    barrier(world)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(pipe.save_stream)
    launches0 = pipe.launches
    for _ in range(args.steps):
        step()
    t1.record(pipe.copy_stream)
    torch.cuda.synchronize(device)
    barrier(world)
    ms = max_over_ranks(t0.elapsed_time(t1), world, device)
    ok = all(torch.equal(host[layer][r][: wl.fmts[r].packed_bytes], wl.packed[layer][r].cpu())
             for layer in range(wl.layers) for r in range(wl.requests)) and int(err.item()) == 0
    value = wl.kv_bytes_per_step * world * args.steps / (ms / 1e3) / GB
    d2h = wl.packed_bytes_per_step
    return {"value": round(value, 1), "unit": "GB/s", "h2d_bytes_per_step": sum(t.numel() * 8 for t in ids_host),
            "d2h_bytes_per_step": d2h, "ms_per_step": round(ms / args.steps, 3),
            "pcie_d2h_gbs": round(d2h * args.steps / (ms / 1e3) / GB, 2),
            "gpu_launches": pipe.launches - launches0,
            "pipeline": "save stream pack -> 3-slot ring -> copy stream D2H into pinned host", "ok": ok}


def run_pipeline_c4(args, device, world):
    """Exposed restore time per layer for one rank of C4 (Llama-3-70B KV at TP=8: 1 KV head,
    4 x 131072 tokens, fp16, block 32): per-layer pinned H2D + restore through
    RestorePipeline overlapped with a bf16 8192^3 prefill GEMM per layer on the model's
    stream, which waits on each layer's event (the wait_for_layer_load contract)."""
    import torch

    from origami_b200 import BYTE_PLANES, LayerFormat, workloads
    from origami_b200.layer import pack_layer
    from origami_b200.pipeline import RestorePipeline

    cfg = workloads.C4
    L = max(2, args.pipeline_layers)
    heads, T, bs, R = 1, cfg.tokens[0], cfg.block_size, len(cfg.tokens)
    nb = T // bs
    fmt = LayerFormat(T, heads, cfg.head_dim, BYTE_PLANES)
    pool = workloads.permuted_block_table(nb * R, nb * R, workloads.SEED + 4)
    ids = [pool[r * nb:(r + 1) * nb].to(device) for r in range(R)]
    caches, hosts, origs = [], [], []
    for layer in range(L):
        cache = torch.empty((2, nb * R, bs, heads, cfg.head_dim), dtype=cfg.dtype, device=device)
        row = []
        for r in range(R):
            kv = workloads.kv_values(T, heads, cfg.head_dim, cfg.dtype, seed=workloads.SEED + 77 * layer + r,
                                     v_std=cfg.v_std, device=device)
            workloads.scatter_into_cache(cache, kv, ids[r])
            h = torch.empty((fmt.packed_bytes,), dtype=torch.uint8, pin_memory=True)
            h.copy_(pack_layer(cache, ids[r], fmt))
            row.append(h)
        origs.append(cache.clone())
        caches.append(cache)
        hosts.append(row)
    torch.cuda.synchronize(device)
    a = torch.randn((8192, 8192), dtype=torch.bfloat16, device=device)
    b = torch.randn((8192, 8192), dtype=torch.bfloat16, device=device)
    c = torch.empty((8192, 8192), dtype=torch.bfloat16, device=device)
    model = torch.cuda.Stream(device)
    pipe = RestorePipeline(device, fmt.packed_bytes, slots=3)
    err = torch.zeros(1, dtype=torch.int32, device=device)

    def timed(fn):
        torch.cuda.synchronize(device)
        barrier(world)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(model)
        fn()
        t1.record(model)
        torch.cuda.synchronize(device)
        return max_over_ranks(t0.elapsed_time(t1), world, device)

    def compute_only():
        with torch.cuda.stream(model):
            for _ in range(L):
                torch.matmul(a, b, out=c)

    def restore_only():
        ev = None
        pipe.copy_stream.wait_stream(model)
        for layer in range(L):
            for r in range(R):
                ev = pipe.enqueue(hosts[layer][r], fmt, caches[layer], ids[r], error_count=err)
        model.wait_event(ev)

    def pipelined():
        pipe.copy_stream.wait_stream(model)
        evs = [[pipe.enqueue(hosts[layer][r], fmt, caches[layer], ids[r], error_count=err) for r in range(R)]
               for layer in range(L)]
        with torch.cuda.stream(model):
            for layer in range(L):
                for ev in evs[layer]:
                    model.wait_event(ev)  # wait_for_layer_load(layer)
                torch.matmul(a, b, out=c)

    def unpipelined():
        from origami_b200.layer import restore_layer

        slot = pipe.slots[0].buf
        with torch.cuda.stream(model):
            for layer in range(L):
                for r in range(R):
                    slot[: fmt.packed_bytes].copy_(hosts[layer][r], non_blocking=True)
                    restore_layer(slot[: fmt.packed_bytes], fmt, caches[layer], ids[r], stream=model, error_count=err)

    for fn in (compute_only, restore_only, pipelined, unpipelined):  # warm-up
        fn()
    for cc in caches:
        cc.zero_()
    t_compute = timed(compute_only)
    t_restore = timed(restore_only)
    t_unpipe = timed(unpipelined)
    for cc in caches:
        cc.zero_()
    t_pipe = timed(pipelined)
    ok = all(torch.equal(x.view(torch.int16), y.view(torch.int16)) for x, y in zip(caches, origs)) and int(err.item()) == 0
    exposed = (t_pipe - t_compute) / L
    unpipe_per_layer = t_unpipe / L
    h2d_bytes = L * R * fmt.packed_bytes
    # Lower bound of the pipelined time: layer L's GEMM needs layer L restored, so at best
    # the restores run back to back and only the last layer's GEMM follows them (or the
    # GEMMs run back to back behind the first restore, when compute is the longer chain).
    t_best = max(t_restore + t_compute / L, t_compute + t_restore / L)
    return {
        "workload": f"C4 one rank at TP=8: {L} of 80 layers, 1 KV head, {R} x {T} tokens, fp16, block {bs}, "
                    "byte planes; per layer a bf16 8192x8192x8192 GEMM on the model stream",
        "exposed_restore_ms_per_layer": round(exposed, 4),
        "unpipelined_restore_ms_per_layer": round(unpipe_per_layer, 4),
        "exposed_frac_of_unpipelined": round(exposed / unpipe_per_layer, 4),
        "compute_only_ms_per_layer": round(t_compute / L, 4),
        "restore_only_ms_per_layer": round(t_restore / L, 4),
        "pipelined_ms_per_layer": round(t_pipe / L, 4),
        "pcie_h2d_gbs": round(h2d_bytes / (t_restore / 1e3) / GB, 2),
        "overlap_frac_of_ideal": round((t_compute + t_restore - t_pipe) / min(t_compute, t_restore), 4),
        # the overlap the layer dependency allows, and the share of it achieved
        "overlap_frac_of_achievable": round((t_compute + t_restore - t_pipe) / (t_compute + t_restore - t_best), 4),
        # floor of exposed_frac_of_unpipelined set by PCIe: a layer's H2D cannot hide behind
        # less compute than it takes ((t_restore - t_compute) / t_unpipelined per layer)
        "exposed_floor_frac": round(max(0.0, t_restore - t_compute) / t_unpipe, 4),
        "bytes_per_layer": R * fmt.packed_bytes,
        "ok": ok,
    }


def host_cpu() -> dict:
    """The host the CPU baselines ran on: threads, CPU model and NUMA nodes."""
    model = None
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                model = ln.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    nodes = len([n for n in Path("/sys/devices/system/node").glob("node[0-9]*")]) or None
    return {"nproc": os.cpu_count(), "cpu_model": model, "numa_nodes": nodes}


def cpu_baseline(args, wl):
    """CPU baselines on the host cores over bounded samples of the config's layers
    (request 0), each about args.cpu_seconds: the oracle port of the layout (restore; pack
    for C5) on all host threads (the headline entry) and on one thread, and for restores
    the reference connector's own CPU lossless restore of the raw-bytes layout (zlib level 1
    chunks -> cat -> view -> index_copy_, oracle/ref_lossless.py)."""
    import torch

    sys.path.insert(0, str(REPO / "oracle"))
    import oracle

    fmt, T = wl.fmts[0], wl.tokens[0]
    ids = wl.block_ids[0].cpu().numpy()
    pack_dir = args.config == "C5"
    layers = min(wl.layers, 8)
    if pack_dir:
        caches = [o.cpu().view(torch.int16).numpy().view(np.uint16) for o in wl.orig[:layers]]
    else:
        packed = [wl.packed[layer][0].cpu().numpy() for layer in range(layers)]
        cache = np.zeros((2, wl.NB, wl.bs, wl.heads, wl.cfg.head_dim), dtype=np.uint16)
    what = "pack_layer" if pack_dir else "restore_layer"

    def port(threads: int) -> dict:
        oracle.set_threads(threads)
        done = 0
        t0 = time.perf_counter()
        while done < layers:
            if pack_dir:
                oracle.pack_layer(caches[done], 0, ids, T, wl.planes.shifts, wl.planes.bits, fmt.specs)
            else:
                oracle.restore_layer(packed[done], wl.planes.shifts, wl.planes.bits, fmt.specs, cache, 0, ids, T)
            done += 1
            if time.perf_counter() - t0 > args.cpu_seconds:
                break
        dt = time.perf_counter() - t0
        return {"value": round(done * fmt.kv_bytes / dt / GB, 3), "unit": "GB/s", "cores": oracle.max_threads(),
                "kind": "port", "sample": f"{done} {args.config} layers x 1 request ({done * fmt.kv_bytes / 2**20:.0f} "
                f"MiB KV), oracle {what}, {dt:.1f} s"}

    full = port(os.cpu_count() or 1)
    entries = [full, port(1)]
    oracle.set_threads(os.cpu_count() or 1)
    if not pack_dir:
        import ref_lossless

        # request 0's blocks of each sampled layer (the restored, verified cache) saved the
        # reference's way; the restore scatters them over a pool of the request's size in
        # a seeded block order (the scatter pattern, without a 120 GB host pool for C3)
        nb = len(ids)
        ids_list = [int(i) for i in np.random.default_rng(5).permutation(nb)]
        host_cache = torch.zeros((2, nb, wl.bs, wl.heads, wl.cfg.head_dim), dtype=wl.cfg.dtype)
        saved = [ref_lossless.save_gathered(torch.index_select(wl.caches[layer], 1, wl.block_ids[0]).cpu())
                 for layer in range(layers)]
        done = 0
        t0 = time.perf_counter()
        while done < layers:
            ref_lossless.restore_layer(saved[done], host_cache, ids_list)
            done += 1
            if time.perf_counter() - t0 > args.cpu_seconds:
                break
        dt = time.perf_counter() - t0
        entries.append({"value": round(done * fmt.kv_bytes / dt / GB, 3), "unit": "GB/s", "cores": 1,
                        "kind": "reference-restated",
                        "sample": f"{done} {args.config} layers x 1 request ({done * fmt.kv_bytes / 2**20:.0f} MiB KV), "
                                  "the reference's CPU lossless restore of the raw-bytes layout: zlib level-1 1 MiB "
                                  f"chunks -> torch.cat -> view -> index_copy_ (one Python thread), {dt:.1f} s"})
    return full, entries


def run_reference(args, rank, world):
    """CPU implementation of the path on the host cores (rank 0 only): the oracle port of
    the reference layout on one request of the config per step (restore; pack for C5)."""
    if rank != 0:
        return 0
    import torch

    sys.path.insert(0, str(REPO / "oracle"))
    import oracle
    from origami_b200 import LayerFormat, plane_spec, workloads

    cfg = {"C2": workloads.C2, "C3": workloads.c3_config(), "C5": workloads.C5}[args.config]
    heads = cfg.heads // world
    T, bs = cfg.tokens[0], cfg.block_size
    nb = (T + bs - 1) // bs
    planes = plane_spec(args.planes, cfg.dtype)
    cb = args.chunk_bytes
    fmt = LayerFormat(T, heads, cfg.head_dim, planes, cb, cb, cb)
    threads = os.cpu_count() or 1
    oracle.set_threads(threads)
    ids = workloads.permuted_block_table(nb, nb, workloads.SEED).numpy()
    kv = workloads.kv_values(T, cfg.heads, cfg.head_dim, cfg.dtype, seed=workloads.SEED, v_std=cfg.v_std)
    cache = torch.zeros((2, nb, bs, heads, cfg.head_dim), dtype=cfg.dtype)
    workloads.scatter_into_cache(cache, kv[:, :, :heads].contiguous(), torch.from_numpy(ids))
    c16 = cache.view(torch.int16).numpy().view(np.uint16).copy()
    packed, _ = oracle.pack_layer(c16, 0, ids, T, planes.shifts, planes.bits, fmt.specs)
    dst = np.zeros_like(c16)
    pack_dir = args.config == "C5"

    def step():
        if pack_dir:
            oracle.pack_layer(c16, 0, ids, T, planes.shifts, planes.bits, fmt.specs)
        else:
            oracle.restore_layer(packed, planes.shifts, planes.bits, fmt.specs, dst, 0, ids, T)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    ok = True if pack_dir else bool(np.array_equal(dst, c16))
    value = fmt.kv_bytes * args.steps / dt / GB
    sample = f"1 {args.config} layer x 1 request per step ({fmt.kv_bytes / 2**20:.0f} MiB KV), {heads} heads"
    metric = ("KV pack GB/s (gather + plane split + bitpack), whole job" if pack_dir else
              "KV restore GB/s (unpack + plane merge + paged scatter), whole job")
    line = {
        "impl": "reference",
        "metric": metric,
        "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3 / args.steps, 2), "higher_is_better": True,
        "scaling": "weak" if args.config == "C2" else "strong",
        "vs_baseline": None, "dtype": "u16 (bf16/fp16 bit patterns)", "data": "synthetic",
        "config": {"workload": f"{args.config} (bounded CPU sample)", "planes": planes.name, "chunk_bytes": cb},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": oracle.max_threads(), "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "verified": ok,
        "note": "the reference's CPU layout packer/unpacker is a stub (native_cpu.py:137-161); this is the "
                "oracle restatement of its format, timed on the host cores",
    }
    print(json.dumps(with_nominal(line)), flush=True)
    return 0


# ----------------------------------------------------------------------------------------
# quantized restore paths: CacheGen / KIVI dequantize-to-cache (--config CG | KIVI)
# ----------------------------------------------------------------------------------------
QUANT = {
    # Llama-3-8B-shaped request of C2 (32 layers, 8 KV heads, head_dim 128, 32768 tokens,
    # block 16, bf16 cache); CacheGen bins of the reference's quant level 2 fallback
    # (cachegen_adapter.py:49-57: key 32 / value 16 bins -> 5 / 4 bits, fp16 per-token max);
    # KIVI defaults of kivi_adapter.py:138-145 (2 bits, group 64, 128 sink tokens, fp16
    # scale / zero / sink).
    "CG": dict(layers=32, T=32768, H=8, D=128, bs=16, key_bins=32, value_bins=16),
    "KIVI": dict(layers=32, T=32768, H=8, D=128, bs=16, bits=2, group_size=64, sink=128),
}


class QuantWorkload:
    """Per-layer quantized payloads (seeded random streams and metadata, the same bytes
    for both arms) and a paged bf16 cache per layer, all resident on the device."""

    def __init__(self, kind: str, layers: int, device, seed: int = 7):
        import torch

        q = QUANT[kind]
        self.kind, self.q = kind, q
        self.layers = layers
        T, H, D, bs = q["T"], q["H"], q["D"], q["bs"]
        C = H * D
        self.T, self.H, self.D, self.bs, self.C = T, H, D, bs, C
        nb = (T + bs - 1) // bs
        self.NB = nb + 64
        g = torch.Generator(device="cpu").manual_seed(seed)
        self.ids = torch.randperm(self.NB, generator=g)[:nb].to(device)
        gd = torch.Generator(device=device).manual_seed(seed)

        def rbytes(n):
            return torch.randint(0, 256, (n,), generator=gd, dtype=torch.uint8, device=device)

        # One blob per layer, as the adapters lay out their raw payload (the symbol streams
        # followed by the fp16 metadata, cachegen_adapter.py:288-300, kivi_adapter.py:361-392);
        # the ops read typed views of it.
        parts: list[tuple[str, int, str]] = []  # name, bytes, dtype
        if kind == "CG":
            kb = (q["key_bins"] - 1).bit_length()
            vb = (q["value_bins"] - 1).bit_length()
            self.key_bits, self.value_bits = kb, vb
            self.klen, self.vlen = (T * C * kb + 7) // 8, (T * C * vb + 7) // 8
            parts = [("key", self.klen, "u8"), ("value", self.vlen, "u8"), ("max_key", 2 * T, "f16"),
                     ("max_value", 2 * T, "f16")]
        else:
            b, gs, sink = q["bits"], q["group_size"], q["sink"]
            body = T - sink
            slen = (body * C * b + 7) // 8
            kg, vg = (body + gs - 1) // gs, (C + gs - 1) // gs
            self.klen = self.vlen = slen
            parts = [("key", slen, "u8"), ("value", slen, "u8"), ("key_scale", 2 * kg * C, "f16"),
                     ("key_zero", 2 * kg * C, "f16"), ("value_scale", 2 * body * vg, "f16"),
                     ("value_zero", 2 * body * vg, "f16"), ("key_sink", 2 * sink * C, "f16"),
                     ("value_sink", 2 * sink * C, "f16")]
        self.offsets, off = {}, 0
        for name, n, _ in parts:
            off = (off + 15) // 16 * 16
            self.offsets[name] = (off, n)
            off += n
        self.blob_bytes = off
        self.in_bytes = sum(n for _, n, _ in parts)
        ranges = {"max_key": (0.0, 1.0), "max_value": (0.0, 1.0), "key_scale": (0.001, 0.5),
                  "value_scale": (0.001, 0.5), "key_zero": (-2, 2), "value_zero": (-2, 2), "key_sink": (-8, 8),
                  "value_sink": (-8, 8)}
        self.blobs = []
        for _ in range(layers):
            blob = torch.zeros(self.blob_bytes, dtype=torch.uint8, device=device)
            for name, n, dt in parts:
                o = self.offsets[name][0]
                if dt == "u8":
                    blob[o:o + n] = rbytes(n)
                elif name.startswith("max"):
                    blob[o:o + n].view(torch.float16)[:] = torch.exp(
                        torch.randn(n // 2, generator=gd, device=device)).half()
                else:
                    lo, hi = ranges[name]
                    blob[o:o + n].view(torch.float16)[:] = (
                        torch.rand(n // 2, generator=gd, device=device) * (hi - lo) + lo).half()
            self.blobs.append(blob)
        self.kv_bytes = 2 * T * C * 2
        self.caches = [torch.zeros((2, self.NB, bs, H, D), dtype=torch.bfloat16, device=device)
                       for _ in range(layers)]

    def view(self, blob, name):
        import torch

        o, n = self.offsets[name]
        return blob[o:o + n].view(torch.float16)

    def call(self, fn_cg, fn_kivi, layer: int, blob=None, error_count=None):
        """One layer's fused restore from `blob` (default: the layer's resident blob)."""
        q = self.q
        blob = self.blobs[layer] if blob is None else blob
        kw = {} if error_count is None else {"error_count": error_count}
        ko, vo = self.offsets["key"][0], self.offsets["value"][0]
        if self.kind == "CG":
            fn_cg(blob, ko, self.klen, vo, self.vlen, self.key_bits, self.value_bits, q["key_bins"],
                  q["value_bins"], self.view(blob, "max_key"), self.view(blob, "max_value"), self.caches[layer],
                  self.ids, self.T, self.H, self.D, **kw)
        else:
            fn_kivi(blob, ko, self.klen, vo, self.vlen, q["bits"], q["group_size"], q["sink"],
                    self.view(blob, "key_scale"), self.view(blob, "key_zero"), self.view(blob, "value_scale"),
                    self.view(blob, "value_zero"), self.view(blob, "key_sink"), self.view(blob, "value_sink"),
                    self.caches[layer], self.ids, self.T, self.H, self.D, **kw)

    def oracle_layer(self, layer: int) -> np.ndarray:
        """The CPU oracle's cache for one layer (checker; also the timed CPU sample)."""
        sys.path.insert(0, str(REPO / "oracle"))
        import oracle

        q = self.q
        cache = np.zeros((2, self.NB, self.bs, self.H, self.D), dtype=np.uint16)
        blob = self.blobs[layer].cpu().numpy()
        ids = self.ids.cpu().numpy()
        ko, vo = self.offsets["key"][0], self.offsets["value"][0]

        def h(name):
            o, n = self.offsets[name]
            return blob[o:o + n].view(np.float16)

        if self.kind == "CG":
            oracle.cachegen_to_cache(blob, ko, self.klen, vo, self.vlen, self.key_bits, self.value_bits,
                                     q["key_bins"], q["value_bins"], h("max_key"), h("max_value"), cache, False, ids,
                                     self.T, True)
        else:
            oracle.kivi_to_cache(blob, ko, self.klen, vo, self.vlen, q["bits"], q["group_size"], q["sink"],
                                 h("key_scale"), h("key_zero"), h("value_scale"), h("value_zero"), h("key_sink"),
                                 h("value_sink"), cache, False, ids, self.T, True)
        return cache


def _graph_timed(step_fn, args, world, device):
    """Warm-up, per-launch CUDA events (eager, behind a sleep head start), then CUDA-graph
    replays of the step; the same method as the C2 line."""
    import torch

    stream = torch.cuda.current_stream(device)
    for _ in range(args.warmup):
        step_fn()
    torch.cuda.synchronize(device)
    for _attempt in range(4):
        ev = []
        torch.cuda._sleep(HEAD_START_CYCLES)
        t_host = time.perf_counter()
        step_fn(ev)
        host_s = time.perf_counter() - t_host
        torch.cuda.synchronize(device)
        if host_s < HEAD_START_S:
            break
    launch_ms = [a.elapsed_time(b) for a, b in ev]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step_fn()
    for _ in range(args.warmup):
        graph.replay()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _attempt in range(4):
        barrier(world)
        torch.cuda.synchronize(device)
        torch.cuda._sleep(HEAD_START_CYCLES)
        t_host = time.perf_counter()
        t0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        t1.record(stream)
        host_s = time.perf_counter() - t_host
        torch.cuda.synchronize(device)
        if not any_over_ranks(host_s >= HEAD_START_S, world, device):
            break
    barrier(world)
    ms = max_over_ranks(t0.elapsed_time(t1), world, device)
    del graph
    return ms, launch_ms


def run_quant(args, rank, world, local, impl: str):
    """--config CG | KIVI: the fused dequantize-to-cache restore of one request's layers.
    `impl` origami times liborigami_b200.so; reference times the reference's own CUDA
    kernels (csrc/origami/bitpack_layout_cuda.cu:348-423, 577-683) built from its sources
    into oracle/_ref (rank 0 only)."""
    import torch

    kind = args.config
    metric = {"CG": "KV restore GB/s (CacheGen unpack + dequantize + paged scatter), whole job",
              "KIVI": "KV restore GB/s (KIVI unpack + dequantize + paged scatter), whole job"}[kind]
    if impl == "reference":
        if rank != 0:
            return 0
        sys.path.insert(0, str(REPO / "tests" / "golden"))
        from make_ref_vectors import load_reference_extension

        ext = load_reference_extension()
        if ext is None:
            print(json.dumps({"impl": "reference", "unavailable": "reference extension not built in oracle/_ref "
                              "(python oracle/build_ref.py needs the reference sources)"}), flush=True)
            return 0
        fn_cg, fn_kivi = ext.cachegen_unpack_dequantize_to_kv_cache_cuda, ext.kivi_dequantize_to_kv_cache_cuda
        world_eff = 1
    else:
        from origami_b200 import quant

        fn_cg, fn_kivi = quant.cachegen_unpack_dequantize_to_kv_cache_cuda, quant.kivi_dequantize_to_kv_cache_cuda
        world_eff = world
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    layers = args.layers or QUANT[kind]["layers"]
    wl = QuantWorkload(kind, layers, device, seed=7 + rank)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device)

    def step(events=None):
        for layer in range(layers):
            if events is not None:
                events.append((torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)))
                events[-1][0].record(stream)
            if impl == "reference":
                wl.call(fn_cg, fn_kivi, layer)
            else:
                wl.call(fn_cg, fn_kivi, layer, error_count=err)
            if events is not None:
                events[-1][1].record(stream)

    clocks = ClockSampler(local)
    clocks.start()
    ms, launch_ms = _graph_timed(step, args, world_eff, device)
    clock_info = clocks.stop()
    steps = args.steps
    kv_gbs = wl.kv_bytes * layers * world_eff * steps / (ms / 1e3) / GB
    alg = wl.kv_bytes + wl.in_bytes
    peak, peak_kind = measured_hbm_peak()
    mean_launch = sum(launch_ms) / len(launch_ms)
    # the configs' kernels: CG 5 / 4-bit symbols (staged rows), KIVI 2 bits with group 64
    kernel = {"CG": "cachegen_staged", "KIVI": "kivi2_to_cache"}[kind]
    if impl == "reference":
        kernel = {"CG": "cachegen_unpack_dequantize_to_kv_cache_kernel",
                  "KIVI": "kivi_dequantize_to_kv_cache_kernel"}[kind]
    roof = {"kernel": kernel, "bound": "hbm", "achieved": round(alg / (mean_launch / 1e3) / GB, 1), "peak": peak,
            "peak_kind": peak_kind, "unit": "GB/s", "frac": round(alg / (mean_launch / 1e3) / GB / peak, 4),
            "traffic": (profiled_traffic(kernel, {"CG": "CG_layer_T32768_H8_D128_k5_v4",
                                                  "KIVI": "KIVI_layer_T32768_H8_D128_b2_g64"}[kind], 1)
                        if impl == "origami" else None),
            "algorithmic_bytes_per_launch": alg, "launch_ms": round(mean_launch, 5)}
    q = QUANT[kind]
    cfgd = {"workload": f"{kind}: Llama-3-8B-shaped request, {q['T']} tokens, {q['H']} KV heads per rank, "
                        f"head_dim {q['D']}, block {q['bs']}, bf16 paged cache, seeded permuted block table",
            "layers": layers, "requests": world_eff, **{k: v for k, v in q.items() if k != "layers"},
            "parallelism": f"kv-head shard x{world_eff}, no collective",
            "l2": f"inputs larger than L2 ({layers * (wl.kv_bytes + wl.in_bytes) / 2**30:.1f} GiB per rank per step)"}

    # verification and CPU sample: layer 0 against the oracle
    ok = True
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        t0 = time.perf_counter()
        want = wl.oracle_layer(0)
        dt = time.perf_counter() - t0
        got = wl.caches[0].view(torch.int16).cpu().numpy().view(np.uint16)
        ok = bool(np.array_equal(got, want))
        cpu = {"value": round(wl.kv_bytes / dt / GB, 3), "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": f"1 layer ({wl.kv_bytes / 2**20:.0f} MiB KV), oracle {kind} restatement, {dt:.1f} s"}
    if impl == "origami":
        ok = ok and int(err.item()) == 0

    e2e = None
    if impl == "origami" and not args.no_e2e:
        host = [b.cpu().pin_memory() for b in wl.blobs]
        dev = torch.empty_like(wl.blobs[0])
        err_h = torch.zeros(1, dtype=torch.int32).pin_memory()

        def e2e_step():
            for layer in range(layers):
                dev.copy_(host[layer], non_blocking=True)
                wl.call(fn_cg, fn_kivi, layer, blob=dev, error_count=err)
            err_h.copy_(err, non_blocking=True)

        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize(device)
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            e2e_step()
        b.record(stream)
        torch.cuda.synchronize(device)
        ms_e2e = max_over_ranks(a.elapsed_time(b), world, device)
        h2d = sum(int(h.numel()) for h in host)
        e2e = {"value": round(wl.kv_bytes * layers * world * steps / (ms_e2e / 1e3) / GB, 1), "unit": "GB/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4, "ms_per_step": round(ms_e2e / steps, 3),
               "note": "each layer's payload blob (streams + metadata) copied from pinned host, then the fused "
                       "restore"}

    if rank == 0:
        line = {"metric": metric, "value": round(kv_gbs, 1), "unit": "GB/s", "n_gpus": world_eff, "steps": steps,
                "warmup": args.warmup, "ms_per_step": round(ms / steps, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16 out (fp32 dequant math)",
                "data": "synthetic (seeded random symbol streams and metadata)", "config": cfgd, "roofline": roof,
                "gpu_launches": layers if impl == "origami" else 0, "clocks": clock_info, "verified": ok}
        if impl == "reference":
            line["impl"] = "reference"
            line["cpu_baseline"] = {"value": round(kv_gbs, 1), "unit": "GB/s", "cores": 0, "kind": "reference",
                                    "sample": "the reference's CUDA kernel on the GPU (no CPU implementation exists)"}
            line["e2e"] = {"value": round(kv_gbs, 1), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
        else:
            if cpu is not None:
                line["cpu_baseline"] = cpu
            if e2e is not None:
                line["e2e"] = e2e
        print(json.dumps(with_nominal(line)), flush=True)
    return 0



# ----------------------------------------------------------------------------------------
# compressed-prefix fused attention (--config ATTN)
# ----------------------------------------------------------------------------------------
# One decode step of a Llama-3-8B-shaped model over a C2-length request whose first 32768
# tokens are a KIVI 2-bit prefix (kivi_adapter.py:138-145 defaults: group 64, 128 sink
# tokens, fp16 metadata) and whose last `suffix` tokens sit in the paged bf16 cache; the
# query is the newest token (32 query heads over 8 KV heads).
ATTN = dict(layers=32, T=32768, suffix=256, H=8, QH=32, D=128, bs=16, bits=2, group_size=64, sink=128)


class AttnWorkload:
    """Per-layer KIVI prefix blobs (streams then fp16 metadata, 16-byte aligned parts),
    paged caches holding the suffix, queries and outputs, all resident on the device."""

    def __init__(self, layers: int, queries: int, device, seed: int = 11):
        import torch

        q = ATTN
        self.layers, self.queries = layers, queries
        T, H, D, bs, b, gs, sink = q["T"], q["H"], q["D"], q["bs"], q["bits"], q["group_size"], q["sink"]
        C = H * D
        self.T, self.H, self.QH, self.D, self.C = T, H, q["QH"], D, C
        self.seq = T + q["suffix"]
        self.q_start = self.seq - queries
        body = T - sink
        slen = (body * C * b + 7) // 8
        kg, vg = (body + gs - 1) // gs, (C + gs - 1) // gs
        self.slen = slen
        parts = [("key", slen), ("value", slen), ("key_scale", 2 * kg * C), ("key_zero", 2 * kg * C),
                 ("value_scale", 2 * body * vg), ("value_zero", 2 * body * vg), ("key_sink", 2 * sink * C),
                 ("value_sink", 2 * sink * C)]
        self.offsets, off = {}, 0
        for name, n in parts:
            off = (off + 15) // 16 * 16
            self.offsets[name] = (off, n)
            off += n
        self.blob_bytes = off
        self.prefix_bytes = sum(n for _, n in parts)
        gd = torch.Generator(device=device).manual_seed(seed)
        levels = (1 << b) - 1
        self.blobs = []
        for _ in range(layers):
            blob = torch.zeros(self.blob_bytes, dtype=torch.uint8, device=device)
            for name, n in parts:
                o = self.offsets[name][0]
                if name in ("key", "value"):
                    blob[o:o + n] = torch.randint(0, 256, (n,), generator=gd, dtype=torch.uint8, device=device)
                    continue
                v = blob[o:o + n].view(torch.float16)
                r = torch.rand(n // 2, generator=gd, device=device)
                if name.endswith("scale"):
                    v[:] = ((0.5 + r) * 2.0 / levels).half()
                elif name.endswith("zero"):
                    v[:] = (-1.2 + 0.4 * r).half()
                else:
                    v[:] = torch.randn(n // 2, generator=gd, device=device).half()
            self.blobs.append(blob)
        nb = (self.seq + bs - 1) // bs
        self.NB = nb + 64
        g = torch.Generator(device="cpu").manual_seed(seed)
        self.table = torch.randperm(self.NB, generator=g)[:nb].to(torch.int32).to(device)
        self.caches = [torch.randn((2, self.NB, bs, H, D), generator=gd, device=device).to(torch.bfloat16)
                       for _ in range(layers)]
        self.query = [torch.randn((queries, self.QH, D), generator=gd, device=device).to(torch.bfloat16)
                      for _ in range(layers)]
        self.out = [torch.empty_like(x) for x in self.query]
        self.scale = 1.0 / math.sqrt(D)
        # bytes one launch must read: the compressed prefix, the suffix K/V rows, the query
        # (and write the output)
        self.alg_bytes = self.prefix_bytes + 2 * q["suffix"] * C * 2 + 2 * queries * self.QH * D * 2
        # bf16-equivalent K/V attended per step and layer
        self.kv_equiv = 2 * self.seq * C * 2

    def view(self, blob, name):
        import torch

        o, n = self.offsets[name]
        return blob[o:o + n].view(torch.float16)

    def args(self, layer: int, blob=None):
        q = ATTN
        blob = self.blobs[layer] if blob is None else blob
        return [blob, self.offsets["key"][0], self.slen, self.offsets["value"][0], self.slen, 0, q["bits"],
                q["group_size"], q["sink"], self.view(blob, "key_scale"), self.view(blob, "key_zero"),
                self.view(blob, "value_scale"), self.view(blob, "value_zero"), self.view(blob, "key_sink"),
                self.view(blob, "value_sink"), self.query[layer], self.caches[layer], self.table, self.T,
                self.q_start, self.seq, self.scale, self.out[layer]]

    def oracle_layer(self, layer: int) -> np.ndarray:
        """The CPU oracle's output for one layer (checker; also the timed CPU sample)."""
        sys.path.insert(0, str(REPO / "oracle"))
        import oracle

        q = ATTN
        blob = self.blobs[layer].cpu().numpy()

        def h(name):
            o, n = self.offsets[name]
            return blob[o:o + n].view(np.float16)

        u16 = lambda t: t.view(__import__("torch").int16).cpu().numpy().view(np.uint16)  # noqa: E731
        return oracle.fused_prefix_attention(
            blob, self.offsets["key"][0], self.slen, self.offsets["value"][0], self.slen, 0, q["bits"],
            q["group_size"], q["sink"], h("key_scale"), h("key_zero"), h("value_scale"), h("value_zero"),
            h("key_sink"), h("value_sink"), u16(self.query[layer]), True, u16(self.caches[layer]), True, False,
            self.table.cpu().numpy(), self.T, self.q_start, self.seq, self.scale)


def _oracle_cores() -> int:
    sys.path.insert(0, str(REPO / "oracle"))
    import oracle

    return oracle.max_threads()


def run_attention(args, rank, world, local, impl: str):
    """--config ATTN: the fused attention over a quantized prefix, one decode step over all
    layers. `impl` origami times liborigami_b200.so (tcgen05 kernel); reference times the
    reference's own kernel (csrc/origami/bitpack_layout_cuda.cu:873-1091) built from its
    sources into oracle/_ref (rank 0 only)."""
    import torch

    if impl == "reference":
        if rank != 0:
            return 0
        sys.path.insert(0, str(REPO / "tests" / "golden"))
        from make_ref_vectors import load_reference_extension

        ext = load_reference_extension()
        if ext is None:
            print(json.dumps({"impl": "reference", "unavailable": "reference extension not built in oracle/_ref "
                              "(python oracle/build_ref.py needs the reference sources)"}), flush=True)
            return 0
        fn = ext.fused_prefix_attention_cuda
        world_eff = 1
    else:
        from origami_b200 import attention

        fn = attention.fused_prefix_attention_cuda
        world_eff = world
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    layers = args.layers or ATTN["layers"]
    wl = AttnWorkload(layers, args.attn_queries, device, seed=11 + rank)
    stream = torch.cuda.current_stream(device)
    kw = {}
    flags = None
    if impl == "origami":
        from origami_b200 import attention

        need = attention.workspace_bytes(wl.queries, wl.QH, wl.H, wl.q_start, wl.seq, device)
        flags = torch.zeros(1, dtype=torch.int32, device=device)
        kw = {"error_flags": flags}
        if need:
            kw["workspace"] = torch.zeros(need, dtype=torch.uint8, device=device)

    def step(events=None):
        for layer in range(layers):
            if events is not None:
                events.append((torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)))
                events[-1][0].record(stream)
            fn(*wl.args(layer), **kw)
            if events is not None:
                events[-1][1].record(stream)

    clocks = ClockSampler(local)
    clocks.start()
    ms, launch_ms = _graph_timed(step, args, world_eff, device)
    clock_info = clocks.stop()
    steps = args.steps
    kv_gbs = wl.kv_equiv * layers * world_eff * steps / (ms / 1e3) / GB
    peak, peak_kind = measured_hbm_peak()
    mean_launch = sum(launch_ms) / len(launch_ms)
    kernel = "prefix_attention_sym" if impl == "origami" else "origami_fused_prefix_attention_kernel"
    achieved = wl.alg_bytes / (mean_launch / 1e3) / GB
    # one launch per layer; the committed ncu figure is for the default one-query decode
    traffic = (profiled_traffic(kernel, "ATTN_layer_T32768_H8_D128_b2_g64_q1", 1)
               if impl == "origami" and wl.queries == 1 else None)
    roof = {"kernel": kernel, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind,
            "unit": "GB/s", "frac": round(achieved / peak, 4), "traffic": traffic,
            "algorithmic_bytes_per_launch": wl.alg_bytes, "launch_ms": round(mean_launch, 5),
            "us_per_layer": round(ms / steps / layers * 1e3, 2)}
    q = ATTN
    cfgd = {"workload": f"ATTN: Llama-3-8B decode step over a {q['T']}-token KIVI {q['bits']}-bit prefix "
                        f"(group {q['group_size']}, {q['sink']} sink tokens) + {q['suffix']} paged bf16 tokens, "
                        f"{wl.QH} query / {wl.H} KV heads, head_dim {q['D']}",
            "layers": layers, "query_tokens": wl.queries, "requests": world_eff,
            **{k: v for k, v in q.items() if k != "layers"}, "parallelism": f"replicas x{world_eff}, no collective",
            "l2": f"inputs larger than L2 ({layers * wl.alg_bytes / 2**30:.2f} GiB read per rank per step)"}

    ok = True
    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        t0 = time.perf_counter()
        want = wl.oracle_layer(0)
        dt = time.perf_counter() - t0
        got = wl.out[0].float().cpu().numpy()
        ref = (want.astype(np.uint32) << 16).view(np.float32)
        ok = bool(np.allclose(got, ref, atol=3e-2, rtol=3e-2))
        cpu = {"value": round(wl.kv_equiv / dt / GB, 3), "unit": "GB/s", "cores": _oracle_cores(),
               "kind": "port", "sample": f"1 layer ({wl.QH} query heads x {wl.seq} keys), oracle restatement of the "
                                         f"reference kernel, {dt:.1f} s"}
    if impl == "origami":
        ok = ok and int(flags.item()) == 0

    e2e = None
    if impl == "origami" and not args.no_e2e:
        host = [b.cpu().pin_memory() for b in wl.blobs]
        dev = torch.empty_like(wl.blobs[0])
        out_h = [torch.empty_like(o, device="cpu").pin_memory() for o in wl.out]

        def e2e_step():
            for layer in range(layers):
                dev.copy_(host[layer], non_blocking=True)
                fn(*wl.args(layer, blob=dev), **kw)
                out_h[layer].copy_(wl.out[layer], non_blocking=True)

        for _ in range(args.warmup):
            e2e_step()
        torch.cuda.synchronize(device)
        barrier(world)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            e2e_step()
        b.record(stream)
        torch.cuda.synchronize(device)
        ms_e2e = max_over_ranks(a.elapsed_time(b), world, device)
        e2e = {"value": round(wl.kv_equiv * layers * world * steps / (ms_e2e / 1e3) / GB, 1), "unit": "GB/s",
               "h2d_bytes_per_step": sum(int(h.numel()) for h in host),
               "d2h_bytes_per_step": sum(int(o.numel()) * 2 for o in out_h), "ms_per_step": round(ms_e2e / steps, 3),
               "note": "each layer's compressed prefix blob copied from pinned host, the fused attention, the output "
                       "copied back"}

    if rank == 0:
        line = {"metric": "prefix attention: bf16-equivalent KV GB/s attended per decode step, whole job",
                "value": round(kv_gbs, 1), "unit": "GB/s", "n_gpus": world_eff, "steps": steps,
                "warmup": args.warmup, "ms_per_step": round(ms / steps, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (fp32 dequant, fp32 accumulate)",
                "data": "synthetic (seeded random symbol streams, metadata, suffix cache and queries)",
                "config": cfgd, "roofline": roof, "gpu_launches": layers if impl == "origami" else 0,
                "clocks": clock_info, "verified": ok}
        if impl == "reference":
            line["impl"] = "reference"
            line["cpu_baseline"] = {"value": round(kv_gbs, 1), "unit": "GB/s", "cores": 0, "kind": "reference",
                                    "sample": "the reference's CUDA kernel on the GPU (no CPU implementation exists)"}
            line["e2e"] = {"value": round(kv_gbs, 1), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
        else:
            if cpu is not None:
                line["cpu_baseline"] = cpu
            if e2e is not None:
                line["e2e"] = e2e
        print(json.dumps(with_nominal(line)), flush=True)
    return 0


def main():
    args = parse_args()
    if args.config in QUANT:
        rank, world, local = init_dist("nccl")
        rc = run_quant(args, rank, world, local, args.impl)
    elif args.config == "ATTN":
        rank, world, local = init_dist("nccl")
        rc = run_attention(args, rank, world, local, args.impl)
    elif args.impl == "reference":
        rank, world, _ = init_dist("gloo")
        rc = run_reference(args, rank, world)
    else:
        rank, world, local = init_dist("nccl")
        rc = run_origami(args, rank, world, local)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return rc


if __name__ == "__main__":
    sys.exit(main())
