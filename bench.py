"""Benchmark of the specgrove_b200 packed tree-verification step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload verify|verify4b|accept]

One JSON line is printed by rank 0.  Under torchrun (N > 1) every rank runs
its own shard of requests with a full model replica (data parallel, no
data-path collective; weak scaling); the step time is the max over ranks of
the CUDA-event time and `value` aggregates the accepted tokens of all ranks.

Workload `verify` (default): Qwen3-8B shape
(36 layers, hidden 4096, 32 q / 8 kv heads, head_dim 128, intermediate 12288,
vocab 151936), random-init bf16 weights, 64 requests per GPU with cache
prefixes uniform in [1024, 4096] (synthetic KV), one canonical best-first
tree per request cut to its tier (tier mix 40x16 + 12x32 + 8x64 + 4x128 rows
= 2048 rows).  One step = one packed verify pass: target forward over the
2048 rows, LM head fused with online softmax and Gumbel-max sampling, tree
walk, and commit of the accepted rows' KV.  Weights (16.4 GB) and KV
(~24 GB read per step) are far larger than L2, so no flush is needed.
`verify4b` is configuration 3 (Qwen3-4B shape, 16 requests, 512 rows);
`accept` is the kernel-isolated acceptance sweep (configuration 2).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

KV_BYTES_PER_TOKEN = 36 * 8 * 128 * 2 * 2  # layers x kv heads x head_dim x bf16 x {K,V}

# DRAM bytes (read + write) of one layer's tree-attention launch on the
# configuration-4 wave, from an ncu capture of that launch
# (dram__bytes_read.sum 736.3 MB + dram__bytes_write.sum 15.5 MB).
NCU_ATTENTION_TRAFFIC_CFG4 = 736.310016e6 + 15.491584e6
# Same for one gate/up + SwiGLU GEMM launch on the configuration-4 rows
# (dram__bytes_read.sum 218.2 MB + dram__bytes_write.sum 41.1 MB).
NCU_SWIGLU_TRAFFIC_CFG4 = 218.232576e6 + 41.149184e6
# Same for one acceptance launch of the configuration-2 sweep
# (dram__bytes_read.sum 53.6 MB + dram__bytes_write.sum 0.81 MB).
NCU_ACCEPT_TRAFFIC_CFG2 = 53.622528e6 + 0.811264e6


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi sampling during the timed region (median SM MHz, reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.gpu_id = self._smi_id(device_index)
        self.proc = None
        self.path = None

    @staticmethod
    def _smi_id(device_index: int) -> str:
        """nvidia-smi --id for a torch device: its UUID (immune to
        CUDA_VISIBLE_DEVICES remapping), else the visible-device mapping."""
        visible = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [v.strip() for v in visible.split(",") if v.strip()]
        fallback = ids[device_index] if device_index < len(ids) else str(device_index)
        try:
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            if not uuid:
                return fallback
            uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            probe = subprocess.run(["nvidia-smi", f"--id={uuid}", "--query-gpu=index", "--format=csv,noheader"],
                                   capture_output=True, text=True, timeout=10)
            return uuid if probe.returncode == 0 and probe.stdout.strip() else fallback
        except Exception:  # no device properties or no nvidia-smi: keep the index mapping
            return fallback

    def _cmd(self, loop: bool):
        cmd = ["nvidia-smi", f"--id={self.gpu_id}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits"]
        return cmd + ["-lms", "50"] if loop else cmd

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(self._cmd(True), stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            # one more sample taken at the end of the timed region, so short
            # runs report at least one reading
            try:
                out = subprocess.run(self._cmd(False), capture_output=True, text=True, timeout=10).stdout
                with open(self.path, "a") as f:
                    f.write(out)
            except (OSError, subprocess.SubprocessError):
                pass
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.path is None:
            return None
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), max=float(parts[2]), power=float(parts[3]),
                                 hw=parts[5], hwt=parts[6], swt=parts[7], swp=parts[8]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return None
        reasons = set()
        for r in rows:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                              ("swt", "sw_thermal_slowdown"), ("swp", "sw_power_cap")):
                if r[key].lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in rows), "sm_max_mhz": max(r["max"] for r in rows),
                "samples": len(rows), "power_w_max": max(r["power"] for r in rows), "reasons": sorted(reasons)}


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ---------------------------------------------------------------------------
# Acceptance sweep workload
# ---------------------------------------------------------------------------
class AcceptWorkload:
    name = "acceptance_sweep: 64 trees / 4096 nodes / V=151936 fp32 probs + KV commit 36x8x128 bf16"

    def __init__(self, rank: int):
        from specgrove_b200 import workloads
        from specgrove_b200.arena import PersistentKVArena
        from specgrove_b200.sampling import PackedTrees
        self.batch, self.probs = workloads.acceptance_sweep(seed=rank, device="cuda")
        self.trees = PackedTrees(self.batch.parents, self.batch.tokens, "cuda")
        self.D = self.trees.max_depth
        self.T = self.trees.count
        self.vocab = self.probs.shape[1]
        rng = np.random.default_rng(rank)
        self.lengths0 = rng.integers(64, 257, size=self.T)
        # a node's tree row sits at length + node in its slot's tail
        capacity = int(self.lengths0.max()) + self.trees.max_nodes
        self.arena = PersistentKVArena(36, 8, 128, self.T, capacity, dtype=torch.bfloat16)
        self.slots = torch.arange(self.T, dtype=torch.long, device="cuda")
        self.len_in = torch.from_numpy(self.lengths0.astype(np.int64)).cuda()
        self.len_out = torch.empty_like(self.len_in)
        self.request_ids = torch.arange(self.T, dtype=torch.long, device="cuda") + 1000 * rank
        self.status = torch.zeros(1, dtype=torch.int32, device="cuda")
        torch.cuda.empty_cache()   # release the generator's temporaries

    def step(self, seed: int, out: torch.Tensor, events=None):
        from specgrove_b200 import _lib
        from specgrove_b200._lib import check, ptr, stream_ptr
        from specgrove_b200.sampling import accept_packed
        if events is not None:
            events[0].record()
        accept_packed(self.probs, self.trees, seed=seed, request_ids=self.request_ids, out=out,
                      status=self.status)
        if events is not None:
            events[1].record()
        a = self.arena
        st = _lib.load().sg_kv_commit_accepted(
            ptr(a.storage), a.plane_rows, a.num_planes, a.row_bytes, a.capacity, ptr(self.slots),
            ptr(self.len_in), ptr(self.len_out), ptr(out), self.T, self.D, ptr(self.status),
            stream_ptr())
        check(st, "sg_kv_commit_accepted")
        if events is not None:
            events[2].record()

    def units(self, outs: torch.Tensor) -> int:
        """accepted tokens (accepted nodes + bonus) over the given step outputs."""
        return int((outs[..., self.D] + 1).sum())


class VerifyWorkload:
    def __init__(self, rank: int, config: str, layers: int | None = None):
        from specgrove_b200 import workloads
        from specgrove_b200.engine import QWEN3_4B, QWEN3_8B, B200Engine, Wave, Weights
        if config == "verify4b":
            self.shape, mix, prefix = QWEN3_4B, workloads.TIER_MIX_CONFIG3, (512, 2048)
            self.name = "config3: Qwen3-4B shape, 16 requests, prefixes U[512,2048], tiers {16,32,64}, 512 rows"
        else:
            self.shape, mix, prefix = QWEN3_8B, workloads.TIER_MIX_CONFIG4, (1024, 4096)
            self.name = "config4: Qwen3-8B shape, 64 requests, prefixes U[1024,4096], tiers {16,32,64,128}, 2048 rows"
        if layers is not None and layers != self.shape.num_layers:
            import dataclasses
            # profiling captures only: fewer layers keep an ncu capture small
            self.shape = dataclasses.replace(self.shape, num_layers=layers)
            self.name += f" [PROFILING ONLY: {layers} layers]"
        self.weights = Weights.random(self.shape, seed=1234)           # full replica on every rank
        self.wl = workloads.verify_workload(self.shape.vocab, mix, prefix, seed=rank)
        R = len(self.wl.trees)
        rows = sum(len(t[0]) for t in self.wl.trees)
        self.capacity = prefix[1] + max(self.wl.tiers) + 16
        self.engine = B200Engine(self.weights, num_slots=R, capacity=self.capacity, max_rows=rows)
        g = torch.Generator(device="cuda").manual_seed(rank)
        self.engine.arena.storage.normal_(0.0, 1.0, generator=g)       # synthetic cache prefixes
        self.wave = Wave(self.wl.trees, list(range(R)), self.wl.cache_lengths,
                         request_ids=[rank * 1_000_000 + i for i in range(R)])
        self.dw = self.wave.to("cuda")
        self.R, self.rows, self.D = R, rows, self.wave.max_depth
        self.lengths_out = torch.empty(R, dtype=torch.long, device="cuda")
        # Per-wave allocator score exchange across data-parallel ranks (the
        # only collective of the step; a few KB over NCCL).
        self.exchange = None
        import torch.distributed as dist
        if dist.is_initialized() and dist.get_world_size() > 1:
            from specgrove_b200.allocator import RequestScores, ScoreExchange
            rng = np.random.default_rng(1000 + rank)
            self.scores = RequestScores(progress=[0] * R, ages=[0] * R,
                                        service_weights=[float(x) for x in rng.choice([1.0, 2.0, 4.0], size=R)],
                                        utilities=self.wl.utilities)
            self.exchange = ScoreExchange(R, len(self.wl.tier_options), "cuda")
            self.exchange.pack(self.scores)

    def step(self, seed: int, out: torch.Tensor, trace=None):
        if self.exchange is not None:
            self.exchange.exchange()
        self.engine.verify_device(self.dw, seed=seed, commit=True, accept_out=out, lengths_out=self.lengths_out,
                                  trace=trace)

    def units(self, outs: torch.Tensor) -> int:
        return int((outs[..., self.D] + 1).sum())

    def attention_bytes(self) -> float:
        s = self.shape
        per_token = s.num_kv_heads * s.head_dim * 2 * 2
        return float(sum((L + len(t[0])) * per_token for L, t in zip(self.wl.cache_lengths, self.wl.trees)))

    def pass_flops(self) -> float:
        s = self.shape
        f = self.rows * s.gemm_flops_per_row()
        for L, (par, _) in zip(self.wl.cache_lengths, self.wl.trees):
            depth = [0] * len(par)
            for j in range(1, len(par)):
                depth[j] = depth[par[j]] + 1
            f += sum(s.attention_flops(L + d + 1) for d in depth)
        return float(f)


def make_events(n):
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
    for e in evs:           # materialise the cudaEvent_t handles
        e.record()
    torch.cuda.synchronize()
    return evs


def run_verify(args, world, rank):
    from specgrove_b200 import _lib
    from specgrove_b200.engine import TRACE_EVENTS, TRACE_STAGES
    hbm, tc, tc_sus, peak_kind = peaks()
    wl = VerifyWorkload(rank, args.workload, args.layers)
    K, W = args.steps, args.warmup
    outs = torch.empty((K, wl.R, wl.D + 2), dtype=torch.long, device="cuda")
    warm = torch.empty((wl.R, wl.D + 2), dtype=torch.long, device="cuda")
    for i in range(W):
        wl.step(10_000 + i, warm)
    torch.cuda.synchronize()
    traces = [make_events(TRACE_EVENTS) for _ in range(K)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = _lib.launch_count()
    with ClockSampler(torch.cuda.current_device()) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        start.record()
        for i in range(K):
            wl.step(i, outs[i], traces[i])
        stop.record()
        torch.cuda.synchronize()
        barrier(world)
    launches = _lib.launch_count() - launches0
    if int(wl.engine.status) != 0:
        raise RuntimeError(f"device status {int(wl.engine.status)}")
    ms = max_over_ranks(start.elapsed_time(stop) / K, world)
    total_units = sum_over_ranks(wl.units(outs), world)
    value = total_units / (ms * K / 1000.0)
    stages = {name: statistics.mean(t[i].elapsed_time(t[i + 1]) for t in traces)
              for i, name in enumerate(TRACE_STAGES)}
    attn_ms = stages["L0 attention"]
    attn_bytes = wl.attention_bytes()                  # one layer's K/V reads
    attn_gbs = attn_bytes / (attn_ms / 1000) / 1e9
    flops = wl.pass_flops()
    pass_tflops = flops / (ms / 1000) / 1e12
    gu_ms = stages["L0 gate/up gemm"]
    gu_flops = 2.0 * wl.rows * (2 * wl.shape.intermediate) * wl.shape.hidden
    gu_tflops = gu_flops / (gu_ms / 1000) / 1e12
    cfg4 = wl.name.startswith("config4")
    e2e = e2e_verify(wl, args, world)
    cpu = cpu_baseline_verify(wl) if (rank == 0 and world == 1 and not args.no_cpu) else None
    clk = clocks.summary()
    line = {
        "metric": "accepted tokens/s/GPU", "value": value, "unit": "accepted tokens/s",
        "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, "
        "synthetic KV prefixes, seeded best-first trees)",
        "config": {"workload": wl.name, "model": "Qwen3-8B shape" if wl.shape.hidden == 4096 else "Qwen3-4B shape",
                   "collective": "per-step NCCL all_gather_into_tensor of allocator scores" if world > 1 else None,
                   "requests_per_gpu": wl.R, "rows_per_gpu": wl.rows, "global_batch_rows": wl.rows * world,
                   "verify_pass_us_per_row": ms * 1000 / wl.rows, "temperature": 1.0,
                   "parallelism": f"dp{world}", "l2": "inputs larger than L2 (16.4 GB weights, ~24 GB KV/step)"},
        # dominant kernel by time: the gate/up GEMM with the SwiGLU epilogue
        # (timed inside the step, so against the sustained bf16 peak)
        "roofline": {"bound": "tensor", "kernel": "gemm_kernel<EpiSwiGlu> (layer 0 gate/up)",
                     "achieved": gu_tflops, "peak": tc_sus, "peak_kind": peak_kind + " sustained",
                     "unit": "TFLOP/s", "frac": gu_tflops / tc_sus,
                     "traffic": NCU_SWIGLU_TRAFFIC_CFG4 if cfg4 else None,
                     "algorithmic_flops_per_launch": gu_flops, "launch_ms": gu_ms,
                     "attention": {"bound": "hbm", "kernel": "tree_attention_tm_kernel (layer 0)",
                                   "achieved": attn_gbs, "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s",
                                   "frac": attn_gbs / hbm,
                                   "traffic": NCU_ATTENTION_TRAFFIC_CFG4 if cfg4 else None,
                                   "algorithmic_bytes_per_launch": attn_bytes, "launch_ms": attn_ms},
                     "pass": {"bound": "tensor", "achieved": pass_tflops, "peak": tc_sus, "unit": "TFLOP/s",
                              "frac": pass_tflops / tc_sus, "algorithmic_flops_per_step": flops,
                              "peak_kind": peak_kind + " sustained"}},
        "stages_ms": {k: round(v, 4) for k, v in stages.items()},
        "profiling_only": args.layers is not None and args.layers != 36,
        "cpu_baseline": cpu, "clocks": clk, "e2e": e2e, "gpu_launches": launches,
    }
    return line


def e2e_verify(wl, args, world):
    """Through the public API with host buffers: the wave (tree metadata,
    tokens, lengths) is copied from pinned host memory, the pass runs, the
    decisions are read back, every step."""
    host = wl.wave.host.pin_memory()
    dev = wl.dw.buf
    out_dev = torch.empty((wl.R, wl.D + 2), dtype=torch.long, device="cuda")
    out_host = torch.empty_like(out_dev, device="cpu").pin_memory()
    steps = max(3, min(args.steps, 10))

    def one(seed):
        dev.copy_(host, non_blocking=True)
        wl.step(seed, out_dev)
        out_host.copy_(out_dev, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return int((out_host[:, wl.D] + 1).sum())

    one(777)
    barrier(world)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    units = 0
    start.record()
    for i in range(steps):
        units += one(50_000 + i)
    stop.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(stop) / steps, world)
    total = sum_over_ranks(units, world)
    return {"value": total / (ms * steps / 1000.0), "unit": "accepted tokens/s",
            "h2d_bytes_per_step": host.numel() * 8, "d2h_bytes_per_step": out_host.numel() * 8,
            "steps": steps, "ms_per_step": ms}


def cpu_baseline_verify(wl, requests: int = 4, budget_s: float = 20.0):
    """The reference's step restated on the host (oracle/forward.py: torch fp32
    target pass with the packed tree mask, fp32 softmax, fp64 walk) on a
    bounded slice: the first `requests` requests of the wave, all layers."""
    from oracle.forward import CpuWeights, verify_step
    torch.set_num_threads(os.cpu_count())
    cw = CpuWeights(wl.weights)
    trees = wl.wl.trees[:requests]
    lengths = wl.wl.cache_lengths[:requests]
    store = wl.engine.arena
    prefixes = []
    for i, L in enumerate(lengths):
        base = i * store.capacity
        prefixes.append([(store.key_storage[l][:, base:base + L].float().cpu(),
                          store.value_storage[l][:, base:base + L].float().cpu())
                         for l in range(wl.shape.num_layers)])
    rows = sum(len(t[0]) for t in trees)
    units, seconds, reps = 0, 0.0, 0
    while reps < 1 or (seconds < budget_s and reps < 5):
        t0 = time.perf_counter()
        res, _ = verify_step(cw, prefixes, trees, lengths, seed=reps)
        seconds += time.perf_counter() - t0
        units += sum(len(nodes) + 1 for nodes, _ in res)
        reps += 1
    return {"value": units / seconds, "unit": "accepted tokens/s", "cores": os.cpu_count(), "kind": "port",
            "us_per_row": seconds / reps / rows * 1e6,
            "sample": f"{reps} step(s) of {requests} requests ({rows} rows), all {wl.shape.num_layers} layers, "
                      f"torch fp32 on {torch.get_num_threads()} threads"}


def run_b200(args, world, rank):
    from specgrove_b200 import _lib
    hbm, tc, tc_sus, peak_kind = peaks()
    wl = AcceptWorkload(rank)
    K, W = args.steps, args.warmup
    outs = torch.empty((K, wl.T, wl.D + 2), dtype=torch.long, device="cuda")
    warm = torch.empty((wl.T, wl.D + 2), dtype=torch.long, device="cuda")
    for i in range(W):
        wl.step(10_000 + i, warm)
    torch.cuda.synchronize()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(K)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # The rows a step visits (~55 MB, the 64 roots every step) fit in L2, so
    # L2 is flushed between timed steps by writing a buffer four times its
    # size; each step is timed by its own events, which exclude the flush.
    flush = torch.empty(512 << 20, dtype=torch.uint8, device="cuda")
    launches0 = _lib.launch_count()
    with ClockSampler(torch.cuda.current_device()) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        # A step is two short kernels (~tens of us), less than the host needs
        # to enqueue it; a device sleep ahead of the start event lets the host
        # queue all K steps first, so the events time the kernels back to
        # back instead of the host's enqueue gaps.
        torch.cuda._sleep(int(4_000_000 * K))
        start.record()
        for i in range(K):
            flush.fill_(i & 0xFF)
            wl.step(i, outs[i], ev[i])
        stop.record()
        torch.cuda.synchronize()
        barrier(world)
    launches = _lib.launch_count() - launches0
    ms_with_flush = start.elapsed_time(stop) / K
    ms_local = statistics.mean(e[0].elapsed_time(e[2]) for e in ev)
    ms = max_over_ranks(ms_local, world)
    units_local = wl.units(outs)
    total_units = sum_over_ranks(units_local, world)
    value = total_units / (ms * K / 1000.0)
    if int(wl.status) != 0:
        raise RuntimeError(f"device status {int(wl.status)}")
    # roofline of the dominant kernel (acceptance): visited rows x V x 4 bytes per launch
    accept_ms = [e[0].elapsed_time(e[1]) for e in ev]
    commit_ms = [e[1].elapsed_time(e[2]) for e in ev]
    visited = (outs[..., wl.D] + 1).double()        # scan rule: accepted + exit row
    accept_bytes = float(visited.sum()) / K * wl.vocab * 4
    # kept tokens x 147,456 B, read and written (the reference's append copies
    # every kept row); here the root row and rows already at their final
    # position never move, so the bytes actually moved are fewer
    commit_bytes = float(visited.sum()) / K * KV_BYTES_PER_TOKEN * 2
    moved = outs[..., :wl.D] >= 0
    depth_idx = torch.arange(1, wl.D + 1, device=outs.device).expand_as(moved)
    moved_rows = float((moved & (outs[..., :wl.D] != depth_idx)).sum()) / K
    moved_bytes = moved_rows * KV_BYTES_PER_TOKEN * 2
    accept_gbs = accept_bytes / (statistics.mean(accept_ms) / 1000) / 1e9
    commit_gbs = commit_bytes / (statistics.mean(commit_ms) / 1000) / 1e9
    # e2e through the public API with host buffers: probabilities and tree
    # metadata copied from pinned host memory, decisions read back, per step.
    e2e = e2e_accept(wl, args, world)
    cpu = cpu_baseline_accept(wl) if (rank == 0 and world == 1 and not args.no_cpu) else None
    clk = clocks.summary()
    line = {
        "metric": "accepted tokens/s/GPU", "value": value, "unit": "accepted tokens/s",
        "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": wl.name, "trees_per_gpu": wl.T, "nodes_per_gpu": wl.trees.total_rows,
                   "vocab": wl.vocab, "rule": "scan (Philox per node)", "parallelism": f"dp{world}",
                   "l2": "flushed between timed steps (512 MB write); ms_per_step = mean per-step event span "
                         "(acceptance + commit), flush excluded",
                   "ms_per_step_with_flush": ms_with_flush},
        "roofline": {"bound": "hbm", "kernel": "accept_probs_kernel", "achieved": accept_gbs, "peak": hbm,
                     "peak_kind": peak_kind, "unit": "GB/s", "frac": accept_gbs / hbm,
                     "traffic": NCU_ACCEPT_TRAFFIC_CFG2,
                     "algorithmic_bytes_per_launch": accept_bytes,
                     "launch_ms": statistics.mean(accept_ms),
                     "commit": {"achieved": commit_gbs, "frac": commit_gbs / hbm,
                                "bytes_per_launch": commit_bytes, "moved_bytes_per_launch": moved_bytes,
                                "launch_ms": statistics.mean(commit_ms)}},
        "cpu_baseline": cpu, "clocks": clk, "e2e": e2e, "gpu_launches": launches,
    }
    return line


def e2e_accept(wl, args, world):
    from specgrove_b200.sampling import PackedTrees, accept_packed
    probs_host = wl.probs.cpu().pin_memory()
    parents, tokens = wl.batch.flat()
    meta_host = torch.from_numpy(np.concatenate([np.asarray(wl.batch.row_offsets, np.int64), parents,
                                                 tokens])).pin_memory()
    probs_dev = torch.empty_like(wl.probs)
    meta_dev = torch.empty_like(meta_host, device="cuda")
    out_host = torch.empty((wl.T, wl.D + 2), dtype=torch.long).pin_memory()
    out_dev = torch.empty((wl.T, wl.D + 2), dtype=torch.long, device="cuda")
    n = len(wl.batch.row_offsets)
    trees = PackedTrees.__new__(PackedTrees)
    trees.count, trees.max_depth, trees.max_nodes = wl.T, wl.D, wl.trees.max_nodes
    trees.total_rows = wl.trees.total_rows
    trees.row_offsets = meta_dev[:n]
    trees.parents = meta_dev[n:n + trees.total_rows]
    trees.tokens = meta_dev[n + trees.total_rows:]
    steps = max(2, min(args.steps, 5))
    units = 0

    def one(seed):
        probs_dev.copy_(probs_host, non_blocking=True)
        meta_dev.copy_(meta_host, non_blocking=True)
        accept_packed(probs_dev, trees, seed=seed, request_ids=wl.request_ids, out=out_dev)
        out_host.copy_(out_dev, non_blocking=True)

    one(123)
    torch.cuda.synchronize()
    barrier(world)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for i in range(steps):
        one(i)
        torch.cuda.current_stream().synchronize()
        units += int((out_host[:, wl.D] + 1).sum())
    stop.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(start.elapsed_time(stop) / steps, world)
    total = sum_over_ranks(units, world)
    return {"value": total / (ms * steps / 1000.0), "unit": "accepted tokens/s",
            "h2d_bytes_per_step": probs_host.numel() * 4 + meta_host.numel() * 8,
            "d2h_bytes_per_step": out_host.numel() * 8, "steps": steps, "ms_per_step": ms}


def cpu_baseline_accept(wl, arith=None):
    """The reference's rule (sequential fp64 running sums, the CPU helper of
    fused_tree_sampling.py:2607-2612) over the same trees, all host cores."""
    from oracle import cpu as oracle
    probs = wl.probs.cpu().numpy()
    parents, tokens = wl.batch.flat()
    arith = oracle.ARITH_FP64 if arith is None else arith
    rng = np.random.default_rng(0)
    units, seconds, reps = 0, 0.0, 0
    while seconds < 10.0 and reps < 50:
        uniforms = rng.random((wl.T, wl.D + 1))
        t0 = time.perf_counter()
        out, _ = oracle.accept_probs(probs, wl.batch.row_offsets, parents, tokens, wl.D, uniforms=uniforms,
                                     arith=arith)
        seconds += time.perf_counter() - t0
        units += int((out[:, wl.D] + 1).sum())
        reps += 1
    return {"value": units / seconds, "unit": "accepted tokens/s", "cores": os.cpu_count(),
            "kind": "port", "sample": f"{reps} full acceptance steps (64 trees, explicit uniforms, "
                                      "fp64 running-sum rule); KV commit not included"}


def run_reference(args, world, rank):
    """The reference's CPU path for the same workload and metric: the oracle
    port (the reference's step restated in torch fp32 / C), all host cores."""
    if rank != 0:
        return None
    if args.workload == "accept":
        wl = AcceptWorkload(rank)
        cpu = cpu_baseline_accept(wl)
        dtype = "fp64"
    else:
        wl = VerifyWorkload(rank, args.workload, args.layers)
        cpu = cpu_baseline_verify(wl, requests=2, budget_s=10.0)
        dtype = "fp32"
    line = {"impl": "reference", "metric": "accepted tokens/s/GPU", "value": cpu["value"],
            "unit": "accepted tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype,
            "data": "synthetic", "config": {"workload": wl.name, "parallelism": "cpu"},
            "cpu_baseline": cpu, "e2e": {"value": cpu["value"], "unit": "accepted tokens/s",
                                         "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    return line


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="verify", choices=["verify", "verify4b", "accept"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--layers", type=int, default=None,
                    help="profiling only: build the model with this many layers (not a benchmark number)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            line = run_reference(args, world, rank)
        elif args.workload == "accept":
            line = run_b200(args, world, rank)
        else:
            line = run_verify(args, world, rank)
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
