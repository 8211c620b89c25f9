"""Benchmark of the specgrove_b200 packed tree-verification step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                    [--workload verify|verify4b|accept]

One JSON line is printed by rank 0.  Under torchrun (N > 1) every rank runs
its own shard of requests with a full model replica (data parallel, no
data-path collective; weak scaling); the step time is the max over ranks of
the CUDA-event time and `value` is the accepted tokens of ALL ranks per
second (`per_gpu` divides it by N).

Workload `verify` (default): Qwen3-8B shape
(36 layers, hidden 4096, 32 q / 8 kv heads, head_dim 128, intermediate 12288,
vocab 151936), random-init bf16 weights, 64 requests per GPU with cache
prefixes uniform in [1024, 4096] (synthetic KV), one canonical best-first
tree per request cut to its tier (tier mix 40x16 + 12x32 + 8x64 + 4x128 rows
= 2048 rows).  One step = one packed verify pass: target forward over the
2048 rows, LM head fused with softmax and sampling, tree walk, and commit of
the accepted rows' KV.  Weights (16.4 GB) and KV (~24 GB read per step) are
far larger than L2, so no flush is needed.  At N = 1 the same line nests the
configuration-2 acceptance sweep and the configuration-3 (Qwen3-4B shape)
pass, measured in the same run.
`verify4b` is configuration 3 (Qwen3-4B shape, 16 requests, 512 rows);
`accept` is the kernel-isolated acceptance sweep (configuration 2);
`draft` prints only the nested drafter block (below).

Also nested at N = 1: `draft`, the step before each wave at the
configuration-4 geometry (DFlash drafter of Qwen3-8B shape over the 64
requests' draft caches, then the on-device wave plan: proposals, trees, tier
knapsack, packed wave), and at every N `config5`, the open-loop serving run.

`--impl reference` times the reference's CPU path (restated in oracle/: torch
fp32 target pass with the packed tree mask, fp32 softmax, the reference's
fp64 inverse-CDF walk, KV commit) on the host cores, on a bounded sample of
the same wave; it never loads the CUDA library.
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
METRIC = "accepted tokens/s (total over GPUs)"
UNIT = "accepted tokens/s"

# DRAM bytes (read + write) per launch from ncu captures of the same kernels
# (profiles/): the layer-0 tree attention and gate/up + SwiGLU GEMM on the
# configuration-4 wave, and the acceptance launch of the configuration-2 sweep.
NCU_ATTENTION_TRAFFIC_CFG4 = 736.275200e6 + 15.357440e6
NCU_SWIGLU_TRAFFIC_CFG4 = 218.211840e6 + 39.758592e6
NCU_ACCEPT_TRAFFIC_CFG2 = 53.622528e6 + 0.811264e6


def peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    return 6650.0, 1590.0, 1400.0, "fallback"


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def product_library_loaded() -> bool:
    """Whether this process has mapped libspecgrove_b200.so."""
    try:
        return "libspecgrove_b200.so" in Path("/proc/self/maps").read_text()
    except OSError:
        return False


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
    elif torch.cuda.is_available():
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


def make_events(n):
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
    for e in evs:           # materialise the cudaEvent_t handles
        e.record()
    torch.cuda.synchronize()
    return evs


# ---------------------------------------------------------------------------
# Acceptance sweep (configuration 2)
# ---------------------------------------------------------------------------
class AcceptWorkload:
    name = "config2: acceptance sweep, 64 trees / 4096 nodes / V=151936 fp32 probs + KV commit 36x8x128 bf16"

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


def measure_accept(args, world, rank, wl=None):
    """Acceptance + commit steps of configuration 2, L2 flushed between steps."""
    from specgrove_b200 import _lib
    hbm, _, _, peak_kind = peaks()
    wl = wl or AcceptWorkload(rank)
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
    barrier(world)
    torch.cuda.synchronize()
    # A step is two short kernels (~tens of us), less than the host needs to
    # enqueue it; a device sleep ahead of the start event lets the host queue
    # all K steps first, so the events time the kernels back to back instead
    # of the host's enqueue gaps.
    torch.cuda._sleep(int(4_000_000 * K))
    start.record()
    for i in range(K):
        flush.fill_(i & 0xFF)
        wl.step(i, outs[i], ev[i])
    stop.record()
    torch.cuda.synchronize()
    barrier(world)
    launches = _lib.launch_count() - launches0
    ms_local = statistics.mean(e[0].elapsed_time(e[2]) for e in ev)
    ms = max_over_ranks(ms_local, world)
    total_units = sum_over_ranks(wl.units(outs), world)
    if int(wl.status) != 0:
        raise RuntimeError(f"device status {int(wl.status)}")
    accept_ms = [e[0].elapsed_time(e[1]) for e in ev]
    commit_ms = [e[1].elapsed_time(e[2]) for e in ev]
    visited = (outs[..., wl.D] + 1).double()        # scan rule: accepted + exit row
    accept_bytes = float(visited.sum()) / K * wl.vocab * 4
    # kept tokens x 147,456 B, read and written (the reference's append copies
    # every kept row); the root row and rows already at their final position
    # never move, so the bytes actually moved are fewer
    commit_bytes = float(visited.sum()) / K * KV_BYTES_PER_TOKEN * 2
    moved = outs[..., :wl.D] >= 0
    depth_idx = torch.arange(1, wl.D + 1, device=outs.device).expand_as(moved)
    moved_rows = float((moved & (outs[..., :wl.D] != depth_idx)).sum()) / K
    accept_gbs = accept_bytes / (statistics.mean(accept_ms) / 1000) / 1e9
    commit_gbs = commit_bytes / (statistics.mean(commit_ms) / 1000) / 1e9
    # The decoder's default verifier (terminal mass) on the same trees: it
    # reads every internal node's row once plus each tree's terminal row.
    from specgrove_b200.sampling import terminal_mass_packed
    tm_out = torch.empty((wl.T, wl.D + 2), dtype=torch.long, device="cuda")
    for i in range(W):
        terminal_mass_packed(wl.probs, wl.trees, seed=20_000 + i, request_ids=wl.request_ids, out=tm_out,
                             status=wl.status)
    tm_ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    torch.cuda.synchronize()
    for i in range(K):
        flush.fill_(i & 0xFF)
        tm_ev[i][0].record()
        terminal_mass_packed(wl.probs, wl.trees, seed=30_000 + i, request_ids=wl.request_ids, out=tm_out,
                             status=wl.status)
        tm_ev[i][1].record()
    torch.cuda.synchronize()
    if int(wl.status) != 0:
        raise RuntimeError(f"device status {int(wl.status)}")
    tm_ms = statistics.mean(a.elapsed_time(b) for a, b in tm_ev)
    internal_rows = sum(len(set(p[1:])) for p in wl.batch.parents)
    tm_bytes = float(internal_rows + wl.T) * wl.vocab * 4
    return {
        "workload": wl.name, "value": total_units / (ms * K / 1000.0), "unit": UNIT, "ms_per_step": ms,
        "launches": launches, "rule": "scan (Philox per node)",
        "l2": "flushed between timed steps (512 MB write); ms_per_step = mean per-step event span "
              "(acceptance + commit), flush excluded",
        "ms_per_step_with_flush": start.elapsed_time(stop) / K,
        "acceptance": {"bound": "hbm", "kernel": "accept_probs_kernel", "achieved": accept_gbs, "peak": hbm,
                       "peak_kind": peak_kind, "unit": "GB/s", "frac": accept_gbs / hbm,
                       "traffic": NCU_ACCEPT_TRAFFIC_CFG2, "algorithmic_bytes_per_launch": accept_bytes,
                       "launch_ms": statistics.mean(accept_ms)},
        "terminal_mass": {"bound": "hbm", "kernel": "row_mass_kernel + terminal_kernel (two launches)",
                          "achieved": tm_bytes / (tm_ms / 1000) / 1e9, "peak": hbm, "unit": "GB/s",
                          "frac": tm_bytes / (tm_ms / 1000) / 1e9 / hbm, "algorithmic_bytes_per_call": tm_bytes,
                          "internal_rows": internal_rows, "call_ms": tm_ms},
        "commit": {"bound": "hbm", "kernel": "kv_commit_accepted_kernel", "achieved": commit_gbs, "peak": hbm,
                   "unit": "GB/s", "frac": commit_gbs / hbm, "algorithmic_bytes_per_launch": commit_bytes,
                   "moved_bytes_per_launch": moved_rows * KV_BYTES_PER_TOKEN * 2,
                   "launch_ms": statistics.mean(commit_ms)},
    }


# ---------------------------------------------------------------------------
# Verify pass (configurations 3 and 4)
# ---------------------------------------------------------------------------
def wave_spec(config: str):
    from specgrove_b200 import workloads
    from specgrove_b200.engine import QWEN3_4B, QWEN3_8B
    if config == "verify4b":
        return (QWEN3_4B, workloads.TIER_MIX_CONFIG3, (512, 2048),
                "config3: Qwen3-4B shape, 16 requests, prefixes U[512,2048], tiers {16,32,64}, 512 rows")
    return (QWEN3_8B, workloads.TIER_MIX_CONFIG4, (1024, 4096),
            "config4: Qwen3-8B shape, 64 requests, prefixes U[1024,4096], tiers {16,32,64,128}, 2048 rows")


class VerifyWorkload:
    def __init__(self, rank: int, config: str, layers: int | None = None):
        from specgrove_b200 import workloads
        from specgrove_b200.engine import B200Engine, Wave, Weights
        self.shape, mix, prefix, self.name = wave_spec(config)
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

    def close(self):
        self.engine.close()
        del self.engine, self.weights, self.dw

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


def measure_verify(args, world, rank, wl):
    """K untraced steps timed as one event span (max over ranks), then a few
    traced steps for the per-stage split."""
    from specgrove_b200 import _lib
    from specgrove_b200.engine import TRACE_EVENTS, TRACE_STAGES
    K, W = args.steps, args.warmup
    outs = torch.empty((K, wl.R, wl.D + 2), dtype=torch.long, device="cuda")
    warm = torch.empty((wl.R, wl.D + 2), dtype=torch.long, device="cuda")
    for i in range(W):
        wl.step(10_000 + i, warm)
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = _lib.launch_count()
    with ClockSampler(torch.cuda.current_device()) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        start.record()
        for i in range(K):
            wl.step(i, outs[i])
        stop.record()
        torch.cuda.synchronize()
        barrier(world)
    launches = _lib.launch_count() - launches0
    if int(wl.engine.status) != 0:
        raise RuntimeError(f"device status {int(wl.engine.status)}")
    ms = max_over_ranks(start.elapsed_time(stop) / K, world)
    total_units = sum_over_ranks(wl.units(outs), world)
    # stage split from separate traced steps (events between the kernels)
    traces = [make_events(TRACE_EVENTS) for _ in range(3)]
    for i, t in enumerate(traces):
        wl.step(20_000 + i, warm, t)
    torch.cuda.synchronize()
    stages = {name: statistics.mean(t[i].elapsed_time(t[i + 1]) for t in traces)
              for i, name in enumerate(TRACE_STAGES)}
    return dict(ms=ms, units=total_units, value=total_units / (ms * K / 1000.0), launches=launches,
                stages=stages, clocks=clocks.summary(), outs=outs)


def verify_rooflines(wl, m):
    hbm, tc, tc_sus, peak_kind = peaks()
    stages, ms = m["stages"], m["ms"]
    attn_ms = stages["L0 attention"]
    attn_bytes = wl.attention_bytes()                  # one layer's K/V reads
    attn_gbs = attn_bytes / (attn_ms / 1000) / 1e9
    flops = wl.pass_flops()
    pass_tflops = flops / (ms / 1000) / 1e12
    gu_ms = stages["L0 gate/up gemm"]
    gu_flops = 2.0 * wl.rows * (2 * wl.shape.intermediate) * wl.shape.hidden
    gu_tflops = gu_flops / (gu_ms / 1000) / 1e12
    cfg4 = wl.name.startswith("config4")
    # dominant kernel by time: the gate/up GEMM with the SwiGLU epilogue
    # (timed inside the step, so against the sustained bf16 peak)
    return {"bound": "tensor", "kernel": "gemm_kernel<EpiSwiGlu> (layer 0 gate/up)",
            "achieved": gu_tflops, "peak": tc_sus, "peak_kind": peak_kind + " sustained",
            "unit": "TFLOP/s", "frac": gu_tflops / tc_sus,
            "traffic": NCU_SWIGLU_TRAFFIC_CFG4 if cfg4 else None,
            "traffic_source": "ncu capture, profiles/gemm_swiglu_cfg4_small.md" if cfg4 else None,
            "algorithmic_flops_per_launch": gu_flops, "launch_ms": gu_ms,
            "attention": {"bound": "hbm", "kernel": "tree_attention_tm_kernel (layer 0)",
                          "achieved": attn_gbs, "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s",
                          "frac": attn_gbs / hbm,
                          "traffic": NCU_ATTENTION_TRAFFIC_CFG4 if cfg4 else None,
                          "algorithmic_bytes_per_launch": attn_bytes, "launch_ms": attn_ms},
            "pass": {"bound": "tensor", "achieved": pass_tflops, "peak": tc_sus, "unit": "TFLOP/s",
                     "frac": pass_tflops / tc_sus, "algorithmic_flops_per_step": flops,
                     "peak_kind": peak_kind + " sustained",
                     "vs_burst_peak": {"peak": tc, "frac": pass_tflops / tc}}}


def run_verify(args, world, rank):
    wl = VerifyWorkload(rank, args.workload, args.layers)
    m = measure_verify(args, world, rank, wl)
    e2e = e2e_verify(wl, args, world)
    ms, value = m["ms"], m["value"]
    line = {
        "metric": METRIC, "value": value, "unit": UNIT,
        "per_gpu": {"metric": "accepted tokens/s/GPU", "value": value / world},
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, "
        "synthetic KV prefixes, seeded best-first trees)",
        "config": {"workload": wl.name, "model": "Qwen3-8B shape" if wl.shape.hidden == 4096 else "Qwen3-4B shape",
                   "collective": "per-step NCCL all_gather_into_tensor of allocator scores" if world > 1 else None,
                   "requests_per_gpu": wl.R, "rows_per_gpu": wl.rows, "global_batch_rows": wl.rows * world,
                   "verify_pass_us_per_row": ms * 1000 / wl.rows, "temperature": 1.0,
                   "parallelism": f"dp{world}", "l2": "inputs larger than L2 (16.4 GB weights, ~24 GB KV/step)",
                   "timing": "K untraced steps between two events; stages_ms from 3 separate traced steps"},
        "roofline": verify_rooflines(wl, m),
        "stages_ms": {k: round(v, 4) for k, v in m["stages"].items()},
        "profiling_only": args.layers is not None and args.layers != 36,
        "clocks": m["clocks"], "e2e": e2e, "gpu_launches": m["launches"],
    }
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline_verify(wl)
    line["cpu_baseline"] = cpu
    if not args.no_nested and args.layers is None and args.workload == "verify":
        weights = wl.weights
        wl.close()
        del wl
        torch.cuda.empty_cache()
        nested = nested_configs(args, world, rank) if world == 1 else {}
        if world == 1:
            nested["draft"] = measure_draft(args, world, rank, weights)
        nested["config5"] = measure_serving(args, world, rank, weights)
        line["nested"] = nested
    return line


# Synthetic monotone wave-cost curve (rows -> ms) for the allocator, shaped
# like the measured configuration-4 pass (a fixed part, then ~17 us per row).
SERVE_COST_CURVE = [(16, 2.0), (256, 5.5), (512, 9.0), (1024, 17.5), (2048, 34.7)]


def measure_serving(args, world, rank, weights=None):
    """Configuration 5: open-loop serving of the Qwen3-8B shape, requests
    partitioned over the ranks, with the per-wave NCCL allgather of allocator
    scores.  Default mode `spec`: the full speculative step (real chunked
    prefill of each admitted prompt into the target's arena and the draft
    cache, then per wave the DFlash drafter, the on-device wave plan and one
    verify pass); mode `synthetic`: synthetic prompt KV and host-built trees,
    one verify pass per wave.  The makespan is the CUDA-event span of the
    whole serving loop on each rank (max over ranks)."""
    if args.serve_mode == "spec":
        return measure_serving_spec(args, world, rank, weights)
    from specgrove_b200 import _lib
    from specgrove_b200.allocator import ScoreExchange
    from specgrove_b200.engine import QWEN3_8B, B200Engine, Wave, Weights
    from specgrove_b200.serving import OpenLoopServer, make_requests
    shape = QWEN3_8B
    weights = weights or Weights.random(shape, seed=1234)
    tiers = [16, 32, 64, 128]
    n_req, rate, max_new = args.serve_requests, 8.0 * world, 256
    requests = make_requests(n_req, rate, (256, 8192), tiers, shape.vocab, seed=5)
    slots = 64
    capacity = 8192 + max_new + max(tiers) + 16
    engine = B200Engine(weights, num_slots=slots, capacity=capacity, max_rows=2048, max_requests=slots)
    gen = torch.Generator(device="cuda").manual_seed(77 + rank)
    engine.arena.storage.normal_(0.0, 1.0, generator=gen)            # synthetic prompt KV

    def step(trees, slot_ids, lengths, rids, seed):
        wave = Wave(trees, slot_ids, lengths, request_ids=rids)
        out = engine.verify_device(wave.to("cuda"), seed=seed, commit=True)
        return out[:, wave.max_depth].cpu().tolist()

    exchange = ScoreExchange(slots, len(tiers), "cuda")
    server = OpenLoopServer(requests, step, rank=rank, world=world, exchange=exchange, num_slots=slots,
                            capacity=capacity, tier_rows=tiers, row_budget=2048, max_new_tokens=max_new,
                            row_cost_curve=SERVE_COST_CURVE)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = _lib.launch_count()
    with ClockSampler(torch.cuda.current_device()) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        start.record()
        stats = server.run(seed=1_000_000 * rank)
        stop.record()
        torch.cuda.synchronize()
        barrier(world)
    if int(engine.status) != 0:
        raise RuntimeError(f"device status {int(engine.status)}")
    span_ms = start.elapsed_time(stop)
    makespan = max_over_ranks(span_ms, world)
    tokens = sum_over_ranks(stats.tokens, world)
    waves = max_over_ranks(stats.waves, world)
    lat = sorted(stats.finish_times)
    engine.close()
    del engine
    torch.cuda.empty_cache()
    return {"workload": f"config5: Qwen3-8B shape, {n_req} requests, Poisson {8.0:g} req/s per GPU, prompts "
                        f"log-uniform [256, 8192] (synthetic KV), {max_new} tokens each, tiers {{16,32,64,128}}, "
                        "service weights U{1,2,4}, 2048-row budget per GPU, least-loaded admission",
            "metric": METRIC, "value": tokens / (makespan / 1000.0), "unit": UNIT, "n_gpus": world,
            "makespan_ms": makespan, "tokens": tokens, "waves_max_rank": waves,
            "rows_per_wave_rank0": stats.rows / max(1, stats.waves), "host_ms_rank0": stats.host_ms,
            "requests_rank0": stats.requests, "exchanges": stats.exchanges,
            "latency_s_rank0": {"p50": lat[len(lat) // 2] if lat else None, "max": lat[-1] if lat else None},
            "collective": "per-wave NCCL all_gather_into_tensor of allocator scores + clock/load/done header"
                          if world > 1 else "none (one rank)",
            "gpu_launches": _lib.launch_count() - launches0, "clocks": clocks.summary()}


def measure_serving_spec(args, world, rank, weights=None):
    from specgrove_b200 import _lib
    from specgrove_b200.allocator import ScoreExchange
    from specgrove_b200.drafter import QWEN3_8B_DFLASH, QWEN3_8B_DFLASH_FEATURE_LAYERS, B200Drafter, DraftWeights
    from specgrove_b200.engine import QWEN3_8B, B200Engine, Weights
    from specgrove_b200.serving import SpecServer, make_prompts, make_requests
    from specgrove_b200.speculative import SpecDecoder
    shape = QWEN3_8B
    weights = weights or Weights.random(shape, seed=1234)
    dweights = DraftWeights.random(QWEN3_8B_DFLASH, weights, seed=4321)
    tiers = [16, 32, 64, 128]
    n_req, rate, max_new = args.serve_requests, 8.0 * world, 256
    requests = make_requests(n_req, rate, (256, 8192), tiers, shape.vocab, seed=5)
    prompts = make_prompts(requests, shape.vocab, seed=6)
    slots = 64
    capacity = 8192 + max_new + max(tiers) + 16
    target = B200Engine(weights, num_slots=slots, capacity=capacity, max_rows=2048, max_requests=slots)
    drafter = B200Drafter(dweights, num_slots=slots, capacity=capacity, max_requests=slots, max_update_rows=2048)
    decoder = SpecDecoder(target, drafter, QWEN3_8B_DFLASH_FEATURE_LAYERS, tiers=[t - 1 for t in tiers],
                          row_budget=2048, temperature=1.0, row_cost_curve=SERVE_COST_CURVE, seed=1_000_000 * rank)
    exchange = ScoreExchange(slots, len(tiers), "cuda")
    server = SpecServer(requests, decoder, prompts, rank=rank, world=world, exchange=exchange,
                        num_tiers=len(tiers), max_new_tokens=max_new)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    launches0 = _lib.launch_count()
    with ClockSampler(torch.cuda.current_device()) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        start.record()
        stats = server.run()
        stop.record()
        torch.cuda.synchronize()
        barrier(world)
    span_ms = start.elapsed_time(stop)
    makespan = max_over_ranks(span_ms, world)
    tokens = sum_over_ranks(stats.tokens, world)
    waves = max_over_ranks(stats.waves, world)
    lat = sorted(stats.finish_times)
    prompt_tokens = sum(r.prompt_len for r in requests if r.rank == rank)
    target.close()
    drafter.close()
    del target, drafter, decoder
    torch.cuda.empty_cache()
    return {"workload": f"config5: Qwen3-8B shape + DFlash drafter (5 layers, block 16), {n_req} requests, Poisson "
                        f"{8.0:g} req/s per GPU, prompts log-uniform [256, 8192] (random tokens, prefilled into the "
                        f"target arena and the draft cache on admission), {max_new} tokens each, tiers "
                        "{16,32,64,128}, service weights U{1,2,4}, 2048-row budget per GPU, least-loaded admission; "
                        "each wave = drafter + on-device plan + verify",
            "mode": "spec", "metric": METRIC, "value": tokens / (makespan / 1000.0), "unit": UNIT, "n_gpus": world,
            "makespan_ms": makespan, "tokens": tokens, "waves_max_rank": waves,
            "prompt_tokens_rank0": prompt_tokens, "decoder_steps_rank0": stats.waves,
            "rows_committed_rank0": stats.rows, "rows_per_wave_rank0": stats.rows_verified / max(1, stats.waves),
            "prefill_ms_rank0": stats.admit_ms, "step_ms_rank0": stats.step_ms,
            "step_ms_per_wave_rank0": stats.step_ms / max(1, stats.waves), "host_ms_rank0": stats.host_ms,
            "requests_rank0": stats.requests, "exchanges": stats.exchanges,
            "latency_s_rank0": {"p50": lat[len(lat) // 2] if lat else None, "max": lat[-1] if lat else None},
            "collective": "per-wave NCCL all_gather_into_tensor of allocator scores + clock/load/done header"
                          if world > 1 else "none (one rank)",
            "gpu_launches": _lib.launch_count() - launches0, "clocks": clocks.summary()}


def measure_plan(args):
    """The on-device wave plan alone (a small, profiler-sized case): 64
    requests x 15 draft positions x the Qwen3 vocabulary of N(0, 2.5^2) bf16
    logits, top-128 proposals, 128-node trees, tiers {16, 32, 64, 128}, the
    2048-row knapsack on the serving cost curve and the packed wave."""
    from specgrove_b200 import _lib
    from specgrove_b200.draft_tree import plan_wave
    R, D, V = 64, 15, 151936
    g = torch.Generator(device="cuda").manual_seed(17)
    logits = (torch.randn((R, D, V), generator=g, device="cuda") * 2.5).to(torch.bfloat16)
    anchors = torch.randint(0, V, (R,), generator=g, device="cuda")
    wts = 1.0 + torch.rand(R, generator=g, device="cuda", dtype=torch.float64)
    tiers = [16, 32, 64, 128]

    def once():
        return plan_wave(logits, 1.0, tiers, wts, anchors, row_budget=2048, row_cost_curve=SERVE_COST_CURVE)

    for _ in range(args.warmup):
        once()
    torch.cuda.synchronize()
    launches0 = _lib.launch_count()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        plan = once()
    stop.record()
    torch.cuda.synchronize()
    if int(plan.status.max()) != 0:
        raise RuntimeError(f"plan status {plan.status.tolist()}")
    return {"workload": "plan: 64 requests x 15 positions x 151936 vocab (bf16 N(0, 2.5^2)), top-128, 128-node "
                        "trees, tiers {16,32,64,128}, 2048-row knapsack, packed wave",
            "ms_per_plan_eager": start.elapsed_time(stop) / args.steps, "steps": args.steps,
            "gpu_launches": _lib.launch_count() - launches0, "rows": int(plan.row_offsets[-1])}


def measure_draft(args, world, rank, weights):
    """The step before each wave at the configuration-4 geometry: the DFlash
    drafter of Qwen3-8B shape (5 layers, block 16) over 64 requests whose
    draft caches hold L_i ~ U[1024, 4096] context rows (synthetic K/V), each
    appending 1-4 new context rows (the previous wave's kept rows), then the
    on-device wave plan from block rows 1..15: top-128 proposals per depth,
    128-node best-first trees, tier utilities for {16, 32, 64, 128}, the
    2048-row tier knapsack and the packed wave.  Device-timed with events."""
    from specgrove_b200 import _lib
    from specgrove_b200.allocator import allocate_tree_budgets_device
    from specgrove_b200.draft_tree import build_draft_trees, pack_tree_wave, plan_wave, proposal_topk
    from specgrove_b200.drafter import QWEN3_8B_DFLASH, B200Drafter, DraftWeights
    shape = QWEN3_8B_DFLASH
    dw = DraftWeights.random(shape, weights, seed=99)
    R, B, V, H = 64, shape.block_size, shape.vocab, shape.hidden
    g = torch.Generator().manual_seed(4321)
    prefix = torch.randint(1024, 4097, (R,), generator=g)
    upd = torch.randint(1, 5, (R,), generator=g)
    U = int(upd.sum())
    capacity = 4096 + 4 + B + 12
    drafter = B200Drafter(dw, num_slots=R, capacity=capacity, max_requests=R, max_update_rows=U)
    drafter.arena.storage.normal_(0.0, 1.0, generator=torch.Generator(device="cuda").manual_seed(5 + rank))
    dev = "cuda"
    slots = torch.arange(R, device=dev)
    cache_len = prefix.to(dev)
    offsets = torch.cat([torch.zeros(1, dtype=torch.long), upd.cumsum(0)]).to(dev)
    feats = (torch.randn((U, shape.num_feature_layers * H), generator=g) * 2).to(torch.bfloat16).to(dev)
    anchors = torch.randint(0, V, (R,), generator=g).to(dev)
    logits = torch.empty((R, B, V), dtype=torch.bfloat16, device=dev)
    tiers = [16, 32, 64, 128]
    wts = (1.0 + torch.rand(R, generator=g, dtype=torch.float64)).to(dev)

    def draft():
        drafter.draft_device(slots, cache_len, offsets, feats, anchors, U, logits_out=logits)

    def plan():
        return plan_wave(logits[:, 1:B], 1.0, tiers, wts, anchors, row_budget=2048, row_cost_curve=SERVE_COST_CURVE)

    def timed(fn, steps):
        """Eager calls: host enqueue included (Python, ctypes, allocations)."""
        ev = make_events(2)
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        ev[0].record()
        for _ in range(steps):
            fn()
        ev[1].record()
        torch.cuda.synchronize()
        return ev[0].elapsed_time(ev[1]) / steps

    def graphed(fn, steps):
        """The calls captured once in a CUDA graph and replayed: device time
        of the kernels, without the host's per-call enqueue work."""
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for _ in range(args.warmup):
                fn()
        torch.cuda.current_stream().wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        for _ in range(args.warmup):
            graph.replay()
        ev = make_events(2)
        ev[0].record()
        for _ in range(steps):
            graph.replay()
        ev[1].record()
        torch.cuda.synchronize()
        del graph
        return ev[0].elapsed_time(ev[1]) / steps

    steps = max(3, args.steps)
    launches0 = _lib.launch_count()
    lq, ids = proposal_topk(logits[:, 1:B], 1.0, 128)
    trees = build_draft_trees(lq, ids, 128, tiers=tiers)
    alloc = allocate_tree_budgets_device(wts, tiers, trees.utilities, row_budget=2048,
                                         row_cost_curve=SERVE_COST_CURVE)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        draft_ms = graphed(draft, steps)
        plan_ms = graphed(plan, steps)
        both_ms = graphed(lambda: (draft(), plan()), steps)
        eager_ms = timed(lambda: (draft(), plan()), steps)
        launches = (_lib.launch_count() - launches0) / (4 * (steps + args.warmup) + 3)
        topk_ms = graphed(lambda: proposal_topk(logits[:, 1:B], 1.0, 128), steps)
        trees_ms = graphed(lambda: build_draft_trees(lq, ids, 128, tiers=tiers), steps)
        alloc_ms = graphed(lambda: allocate_tree_budgets_device(wts, tiers, trees.utilities, row_budget=2048,
                                                                row_cost_curve=SERVE_COST_CURVE), steps)
        pack_ms = graphed(lambda: pack_tree_wave(trees, alloc, anchors, 2048), steps)
    p = plan()
    torch.cuda.synchronize()
    if int(drafter.status.item()) != 0 or int(p.status.item()) != 0:
        raise RuntimeError(f"drafter status {int(drafter.status.item())}, plan status {int(p.status.item())}")
    s = shape
    qkvo = H * (s.num_q_heads + 2 * s.num_kv_heads) * s.head_dim + s.num_q_heads * s.head_dim * H
    per_layer = qkvo + 3 * H * s.intermediate
    Q = R * B
    gemm_flops = 2 * (Q * s.num_layers * per_layer + U * (s.num_feature_layers * H * H +
                      s.num_layers * 2 * s.num_kv_heads * s.head_dim * H) + Q * H * V)
    keys = float(((prefix + upd + B) * B).sum())
    attn_flops = 4 * s.num_q_heads * s.head_dim * s.num_layers * keys
    flops = gemm_flops + attn_flops
    hbm, _, tf_sustained, peak_kind = peaks()
    topk_bytes = R * (B - 1) * V * 2
    result = {
        "workload": "DFlash drafter (Qwen3-8B shape, 5 layers, block 16) over 64 requests, draft caches "
                    "U[1024,4096] + 1-4 new context rows, then top-128 proposals x 15 depths, 128-node trees, "
                    "tiers {16,32,64,128}, 2048-row knapsack, packed wave",
        "timing": "CUDA-graph replays (device time); eager_draft_plus_plan_ms: the same calls enqueued from "
                  "Python each step",
        "draft_ms": draft_ms, "plan_ms": plan_ms, "draft_plus_plan_ms": both_ms,
        "eager_draft_plus_plan_ms": eager_ms,
        "plan_parts_ms": {"proposal_topk": topk_ms, "trees": trees_ms, "allocate": alloc_ms, "pack": pack_ms},
        "draft_pass": {"tflop": flops / 1e12, "achieved_tflops": flops / (draft_ms * 1e-3) / 1e12,
                       "frac_of_sustained": flops / (draft_ms * 1e-3) / 1e12 / tf_sustained,
                       "peak": f"{tf_sustained} TFLOP/s sustained bf16 ({peak_kind})"},
        "proposal_topk": {"algorithmic_gb": topk_bytes / 1e9,
                          "achieved_gbs": topk_bytes / (topk_ms * 1e-3) / 1e9,
                          "frac_of_hbm": topk_bytes / (topk_ms * 1e-3) / 1e9 / hbm,
                          "peak": f"{hbm} GB/s ({peak_kind})"},
        "gpu_launches_per_call": launches, "clocks": clocks.summary()}
    drafter.close()
    del drafter, dw
    torch.cuda.empty_cache()
    return result


def nested_configs(args, world, rank):
    """Configurations 2 and 3 measured in the same run as the headline."""
    out = {}
    acc = AcceptWorkload(rank)
    out["config2"] = measure_accept(args, world, rank, acc)
    del acc
    torch.cuda.empty_cache()
    wl3 = VerifyWorkload(rank, "verify4b")
    m3 = measure_verify(args, world, rank, wl3)
    r3 = verify_rooflines(wl3, m3)
    out["config3"] = {"workload": wl3.name, "value": m3["value"], "unit": UNIT, "ms_per_step": m3["ms"],
                      "verify_pass_us_per_row": m3["ms"] * 1000 / wl3.rows, "rows": wl3.rows,
                      "pass": r3["pass"], "gate_up_gemm": {k: r3[k] for k in ("achieved", "frac", "launch_ms")},
                      "attention": {k: r3["attention"][k] for k in ("achieved", "frac", "launch_ms")},
                      "stages_ms": {k: round(v, 4) for k, v in m3["stages"].items()}}
    wl3.close()
    del wl3
    torch.cuda.empty_cache()
    return out


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
    return {"value": total / (ms * steps / 1000.0), "unit": UNIT,
            "h2d_bytes_per_step": host.numel() * 8, "d2h_bytes_per_step": out_host.numel() * 8,
            "steps": steps, "ms_per_step": ms}


# ---------------------------------------------------------------------------
# CPU path: the reference's step restated in oracle/ (torch fp32 + C walk)
# ---------------------------------------------------------------------------
class HostWeights:
    """Random-init fp32 weights of a Qwen3 shape on the host, in the engine's
    packed layout (oracle.forward.CpuWeights reads them).  One random layer
    is generated and used by every layer: each layer's arithmetic is that of a
    distinct random layer, without generating 8 B distinct host values."""

    def __init__(self, shape, seed: int):
        g = torch.Generator().manual_seed(seed)
        H, D, I = shape.hidden, shape.head_dim, shape.intermediate
        nq, nkv = shape.num_q_heads, shape.num_kv_heads
        normal = lambda *size: torch.empty(size).normal_(0.0, 0.02, generator=g)
        ones = lambda n: torch.ones(n)
        self.shape = shape
        self.embed = normal(shape.vocab, H)
        self.lm_head = normal(shape.vocab, H)
        self.final_norm = ones(H)
        D2 = torch.arange(0, D, 2, dtype=torch.int64).float() / D
        self.inv_freq = 1.0 / (shape.rope_theta ** D2)
        layer = [ones(H), normal((nq + 2 * nkv) * D, H), ones(D), ones(D), normal(H, nq * D), ones(H),
                 normal(2 * I, H), normal(H, I)]
        self.layers = [layer] * shape.num_layers

    def nbytes(self):
        return 0


def cpu_sample_requests(tiers, want=(16, 16, 32, 64)):
    """Indices of a representative request sample: the first requests with
    the given tiers (16, 16, 32, 64 rows: 32 rows per request, the wave's
    own mean for configurations 3 and 4)."""
    picked, used = [], set()
    for t in want:
        for i, ti in enumerate(tiers):
            if ti == t and i not in used:
                picked.append(i)
                used.add(i)
                break
    return picked


class CpuStep:
    """One CPU verify step over a request sample: target pass (oracle.forward),
    fp32 softmax, the reference's fp64 inverse-CDF walk (oracle C library,
    Philox uniforms per node), and commit of the kept rows' K/V into each
    request's tail (append_packed_sequence, decode.py:215-261)."""

    def __init__(self, cw, trees, lengths, seed: int):
        s = cw.shape
        g = torch.Generator().manual_seed(seed)
        self.cw, self.trees, self.lengths = cw, trees, lengths
        self.prefixes = [[(torch.randn((s.num_kv_heads, L, s.head_dim), generator=g),
                           torch.randn((s.num_kv_heads, L, s.head_dim), generator=g))
                          for _ in range(s.num_layers)] for L in lengths]
        self.tails = [[torch.zeros((2, s.num_kv_heads, len(par), s.head_dim)) for _ in range(s.num_layers)]
                      for par, _ in trees]
        self.parents = np.asarray([p for par, _ in trees for p in par], np.int64)
        self.tokens = np.asarray([t if j else -1 for par, tok in trees for j, t in enumerate(tok)], np.int64)
        self.depth = 0
        for par, _ in trees:
            d = [0] * len(par)
            for j in range(1, len(par)):
                d[j] = d[par[j]] + 1
            self.depth = max(self.depth, max(d))
        self.rows = len(self.parents)

    def __call__(self, seed: int) -> int:
        from oracle import cpu as oracle
        from oracle.forward import verify_logits
        logits, offsets, kv = verify_logits(self.cw, self.prefixes, self.trees, self.lengths, return_kv=True)
        probs = torch.softmax(logits, dim=-1).numpy()
        out, _ = oracle.accept_probs(probs, offsets, self.parents, self.tokens, self.depth, seed=seed,
                                     request_ids=np.arange(len(self.trees)), arith=oracle.ARITH_FP64)
        units = 0
        for i, (r0, tail) in enumerate(zip(offsets, self.tails)):
            count = int(out[i, self.depth])
            keep = torch.tensor([0] + out[i, :count].tolist()) + r0
            for l, (k, v) in enumerate(kv):
                tail[l][0, :, :len(keep)] = k[keep].transpose(0, 1)
                tail[l][1, :, :len(keep)] = v[keep].transpose(0, 1)
            units += count + 1
        return units


def cpu_verify_arm(config: str, rank: int = 0):
    """Host-only construction of the CPU step for a verify workload (no CUDA
    library, no GPU memory): same shape, tier mix, prefix lengths and seeds."""
    from oracle.forward import CpuWeights
    from specgrove_b200 import workloads
    shape, mix, prefix, name = wave_spec(config)
    wl = workloads.verify_workload(shape.vocab, mix, prefix, seed=rank, device="cpu")
    idx = cpu_sample_requests(wl.tiers)
    cw = CpuWeights(HostWeights(shape, seed=1234), lazy=False)
    step = CpuStep(cw, [wl.trees[i] for i in idx], [wl.cache_lengths[i] for i in idx], seed=rank)
    return name, step, idx, wl


def cpu_baseline_verify(wl, budget_s: float = 20.0):
    """The CPU leg of the headline line (rank 0, N = 1): the CPU step over a
    representative sample of the same wave, all host threads."""
    torch.set_num_threads(os.cpu_count())
    name, step, idx, _ = cpu_verify_arm("verify4b" if wl.name.startswith("config3") else "verify")
    units, seconds, reps = 0, 0.0, 0
    while reps < 1 or (seconds < budget_s and reps < 5):
        t0 = time.perf_counter()
        units += step(reps)
        seconds += time.perf_counter() - t0
        reps += 1
    return {"value": units / seconds, "unit": UNIT, "cores": torch.get_num_threads(), "cpu_model": cpu_model(),
            "kind": "port", "us_per_row": seconds / reps / step.rows * 1e6,
            "sample": f"{reps} step(s) of {len(idx)} requests (tiers 16/16/32/64, {step.rows} rows) of the same "
                      f"wave, all {step.cw.shape.num_layers} layers, torch fp32 + fp64 walk + KV commit on "
                      f"{torch.get_num_threads()} threads"}


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
    return {"value": units / seconds, "unit": UNIT, "cores": 1, "cpu_model": cpu_model(),
            "kind": "port", "sample": f"{reps} full acceptance steps (64 trees, explicit uniforms, "
                                      "fp64 running-sum rule, one thread); KV commit not included"}


def run_accept(args, world, rank):
    wl = AcceptWorkload(rank)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        m = measure_accept(args, world, rank, wl)
    e2e = e2e_accept(wl, args, world)
    cpu = cpu_baseline_accept(wl) if (rank == 0 and world == 1 and not args.no_cpu) else None
    roof = dict(m["acceptance"])
    roof["commit"] = m["commit"]
    roof["terminal_mass"] = m["terminal_mass"]
    return {
        "metric": METRIC, "value": m["value"], "unit": UNIT,
        "per_gpu": {"metric": "accepted tokens/s/GPU", "value": m["value"] / world},
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": m["ms_per_step"],
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": wl.name, "trees_per_gpu": wl.T, "nodes_per_gpu": wl.trees.total_rows,
                   "vocab": wl.vocab, "rule": m["rule"], "parallelism": f"dp{world}", "l2": m["l2"],
                   "ms_per_step_with_flush": m["ms_per_step_with_flush"]},
        "roofline": roof, "cpu_baseline": cpu, "clocks": clocks.summary(), "e2e": e2e,
        "gpu_launches": m["launches"],
    }


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
    return {"value": total / (ms * steps / 1000.0), "unit": UNIT,
            "h2d_bytes_per_step": probs_host.numel() * 4 + meta_host.numel() * 8,
            "d2h_bytes_per_step": out_host.numel() * 8, "steps": steps, "ms_per_step": ms}


def run_reference(args, world, rank):
    """The reference's CPU path for the same workload, metric and config, on
    the host cores; never loads the CUDA library.  Under torchrun only rank 0
    runs it."""
    if rank != 0:
        return None
    torch.set_num_threads(os.cpu_count())
    K, W = args.steps, args.warmup
    if args.workload == "accept":
        from oracle import cpu as oracle
        from specgrove_b200 import workloads
        batch, probs = workloads.acceptance_sweep(seed=rank, device="cpu")
        probs = probs.numpy()
        parents, tokens = batch.flat()
        D = batch.max_depth
        rng = np.random.default_rng(0)

        def step(i):
            u = rng.random((len(batch.parents), D + 1))
            out, _ = oracle.accept_probs(probs, batch.row_offsets, parents, tokens, D, uniforms=u,
                                         arith=oracle.ARITH_FP64)
            return int((out[:, D] + 1).sum())
        name, sample, dtype = AcceptWorkload.name, "every step: the full 64-tree sweep, fp64 rule", "fp64"
        rows = batch.total_rows
    else:
        name, cstep, idx, wl = cpu_verify_arm(args.workload, rank)
        step = cstep
        rows = cstep.rows
        sample = (f"every step: {len(idx)} of the wave's {len(wl.trees)} requests (tiers 16/16/32/64, "
                  f"{rows} rows, 32 rows per request like the full wave), all layers; torch fp32 target pass, "
                  f"fp32 softmax, fp64 inverse-CDF walk, KV commit")
        dtype = "fp32"
    for i in range(W):
        step(10_000 + i)
    units, t0 = 0, time.perf_counter()
    for i in range(K):
        units += step(i)
    seconds = time.perf_counter() - t0
    value = units / seconds
    cpu = {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "cpu_model": cpu_model(),
           "kind": "port", "sample": sample, "us_per_row": seconds / K / rows * 1e6}
    return {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
            "n_gpus": world, "steps": K, "warmup": W, "ms_per_step": seconds / K * 1000,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype,
            "data": "synthetic", "config": {"workload": name, "parallelism": "cpu", "same_config": True,
                                            "rows_per_step": rows},
            "cpu_baseline": cpu, "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                                         "d2h_bytes_per_step": 0},
            "product_library_loaded": product_library_loaded()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="verify", choices=["verify", "verify4b", "accept", "draft", "serve", "plan"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-nested", action="store_true", help="skip the nested configuration-2/3/5 blocks")
    ap.add_argument("--serve-requests", type=int, default=256, help="configuration-5 request count")
    ap.add_argument("--serve-mode", default="spec", choices=["spec", "synthetic"],
                    help="configuration 5: full speculative step with real prefill, or synthetic KV + host trees")
    ap.add_argument("--layers", type=int, default=None,
                    help="profiling only: build the model with this many layers (not a benchmark number)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        # host-only: no process group, no CUDA context; rank 0 alone measures
        world, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
        line = run_reference(args, world, rank)
        if rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
        return
    world, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            line = run_reference(args, world, rank)
        elif args.workload == "accept":
            line = run_accept(args, world, rank)
        elif args.workload == "draft":
            # the nested drafter + wave-plan block alone (development runs)
            from specgrove_b200.engine import QWEN3_8B, ModelShape, Weights
            s = QWEN3_8B
            target = Weights.random(ModelShape(1, s.hidden, s.num_q_heads, s.num_kv_heads, s.head_dim,
                                               s.intermediate, s.vocab), seed=1234)
            line = {"workload": "draft", "draft": measure_draft(args, world, rank, target)}
        elif args.workload == "plan":
            line = measure_plan(args)
        elif args.workload == "serve":
            # the nested configuration-5 block alone (development runs)
            line = {"workload": "serve", "config5": measure_serving(args, world, rank)}
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
