"""Benchmark of the sm_100a attention forward (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C2] [--impl ours|reference]

A step is one attention forward over one batch of the workload. At N=1 the
workload is C2 (B=1, H=24, Sq=Skv=4096, D=128, fp16; the configuration the
north-star target is quoted on). Under torchrun with N ranks every rank runs
its own C2-sized batch of (batch x head) units -- the path shards by
(batch x head) with no data exchange -- so the scaling is weak and `value`
is the whole-job TFLOP/s = N * flops / max-over-ranks time.

Timing: W untimed warm-up steps, then K steps back to back between CUDA
events on the launching stream, bracketed by a barrier and
torch.cuda.synchronize() on both sides. Inputs rotate over enough distinct
sets that their total is larger than the 126 MB L2, so no step reads inputs
the previous step left in L2. SM clocks and throttle reasons are sampled
through NVML while the timed steps run.

`e2e` repeats the measurement through the public host-memory entry point
(`gfx906_b200.attn_host`) with the inputs in pinned host memory: each step
copies all of q, k, v host->device and all of o back, inside the timed
region; the copies of one block of (batch x head) units overlap the kernel of
the previous block and the download of the one before.

`strong` (a list in the same line) is the strong-scaling record of the
path's multi-GPU form: C5 (and C5 at S=32768) with query rows cut over the N
ranks, K/V broadcast from rank 0 and O all-gathered over NCCL; it gives the
kernel-only time and the time with the collectives, both max over ranks.

`--impl reference` times the reference's CPU path (fp32 SDPA MATH on the host
cores, from the CPU oracle) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

from gfx906_b200.configs import CONFIGS, AttnConfig, make_qkv  # noqa: E402

METRIC = "attn fwd TFLOP/s (4*B*H*Sq*Skv*D)"
UNIT = "TFLOP/s"
L2_BYTES = 126 * 1024 * 1024


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", default="C2", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--strong-steps", type=int, default=10,
                    help="steps of each leg of the strong-scaling record (C5, C5s rows-sharded)")
    ap.add_argument("--no-strong", action="store_true", help="skip the strong-scaling record")
    ap.add_argument("--strong-reps", type=int, default=2, help="interleaved repeats of the strong legs (best kept)")
    ap.add_argument("--reserve-sms", type=int, default=16,
                    help="SMs the pipelined strong leg leaves to the NCCL kernels (the attention kernel takes the rest)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--layout", default="rows", choices=["rows", "dmajor"],
                    help="dmajor: D=512 configs on transposed [B,H,D,S] tensors (VAE feature maps)")
    ap.add_argument("--shard", default="heads", choices=["heads", "rows"],
                    help="heads: every rank its own batch of (batch x head) units (weak scaling); "
                         "rows: one problem, query rows split over ranks, K/V broadcast (strong scaling)")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), float(d.get("hbm_gbs", 6650.0)), "measured"
    return 1590.0, 6650.0, "fallback"


def profiled_traffic(cfg_name: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary."""
    f = ROOT / "profiles" / f"attn_fwd_{cfg_name}_traffic.txt"
    if not f.is_file():
        return None
    for line in f.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch:"):
            return float(line.split(":", 1)[1])
    return None


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML in a thread."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
        "display_clocks_setting": 0x100,
    }

    def __init__(self, device_index: int, period_s: float = 0.005):
        self.period = period_s
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            uuid = torch.cuda.get_device_properties(device_index).uuid
            h = None
            try:
                h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + str(uuid)).encode())
            except Exception:  # noqa: BLE001
                h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self._h = h
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - no NVML: clocks stay unknown
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for name, bit in self.REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self):
        med = statistics.median(self.samples) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


def barrier(world):
    if world > 1:
        torch.distributed.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def rank_config(cfg: AttnConfig, rank: int) -> AttnConfig:
    """Rank r's own batch of (batch x head) units: same shape, its own seed."""
    return AttnConfig(cfg.name, cfg.B, cfg.H, cfg.Sq, cfg.Skv, cfg.D, cfg.seed + 1000 * rank, cfg.std)


def cpu_baseline(cfg: AttnConfig, seconds: float):
    """The reference's CPU path (fp32 SDPA MATH) on a bounded sample of cfg."""
    from oracle.sdpa_math import sdpa_math_fp32

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    q, k, v = make_qkv(1, 1, min(cfg.Sq, 512), cfg.Skv, cfg.D, seed=cfg.seed, std=cfg.std)
    sdpa_math_fp32(q, k, v, cfg.scale)  # warm-up
    t0 = time.perf_counter()
    sdpa_math_fp32(q, k, v, cfg.scale)
    probe = time.perf_counter() - t0
    rate_rows = q.shape[2] / max(probe, 1e-6)  # query rows per second (one head)
    rows = int(min(cfg.Sq, max(64, rate_rows * seconds / 3)))
    heads = max(1, min(cfg.B * cfg.H, int(rate_rows * seconds / max(rows, 1) / 1.0)))
    heads = min(heads, cfg.B * cfg.H)
    q, k, v = make_qkv(1, heads, rows, cfg.Skv, cfg.D, seed=cfg.seed, std=cfg.std)
    t0 = time.perf_counter()
    sdpa_math_fp32(q, k, v, cfg.scale)
    dt = time.perf_counter() - t0
    flops = 4.0 * heads * rows * cfg.Skv * cfg.D
    return {
        "value": flops / dt / 1e12,
        "unit": UNIT,
        "cores": torch.get_num_threads(),
        "kind": "port",
        "sample": (f"fp32 SDPA MATH on the host CPU over {heads} head(s) x {rows} query rows x "
                   f"{cfg.Skv} keys x D={cfg.D} of {cfg.name} ({flops / 1e9:.1f} GFLOP, {dt:.2f} s)"),
    }


def run_reference(args, rank, world):
    """--impl reference: the reference's CPU path on the host cores (rank 0 only)."""
    if rank != 0:
        return
    from oracle.sdpa_math import sdpa_math_fp32

    cfg = CONFIGS[args.config]
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    budget = 90.0  # seconds for all warm-up + timed steps together
    q, k, v = make_qkv(1, 1, min(cfg.Sq, 256), cfg.Skv, cfg.D, seed=cfg.seed, std=cfg.std)
    sdpa_math_fp32(q, k, v, cfg.scale)
    t0 = time.perf_counter()
    sdpa_math_fp32(q, k, v, cfg.scale)
    rate_rows = q.shape[2] / max(time.perf_counter() - t0, 1e-6)
    per_step = budget / max(1, args.steps + args.warmup)
    rows = int(max(16, min(cfg.Sq, rate_rows * per_step)))
    q, k, v = make_qkv(1, 1, rows, cfg.Skv, cfg.D, seed=cfg.seed, std=cfg.std)
    for _ in range(args.warmup):
        sdpa_math_fp32(q, k, v, cfg.scale)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        sdpa_math_fp32(q, k, v, cfg.scale)
    dt = time.perf_counter() - t0
    flops = 4.0 * rows * cfg.Skv * cfg.D * args.steps
    value = flops / dt / 1e12
    sample = (f"each step: fp32 SDPA MATH over 1 head x {rows} query rows x {cfg.Skv} keys x "
              f"D={cfg.D} of {cfg.name} (host CPU, {torch.get_num_threads()} threads)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": f"{cfg.name}: {cfg.describe()}", "sample_rows": rows},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def strong_rows(cfg: AttnConfig, rank: int, world: int, local: int, steps: int, warmup: int,
                reserve_sms: int = 16, reps: int = 2) -> dict:
    """Strong scaling of one problem: cfg's query rows cut over the ranks in
    whole 256-row blocks, K and V broadcast from rank 0 with NCCL, O gathered
    with all_gather_into_tensor (gfx906_b200.shard.attention_by_rows). Times,
    each the max over ranks of CUDA events on the launching stream: the kernel
    alone, the kernel alone on all SMs but `reserve_sms`, the broadcast alone,
    the gather alone, the three in sequence, and the three pipelined across
    calls (shard.attention_by_rows_pipelined: the next call's K/V broadcast
    and this call's gather run beside the next kernel on the reserved SMs),
    the same with K/V pulled on the copy engines instead of broadcast
    (shard.attention_by_rows_copy_engine, the kernel on every SM, the NCCL
    gather after it), and with the output rows pushed on the copy engines as
    well (B * H == 1). The legs run interleaved `reps` times; each figure is
    the best repeat."""
    import gfx906_b200
    from gfx906_b200 import shard

    dev = torch.device("cuda", local)
    q, k, v = make_qkv(cfg.B, cfg.H, cfg.Sq, cfg.Skv, cfg.D, cfg.seed, cfg.std)
    sh = shard.row_shard(cfg.Sq, rank, world)
    q_rows = q[:, :, sh.start:sh.stop].contiguous().to(dev)
    kd, vd = k.to(dev), v.to(dev)
    del q, k, v
    out_full = torch.empty(cfg.B, cfg.H, cfg.Sq, cfg.D, dtype=torch.float16, device=dev)
    stream = torch.cuda.current_stream(dev)
    local_out = gfx906_b200.attn(q_rows, kd, vd, cfg.scale)
    counts = [shard.row_shard(cfg.Sq, r, world).size for r in range(world)]

    def bcast():
        if world > 1:
            torch.distributed.broadcast(kd, src=0)
            torch.distributed.broadcast(vd, src=0)

    def gather():
        if world > 1:
            shard._gather_dim(local_out, counts, 2, None, out=out_full)

    # pipelined: every call still broadcasts its K/V, runs the kernel and
    # gathers its O, but the next call's broadcast (other buffers) and this
    # call's gather run on the collective stream beside the next kernel
    kbuf, vbuf = [kd, kd.clone()], [vd, vd.clone()]
    obuf = [out_full, torch.empty_like(out_full)]

    def pipelined(n):
        calls = [(q_rows, kbuf[i % 2], vbuf[i % 2], cfg.scale, obuf[i % 2]) for i in range(n)]
        shard.attention_by_rows_pipelined(calls, cfg.Sq, src=0, reserve_sms=reserve_sms)

    n_sms = torch.cuda.get_device_properties(dev).multi_processor_count

    def kernel_reserved(n):
        with gfx906_b200.sm_limit(max(2, n_sms - reserve_sms)):
            for _ in range(n):
                gfx906_b200.attn(q_rows, kd, vd, cfg.scale)

    legs = {
        "kernel": (lambda n: [gfx906_b200.attn(q_rows, kd, vd, cfg.scale) for _ in range(n)]),
        "kernel_reserved": kernel_reserved,
        "broadcast": (lambda n: [bcast() for _ in range(n)]),
        "gather": (lambda n: [gather() for _ in range(n)]),
        "with_collectives": (lambda n: [shard.attention_by_rows(q_rows, kd, vd, cfg.scale, cfg.Sq, src=0,
                                                                out=out_full) for _ in range(n)]),
        "pipelined": pipelined,
    }
    # copy engines: K/V pulled from rank 0's ring over CUDA IPC while the
    # previous call's kernel runs on every SM (gfx906_b200.peer.KVBroadcast);
    # set up collectively, used only if it came up on every rank
    ce, ce_error = None, None
    if world > 1:
        try:
            from gfx906_b200.peer import KVBroadcast

            ce = KVBroadcast(tuple(kd.shape), dtype=kd.dtype, src=0)
            if rank == 0:  # the same K/V every call: both ring pairs hold them
                for b in range(ce.depth):
                    ce.k[b].copy_(kd)
                    ce.v[b].copy_(vd)
        except Exception as e:  # noqa: BLE001 - reported in the record
            ce_error = f"{type(e).__name__}: {e}"
        up = torch.tensor([0 if ce_error else 1], device=dev)
        torch.distributed.all_reduce(up, op=torch.distributed.ReduceOp.MIN)
        if int(up.item()) == 0:
            ce_error = ce_error or "not available on another rank"
            ce = None  # not closed: close() is collective and the other rank has none
    rg = None
    if ce is not None:
        legs["pipelined_copy_engine"] = lambda n: shard.attention_by_rows_copy_engine(
            [q_rows] * n, ce, cfg.scale, cfg.Sq, [obuf[i % 2] for i in range(n)])
        if cfg.B * cfg.H == 1:
            # the output rows pushed to every rank on the copy engines as well
            from gfx906_b200.peer import RowGather

            rows = [(shard.row_shard(cfg.Sq, r, world).start, shard.row_shard(cfg.Sq, r, world).stop)
                    for r in range(world)]
            try:
                rg = RowGather(tuple(out_full.shape), rows)
            except Exception as e:  # noqa: BLE001 - reported in the record
                ce_error = f"row gather: {type(e).__name__}: {e}"
            up = torch.tensor([0 if rg is None else 1], device=dev)
            torch.distributed.all_reduce(up, op=torch.distributed.ReduceOp.MIN)
            if int(up.item()) == 0:
                rg = None  # not closed: close() is collective and another rank has none
            else:
                legs["copy_engine_all"] = lambda n: shard.attention_by_rows_copy_engine(
                    [q_rows] * n, ce, cfg.scale, cfg.Sq, rg=rg)
    ms = {}
    for rep in range(reps):  # legs interleaved, best of `reps` (each the max over ranks)
        for name, fn in legs.items():  # every rank runs the same legs in the same order
            if rep == 0:
                fn(max(3, warmup))  # NCCL's lazy set-up stays out of the timing
            torch.cuda.synchronize()
            barrier(world)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            # ~0.5 ms of GPU spin ahead of the start event: the host queues the
            # first calls meanwhile, so its launch latency stays out of the timing
            torch.cuda._sleep(1 << 20)
            e0.record(stream)
            fn(steps)
            e1.record(stream)
            torch.cuda.synchronize()
            barrier(world)
            t = max_over_ranks(e0.elapsed_time(e1), world) / steps
            ms[name] = min(ms.get(name, t), t)
    if rg is not None:
        rg.close()
    if ce is not None:
        ce.close()
    kv_bytes = 2 * kd.numel() * kd.element_size()
    o_bytes = out_full.numel() * out_full.element_size()
    return {
        "workload": f"{cfg.name}: {cfg.describe()}",
        "ranks": world, "rows_per_rank": sh.size, "steps": steps, "repeats": reps,
        "kernel_ms": ms["kernel"], "kernel_reserved_ms": ms["kernel_reserved"], "reserve_sms": reserve_sms,
        "broadcast_ms": ms["broadcast"], "gather_ms": ms["gather"],
        "with_collectives_ms": ms["with_collectives"], "pipelined_ms": ms["pipelined"],
        "pipelined_copy_engine_ms": ms.get("pipelined_copy_engine"),
        "copy_engine_all_ms": ms.get("copy_engine_all"),
        "copy_engine_error": ce_error,
        "value_kernel": cfg.flops / (ms["kernel"] * 1e-3) / 1e12,
        "value_with_collectives": cfg.flops / (ms["with_collectives"] * 1e-3) / 1e12,
        "value_pipelined": cfg.flops / (ms["pipelined"] * 1e-3) / 1e12,
        "value_pipelined_copy_engine": (cfg.flops / (ms["pipelined_copy_engine"] * 1e-3) / 1e12
                                        if "pipelined_copy_engine" in ms else None),
        "value_copy_engine_all": (cfg.flops / (ms["copy_engine_all"] * 1e-3) / 1e12
                                  if "copy_engine_all" in ms else None),
        "unit": UNIT,
        "collectives": (f"NCCL broadcast of K and V from rank 0 ({kv_bytes / 2**20:.0f} MiB) and "
                        f"all_gather_into_tensor of O ({o_bytes / 2**20:.0f} MiB) over {world} rank(s)"
                        if world > 1 else "none (one rank)"),
    }


def run_rows(args, rank, world, local):
    """--shard rows: the strong-scaling leg alone, as the line's value."""
    import gfx906_b200

    torch.cuda.set_device(local)
    if gfx906_b200.load_attention() is None:
        raise RuntimeError(f"sm_100 attention operator unavailable: {gfx906_b200.last_error()}")
    cfg = CONFIGS[args.config]
    sampler = ClockSampler(local)
    with sampler:
        rec = strong_rows(cfg, rank, world, local, args.steps, args.warmup, args.reserve_sms, args.strong_reps)
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": rec["value_kernel"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": rec["kernel_ms"], "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f16", "data": "synthetic",
        "config": {"workload": rec["workload"],
                   "parallelism": f"query rows split over {world} GPU(s) in 256-row blocks, K/V broadcast"},
        "strong": rec,
        "clocks": sampler.summary(),
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, local):
    import gfx906_b200

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    mod = gfx906_b200.load_attention()
    if mod is None:
        raise RuntimeError(f"sm_100 attention operator unavailable: {gfx906_b200.last_error()}")
    base = CONFIGS[args.config]
    cfg = rank_config(base, rank)
    scale = cfg.scale

    # distinct input sets so that the rotation exceeds L2
    set_bytes = cfg.io_bytes
    nsets = max(2, math.ceil(2 * L2_BYTES / set_bytes) + 1)
    nsets = min(nsets, 8)
    q0, k0, v0 = make_qkv(cfg.B, cfg.H, cfg.Sq, cfg.Skv, cfg.D, cfg.seed, cfg.std)
    sets = []
    for i in range(nsets):
        # same values, distinct buffers (the kernel's time does not depend on values)
        sets.append((q0.to(dev), k0.to(dev), v0.to(dev)))
    outs = [torch.empty_like(s[0]) for s in sets]
    dmajor = args.layout == "dmajor"
    if dmajor and cfg.D != 512:
        raise SystemExit("--layout dmajor needs a D=512 config (C4)")
    # d-major: the same buffers read as [B,H,D,S] (values do not change the timing)
    lib_launch = _c_launcher(dmajor)
    stream = torch.cuda.current_stream(dev)

    def step(i):
        q, k, v = sets[i % nsets]
        o = outs[i % nsets]
        rc = lib_launch(q, k, v, o, cfg, scale, stream)
        if rc != 0:
            raise RuntimeError(f"launch failed with status {rc}")

    for i in range(max(3, args.warmup)):
        step(i)
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    with sampler:
        start.record(stream)
        for i in range(args.steps):
            step(i)
        end.record(stream)
        torch.cuda.synchronize()
    barrier(world)
    ms = start.elapsed_time(end)
    ms_max = max_over_ranks(ms, world)
    if mod.device_status(False) != 0:
        raise RuntimeError("a kernel wait timed out during the benchmark")

    flops_step = cfg.flops
    value = world * flops_step * args.steps / (ms_max * 1e-3) / 1e12
    per_launch_ms = ms / args.steps
    achieved = flops_step / (per_launch_ms * 1e-3) / 1e12

    # ---- e2e through the public operator, host buffers, copies in the timed region
    hq = q0.pin_memory()
    hk = k0.pin_memory()
    hv = v0.pin_memory()
    hout = torch.empty(hq.shape, dtype=hq.dtype, pin_memory=True)
    e2e_steps = max(1, args.e2e_steps)

    def e2e_step():
        if dmajor:  # public transposed-layout operator, copies in and out each step
            shp = (cfg.B, cfg.H, cfg.D, cfg.Sq)
            o = gfx906_b200.attn_dmajor(hq.view(shp).to(dev, non_blocking=True),
                                        hk.view(cfg.B, cfg.H, cfg.D, cfg.Skv).to(dev, non_blocking=True),
                                        hv.view(cfg.B, cfg.H, cfg.D, cfg.Skv).to(dev, non_blocking=True), scale)
            hout.view(shp).copy_(o, non_blocking=True)
            return
        # public host-memory entry point: every step uploads q, k, v and downloads
        # o; blocks of (batch x head) units overlap upload, kernel and download
        gfx906_b200.attn_host(hq, hk, hv, scale, out=hout, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world)
    e2e_value = world * flops_step * e2e_steps / (e2e_ms * 1e-3) / 1e12
    h2d = (hq.numel() + hk.numel() + hv.numel()) * hq.element_size()
    d2h = hout.numel() * hout.element_size()

    # strong scaling of the long single-head configs (query rows over the ranks,
    # K/V broadcast, O gathered): the multi-GPU path with its collectives
    strong = []
    if not args.no_strong:
        for name in ("C5", "C5s"):
            strong.append(strong_rows(CONFIGS[name], rank, world, local, args.strong_steps, 3, args.reserve_sms,
                                      args.strong_reps))

    if rank != 0:
        return
    peak_tf, _, peak_kind = load_peaks()
    traffic = profiled_traffic(base.name + ("_dmajor" if dmajor else ""))
    clocks = sampler.summary()
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms_max / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic",
        "config": {
            "workload": f"{base.name}: {base.describe()}" + (
                "; tensors stored transposed [B,H,D,S] (VAE feature-map layout)" if dmajor else ""),
            "per_rank": f"each rank its own B*H={cfg.B * cfg.H} heads (weak scaling over (batch x head))",
            "l2": f"inputs rotate over {nsets} distinct sets ({nsets * set_bytes / 2**20:.0f} MiB > 126 MB L2)",
            "parallelism": f"shard (batch x head) over {world} GPU(s), no collective on the data path",
        },
        "roofline": {
            "bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": UNIT,
            "frac": achieved / peak_tf,
            "peak_source": f"{peak_kind} bf16 dense burst (MEASURED_PEAKS.json bf16_tflops)",
            "traffic": traffic,
            "algorithmic_bytes": cfg.io_bytes,
            "kernel": f"attn_fwd_kernel<{128 if cfg.D == 128 else 64}>" if cfg.D <= 128
            else f"attn_fwd_d512_pair_kernel<{'true' if dmajor else 'false'}>",
        },
        "clocks": clocks,
        "gpu_launches": args.steps * _launches_per_call(cfg, dmajor),
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps,
                "ms_per_step": e2e_ms / e2e_steps},
    }
    if strong:
        line["strong"] = strong
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(base, args.cpu_seconds)
    print(json.dumps(line), flush=True)


def _launches_per_call(cfg: AttnConfig, dmajor: bool = False) -> int:
    """Kernels one call launches: the attention kernel, plus the combine
    kernel when the plan splits and combines pieces in a second kernel."""
    if dmajor:
        return 1
    from gfx906_b200 import build
    from gfx906_b200.cabi import CABI

    rc, pl = CABI(build.LIB_PATH).plan(cfg.B, cfg.H, cfg.Sq, cfg.Skv, cfg.D, with_workspace=True)
    return 2 if rc == 0 and pl["split"] == 2 else 1


def _c_launcher(dmajor: bool = False):
    """Direct C-ABI launch on preallocated outputs and workspace (no allocation
    in the timed loop): the split schedule the torch op uses. dmajor: the
    transposed-layout entry point (D=512)."""
    from gfx906_b200 import build
    from gfx906_b200.cabi import CABI

    lib = CABI(build.LIB_PATH)
    cache = {}

    def launch(q, k, v, o, cfg, scale, stream):
        if dmajor:
            return lib.launch_dmajor_status(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), cfg.B, cfg.H,
                                            cfg.Sq, cfg.Skv, cfg.D, scale, stream.cuda_stream)
        n = lib.workspace_size(cfg.B, cfg.H, cfg.Sq, cfg.Skv, cfg.D)
        ws = cache.get(q.device)
        if n and (ws is None or ws.numel() < n):
            ws = cache[q.device] = torch.zeros(n, dtype=torch.uint8, device=q.device)
        return lib.launch_ws_status(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), cfg.B, cfg.H,
                                    cfg.Sq, cfg.Skv, cfg.D, scale, ws.data_ptr() if n else None, n,
                                    stream.cuda_stream)

    return launch


def main():
    args = parse_args()
    rank, world, local = dist_env()
    if world > 1:
        import datetime

        if args.impl == "reference":
            # only rank 0 works; the other ranks exit without joining anything
            run_reference(args, rank, world)
            return
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif args.shard == "rows":
            run_rows(args, rank, world, local)
        else:
            run_ours(args, rank, world, local)
    finally:
        if world > 1 and torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
