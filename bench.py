#!/usr/bin/env python3
"""Benchmark of the Neso B200 hot path; prints ONE JSON line (rank 0).

Headline workload (BASELINE.json metric "FA2 fwd TFLOP/s (D=64,S=2048)"):
Flash Attention 2 forward, fp16 Q/K/V [B=16, H=16, S=2048, D=64] drawn N(0,1)
from a seed, softmax scale 1/8, fp32 accumulation and fp32 O, non-causal.
One step = one FA2 forward over the whole batch. The inputs (3 x 64 MiB fp16
+ 128 MiB fp32 out at N=1) are larger than the 126 MB L2, so no L2 flush is
needed between steps.

Multi-GPU (``torchrun --nproc-per-node N``): the fixed 16 x 16 heads are
partitioned along flattened batch x heads (``neso_b200.shard``), 256/N heads
per rank, one launch per rank and step, no collective in the step ->
"scaling": "strong". ``value`` = total FLOPs / the step time, the max over
ranks of the CUDA-event time. After timing, the ranks' outputs are
all-gathered over NCCL and rank 0 checks sampled heads against the CPU oracle
(``verified``). The timed region (K steps between barrier + synchronize) is
repeated until about a third of a second of device time has been sampled, so
the clock sampler sees the kernel; ``ms_per_step`` is the median region.

``--impl reference`` times the reference algorithm's CPU implementation (the
torch-fp32 oracle port: the reference's own kernels are Metal/HLSL and cannot
run here) on the host cores, one bounded sample per step; under torchrun only
rank 0 runs it.

Also reported (not part of ``value``), each sharded over the ranks the same
way as the headline (heads for attention, output columns for the matmuls,
element ranges for the elementwise kernels) and timed as the max over ranks:
every BASELINE config with its roofline fraction (``baseline_configs``), the
e2e number through the public API with pinned host buffers, the roofline of
the headline kernel and the CPU baseline. A BASELINE config's time is the
device time per launch with the launches replayed from one CUDA graph (its
roofline fraction uses it); the same calls issued eagerly from Python are
reported beside it (``ms_eager`` / ``us_eager``), which for problems of a
few microseconds is the host's per-call cost.
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
sys.path.insert(0, str(ROOT))

B, H, S, D = 16, 16, 2048, 64
SEED = 1234
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
METRIC = "FA2 fwd TFLOP/s (D=64,S=2048) & quant-GEMM TFLOP/s at 1/2/4/8 B200"
L2_FLOOR = 256 << 20  # rotate input sets until they exceed twice the 126 MB L2
QK, QN = 4096, 11008   # quantized matmul weight shape


def fa2_flops(b=B, h=H, s=S, d=D, causal=False) -> float:
    f = 4.0 * b * h * s * s * d  # tests/test_flash_attention.py:387
    return f / 2 if causal else f


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


_JSON_OUT = sys.stdout  # replaced in main() by a duplicate of the original stdout


def load_traffic(kernel_key: str):
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text()).get(kernel_key)
    except Exception:
        return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, device_index: int, interval_s: float = 0.005):
        self.idx = device_index
        self.interval = interval_s
        self.samples: list[int] = []
        self.reasons: set[str] = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.ok = False

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            return self
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def _run(self):
        nv = self._nvml
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                for name, bit in self.REASONS.items():
                    if mask & bit and name != "gpu_idle":
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(self.interval)

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=1.0)

    def summary(self) -> dict:
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml-unavailable"]}
        med = statistics.median(self.samples) if self.samples else None
        return {"sm_mhz": med, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


def cpu_fa2_sample(budget_s: float, threads: int) -> dict:
    """Time the torch-fp32 CPU oracle on whole heads of the workload until the
    budget is used (at least one head)."""
    import torch
    import oracle

    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(SEED)
    q, k, v = (torch.randn(1, 1, S, D, generator=g).half() for _ in range(3))
    oracle.attention(q[:, :, :256], k[:, :, :256], v[:, :, :256], 1 / math.sqrt(D))  # warm the thread pool
    heads = 0
    t0 = time.perf_counter()
    while True:
        oracle.attention(q, k, v, 1 / math.sqrt(D))
        heads += 1
        el = time.perf_counter() - t0
        if el >= budget_s or heads >= 4096:
            break
    tflops = fa2_flops(1, heads, S, D) / el / 1e12
    return {"value": tflops, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{heads} head(s) of [S={S}, D={D}] fp32 softmax attention (torch CPU oracle), "
                      f"{el:.2f} s"}


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_reference(args, rank: int, world: int) -> None:
    """--impl reference: the reference algorithm's CPU implementation (torch
    fp32 oracle port) on the host cores, one head of the workload per step.
    Under torchrun rank 0 alone runs it."""
    if rank != 0:
        return
    import torch
    import oracle

    threads = host_threads()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(SEED)
    q, k, v = (torch.randn(1, 1, S, D, generator=g).half() for _ in range(3))
    for _ in range(max(args.warmup, 0)):
        oracle.attention(q, k, v, 1 / math.sqrt(D))
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.attention(q, k, v, 1 / math.sqrt(D))
        times.append(time.perf_counter() - t0)
    per = statistics.median(times)
    value = fa2_flops(1, 1, S, D) / per / 1e12
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": f"FA2 fwd B={B} H={H} S={S} D={D} non-causal (one head per step on CPU)",
                   "global_batch": B, "heads": H, "seq_len": S, "head_dim": D, "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"1 head [S={S}, D={D}] per step, torch CPU fp32 oracle (reference kernels "
                                   f"are Metal/HLSL: unavailable on this box)"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), file=_JSON_OUT, flush=True)


class Ctx:
    """Rank, world, device, stream and the cross-rank max of a time."""

    def __init__(self, world: int, rank: int, dev, stream):
        self.world, self.rank, self.dev, self.stream = world, rank, dev, stream

    @property
    def dist_on(self) -> bool:
        return self.world > 1

    def max_over_ranks(self, ms: float) -> float:
        if not self.dist_on:
            return ms
        import torch
        import torch.distributed as dist
        t = torch.tensor([ms], device=self.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def barrier(self) -> None:
        if self.dist_on:
            import torch.distributed as dist
            dist.barrier()


def time_region(ctx: Ctx, fn, steps: int) -> float:
    """Barrier + sync, `steps` calls between CUDA events on the launching
    stream, barrier + sync. Returns ms per step, max over ranks."""
    import torch

    ctx.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(ctx.stream)
    for _ in range(steps):
        fn()
    end.record(ctx.stream)
    torch.cuda.synchronize()
    ctx.barrier()
    return ctx.max_over_ranks(start.elapsed_time(end) / steps)


def time_rotating(ctx: Ctx, sets: list, launch, iters: int = 20) -> tuple[float, float]:
    """ms per launch of `launch(set)` over rotating input sets (their total
    size exceeds L2, so every launch reads HBM), after one warm-up launch per
    set; max over ranks. Returns (device ms, eager ms): the device time
    replays the `iters` launches from one CUDA graph, so small problems show
    the kernels' time rather than the host's per-call cost; the eager time
    issues the same calls from Python back to back."""
    import torch

    eager = None
    side = torch.cuda.Stream(ctx.dev)
    side.wait_stream(torch.cuda.current_stream(ctx.dev))
    with torch.cuda.stream(side):  # the capture stream gets its per-stream state first
        for st in sets:
            launch(st)
    torch.cuda.synchronize()
    for st in sets:
        launch(st)
    torch.cuda.synchronize()
    eager = time_region(ctx, _Rotor(sets, launch), iters)
    graph = torch.cuda.CUDAGraph()
    rot = _Rotor(sets, launch)
    with torch.cuda.graph(graph, stream=side):
        for _ in range(iters):
            rot()
    graph.replay()
    torch.cuda.synchronize()
    ctx.barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(side):  # replay() runs on the current stream: time it there
        start.record(side)
        graph.replay()
        end.record(side)
    torch.cuda.synchronize()
    ctx.barrier()
    dev_ms = ctx.max_over_ranks(start.elapsed_time(end) / iters)
    del graph
    return dev_ms, eager


class _Rotor:
    def __init__(self, sets, launch):
        self.sets, self.launch, self.i = sets, launch, 0

    def __call__(self):
        self.launch(self.sets[self.i % len(self.sets)])
        self.i += 1


def copies(bytes_per_set: int) -> int:
    return max(1, -(-L2_FLOOR // max(1, bytes_per_set)))


def roofline(flops: float | None, nbytes: float, t_s: float, peaks: dict) -> dict:
    """Per-GPU achieved rate against min(tensor peak, AI x HBM) (tensor-bound
    work) or the HBM peak (byte work)."""
    hbm = float(peaks["hbm_gbs"]) * 1e9
    ten = float(peaks["bf16_tflops"]) * 1e12
    if flops is None:
        ach = nbytes / t_s
        return {"bound": "hbm", "achieved_gbs": ach / 1e9, "frac": ach / hbm}
    ach = flops / t_s
    roof = min(ten, flops / nbytes * hbm)
    return {"bound": "tensor" if roof >= ten else "hbm", "achieved_tflops": ach / 1e12,
            "roof_tflops": roof / 1e12, "frac": ach / roof, "frac_of_tensor_peak": ach / ten}


def baseline_configs(ctx: Ctx, peaks: dict) -> dict:
    """Every BASELINE config, sharded over the ranks like the headline; each
    entry has the aggregate rate, the per-launch time (max over ranks) and the
    per-GPU roofline fraction."""
    import torch
    from neso_b200 import ops, shard

    dev, world, rank = ctx.dev, ctx.world, ctx.rank
    g = torch.Generator(device=dev).manual_seed(SEED + 17)
    out: dict = {}

    # config 2: elementwise, n = 2^28 fp32 (contiguous element ranges)
    n = 1 << 28
    sh = shard.shard_range(n, world, rank, 1024)
    x = torch.rand(sh.size, device=dev, generator=g) * 2 - 1
    y = torch.rand(sh.size, device=dev, generator=g) * 2 - 1
    z = torch.empty_like(x)
    for name, fn, per_el in (("vector_add", lambda _: ops.vector_add(x, y, out=z), 12),
                             ("scale", lambda _: ops.scale(x, 0.5, out=z), 8)):
        ms, ms_e = time_rotating(ctx, [None], fn, 10)
        r = roofline(None, per_el * sh.size, ms * 1e-3, peaks)
        out[name] = {"n": n, "gbs": per_el * n / (ms * 1e-3) / 1e9, "ms": ms, "ms_eager": ms_e, **r}
    del x, y, z

    # config 4: dense GEMM M = N = K, output columns sharded (16-column groups)
    for m in (1024, 2048, 4096, 8192):
        sh = shard.shard_columns(m, world, rank, 16)
        a = (torch.randn(m, m, device=dev, generator=g) / math.sqrt(m)).half()
        bfull = (torch.randn(m, m, device=dev, generator=g) / math.sqrt(m)).half()
        b = bfull[:, sh.slice()].contiguous()
        del bfull
        set_bytes = 2 * m * m + 2 * m * sh.size + 4 * m * sh.size
        sets = [(a, b, torch.empty(m, sh.size, device=dev))]
        for _ in range(copies(set_bytes) - 1):
            sets.append((a.clone(), b.clone(), torch.empty(m, sh.size, device=dev)))
        ms, ms_e = time_rotating(ctx, sets, lambda s: ops.matmul(s[0], s[1], out=s[2]))
        fl = 2.0 * m * sh.size * m
        r = roofline(fl, set_bytes, ms * 1e-3, peaks)
        out[f"gemm_{m}"] = {"tflops": 2.0 * m ** 3 / (ms * 1e-3) / 1e12, "ms": ms, "ms_eager": ms_e,
                            "cols_per_rank": sh.size, **r}
        del sets, a, b

    # configs 1 and 3: FA2, heads sharded
    fa2_cases = [("fa2_b1h8s512d64", 1, 8, 512, 64, False, False)]
    for d in (64, 128):
        for s_ in (128, 256, 512, 1024, 2048):
            fa2_cases.append((f"fa2_s{s_}_d{d}", 16, 16, s_, d, False, False))
        fa2_cases.append((f"fa2_s2048_d{d}_causal", 16, 16, 2048, d, True, False))
        fa2_cases.append((f"fa2_s2048_d{d}_table", 16, 16, 2048, d, False, True))
        fa2_cases.append((f"fa2_s2048_d{d}_causal_table", 16, 16, 2048, d, True, True))
    for name, b_, h_, s_, d_, causal, tab in fa2_cases:
        if any(shard.shard_heads(b_, h_, world, r).size == 0 for r in range(world)):
            continue  # fewer heads than ranks: skipped on every rank alike
        sh = shard.shard_heads(b_, h_, world, rank)
        set_bytes = 10 * sh.size * s_ * d_
        sets = []
        for _ in range(copies(set_bytes)):
            q, k, v = (torch.randn(1, sh.size, s_, d_, device=dev, generator=g).half() for _ in range(3))
            t = None
            if tab:  # the table rows of this shard's heads (head index = flattened index mod H)
                full = torch.randn(h_, 2 * s_ - 1, device=dev, generator=g) * 0.02
                t = full[torch.arange(sh.start, sh.stop, device=dev) % h_].contiguous()
            sets.append((q, k, v, t, torch.empty(1, sh.size, s_, d_, device=dev)))
        sc = 1 / math.sqrt(d_)
        ms, ms_e = time_rotating(ctx, sets, lambda st: ops.flash_attention(st[0], st[1], st[2], sc, causal=causal,
                                                                      table=st[3], out=st[4]))
        fl_rank = fa2_flops(1, sh.size, s_, d_, causal)
        r = roofline(fl_rank, set_bytes + (4 * (2 * s_ - 1) * sh.size if tab else 0), ms * 1e-3, peaks)
        out[name] = {"tflops": fa2_flops(b_, h_, s_, d_, causal) / (ms * 1e-3) / 1e12, "ms": ms, "ms_eager": ms_e,
                     "heads_per_rank": sh.size, **r}
        del sets

    # the reference's rel_pos_fa2_fwd (dense fp16 bias [nh, T, T], fp16 O), heads sharded
    from neso_b200 import kernels
    for nh, t_, d_ in ((64, 2048, 64), (64, 1024, 128)):
        sh = shard.shard_heads(1, nh, world, rank)
        if sh.size == 0:
            continue
        set_bytes = 8 * sh.size * t_ * d_ + 2 * sh.size * t_ * t_
        sets = [(tuple(torch.randn(sh.size, t_, d_, device=dev, generator=g).half() for _ in range(3)),
                 (0.5 * torch.randn(sh.size, t_, t_, device=dev, generator=g)).half(),
                 torch.empty(sh.size, t_, d_, dtype=torch.float16, device=dev)) for _ in range(copies(set_bytes))]
        launch = kernels.rel_pos_fa2_fwd[(t_ // 128, sh.size, 1)]
        sc = 1 / math.sqrt(d_)
        ms, ms_e = time_rotating(ctx, sets, lambda st: launch(*st[0], st[1], st[2], t_, d_, sc, t_ * d_, t_ * t_))
        r = roofline(fa2_flops(1, sh.size, t_, d_, False), set_bytes, ms * 1e-3, peaks)
        out[f"relpos_dense_t{t_}_d{d_}"] = {"tflops": fa2_flops(1, nh, t_, d_, False) / (ms * 1e-3) / 1e12, "ms": ms,
                                           "ms_eager": ms_e, "heads": nh, "heads_per_rank": sh.size, **r}
        del sets

    # config 5: quantized matmul K = 4096, N = 11008, output columns sharded
    sh = shard.shard_columns(QN, world, rank, 16)
    nc = sh.size
    for kind in ("w8a16", "w4a16"):
        if kind == "w8a16":
            wbytes = QK * nc + 2 * nc
            ws = [(torch.randint(-127, 128, (QK, nc), device=dev, dtype=torch.int8, generator=g),
                   (torch.rand(nc, device=dev, generator=g) * 0.019 + 0.001).half()) for _ in range(copies(wbytes))]
        else:
            wbytes = QK * nc // 2 + 2 * (QK // 128) * nc
            ws = [(torch.randint(0, 256, (QK // 2, nc), device=dev, dtype=torch.uint8, generator=g),
                   (torch.rand(QK // 128, nc, device=dev, generator=g) * 0.019 + 0.001).half())
                  for _ in range(copies(wbytes))]
        for m in (1, 16, 128, 2048):
            xq = torch.randn(m, QK, device=dev, generator=g).half()
            yq = torch.empty(m, nc, device=dev)
            if kind == "w8a16":
                fn = lambda st: ops.w8a16_matmul(xq, st[0], st[1], out=yq)  # noqa: E731
            else:
                fn = lambda st: ops.w4a16_g128_matmul(xq, st[0], st[1], out=yq)  # noqa: E731
            ms, ms_e = time_rotating(ctx, ws, fn, 30)
            fl = 2.0 * m * nc * QK
            nbytes = wbytes + 2 * m * QK + 4 * m * nc
            r = roofline(fl, nbytes, ms * 1e-3, peaks)
            out[f"{kind}_m{m}"] = {"tflops": 2.0 * m * QN * QK / (ms * 1e-3) / 1e12, "us": ms * 1e3,
                                   "us_eager": ms_e * 1e3,
                                   "weight_gbs_per_gpu": (QK * nc if kind == "w8a16" else QK * nc // 2) /
                                   (ms * 1e-3) / 1e9, "cols_per_rank": nc, "weight_copies": len(ws), **r}
            del xq, yq
        del ws
    torch.cuda.synchronize()
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="neso", choices=["neso", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU-baseline work (rank 0, N=1)")
    ap.add_argument("--no-extras", action="store_true", help="skip the BASELINE-config and e2e side measurements")
    ap.add_argument("--min-timed-s", type=float, default=0.3,
                    help="repeat the timed region until this much device time has been sampled")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    # One JSON line on stdout: everything else any library writes to file
    # descriptor 1 (NCCL's version banner, for instance, which the
    # environment may ask for) is sent to stderr instead.
    global _JSON_OUT
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    os.environ.setdefault("NCCL_DEBUG", "WARN")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from neso_b200 import ops, shard

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    ctx = Ctx(world, rank, dev, torch.cuda.current_stream(dev))
    peaks, peak_src = load_peaks()

    # This rank's heads of the fixed [16, 16, 2048, 64] batch: every rank draws
    # the whole batch from the same seed and keeps its contiguous heads.
    sh = shard.shard_heads(B, H, world, rank)
    gen = torch.Generator(device=dev).manual_seed(SEED)
    full = [torch.randn(B * H, S, D, device=dev, generator=gen).half() for _ in range(3)]
    q, k, v = (t[sh.slice()].unsqueeze(0).contiguous() for t in full)
    del full
    o = torch.empty(1, sh.size, S, D, device=dev, dtype=torch.float32)
    scale = 1.0 / math.sqrt(D)

    def step():
        ops.flash_attention(q, k, v, scale, out=o)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    regions = []
    with ClockSampler(local_rank) as clk:
        regions.append(time_region(ctx, step, args.steps))
        # the same repeat count on every rank (collectives inside time_region)
        reps = int(min(50, max(3, math.ceil(args.min_timed_s / max(1e-6, regions[0] * 1e-3 * args.steps)))))
        for _ in range(reps - 1):
            regions.append(time_region(ctx, step, args.steps))
    clocks = clk.summary()
    ms = statistics.median(regions)
    value = fa2_flops() / (ms * 1e-3) / 1e12

    # Roofline of the dominant (only) kernel in the step: one launch per rank and step.
    flops_rank = fa2_flops(1, sh.size, S, D)
    achieved = flops_rank / (ms * 1e-3) / 1e12
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    traffic = load_traffic("fa2_fwd_d64_s2048_b16h16")
    roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "traffic": None if traffic is None else traffic["dram_bytes_per_launch"] * sh.size / (B * H),
            "algorithmic_bytes": 10.0 * sh.size * S * D,
            "peak_source": f"{peak_src} bf16_tflops (burst, kernel timed alone)",
            "traffic_source": None if traffic is None else traffic["source"],
            "kernel": "fa2_pair_kernel<64,false,0>"}

    # Verification after timing: NCCL all-gather of every rank's heads, then
    # rank 0 checks sampled heads (first and last of every shard) on the CPU.
    if ctx.dist_on:
        sizes = [shard.shard_heads(B, H, world, r).size for r in range(world)]
        gathered = shard.gather(o[0], sizes)
    else:
        gathered = o[0]
    verified = None
    if rank == 0:
        import oracle
        gv = torch.Generator(device=dev).manual_seed(SEED)
        fullv = [torch.randn(B * H, S, D, device=dev, generator=gv).half() for _ in range(3)]
        picks = sorted({i for r in range(world) for i in (shard.shard_heads(B, H, world, r).start,
                                                           shard.shard_heads(B, H, world, r).stop - 1)})
        ok = True
        for i in picks:
            ref = oracle.attention(fullv[0][i].cpu(), fullv[1][i].cpu(), fullv[2][i].cpu(), scale)
            ok = ok and torch.allclose(gathered[i].cpu(), ref, atol=2e-3, rtol=2e-3)
        verified = bool(ok)
        del fullv
    del gathered
    ctx.barrier()

    extras: dict = {}
    e2e = None
    if not args.no_extras:
        e2e = e2e_run(ctx, q, k, v, o, scale, args.steps)
        extras["baseline_configs"] = baseline_configs(ctx, peaks)

    cpu = None
    if rank == 0 and world == 1:
        cpu = cpu_fa2_sample(args.cpu_budget, host_threads())

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": {"workload": f"FA2 fwd B={B} H={H} S={S} D={D} non-causal, fp16 in, fp32 acc/out, "
                                   f"heads split over {world} GPU(s)",
                       "global_batch": B, "heads": H, "seq_len": S, "head_dim": D,
                       "heads_per_gpu": sh.size,
                       "parallelism": f"batch x heads sharded over {world} GPU(s), no collective in the step",
                       "l2": "inputs > 126 MB L2 at every N (no flush needed)",
                       "timed_regions": len(regions), "region_ms_per_step": regions},
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": args.steps,
            "clocks": clocks, "verified": verified,
        }
        line.update(extras)
        print(json.dumps(line), file=_JSON_OUT, flush=True)
    if ctx.dist_on:
        dist.barrier()
        dist.destroy_process_group()


def e2e_run(ctx: Ctx, q, k, v, o, scale: float, steps: int) -> dict:
    """The headline metric through the public API with host buffers: every
    step copies its Q/K/V in from pinned host memory, runs FA2 and reads O
    back. Steps are pipelined over two device buffer sets on three streams
    (H2D, compute, D2H) as a serving loop would run them; the time is the max
    over ranks, each rank moving its own heads."""
    import torch
    from neso_b200 import ops

    dev, stream = ctx.dev, ctx.stream
    # Q, K and V of a step sit back to back in one pinned host buffer and one
    # device buffer (views), so each step's input is one host-to-device copy.
    hqkv = torch.empty((3,) + tuple(q.shape), dtype=q.dtype).pin_memory()
    for i, t in enumerate((q, k, v)):
        hqkv[i].copy_(t.cpu())
    ho = torch.empty(o.shape, dtype=o.dtype).pin_memory()
    dbuf = [torch.empty_like(hqkv, device=dev) for _ in range(2)]
    dqkv = [(b[0], b[1], b[2]) for b in dbuf]
    dout = [torch.empty_like(o), torch.empty_like(o)]
    s_h2d, s_comp, s_d2h = (torch.cuda.Stream(dev) for _ in range(3))
    nslot = 2

    def run(n: int) -> float:
        comp_done = [None] * nslot
        d2h_done = [None] * nslot
        ctx.barrier()
        torch.cuda.synchronize()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        for st in (s_h2d, s_comp, s_d2h):
            st.wait_event(start)
        for i in range(n):
            b = i % nslot
            dq, dk, dv = dqkv[b]
            with torch.cuda.stream(s_h2d):
                if comp_done[b] is not None:
                    s_h2d.wait_event(comp_done[b])  # FA2 of step i-2 has read this buffer set
                dbuf[b].copy_(hqkv, non_blocking=True)
                h2d_done = torch.cuda.Event()
                h2d_done.record(s_h2d)
            with torch.cuda.stream(s_comp):
                s_comp.wait_event(h2d_done)
                if d2h_done[b] is not None:
                    s_comp.wait_event(d2h_done[b])  # O of step i-2 has been read back
                ops.flash_attention(dq, dk, dv, scale, out=dout[b])
                comp_done[b] = torch.cuda.Event()
                comp_done[b].record(s_comp)
            with torch.cuda.stream(s_d2h):
                s_d2h.wait_event(comp_done[b])
                ho.copy_(dout[b], non_blocking=True)
                d2h_done[b] = torch.cuda.Event()
                d2h_done[b].record(s_d2h)
        for st in (s_h2d, s_comp, s_d2h):
            ev = torch.cuda.Event()
            ev.record(st)
            stream.wait_event(ev)
        end.record(stream)
        torch.cuda.synchronize()
        ctx.barrier()
        return ctx.max_over_ranks(start.elapsed_time(end) / n)

    run(2)
    n = max(3, min(2 * steps, 40))  # a longer pipelined run amortises its fill and drain
    ms = run(n)
    res = {"value": fa2_flops() / (ms * 1e-3) / 1e12, "unit": "TFLOP/s",
           "h2d_bytes_per_step": 3 * q.numel() * q.element_size() * ctx.world,
           "d2h_bytes_per_step": o.numel() * o.element_size() * ctx.world, "ms_per_step": ms,
           "steps": n, "gpu_launches": n,
           "pipelined": "two buffer sets per GPU; H2D, FA2 and D2H of different steps overlap"}
    del hqkv, ho, dbuf, dqkv, dout
    return res


if __name__ == "__main__":
    main()
