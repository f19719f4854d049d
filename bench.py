#!/usr/bin/env python3
"""Benchmark of the Neso B200 hot path; prints ONE JSON line (rank 0).

Headline workload (BASELINE.json metric "FA2 fwd TFLOP/s (D=64,S=2048)"):
Flash Attention 2 forward, fp16 Q/K/V [B=16, H=16, S=2048, D=64] drawn N(0,1)
from a seed, softmax scale 1/8, fp32 accumulation and fp32 O, non-causal.
One step = one FA2 forward over that batch (one kernel launch). The inputs
(3 x 64 MiB fp16 + 128 MiB fp32 out) are larger than the 126 MB L2, so no L2
flush is needed between steps.

Multi-GPU (``torchrun --nproc-per-node N``): every rank owns its own
B x H = 16 x 16 slice of a global batch of 16 N sequences (sharding along
batch x heads, no cross-GPU reduction) -> "scaling": "weak". The step time is
the max over ranks of the CUDA-event time (NCCL all-reduce MAX); after timing,
each rank's first head is all-gathered to rank 0 over NCCL and checked against
the CPU oracle (``verified``).

``--impl reference`` times the reference algorithm's CPU implementation (the
torch-fp32 oracle port: the reference's own kernels are Metal/HLSL and cannot
run here) on the host cores, one bounded sample per step.

Also reported (not part of ``value``): the quantized GEMM (W8A16 / W4A16,
K=4096, N=11008, M in {1, 16, 128, 2048}) TFLOP/s, the e2e number through the
public API with host buffers (each step copies its Q/K/V in from pinned host
memory and reads O back; consecutive steps overlap on separate copy and compute
streams), the roofline of the FA2 kernel and the CPU baseline.
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


def run_reference(args, rank: int) -> None:
    """--impl reference: the reference algorithm's CPU implementation (torch
    fp32 oracle port) on the host cores, one head of the workload per step."""
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
        "impl": "reference", "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": per * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "config": {"workload": f"FA2 fwd B={B} H={H} S={S} D={D} non-causal (one head per step on CPU)",
                   "global_batch": B * args.gpus, "seq_len": S, "parallelism": f"dp{args.gpus}"},
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": threads, "kind": "port",
                         "sample": f"1 head [S={S}, D={D}] per step, torch CPU fp32 oracle (reference kernels "
                                   f"are Metal/HLSL: unavailable on this box)"},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), file=_JSON_OUT, flush=True)


def time_steps(fn, steps: int, stream, dist_on: bool) -> float:
    """Barrier + sync, K steps between CUDA events on `stream`, barrier + sync.
    Returns the step time in ms (max over ranks)."""
    import torch
    import torch.distributed as dist

    if dist_on:
        dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    if dist_on:
        dist.barrier()
    ms = start.elapsed_time(end) / steps
    if dist_on:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="neso", choices=["neso", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=12.0, help="seconds of CPU-baseline work (rank 0, N=1)")
    ap.add_argument("--no-extras", action="store_true", help="skip the quant-GEMM and e2e side measurements")
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
        run_reference(args, rank)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from neso_b200 import _lib, ops

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist_on = world > 1
    if dist_on:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    stream = torch.cuda.current_stream(dev)

    gen = torch.Generator(device=dev).manual_seed(SEED + rank)
    q, k, v = (torch.randn(B, H, S, D, device=dev, generator=gen).half() for _ in range(3))
    o = torch.empty(B, H, S, D, device=dev, dtype=torch.float32)
    scale = 1.0 / math.sqrt(D)

    def step():
        ops.flash_attention(q, k, v, scale, out=o)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        ms = time_steps(step, args.steps, stream, dist_on)
    clocks = clk.summary()
    flops_rank = fa2_flops()
    value = world * flops_rank / (ms * 1e-3) / 1e12

    # Roofline of the dominant (only) kernel in the step: one launch per step.
    peaks, peak_src = load_peaks()
    achieved = flops_rank / (ms * 1e-3) / 1e12
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    traffic = load_traffic("fa2_fwd_d64_s2048")
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": traffic,
                "peak_source": f"{peak_src} bf16_tflops (burst, kernel timed alone)",
                "kernel": "fa2_tile_kernel<64,1,false,0>"}

    # Verification after timing: NCCL all-gather of each rank's first head to rank 0.
    verified = None
    if dist_on:
        head = o[0, 0].contiguous()
        gathered = torch.empty((world,) + tuple(head.shape), device=dev, dtype=head.dtype)
        dist.all_gather_into_tensor(gathered, head)
    else:
        gathered = o[0, 0].unsqueeze(0)

    extras: dict = {}
    e2e = None
    if rank == 0:
        import oracle
        ok = True
        for r in range(world):
            gr = torch.Generator(device=dev).manual_seed(SEED + r)
            qr, kr, vr = (torch.randn(B, H, S, D, device=dev, generator=gr).half() for _ in range(3))
            ref = oracle.attention(qr[0, 0].cpu(), kr[0, 0].cpu(), vr[0, 0].cpu(), scale)
            ok = ok and torch.allclose(gathered[r].cpu(), ref, atol=2e-3, rtol=2e-3)
            del qr, kr, vr
        verified = bool(ok)

    if not args.no_extras and rank == 0:
        # e2e through the public API with host buffers: every step copies its
        # Q/K/V in from pinned host memory, runs FA2 and reads O back. Steps
        # are pipelined over two device buffer sets on three streams (H2D,
        # compute, D2H), so the H2D and D2H copy engines and the SMs work at
        # the same time, as a serving loop would run them.
        hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
        ho = torch.empty(o.shape, dtype=o.dtype).pin_memory()
        dqkv = [tuple(torch.empty_like(q) for _ in range(3)) for _ in range(2)]
        dout = [o, torch.empty_like(o)]
        s_h2d, s_comp, s_d2h = (torch.cuda.Stream(dev) for _ in range(3))
        nslot = 2
        comp_done = [None] * nslot
        d2h_done = [None] * nslot

        def e2e_run(steps: int) -> float:
            for i in range(nslot):
                comp_done[i] = d2h_done[i] = None
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            start.record(stream)
            for st in (s_h2d, s_comp, s_d2h):
                st.wait_event(start)
            for i in range(steps):
                b = i % nslot
                dq, dk, dv = dqkv[b]
                with torch.cuda.stream(s_h2d):
                    if comp_done[b] is not None:
                        s_h2d.wait_event(comp_done[b])  # FA2 of step i-2 has read this buffer set
                    dq.copy_(hq, non_blocking=True)
                    dk.copy_(hk, non_blocking=True)
                    dv.copy_(hv, non_blocking=True)
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
            return start.elapsed_time(end) / steps

        e2e_run(2)
        e2e_steps = max(3, min(args.steps, 20))
        ms_e2e = e2e_run(e2e_steps)
        e2e = {"value": flops_rank / (ms_e2e * 1e-3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": 3 * q.numel() * q.element_size(),
               "d2h_bytes_per_step": o.numel() * o.element_size(), "ms_per_step": ms_e2e,
               "steps": e2e_steps, "gpu_launches": e2e_steps,
               "pipelined": "two buffer sets; H2D, FA2 and D2H of different steps overlap"}
        del hq, hk, hv, ho, dqkv, dout

        # Quantized GEMM side measurements, not part of `value`.
        try:
            extras["quant_gemm"] = quant_side(dev, stream)
        except Exception as e:  # pragma: no cover - reported, not fatal
            extras["quant_gemm"] = {"error": str(e)}

    cpu = None
    if rank == 0 and world == 1:
        cpu = cpu_fa2_sample(args.cpu_budget, host_threads())

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
            "config": {"workload": f"FA2 fwd B={B} H={H} S={S} D={D} non-causal, fp16 in, fp32 acc/out, per GPU",
                       "global_batch": B * world, "heads": H, "seq_len": S, "head_dim": D,
                       "parallelism": f"dp{world} (batch x heads shards, no collective in the step)",
                       "l2": "inputs 320 MiB > 126 MB L2 (no flush needed)"},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": args.steps,
            "clocks": clocks, "verified": verified,
        }
        line.update(extras)
        print(json.dumps(line), file=_JSON_OUT, flush=True)
    if dist_on:
        dist.barrier()
        dist.destroy_process_group()


def quant_side(dev, stream) -> dict:
    """W8A16 / W4A16 TFLOP/s at M = 2048 and weight-stream GB/s at M = 1
    (K = 4096, N = 11008); three weight copies rotate so M = 1 reads HBM."""
    import torch
    from neso_b200 import ops

    K, N = 4096, 11008
    out = {}
    g = torch.Generator(device=dev).manual_seed(7)
    ws = [torch.randint(-127, 128, (K, N), device=dev, dtype=torch.int8, generator=g) for _ in range(3)]
    wq = [torch.randint(0, 256, (K // 2, N), device=dev, dtype=torch.uint8, generator=g) for _ in range(3)]
    s8 = (torch.rand(N, device=dev, generator=g) * 0.019 + 0.001).half()
    s4 = (torch.rand(K // 128, N, device=dev, generator=g) * 0.019 + 0.001).half()
    for M in (1, 16, 128, 2048):
        x = torch.randn(M, K, device=dev, generator=g).half()
        y = torch.empty(M, N, device=dev)
        for name, fn in (("w8a16", lambda i: ops.w8a16_matmul(x, ws[i % 3], s8, out=y)),
                         ("w4a16", lambda i: ops.w4a16_g128_matmul(x, wq[i % 3], s4, out=y))):
            for i in range(3):
                fn(i)
            torch.cuda.synchronize()
            iters = 30
            st, en = torch.cuda.Event(True), torch.cuda.Event(True)
            st.record(stream)
            for i in range(iters):
                fn(i)
            en.record(stream)
            torch.cuda.synchronize()
            t = st.elapsed_time(en) / iters * 1e-3
            wbytes = K * N if name == "w8a16" else K * N // 2
            out[f"{name}_m{M}"] = {"tflops": 2.0 * M * N * K / t / 1e12, "us": t * 1e6,
                                   "weight_gbs": wbytes / t / 1e9}
    return out


if __name__ == "__main__":
    main()
