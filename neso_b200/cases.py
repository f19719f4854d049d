"""Run one kernel of the library on synthetic inputs, for profiling and timing.

    python -m neso_b200.cases fa2 --B 16 --H 16 --S 2048 --D 64 [--causal] [--iters 5]
    python -m neso_b200.cases relpos --H 64 --S 2048 --D 64      (rel_pos_fa2_fwd, dense fp16 bias)
    python -m neso_b200.cases gemm --M 4096 --N 4096 --K 4096
    python -m neso_b200.cases w8a16 --M 1 --N 11008 --K 4096
    python -m neso_b200.cases w4a16 --M 2048 --N 11008 --K 4096
    python -m neso_b200.cases vector_add --n 268435456

Each case launches the op ``--warmup`` times, then ``--iters`` times between
CUDA events on the current stream, and prints one JSON line with the mean
time and the achieved TFLOP/s or GB/s (algorithmic work, as in bench.py).
With ``--graph`` the timed calls are replayed from one CUDA graph instead, so
small problems show their device time rather than the host's per-call cost.
Inputs smaller than twice the 126 MB L2 (quantized-matmul weights, small
attention and GEMM problems) rotate over enough copies to exceed 256 MB, so
every call reads HBM rather than L2.
"""
from __future__ import annotations

import argparse
import json
import math

import torch

from . import ops


GRAPH = False
L2_FLOOR = 256 << 20


def _copies(nbytes: int) -> int:
    return max(1, -(-L2_FLOOR // max(1, nbytes)))


def _time(fn, warmup: int, iters: int) -> float:
    if GRAPH:
        return _time_graph(fn, warmup, iters)
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for i in range(iters):
        fn(i)
    en.record()
    torch.cuda.synchronize()
    return st.elapsed_time(en) / iters * 1e-3


def _time_graph(fn, warmup: int, iters: int) -> float:
    """Device time per call without the host's per-call cost: the warm-up runs
    on the capture stream (so per-stream work counters exist before capture),
    then ``iters`` calls are captured in one CUDA graph and replayed."""
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        for i in range(max(warmup, 1)):
            fn(i)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for i in range(iters):
            fn(i)
    g.replay()
    torch.cuda.synchronize()
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(s):
        st.record()
        g.replay()
        en.record()
    torch.cuda.synchronize()
    return st.elapsed_time(en) / iters * 1e-3


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["fa2", "relpos", "gemm", "w8a16", "w4a16", "vector_add", "scale"])
    ap.add_argument("--B", type=int, default=16)
    ap.add_argument("--H", type=int, default=16)
    ap.add_argument("--S", type=int, default=2048)
    ap.add_argument("--D", type=int, default=64)
    ap.add_argument("--causal", action="store_true")
    ap.add_argument("--table", action="store_true", help="FA2 with the fp32 relative-position table")
    ap.add_argument("--M", type=int, default=4096)
    ap.add_argument("--N", type=int, default=4096)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--n", type=int, default=1 << 28)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--graph", action="store_true",
                    help="time the calls replayed from one CUDA graph (device time, no per-call host cost)")
    a = ap.parse_args()
    global GRAPH
    GRAPH = a.graph
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    res: dict = {"case": a.case}
    if a.case == "fa2":
        sets = [tuple(torch.randn(a.B, a.H, a.S, a.D, device=dev, generator=g).half() for _ in range(3))
                for _ in range(_copies(10 * a.B * a.H * a.S * a.D))]
        o = torch.empty(a.B, a.H, a.S, a.D, device=dev)
        table = torch.randn(a.H, 2 * a.S - 1, device=dev, generator=g) * 0.02 if a.table else None
        n = len(sets)
        t = _time(lambda i: ops.flash_attention(*sets[i % n], 1 / math.sqrt(a.D), causal=a.causal, table=table,
                                                out=o), a.warmup, a.iters)
        flops = 4.0 * a.B * a.H * a.S * a.S * a.D / (2 if a.causal else 1)
        res.update(shape=[a.B, a.H, a.S, a.D], causal=a.causal, table=a.table, us=t * 1e6, tflops=flops / t / 1e12)
    elif a.case == "relpos":
        from . import kernels
        nh, T, d = a.H, a.S, a.D
        sets = [(tuple(torch.randn(nh, T, d, device=dev, generator=g).half() for _ in range(3)),
                 (0.5 * torch.randn(nh, T, T, device=dev, generator=g)).half())
                for _ in range(_copies(2 * nh * T * T + 8 * nh * T * d))]
        o = torch.empty(nh, T, d, dtype=torch.float16, device=dev)
        bm = next(b for b in (128, 64, 32, 16, 8) if T % b == 0)
        launch = kernels.rel_pos_fa2_fwd[(T // bm, nh, 1)]
        n = len(sets)
        t = _time(lambda i: launch(*sets[i % n][0], sets[i % n][1], o, T, d, 1 / math.sqrt(d), T * d, T * T),
                  a.warmup, a.iters)
        res.update(shape=[nh, T, d], us=t * 1e6, tflops=4.0 * nh * T * T * d / t / 1e12,
                   bias_gbs=2.0 * nh * T * T / t / 1e9)
    elif a.case == "gemm":
        x = (torch.randn(a.M, a.K, device=dev, generator=g) / math.sqrt(a.K)).half()
        w = (torch.randn(a.K, a.N, device=dev, generator=g) / math.sqrt(a.K)).half()
        sets = [(x, w)] + [(x.clone(), w.clone()) for _ in range(_copies(2 * (a.M + a.N) * a.K + 4 * a.M * a.N) - 1)]
        c = torch.empty(a.M, a.N, device=dev)
        n = len(sets)
        t = _time(lambda i: ops.matmul(*sets[i % n], out=c), a.warmup, a.iters)
        res.update(shape=[a.M, a.N, a.K], us=t * 1e6, tflops=2.0 * a.M * a.N * a.K / t / 1e12)
    elif a.case in ("w8a16", "w4a16"):
        x = torch.randn(a.M, a.K, device=dev, generator=g).half()
        y = torch.empty(a.M, a.N, device=dev)
        if a.case == "w8a16":
            ws = [torch.randint(-127, 128, (a.K, a.N), device=dev, dtype=torch.int8, generator=g)
                  for _ in range(_copies(a.K * a.N))]
            s = (torch.rand(a.N, device=dev, generator=g) * 0.019 + 0.001).half()
            t = _time(lambda i: ops.w8a16_matmul(x, ws[i % len(ws)], s, out=y), a.warmup, a.iters)
            wbytes = a.K * a.N
        else:
            ws = [torch.randint(0, 256, (a.K // 2, a.N), device=dev, dtype=torch.uint8, generator=g)
                  for _ in range(_copies(a.K * a.N // 2))]
            s = (torch.rand(a.K // 128, a.N, device=dev, generator=g) * 0.019 + 0.001).half()
            t = _time(lambda i: ops.w4a16_g128_matmul(x, ws[i % len(ws)], s, out=y), a.warmup, a.iters)
            wbytes = a.K * a.N // 2
        res.update(shape=[a.M, a.N, a.K], us=t * 1e6, tflops=2.0 * a.M * a.N * a.K / t / 1e12,
                   weight_gbs=wbytes / t / 1e9)
    else:
        x = torch.rand(a.n, device=dev, generator=g) * 2 - 1
        y = torch.rand(a.n, device=dev, generator=g) * 2 - 1
        z = torch.empty_like(x)
        if a.case == "vector_add":
            t = _time(lambda i: ops.vector_add(x, y, out=z), a.warmup, a.iters)
            nbytes = 12 * a.n
        else:
            t = _time(lambda i: ops.scale(x, 0.5, out=z), a.warmup, a.iters)
            nbytes = 8 * a.n
        res.update(n=a.n, us=t * 1e6, gbs=nbytes / t / 1e9)
    res["timing"] = "cuda_graph" if a.graph else "eager"
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
