"""Sharding of the hot-path kernels across the GPUs of one node.

Every kernel here partitions into independent units with no cross-GPU
reduction (one process per GPU, torch.distributed for the plumbing):

* FA2: over batch x heads — rank r owns a contiguous range of the flattened
  (b, h) index;
* dense GEMM and quantized matmul: over output columns (N), in whole column
  groups of ``align`` (16 by default, so int8 / fp16 column slices start on a
  16-byte boundary and stay valid TMA bases);
* elementwise: contiguous element ranges aligned to 1024.

Each rank computes its slice directly into the matching slice of a full-size
output where strides allow (GEMM / W8A16 column slices via the reference
signatures' row strides), and :func:`gather` all-gathers the per-rank pieces
to every rank (NCCL over NVLink on GPUs, gloo on CPU) — used for
verification only, never inside a timed step.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Sequence

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class Shard:
    start: int
    stop: int

    @property
    def size(self) -> int:
        return self.stop - self.start

    def slice(self) -> slice:
        return slice(self.start, self.stop)


def shard_range(n: int, world: int, rank: int, align: int = 1) -> Shard:
    """Split [0, n) into `world` contiguous pieces whose boundaries are
    multiples of `align` (the last piece takes the remainder). Pieces differ in
    size by at most one `align` unit; trailing ranks may be empty."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if n < 0 or align <= 0:
        raise ValueError("n must be >= 0 and align > 0")
    units = (n + align - 1) // align
    base, extra = divmod(units, world)
    u0 = rank * base + min(rank, extra)
    u1 = u0 + base + (1 if rank < extra else 0)
    return Shard(min(n, u0 * align), min(n, u1 * align))


def shard_heads(B: int, H: int, world: int, rank: int) -> Shard:
    """Contiguous range of the flattened (b, h) index owned by `rank`."""
    return shard_range(B * H, world, rank, 1)


def shard_columns(N: int, world: int, rank: int, align: int = 16) -> Shard:
    """Output-column range owned by `rank` (N-tile sharding)."""
    return shard_range(N, world, rank, align)


def gather(local: torch.Tensor, sizes: Sequence[int], dim: int = 0, group=None) -> torch.Tensor:
    """All-gather per-rank pieces of different sizes along `dim` and return the
    concatenation (every rank receives it). Pieces are padded to the largest
    size for the collective and trimmed afterwards."""
    world = dist.get_world_size(group)
    if len(sizes) != world:
        raise ValueError("one size per rank")
    local = local.movedim(dim, 0).contiguous()
    cap = max(sizes) if sizes else 0
    pad = torch.zeros((cap,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    out = torch.empty((world * cap,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, pad, group=group)
    else:
        chunks = list(out.chunk(world))
        dist.all_gather(chunks, pad, group=group)
        out = torch.cat(chunks)
    pieces = [out[r * cap: r * cap + sizes[r]] for r in range(world)]
    return torch.cat(pieces).movedim(0, dim)


def attention_sharded(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, compute: Callable[..., torch.Tensor],
                      world: int, rank: int, **kw) -> tuple[torch.Tensor, Shard]:
    """Run `compute(q, k, v, **kw)` on this rank's (b, h) shard of
    [B, H, S, D] inputs; returns the [heads, S, D] piece and its shard."""
    B, H, S, D = q.shape
    sh = shard_heads(B, H, world, rank)
    flat = lambda t: t.reshape(B * H, S, D)[sh.slice()].reshape(1, sh.size, S, D)
    table = kw.pop("table", None)
    if table is not None and sh.size:
        # heads of the shard may wrap around H (several batches): expand the table per flattened head
        heads = torch.arange(sh.start, sh.stop, device=table.device) % H
        kw["table"] = table[heads]
    out = compute(flat(q), flat(k), flat(v), **kw) if sh.size else q.new_empty((1, 0, S, D), dtype=torch.float32)
    return out.reshape(sh.size, S, D), sh


def matmul_sharded(a: torch.Tensor, b: torch.Tensor, compute: Callable[..., torch.Tensor], world: int,
                   rank: int) -> tuple[torch.Tensor, Shard]:
    """C[:, cols] = compute(A, B[:, cols]) for this rank's column shard."""
    sh = shard_columns(b.shape[1], world, rank)
    return compute(a, b[:, sh.slice()].contiguous()), sh
