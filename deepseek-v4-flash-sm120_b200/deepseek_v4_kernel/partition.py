"""Partition layer for one 8 x B200 box (one process per GPU).

The reference has no multi-GPU code of its own (SGLang runs it with TP=4,
scripts/launch_dsv4_flash_sm120.sh:73, and the kernel sees one TP shard,
csrc/sm120/decode/sparse_decode_kernel.cuh:35).  Sparse decode needs no
collective: query rows are independent.

* Batch sharding: rank r owns requests [batch_range(b, r, N)) and the KV
  pages those requests reference; it runs metadata + decode + combine on
  its slice alone.  No data-path collective.
* Head sharding (mirrors TP): rank r owns heads [head_range(h_q, r, N)) and
  the matching attn_sink slice over a replicated cache; ``all_gather_heads``
  reassembles the bf16 outputs with one NCCL all-gather (used to verify).
"""
from __future__ import annotations

from typing import Tuple

import torch


def even_range(n: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous share of n items for rank (sizes differ by at most 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank / world")
    lo = n * rank // world
    hi = n * (rank + 1) // world
    return lo, hi


def batch_range(b: int, rank: int, world: int) -> Tuple[int, int]:
    return even_range(b, rank, world)


def head_range(h_q: int, rank: int, world: int) -> Tuple[int, int]:
    if h_q % world:
        raise ValueError(f"h_q={h_q} must divide evenly over {world} ranks for head sharding")
    return even_range(h_q, rank, world)


def shard_batch(q, indices, topk_length, rank, world):
    """Slice the per-request inputs of a batch for this rank."""
    lo, hi = batch_range(q.shape[0], rank, world)
    tk = None if topk_length is None else topk_length[lo:hi]
    return q[lo:hi], indices[lo:hi], tk, (lo, hi)


def shard_heads(q, attn_sink, rank, world):
    lo, hi = head_range(q.shape[2], rank, world)
    s = None if attn_sink is None else attn_sink[lo:hi].contiguous()
    return q[:, :, lo:hi].contiguous(), s, (lo, hi)


def all_gather_heads(out_local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """[b, s_q, h/N, d] per rank -> [b, s_q, h, d] on every rank (one
    all_gather_into_tensor; NCCL over NVLink on GPUs, gloo on CPU)."""
    import torch.distributed as dist
    b, s, hl, d = out_local.shape
    buf = torch.empty((world, b, s, hl, d), dtype=out_local.dtype, device=out_local.device)
    if out_local.is_cuda:
        dist.all_gather_into_tensor(buf, out_local.contiguous(), group=group)
    else:
        dist.all_gather(list(buf.unbind(0)), out_local.contiguous(), group=group)
    return buf.permute(1, 2, 0, 3, 4).reshape(b, s, world * hl, d)


def all_gather_batch(out_local: torch.Tensor, b_total: int, world: int, group=None) -> torch.Tensor:
    """Reassemble batch shards (sizes may differ by one) on every rank."""
    import torch.distributed as dist
    shapes = [batch_range(b_total, r, world) for r in range(world)]
    maxb = max(hi - lo for lo, hi in shapes)
    pad = torch.zeros((maxb,) + tuple(out_local.shape[1:]), dtype=out_local.dtype,
                      device=out_local.device)
    pad[: out_local.shape[0]] = out_local
    bufs = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(bufs, pad, group=group)
    return torch.cat([bufs[r][: hi - lo] for r, (lo, hi) in enumerate(shapes)], dim=0)
