"""FlashMLA-compatible Python surface for the sparse FP8 decode path.

The names and arguments are those of FlashMLA's ``flash_mla_interface``
(vLLM 0.22 ``third_party/flashmla/flash_mla_interface.py:9-176``), which
the reference wraps (deepseek_v4_kernel/_patch.py:45-158):

* ``FlashMLASchedMeta``  scheduler state, filled in on the first call and
  reused afterwards (same fields and Config record as upstream).
* ``get_mla_metadata(*args, **kwargs) -> (FlashMLASchedMeta(), None)``.
* ``flash_mla_with_kvcache(q, k_cache, block_table, cache_seqlens,
  head_dim_v, tile_scheduler_metadata, num_splits=None, softmax_scale=None,
  causal=False, is_fp8_kvcache=False, indices=None, attn_sink=None,
  extra_k_cache=None, extra_indices_in_kvcache=None, topk_length=None,
  extra_topk_length=None, out=None) -> (out, lse)``.

Only the sparse path (``indices is not None``) is implemented here; it is
the one this package replaces.  Dense decode raises NotImplementedError
(the patched entry point in ``_patch.py`` routes it to upstream).
"""
from __future__ import annotations

import dataclasses
from typing import Any, Optional, Tuple

import torch

from .ops import sparse_decode_fwd


@dataclasses.dataclass
class FlashMLASchedMeta:
    """Tile-scheduler state (flash_mla_interface.py:9-33)."""

    @dataclasses.dataclass
    class Config:
        b: int
        s_q: int
        h_q: int
        page_block_size: int
        h_k: int
        causal: bool
        is_fp8_kvcache: bool
        topk: Optional[int]
        extra_page_block_size: Optional[int]
        extra_topk: Optional[int]

    have_initialized: bool = False
    config: Optional[Config] = None
    tile_scheduler_metadata: Optional[torch.Tensor] = None
    num_splits: Optional[torch.Tensor] = None


def get_mla_metadata(*args, **kwargs) -> Tuple[FlashMLASchedMeta, None]:
    """Empty scheduler state; the schedule is computed on the device by the
    first ``flash_mla_with_kvcache`` call (flash_mla_interface.py:38-51)."""
    return FlashMLASchedMeta(), None


def _config_of(schedmeta_cls, q, k_cache, causal, is_fp8_kvcache, indices, extra_k_cache,
               extra_indices):
    return schedmeta_cls.Config(
        q.shape[0], q.shape[1], q.shape[2], k_cache.shape[1], k_cache.shape[2],
        causal, is_fp8_kvcache, indices.shape[-1],
        extra_k_cache.shape[1] if extra_k_cache is not None else None,
        extra_indices.shape[-1] if extra_indices is not None else None)


def sparse_with_sched_meta(
    q, k_cache, head_dim_v, sched_meta: Any, num_splits, softmax_scale, causal,
    is_fp8_kvcache, indices, attn_sink, extra_k_cache, extra_indices_in_kvcache,
    topk_length, extra_topk_length, out=None, schedmeta_cls: Any = None,
):
    """Sparse decode with FlashMLA's scheduler-state protocol: accepts a
    FlashMLASchedMeta (any class with the same fields) or raw tensors, runs
    the B200 op, stores the scheduler tensors back and fills the Config on
    first use (reference _patch.py:79-126)."""
    if softmax_scale is None:
        softmax_scale = q.shape[-1] ** (-0.5)
    if causal:
        raise RuntimeError("causal must be False when sparse attention is enabled")
    if not is_fp8_kvcache:
        raise RuntimeError("is_fp8_kvcache must be True when sparse attention is enabled")
    is_meta = schedmeta_cls is not None and isinstance(sched_meta, schedmeta_cls)
    if is_meta:
        tsm, ns = sched_meta.tile_scheduler_metadata, sched_meta.num_splits
    elif isinstance(sched_meta, torch.Tensor):
        tsm, ns = sched_meta, num_splits
    else:
        tsm = ns = None
    o, lse, tsm, ns = sparse_decode_fwd(
        q, k_cache, indices, topk_length, attn_sink, tsm, ns, extra_k_cache,
        extra_indices_in_kvcache, extra_topk_length, head_dim_v, float(softmax_scale), out=out)
    if is_meta:
        sched_meta.tile_scheduler_metadata = tsm
        sched_meta.num_splits = ns
        if not sched_meta.have_initialized:
            sched_meta.have_initialized = True
            sched_meta.config = _config_of(schedmeta_cls, q, k_cache, causal, is_fp8_kvcache,
                                           indices, extra_k_cache, extra_indices_in_kvcache)
    return o, lse


def flash_mla_with_kvcache(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    block_table: Optional[torch.Tensor],
    cache_seqlens: Optional[torch.Tensor],
    head_dim_v: int,
    tile_scheduler_metadata: Any,
    num_splits: Any = None,
    softmax_scale: Optional[float] = None,
    causal: bool = False,
    is_fp8_kvcache: bool = False,
    indices: Optional[torch.Tensor] = None,
    attn_sink: Optional[torch.Tensor] = None,
    extra_k_cache: Optional[torch.Tensor] = None,
    extra_indices_in_kvcache: Optional[torch.Tensor] = None,
    topk_length: Optional[torch.Tensor] = None,
    extra_topk_length: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor]:
    """Sparse FP8 MLA decode; ``block_table`` / ``cache_seqlens`` are unused
    in sparse mode (indices are page*page_block_size + offset)."""
    if indices is None:
        raise NotImplementedError("dense MLA decode is not part of this package")
    return sparse_with_sched_meta(
        q, k_cache, head_dim_v, tile_scheduler_metadata, num_splits, softmax_scale, causal,
        is_fp8_kvcache, indices, attn_sink, extra_k_cache, extra_indices_in_kvcache,
        topk_length, extra_topk_length, out=out, schedmeta_cls=FlashMLASchedMeta)
