"""Runtime patch that routes FlashMLA's sparse FP8 decode to the B200 kernel.

Same mechanism as the reference (deepseek_v4_kernel/_patch.py:161-265):
``install()`` replaces ``flash_mla.flash_mla_with_kvcache`` (and the
``flash_mla.flash_mla_interface`` attribute) and vLLM's vendored copy
``vllm.third_party.flashmla.flash_mla_interface.flash_mla_with_kvcache``
with a wrapper that takes the sparse + FP8 + bf16-q path on sm_100 GPUs
and defers everything else to the original function.  It also wraps
SGLang's two DeepSeek-V4 indexer fallbacks so that a 2-D ``seq_lens``
reaches them 1-D (reference ``_patch.py:199-236``).

Environment (own prefix, reference style): ``DSV4B_KERNEL_TRACE=1`` logs
each gating decision; ``DSV4B_KERNEL_STRICT=1`` re-raises errors of the
B200 path instead of falling back to upstream FlashMLA (the reference's
DSV4_KERNEL_STRICT); ``DSV4B_KERNEL_DISABLE=1`` makes install() a no-op.
"""
from __future__ import annotations

import logging
import os
from typing import Any, Callable

import torch

from .interface import sparse_with_sched_meta

_log = logging.getLogger("deepseek_v4_kernel.patch_flash_mla")
_INSTALLED = False
_SM100: dict = {}


def _current_is_sm100(device: torch.device) -> bool:
    """Cached per device (the reference queries device 0 on every call,
    _patch.py:35-39)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    v = _SM100.get(idx)
    if v is None:
        v = torch.cuda.is_available() and torch.cuda.get_device_capability(idx) == (10, 0)
        _SM100[idx] = v
    return v


def make_wrapper(original: Callable, schedmeta_cls: Any) -> Callable:
    """Drop-in replacement for ``flash_mla_with_kvcache``."""

    def flash_mla_with_kvcache(q, k_cache, block_table, cache_seqlens, head_dim_v,
                               tile_scheduler_metadata, num_splits=None, softmax_scale=None,
                               causal=False, is_fp8_kvcache=False, indices=None, attn_sink=None,
                               extra_k_cache=None, extra_indices_in_kvcache=None,
                               topk_length=None, extra_topk_length=None, out=None):
        decision = (
            indices is not None,
            isinstance(q, torch.Tensor) and q.is_cuda and _current_is_sm100(q.device),
            bool(is_fp8_kvcache),
            int(q.element_size()) if isinstance(q, torch.Tensor) else None,
        )
        if os.environ.get("DSV4B_KERNEL_TRACE", "0") == "1":
            _log.warning("dsv4b gating: %s q=%s kcache=%s", decision,
                         tuple(q.shape) if isinstance(q, torch.Tensor) else q,
                         tuple(k_cache.shape) if isinstance(k_cache, torch.Tensor) else k_cache)
        if all(decision[:3]) and decision[3] == 2:
            try:
                return sparse_with_sched_meta(
                    q, k_cache, head_dim_v, tile_scheduler_metadata, num_splits, softmax_scale,
                    causal, is_fp8_kvcache, indices, attn_sink, extra_k_cache,
                    extra_indices_in_kvcache, topk_length, extra_topk_length, out=out,
                    schedmeta_cls=schedmeta_cls)
            except Exception as exc:  # mirrors the reference's fallback
                if os.environ.get("DSV4B_KERNEL_STRICT", "0") == "1":
                    raise
                _log.warning("deepseek_v4_kernel (B200) sparse decode failed (%s); "
                             "falling back to upstream flash_mla.", exc)
        kwargs = dict(q=q, k_cache=k_cache, block_table=block_table, cache_seqlens=cache_seqlens,
                      head_dim_v=head_dim_v, tile_scheduler_metadata=tile_scheduler_metadata,
                      num_splits=num_splits, softmax_scale=softmax_scale, causal=causal,
                      is_fp8_kvcache=is_fp8_kvcache, indices=indices, attn_sink=attn_sink,
                      extra_k_cache=extra_k_cache,
                      extra_indices_in_kvcache=extra_indices_in_kvcache,
                      topk_length=topk_length, extra_topk_length=extra_topk_length)
        if out is not None:
            kwargs["out"] = out
        return original(**kwargs)

    flash_mla_with_kvcache.__wrapped__ = original  # type: ignore[attr-defined]
    flash_mla_with_kvcache.__dsv4b_patched__ = True  # type: ignore[attr-defined]
    return flash_mla_with_kvcache


def patch_module(module: Any, also: Any = None) -> bool:
    """Replace ``module.flash_mla_with_kvcache`` (and the same attribute on
    ``also``, a package re-exporting it).  Returns False if absent."""
    original = getattr(module, "flash_mla_with_kvcache", None)
    if original is None:
        return False
    if getattr(original, "__dsv4b_patched__", False):
        return True
    wrapped = make_wrapper(original, getattr(module, "FlashMLASchedMeta", None))
    module.flash_mla_with_kvcache = wrapped
    if also is not None and hasattr(also, "flash_mla_with_kvcache"):
        also.flash_mla_with_kvcache = wrapped
    return True


def _patch_flash_mla_pkg() -> bool:
    try:
        import flash_mla  # type: ignore
        from flash_mla import flash_mla_interface as fmi  # type: ignore
    except Exception:
        return False
    return patch_module(fmi, flash_mla)


def _patch_vllm_pkg() -> bool:
    try:
        from vllm.third_party.flashmla import flash_mla_interface as vfmi  # type: ignore
    except Exception:
        return False
    try:
        from vllm.third_party import flashmla as vpkg  # type: ignore
    except Exception:
        vpkg = None
    return patch_module(vfmi, vpkg)


def squeeze_seq_lens_wrapper(original: Callable) -> Callable:
    """Wrap an indexer-logits function ``f(q_fp8, kvcache_fp8, weight,
    seq_lens, ...)`` so that a ``[b, 1]`` ``seq_lens`` arrives as ``[b]``.

    SGLang's DeepSeek-V4 C4 indexer unsqueezes ``seq_lens`` to 2-D for
    DeepGEMM's signature but its fallbacks assert 1-D; the reference patches
    both fallbacks the same way (deepseek_v4_kernel/_patch.py:199-236).  On
    B200 SGLang normally takes DeepGEMM and never reaches the fallbacks; the
    patch keeps them usable when it does (e.g. DeepGEMM missing)."""
    def wrapper(q_fp8, kvcache_fp8, weight, seq_lens, *args, **kwargs):
        if isinstance(seq_lens, torch.Tensor) and seq_lens.dim() == 2 and seq_lens.shape[-1] == 1:
            seq_lens = seq_lens.squeeze(-1).contiguous()
        return original(q_fp8, kvcache_fp8, weight, seq_lens, *args, **kwargs)

    wrapper.__wrapped__ = original  # type: ignore[attr-defined]
    wrapper.__dsv4b_patched__ = True  # type: ignore[attr-defined]
    return wrapper


# (module, attribute) of SGLang's indexer fallbacks that get the wrapper.
INDEXER_FALLBACKS = (
    ("sglang.srt.layers.attention.nsa.tilelang_kernel", "tilelang_fp8_paged_mqa_logits"),
    ("sglang.srt.layers.attention.compressed.indexer", "fp8_paged_mqa_logits_torch"),
)


def _patch_sglang_indexer_fallbacks() -> int:
    """Wrap the SGLang indexer fallbacks that are importable; returns how
    many are (now) wrapped."""
    import importlib
    n = 0
    for mod_name, attr in INDEXER_FALLBACKS:
        try:
            mod = importlib.import_module(mod_name)
        except Exception:
            continue
        fn = getattr(mod, attr, None)
        if fn is None:
            continue
        if not getattr(fn, "__dsv4b_patched__", False):
            setattr(mod, attr, squeeze_seq_lens_wrapper(fn))
        n += 1
    return n


def install() -> bool:
    """Install the patch (idempotent).  Returns True if anything was patched."""
    global _INSTALLED
    if _INSTALLED:
        return True
    if os.environ.get("DSV4B_KERNEL_DISABLE", "0") == "1":
        return False
    patched = _patch_flash_mla_pkg()
    patched = _patch_vllm_pkg() or patched
    _patch_sglang_indexer_fallbacks()
    if not patched:
        _log.warning("deepseek_v4_kernel: neither flash_mla nor vllm.third_party.flashmla "
                     "was importable; nothing patched.")
        return False
    _INSTALLED = True
    _log.info("deepseek_v4_kernel.patch_flash_mla installed (B200 sm_100a sparse decode).")
    return True
