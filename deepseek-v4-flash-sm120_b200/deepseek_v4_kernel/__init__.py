"""DeepSeek-V4-Flash / V3.2 sparse FP8 MLA decode for B200 (sm_100a).

Drop-in for the reference package's public surface
(deepseek_v4_kernel/__init__.py:1-7): ``sparse_decode_fwd`` and
``patch_flash_mla``; plus the FlashMLA-compatible interface functions
the KV-cache writers that produce the FP8 pages (``cache_ops``) and the
indexer logits that produce ``indices`` (``indexer``).
Importing loads ``libdsv4b.so`` (ImportError if it is not built).
"""
from __future__ import annotations

from ._patch import install as patch_flash_mla  # noqa: F401
from .cache_ops import concat_and_cache_mla, kv_cache_write, quantize_and_insert_k_cache  # noqa: F401
from .indexer import fp8_paged_mqa_logits, get_paged_mqa_logits_metadata  # noqa: F401
from .interface import FlashMLASchedMeta, flash_mla_with_kvcache, get_mla_metadata  # noqa: F401
from .ops import gather_dequant, read_kernel_status, sparse_decode_fwd  # noqa: F401

__all__ = [
    "sparse_decode_fwd",
    "patch_flash_mla",
    "flash_mla_with_kvcache",
    "get_mla_metadata",
    "FlashMLASchedMeta",
    "gather_dequant",
    "read_kernel_status",
    "kv_cache_write",
    "quantize_and_insert_k_cache",
    "concat_and_cache_mla",
    "fp8_paged_mqa_logits",
    "get_paged_mqa_logits_metadata",
]
