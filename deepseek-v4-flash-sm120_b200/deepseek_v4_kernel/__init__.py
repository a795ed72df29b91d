"""DeepSeek-V4-Flash / V3.2 sparse FP8 MLA decode for B200 (sm_100a).

Drop-in for the reference package's public surface
(deepseek_v4_kernel/__init__.py:1-7): ``sparse_decode_fwd`` and
``patch_flash_mla``; plus the FlashMLA-compatible interface functions,
the KV-cache writers that produce the FP8 pages (``cache_ops``), the
indexer logits that produce ``indices`` (``indexer``) and the sparse
prefill ``flash_mla_sparse_fwd`` (``prefill``).

The public names are resolved on first use (PEP 562), so importing a
host-only submodule such as ``deepseek_v4_kernel.kvcache`` or
``deepseek_v4_kernel.partition`` does not map ``libdsv4b.so``.  The first
use of any op loads the library and raises ImportError if it is not built;
there is no fallback path.
"""
from __future__ import annotations

import importlib

# public name -> (submodule, attribute)
_EXPORTS = {
    "patch_flash_mla": ("_patch", "install"),
    "concat_and_cache_mla": ("cache_ops", "concat_and_cache_mla"),
    "kv_cache_write": ("cache_ops", "kv_cache_write"),
    "quantize_and_insert_k_cache": ("cache_ops", "quantize_and_insert_k_cache"),
    "fp8_paged_mqa_logits": ("indexer", "fp8_paged_mqa_logits"),
    "get_paged_mqa_logits_metadata": ("indexer", "get_paged_mqa_logits_metadata"),
    "FlashMLASchedMeta": ("interface", "FlashMLASchedMeta"),
    "flash_mla_sparse_fwd": ("prefill", "flash_mla_sparse_fwd"),
    "flash_mla_with_kvcache": ("interface", "flash_mla_with_kvcache"),
    "get_mla_metadata": ("interface", "get_mla_metadata"),
    "gather_dequant": ("ops", "gather_dequant"),
    "read_kernel_status": ("ops", "read_kernel_status"),
    "sparse_decode_fwd": ("ops", "sparse_decode_fwd"),
}

__all__ = sorted(_EXPORTS)


def __getattr__(name):
    if name in _EXPORTS:
        mod, attr = _EXPORTS[name]
        value = getattr(importlib.import_module(f".{mod}", __name__), attr)
        globals()[name] = value
        return value
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")


def __dir__():
    return sorted(list(globals()) + __all__)
