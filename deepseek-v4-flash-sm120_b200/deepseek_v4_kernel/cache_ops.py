"""KV-cache writer: bf16 tokens -> the FP8 page formats the decode reads.

The producer of the bytes ``sparse_decode_fwd`` consumes.  The reference
reads caches written by SGLang's ``quant_k_cache_v4`` (named at
``tests/reference.py:45-49``); these functions keep the call signatures of
vLLM's writers for the same formats so a serving engine can swap them in:

* ``quantize_and_insert_k_cache(k, k_cache, slot_mapping, block_size,
  is_ue8m0)`` -- MODEL1 (vLLM ``models/deepseek_v4/common/ops/
  cache_utils.py:142-190``): k [n, 512] = 448 NoPE + 64 RoPE, pages of
  block_size x 576-B rows followed by block_size x 8 UE8M0 bytes.
* ``concat_and_cache_mla(kv_c, k_pe, kv_cache, slot_mapping,
  kv_cache_dtype="fp8_ds_mla", scale)`` -- V32 (vLLM
  ``_custom_ops.py:2613-2623``): 656-B records.

Both run one CUDA kernel (``dsv4b_kv_cache_write``) on the current stream;
nothing synchronises, so they can be captured in a CUDA graph.  Tokens
whose slot is negative or past the cache are skipped.  Errors raise
RuntimeError.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from ._lib import check, lib


def _cache_geometry(kv: torch.Tensor, layout: int, block_size: Optional[int]):
    """(num_blocks, page_block, stride_block_bytes, stride_row_bytes)."""
    if kv.dtype not in (torch.uint8, torch.float8_e4m3fn):
        raise RuntimeError(f"kv cache must be uint8 / float8_e4m3fn, got {kv.dtype}")
    e = kv.element_size()
    if kv.dim() == 2:                    # raw page arena [num_blocks, bytes per page]
        if not block_size:
            raise RuntimeError("a 2-D page arena needs block_size")
        row = 656 if layout == _lib.LAYOUT_V32 else 576
        return kv.size(0), int(block_size), kv.stride(0) * e, row
    if kv.dim() in (3, 4):               # [num_blocks, P, (1,) bytes per token]
        if kv.stride(-1) != 1:
            raise RuntimeError("kv cache last dim must be contiguous")
        if block_size and block_size != kv.size(1):
            raise RuntimeError(f"block_size {block_size} != cache page size {kv.size(1)}")
        return kv.size(0), kv.size(1), kv.stride(0) * e, kv.stride(1) * e
    raise RuntimeError(f"kv cache must be 2-D, 3-D or 4-D, got {kv.dim()}-D")


def _rows(t: torch.Tensor, cols: int, name: str) -> torch.Tensor:
    if t.dtype != torch.bfloat16:
        raise RuntimeError(f"{name} must be bf16, got {t.dtype}")
    if t.dim() != 2 or t.size(1) < cols or t.stride(1) != 1:
        raise RuntimeError(f"{name} must be [n, {cols}] with a contiguous last dim")
    return t


def kv_cache_write(layout: int, nope: torch.Tensor, rope: torch.Tensor, slot_mapping: torch.Tensor,
                   kv_cache: torch.Tensor, block_size: Optional[int] = None) -> None:
    """Quantise rows of ``nope`` (V32: 512 latent columns, MODEL1: 448) and
    ``rope`` (64 columns) into ``kv_cache`` at ``slot_mapping`` (int64 or
    int32, flat page * page_block + offset)."""
    n = slot_mapping.numel()
    cols = 512 if layout == _lib.LAYOUT_V32 else 448
    _rows(nope, cols, "nope")
    _rows(rope, 64, "rope")
    if nope.size(0) < n or rope.size(0) < n:
        raise RuntimeError(f"{n} slots for {nope.size(0)} / {rope.size(0)} token rows")
    if slot_mapping.dtype not in (torch.int64, torch.int32):
        raise RuntimeError(f"slot_mapping must be int64 / int32, got {slot_mapping.dtype}")
    slots = slot_mapping.reshape(-1)
    if not slots.is_contiguous():
        slots = slots.contiguous()
    devs = {t.device for t in (nope, rope, slots, kv_cache)}
    if len(devs) != 1 or next(iter(devs)).type != "cuda":
        raise RuntimeError("all tensors must be on one CUDA device")
    nb, page, sb, sr = _cache_geometry(kv_cache, layout, block_size)
    dev = kv_cache.device
    with torch.cuda.device(dev):
        check("dsv4b_kv_cache_write",
              lib.dsv4b_kv_cache_write(layout, nope.data_ptr(), nope.stride(0), rope.data_ptr(),
                                       rope.stride(0), slots.data_ptr(), slots.element_size(), n,
                                       kv_cache.data_ptr(), nb, page, sb, sr,
                                       torch.cuda.current_stream(dev).cuda_stream))


def kv_cache_write_status(device: Optional[torch.device] = None) -> int:
    """Status word of the writer kernels on ``device`` (0 = no error; 1 =
    a wait timed out and a write is incomplete); clears it.  Synchronises."""
    import ctypes
    device = device or torch.device("cuda", torch.cuda.current_device())
    flags = ctypes.c_int()
    with torch.cuda.device(device):
        check("dsv4b_kv_cache_write_status",
              lib.dsv4b_kv_cache_write_status(ctypes.byref(flags), torch.cuda.current_stream(device).cuda_stream))
    return int(flags.value)


def quantize_and_insert_k_cache(k: torch.Tensor, k_cache: torch.Tensor, slot_mapping: torch.Tensor,
                                block_size: int = 64, is_ue8m0: bool = True) -> None:
    """MODEL1 writer, vLLM's signature: k bf16 [n, 512] (448 NoPE | 64 RoPE)."""
    if not is_ue8m0:
        raise RuntimeError("only UE8M0 (power-of-two) scales are defined for MODEL1")
    if k.dim() != 2 or k.size(1) != 512:
        raise RuntimeError(f"k must be [num_tokens, 512], got {tuple(k.shape)}")
    kv_cache_write(_lib.LAYOUT_MODEL1, k, k[:, 448:], slot_mapping, k_cache, block_size)


def concat_and_cache_mla(kv_c: torch.Tensor, k_pe: torch.Tensor, kv_cache: torch.Tensor,
                         slot_mapping: torch.Tensor, kv_cache_dtype: str = "fp8_ds_mla",
                         scale: Optional[torch.Tensor] = None) -> None:
    """V32 writer, vLLM's signature: kv_c bf16 [n, 512], k_pe bf16 [n, 64],
    kv_cache [num_blocks, P, 656] (``scale`` is unused: fp8_ds_mla keeps
    its own per-tile scales)."""
    if kv_cache_dtype not in ("fp8_ds_mla", "fp8"):
        raise RuntimeError(f"kv_cache_dtype {kv_cache_dtype!r}: only fp8_ds_mla is built here")
    if k_pe.dim() == 3:
        k_pe = k_pe.squeeze(1)
    kv_cache_write(_lib.LAYOUT_V32, kv_c, k_pe, slot_mapping, kv_cache)
