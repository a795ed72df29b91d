"""Indexer logits for the top-k selection that produces ``indices``.

``fp8_paged_mqa_logits`` and ``get_paged_mqa_logits_metadata`` keep the
signatures of DeepGEMM's functions as vLLM binds them (vLLM
``utils/deep_gemm.py:386-460``; SGLang's DeepSeek-V4 indexer calls the
same kernel on sm_100).  The reference does not compute this step: it only
wraps SGLang's fallbacks (deepseek_v4_kernel/_patch.py:199-236, mirrored
in ``_patch.squeeze_seq_lens_wrapper``).  Here it is a tcgen05 kernel
(``dsv4b_fp8_paged_mqa_logits``); see include/dsv4b.h for the exact
contract.  One launch on the current stream, no host synchronisation.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple, Union

import torch

from ._lib import check, lib


class MqaLogitsParams(ctypes.Structure):
    _fields_ = [
        ("b", ctypes.c_int32), ("next_n", ctypes.c_int32), ("h", ctypes.c_int32), ("d", ctypes.c_int32),
        ("q", ctypes.c_void_p), ("kv", ctypes.c_void_p),
        ("num_blocks", ctypes.c_int32), ("page_block_size", ctypes.c_int32),
        ("stride_kv_block", ctypes.c_int64),
        ("weights", ctypes.c_void_p), ("context_lens", ctypes.c_void_p), ("block_table", ctypes.c_void_p),
        ("stride_block_table", ctypes.c_int64),
        ("logits", ctypes.c_void_p), ("stride_logits", ctypes.c_int64),
        ("max_model_len", ctypes.c_int32), ("clean_logits", ctypes.c_int32),
    ]


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ctx_1d(context_lens: torch.Tensor) -> torch.Tensor:
    if context_lens.dim() == 2 and context_lens.size(1) == 1:
        context_lens = context_lens.squeeze(1)
    if context_lens.dim() != 1 or context_lens.dtype != torch.int32:
        raise RuntimeError("context_lens must be int32 [B] (or [B, 1])")
    return context_lens.contiguous()


def get_paged_mqa_logits_metadata(context_lens: torch.Tensor, block_size: int, num_sms: int) -> torch.Tensor:
    """int32 [num_sms + 1, 2] schedule: the (request, 128-position tile)
    each CTA starts at.  ``block_size`` is checked, not used (tiles are 128
    positions for every page size)."""
    if block_size not in (32, 64, 128):
        raise RuntimeError(f"block_size {block_size}: 32, 64 or 128 supported")
    ctx = _ctx_1d(context_lens)
    sched = torch.empty(num_sms + 1, 2, dtype=torch.int32, device=ctx.device)
    with torch.cuda.device(ctx.device):
        check("dsv4b_mqa_logits_metadata",
              lib.dsv4b_mqa_logits_metadata(ctx.data_ptr(), ctx.numel(), num_sms, sched.data_ptr(),
                                            _stream(ctx.device)))
    return sched


def fp8_paged_mqa_logits(q: Union[torch.Tensor, Tuple[torch.Tensor, Optional[torch.Tensor]]],
                         kv_cache: torch.Tensor, weights: torch.Tensor, context_lens: torch.Tensor,
                         block_tables: torch.Tensor, schedule_metadata: torch.Tensor, max_model_len: int,
                         clean_logits: bool = True, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """logits fp32 [B * next_n, max_model_len].

    q: float8_e4m3fn [B, next_n, H, 128] (or vLLM's ``(q, None)`` tuple);
    kv_cache: uint8 [num_blocks, P, 1, 132] (per page P x 128 e4m3 then P
    fp32 scales); weights fp32 [B * next_n, H]; context_lens int32 [B];
    block_tables int32 [B, max_pages]; schedule_metadata from
    ``get_paged_mqa_logits_metadata`` (its row count - 1 is the CTA count).
    Positions that are not computed are -inf when ``clean_logits``."""
    if isinstance(q, tuple):
        q, q_scale = q
        if q_scale is not None:
            raise RuntimeError("only the FP8 path (q_scale None) is built")
    if q.dtype != torch.float8_e4m3fn or q.dim() != 4 or q.size(-1) != 128 or not q.is_contiguous():
        raise RuntimeError("q must be contiguous float8_e4m3fn [B, next_n, H, 128]")
    B, nn, H, D = q.shape
    if kv_cache.dtype not in (torch.uint8, torch.float8_e4m3fn) or kv_cache.dim() not in (2, 4):
        raise RuntimeError("kv_cache must be uint8 [num_blocks, P, 1, 132]")
    if kv_cache.dim() == 4:
        nb, P = kv_cache.size(0), kv_cache.size(1)
        if kv_cache.size(-1) != D + 4:
            raise RuntimeError(f"kv_cache last dim must be {D + 4}")
    else:
        raise RuntimeError("pass the 4-D [num_blocks, P, 1, 132] view (P is read from it)")
    if weights.dtype != torch.float32 or tuple(weights.shape) != (B * nn, H) or not weights.is_contiguous():
        raise RuntimeError("weights must be contiguous fp32 [B * next_n, H]")
    ctx = _ctx_1d(context_lens)
    if ctx.numel() != B:
        raise RuntimeError("context_lens must have B entries")
    if block_tables.dtype != torch.int32 or block_tables.dim() != 2 or block_tables.stride(1) != 1:
        raise RuntimeError("block_tables must be int32 [B, max_pages] with a contiguous last dim")
    if schedule_metadata.dtype != torch.int32 or schedule_metadata.dim() != 2 or schedule_metadata.size(1) != 2:
        raise RuntimeError("schedule_metadata must come from get_paged_mqa_logits_metadata")
    dev = q.device
    if out is None:
        out = torch.empty(B * nn, max_model_len, dtype=torch.float32, device=dev)
    elif out.dtype != torch.float32 or out.dim() != 2 or out.size(0) != B * nn or out.size(1) < max_model_len \
            or out.stride(1) != 1:
        raise RuntimeError("out must be fp32 [B * next_n, >= max_model_len]")
    p = MqaLogitsParams(B, nn, H, D, q.data_ptr(), kv_cache.data_ptr(), nb, P, kv_cache.stride(0) * kv_cache.element_size(),
                        weights.data_ptr(), ctx.data_ptr(), block_tables.data_ptr(), block_tables.stride(0),
                        out.data_ptr(), out.stride(0), max_model_len, int(bool(clean_logits)))
    with torch.cuda.device(dev):
        check("dsv4b_fp8_paged_mqa_logits",
              lib.dsv4b_fp8_paged_mqa_logits(ctypes.byref(p), schedule_metadata.data_ptr(),
                                             schedule_metadata.size(0) - 1, _stream(dev)))
    return out


def mqa_logits_status(device: Optional[torch.device] = None) -> int:
    """Status word of the logits kernel (0 = no error); clears it.  Synchronises."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    flags = ctypes.c_int()
    with torch.cuda.device(device):
        check("dsv4b_mqa_logits_status", lib.dsv4b_mqa_logits_status(ctypes.byref(flags), _stream(device)))
    return int(flags.value)
