"""Sparse attention prefill: ``flash_mla_sparse_fwd`` with FlashMLA's
argument list (vLLM ``third_party/flashmla/flash_mla_interface.py:180-217``).

The reference itself has no prefill: its decode kernel flattens s_q into
the batch (``csrc/sm120/decode/sparse_decode_kernel.cuh:38-40``) and the
serving engine runs FlashMLA's sparse prefill next to it.  This is that op
on the B200 path: each query token attends, with all heads, to the top-k
rows of a bf16 KV tensor, through the decode kernel's tcgen05 pipeline
(bf16 rows copied into its swizzled K tile instead of dequantised).

Semantics (checked against vLLM 0.22's FlashMLA kernel on B200):

* indices < 0, >= s_kv, or at positions >= topk_length[i] are left out of
  the softmax;
* lse is the natural-log log-sum-exp of ``sm_scale * q.k`` over the valid
  positions, max_logits their maximum;
* a token with no valid position: lse = +inf, max_logits = -inf, output 0;
* attn_sink scales the output by exp(lse) / (exp(lse) + exp(sink)) and
  leaves lse and max_logits alone (+inf sink: output 0).
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import DecodeParams, check, lib
from .ops import _on_device, _stream, workspace


def flash_mla_sparse_fwd(
    q: torch.Tensor,
    kv: torch.Tensor,
    indices: torch.Tensor,
    sm_scale: float,
    d_v: int = 512,
    attn_sink: Optional[torch.Tensor] = None,
    topk_length: Optional[torch.Tensor] = None,
    out: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """q bf16 [s_q, h_q, d_qk] (d_qk 576 or 512), kv bf16 [s_kv, 1, d_qk],
    indices int32 [s_q, 1, topk] -> (out bf16 [s_q, h_q, 512], max_logits
    fp32 [s_q, h_q], lse fp32 [s_q, h_q]).  RuntimeError on invalid input."""
    if q.dim() != 3 or q.dtype != torch.bfloat16 or q.stride(-1) != 1:
        raise RuntimeError("q must be bf16 [s_q, h_q, d_qk], last dim contiguous")
    s_q, h_q, d_qk = q.shape
    if d_qk not in (576, 512):
        raise RuntimeError(f"d_qk must be 576 or 512, got {d_qk}")
    if int(d_v) != 512:
        raise RuntimeError("d_v must be 512")
    if kv.dim() == 3:
        if kv.shape[1] != 1:
            raise RuntimeError("kv must have h_kv = 1")
        kv2 = kv[:, 0]
    elif kv.dim() == 2:
        kv2 = kv
    else:
        raise RuntimeError("kv must be bf16 [s_kv, 1, d_qk]")
    if kv2.dtype != torch.bfloat16 or kv2.shape[-1] != d_qk or kv2.stride(-1) != 1:
        raise RuntimeError("kv must be bf16 [s_kv, 1, d_qk] matching q, last dim contiguous")
    idx = indices[:, 0] if indices.dim() == 3 else indices
    if indices.dim() == 3 and indices.shape[1] != 1:
        raise RuntimeError("indices must be [s_q, 1, topk]")
    if idx.dtype != torch.int32 or idx.dim() != 2 or idx.shape[0] != s_q or idx.stride(-1) != 1:
        raise RuntimeError("indices must be int32 [s_q, 1, topk], last dim contiguous")
    topk = idx.shape[-1]
    dev = q.device
    for name, t in (("kv", kv2), ("indices", idx)):
        if t.device != dev:
            raise RuntimeError(f"{name} must be on q's device")
    tl = None
    if topk_length is not None:
        tl = topk_length.to(torch.int32).contiguous()
        if tl.numel() != s_q or tl.device != dev:
            raise RuntimeError("topk_length must be int32 [s_q] on q's device")
    sink = None
    if attn_sink is not None:
        sink = attn_sink.to(torch.float32).contiguous()
        if sink.numel() != h_q or sink.device != dev:
            raise RuntimeError("attn_sink must be float32 [h_q] on q's device")
    if out is None:
        out = torch.empty((s_q, h_q, 512), dtype=torch.bfloat16, device=dev)
    elif out.dtype != torch.bfloat16 or tuple(out.shape) != (s_q, h_q, 512) or out.stride(-1) != 1:
        raise RuntimeError("out must be bf16 [s_q, h_q, 512], last dim contiguous")
    max_logits = torch.empty((s_q, h_q), dtype=torch.float32, device=dev)
    lse = torch.empty((s_q, h_q), dtype=torch.float32, device=dev)
    if s_q == 0:
        return out, max_logits, lse

    p = DecodeParams()
    p.layout = _lib.LAYOUT_BF16_576 if d_qk == 576 else _lib.LAYOUT_BF16_512
    p.b, p.s_q, p.h_q, p.d_qk, p.d_v, p.topk = s_q, 1, h_q, d_qk, 512, topk
    p.sm_scale = float(sm_scale)
    p.lse_includes_sink = 0
    p.q = q.data_ptr()
    p.stride_q_b, p.stride_q_s, p.stride_q_h = q.stride(0), 0, q.stride(1)
    p.kv = kv2.data_ptr()
    p.num_blocks, p.page_block_size = kv2.shape[0], 1
    p.stride_kv_block, p.stride_kv_row = kv2.stride(0) * 2, kv2.stride(0) * 2
    p.indices = idx.data_ptr()
    p.stride_idx_b, p.stride_idx_s = idx.stride(0), 0
    p.topk_length = None if tl is None else tl.data_ptr()
    p.attn_sink = None if sink is None else sink.data_ptr()
    p.out = out.data_ptr()
    p.stride_o_b, p.stride_o_s, p.stride_o_h = out.stride(0), 0, out.stride(1)
    p.lse = lse.data_ptr()
    p.prefill = 1
    p.max_logits = max_logits.data_ptr()
    with _on_device(dev):
        ws = workspace(dev, lib.dsv4b_prefill_workspace_bytes(s_q))
        check("dsv4b_sparse_prefill",
              lib.dsv4b_sparse_prefill(ctypes.byref(p), ws.data_ptr(), ws.numel(), _stream(dev)))
    return out, max_logits, lse
