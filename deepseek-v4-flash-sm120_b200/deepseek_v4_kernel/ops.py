"""``sparse_decode_fwd`` with the argument list of the reference op.

Mirrors ``deepseek_v4_kernel.ops.sparse_decode_fwd`` of the reference
(deepseek_v4_kernel/ops.py:17-45 -> csrc/api/sparse_decode.cpp:29-172):
same 12 positional arguments (plus FlashMLA's optional ``out``), same
return value ``(out, lse[b, h_q, s_q], tile_scheduler_metadata,
num_splits)``, RuntimeError on invalid input.  Differences, all on the
B200 side: both KV layouts (656-B V32 and 584-B MODEL1), s_q >= 1, a real
split-KV schedule (computed on the device the first time, then reused
like FlashMLA's scheduler tensors), and the LSE comes out already in
[b, h_q, s_q] (no transpose copy).
"""
from __future__ import annotations

import ctypes
import os
import threading
from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import DecodeParams, check, lib

D_V = 512
BYTES_V32 = 656
BYTES_MODEL1 = 584

_ws_lock = threading.Lock()
_ws_cache: dict = {}
# LSE convention, read once at import: DSV4B_LSE_EXCLUDES_SINK=1 returns the
# FlashMLA-documented LSE without the sink term.
_LSE_INCLUDES_SINK = os.environ.get("DSV4B_LSE_EXCLUDES_SINK", "0") != "1"
# DSV4B_CHECK_STATUS=1 (read once at import): sparse_decode_fwd synchronises
# after each call, reads the kernel status word and raises DSV4BError with
# DSV4B_ERR_KERNEL_TIMEOUT when a bounded wait ran out (the call's outputs
# are then invalid).  Off by default: the check costs a device sync.
CHECK_STATUS = os.environ.get("DSV4B_CHECK_STATUS", "0") == "1"


class _on_device:
    """``torch.cuda.device(device)`` only when ``device`` is not already the
    current device (entering the context costs a few microseconds per call)."""

    __slots__ = ("ctx",)

    def __init__(self, device: torch.device):
        self.ctx = None if device.index == torch.cuda.current_device() else torch.cuda.device(device)

    def __enter__(self):
        if self.ctx is not None:
            self.ctx.__enter__()

    def __exit__(self, *exc):
        if self.ctx is not None:
            return self.ctx.__exit__(*exc)
        return False


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    """Per-device workspace (split partials + kernel status word), grown on
    demand and zero-initialised once.  Calls on one device share it, so
    they must be stream-ordered (the normal case: one decode stream)."""
    key = device.index
    ws = _ws_cache.get(key)
    if ws is not None and ws.numel() >= nbytes:  # fast path: no lock
        return ws
    with _ws_lock:
        ws = _ws_cache.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            _ws_cache[key] = ws
        return ws


def num_sm_parts(device: torch.device, h_q: int) -> int:
    n = ctypes.c_int32()
    check("dsv4b_num_sm_parts", lib.dsv4b_num_sm_parts(device.index, h_q, ctypes.byref(n)))
    return int(n.value)


def kv_layout(kv: torch.Tensor) -> int:
    nbytes = kv.size(-1) * kv.element_size()
    if nbytes == BYTES_V32:
        return _lib.LAYOUT_V32
    if nbytes == BYTES_MODEL1:
        return _lib.LAYOUT_MODEL1
    raise RuntimeError(
        f"kv last dim must be {BYTES_V32} B/token (V32: 512 fp8 + 4 fp32 scales + 64 bf16 "
        f"RoPE) or {BYTES_MODEL1} B/token (MODEL1: 448 fp8 + 64 bf16 RoPE + 8 UE8M0); "
        f"got {nbytes}")


def _check_cache(kv: torch.Tensor, name: str) -> None:
    if not kv.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if kv.dim() != 4:
        raise RuntimeError(f"{name} must be 4-D [num_blocks, page_block, h_kv, bytes]")
    if kv.dtype not in (torch.float8_e4m3fn, torch.uint8, torch.int8):
        raise RuntimeError(f"{name} must be fp8_e4m3 / uint8 / int8 (packed bytes)")
    if kv.size(2) != 1:
        raise RuntimeError("Only MQA (h_kv=1) is supported for sparse decode")
    if kv.stride(-1) != 1:
        raise RuntimeError(f"{name} last dim must be contiguous")


def build_params(q, kv, indices, topk_length, attn_sink, extra_kv, extra_indices,
                 extra_topk_length, d_v, sm_scale, out, lse,
                 lse_includes_sink: bool = True) -> DecodeParams:
    """Validate the torch arguments and fill a dsv4b_decode_params."""
    if not q.is_cuda:
        raise RuntimeError("q and kv must be CUDA tensors")
    if q.dim() != 4:
        raise RuntimeError("q must be 4-D [b, s_q, h_q, d_qk]")
    if indices.dim() != 3:
        raise RuntimeError("indices must be 3-D [b, s_q, topk]")
    if q.dtype != torch.bfloat16:
        raise RuntimeError("q must be bf16")
    if indices.dtype != torch.int32:
        raise RuntimeError("indices must be int32")
    _check_cache(kv, "kv")
    layout = kv_layout(kv)
    b, s_q, h_q, d_qk = q.shape
    want_dqk = 576 if layout == _lib.LAYOUT_V32 else 512
    if d_qk != want_dqk:
        raise RuntimeError(f"this KV layout expects d_qk={want_dqk}, got {d_qk}")
    if int(d_v) != D_V:
        raise RuntimeError("Only d_v=512 supported")
    if tuple(indices.shape[:2]) != (b, s_q) or indices.stride(-1) != 1:
        raise RuntimeError("indices must be [b, s_q, topk] with a contiguous last dim")
    if q.stride(-1) != 1:
        raise RuntimeError("q last dim must be contiguous")
    for name, t, n in (("topk_length", topk_length, b), ("extra_topk_length", extra_topk_length, b),
                       ("attn_sink", attn_sink, h_q)):
        if t is not None:
            want = torch.float32 if name == "attn_sink" else torch.int32
            if t.dtype != want or t.numel() != n or not t.is_contiguous() or t.device != q.device:
                raise RuntimeError(f"{name} must be a contiguous {want} tensor of {n} elements "
                                   f"on {q.device}")
    p = DecodeParams()
    p.layout = layout
    p.b, p.s_q, p.h_q, p.d_qk, p.d_v = b, s_q, h_q, d_qk, int(d_v)
    p.topk = indices.size(2)
    p.sm_scale = float(sm_scale)
    p.lse_includes_sink = 1 if lse_includes_sink else 0
    p.q = q.data_ptr()
    p.stride_q_b, p.stride_q_s, p.stride_q_h = q.stride(0), q.stride(1), q.stride(2)
    esz = kv.element_size()
    p.kv = kv.data_ptr()
    p.num_blocks, p.page_block_size = kv.size(0), kv.size(1)
    p.stride_kv_block, p.stride_kv_row = kv.stride(0) * esz, kv.stride(1) * esz
    p.indices = indices.data_ptr()
    p.stride_idx_b, p.stride_idx_s = indices.stride(0), indices.stride(1)
    p.topk_length = _ptr(topk_length)
    p.attn_sink = _ptr(attn_sink)
    if extra_kv is not None:
        if extra_indices is None:
            raise RuntimeError("extra_indices required when extra_kv is provided")
        _check_cache(extra_kv, "extra_kv")
        if kv_layout(extra_kv) != layout:
            raise RuntimeError("extra_kv must use the same layout as kv")
        if extra_indices.dtype != torch.int32 or extra_indices.dim() != 3 or \
                tuple(extra_indices.shape[:2]) != (b, s_q) or extra_indices.stride(-1) != 1:
            raise RuntimeError("extra_indices must be int32 [b, s_q, extra_topk]")
        e = extra_kv.element_size()
        p.extra_kv = extra_kv.data_ptr()
        p.extra_num_blocks, p.extra_page_block_size = extra_kv.size(0), extra_kv.size(1)
        p.extra_topk = extra_indices.size(2)
        p.stride_extra_kv_block = extra_kv.stride(0) * e
        p.stride_extra_kv_row = extra_kv.stride(1) * e
        p.extra_indices = extra_indices.data_ptr()
        p.stride_extra_idx_b, p.stride_extra_idx_s = extra_indices.stride(0), extra_indices.stride(1)
        p.extra_topk_length = _ptr(extra_topk_length)
    p.out = out.data_ptr()
    p.stride_o_b, p.stride_o_s, p.stride_o_h = out.stride(0), out.stride(1), out.stride(2)
    p.lse = lse.data_ptr()
    return p


def plan_cluster_size(p: DecodeParams, parts: int) -> int:
    """Cluster size of the tile plan for these shapes (1 = no cluster)."""
    c = ctypes.c_int32()
    check("dsv4b_plan_cluster_size", lib.dsv4b_plan_cluster_size(ctypes.byref(p), parts, ctypes.byref(c)))
    return int(c.value)


def get_mla_metadata_tensors(p: DecodeParams, device: torch.device,
                             parts: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Run the on-device scheduler (K2); returns (tile_scheduler_metadata
    int32 [num_sm_parts, 8], num_splits int32 [b*s_q + 1])."""
    if parts is None:
        parts = num_sm_parts(device, p.h_q)
    tsm = torch.empty((parts, 8), dtype=torch.int32, device=device)
    ns = torch.empty((p.b * p.s_q + 1,), dtype=torch.int32, device=device)
    check("dsv4b_get_mla_metadata",
          lib.dsv4b_get_mla_metadata(ctypes.byref(p), parts, tsm.data_ptr(), ns.data_ptr(),
                                     _stream(device)))
    return tsm, ns


def sparse_decode_fwd(
    q: torch.Tensor,
    kv: torch.Tensor,
    indices: torch.Tensor,
    topk_length: Optional[torch.Tensor],
    attn_sink: Optional[torch.Tensor],
    tile_scheduler_metadata: Optional[torch.Tensor],
    num_splits: Optional[torch.Tensor],
    extra_kv: Optional[torch.Tensor],
    extra_indices: Optional[torch.Tensor],
    extra_topk_length: Optional[torch.Tensor],
    d_v: int,
    sm_scale: float,
    out: Optional[torch.Tensor] = None,
    lse_includes_sink: Optional[bool] = None,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """Sparse FP8 MLA decode on B200.  Returns (out [b, s_q, h_q, 512] bf16,
    lse [b, h_q, s_q] fp32, tile_scheduler_metadata, num_splits).

    ``tile_scheduler_metadata`` / ``num_splits``: pass None on the first
    call of a batch; the returned tensors may be reused for later calls
    with the same shapes and the same topk_length / extra_topk_length
    values (FlashMLA's contract, flash_mla_interface.py:83)."""
    if lse_includes_sink is None:
        lse_includes_sink = _LSE_INCLUDES_SINK
    device = q.device
    b, s_q, h_q, _ = q.shape
    if out is None:
        out = torch.empty((b, s_q, h_q, int(d_v)), dtype=torch.bfloat16, device=device)
    elif out.dtype != torch.bfloat16 or tuple(out.shape) != (b, s_q, h_q, int(d_v)) or \
            out.stride(-1) != 1 or out.device != device:
        raise RuntimeError("out must be bf16 [b, s_q, h_q, d_v] on q's device, last dim contiguous")
    lse = torch.empty((b, h_q, s_q), dtype=torch.float32, device=device)
    p = build_params(q, kv, indices, topk_length, attn_sink, extra_kv, extra_indices,
                     extra_topk_length, d_v, sm_scale, out, lse, lse_includes_sink)
    with _on_device(device):
        if tile_scheduler_metadata is None or num_splits is None:
            tile_scheduler_metadata, num_splits = get_mla_metadata_tensors(p, device)
        parts = tile_scheduler_metadata.size(0)
        if tile_scheduler_metadata.dtype != torch.int32 or tile_scheduler_metadata.shape[1:] != (8,) \
                or num_splits.numel() != b * s_q + 1:
            raise RuntimeError("tile_scheduler_metadata / num_splits do not match this batch")
        nbytes = lib.dsv4b_workspace_bytes(b, s_q, h_q, parts)
        ws = workspace(device, nbytes)
        check("dsv4b_sparse_decode",
              lib.dsv4b_sparse_decode(ctypes.byref(p), tile_scheduler_metadata.data_ptr(),
                                      num_splits.data_ptr(), parts, ws.data_ptr(), ws.numel(),
                                      _stream(device)))
        if CHECK_STATUS:
            _raise_on_status(ws, device)
    return out, lse, tile_scheduler_metadata, num_splits


def _raise_on_status(ws: torch.Tensor, device: torch.device) -> None:
    flags = ctypes.c_int()
    check("dsv4b_read_kernel_status",
          lib.dsv4b_read_kernel_status(ws.data_ptr(), ws.numel(), ctypes.byref(flags), _stream(device)))
    if flags.value:
        raise _lib.DSV4BError("sparse_decode_fwd (kernel status)", -6)


def gather_dequant(kv: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
    """Debug: the decode kernel's row decoder applied to flat indices ->
    bf16 [n, d_qk] (zeros for -1 / out-of-range)."""
    _check_cache(kv, "kv")
    layout = kv_layout(kv)
    idx = indices.reshape(-1).to(torch.int32).contiguous()
    d = 576 if layout == _lib.LAYOUT_V32 else 512
    out = torch.empty((idx.numel(), d), dtype=torch.bfloat16, device=kv.device)
    e = kv.element_size()
    with torch.cuda.device(kv.device):
        check("dsv4b_gather_dequant",
              lib.dsv4b_gather_dequant(layout, kv.data_ptr(), kv.size(0), kv.size(1),
                                       kv.stride(0) * e, kv.stride(1) * e, idx.data_ptr(),
                                       idx.numel(), out.data_ptr(), _stream(kv.device)))
    return out


def read_kernel_status(device: Optional[torch.device] = None) -> int:
    """Kernel status word of the device workspace (0 = no error); clears it."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    ws = _ws_cache.get(device.index)
    if ws is None:
        return 0
    flags = ctypes.c_int()
    check("dsv4b_read_kernel_status",
          lib.dsv4b_read_kernel_status(ws.data_ptr(), ws.numel(), ctypes.byref(flags),
                                       _stream(device)))
    return int(flags.value)
