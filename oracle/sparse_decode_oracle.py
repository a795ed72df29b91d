"""CPU oracle for the sparse FP8 MLA decode path (numpy restatement).

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this
module; only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` use it, and only as the checker / timed CPU baseline.

It restates the reference's pure-PyTorch oracle
(0xSero/deepseek-v4-flash-sm120 ``tests/reference.py``) in numpy:

* ``ue8m0_to_scale``            follows ``tests/reference.py:40-42``
* ``unpack_model1_rows``        follows ``tests/reference.py:45-79``
  (fp8 -> fp32, multiply by the fp32 scale, round to bf16, concat RoPE)
* ``unpack_v32_rows``           the DeepSeek-V3.2 656-B/token record
  ``[512 x e4m3 | 4 x fp32 scale | 64 x bf16 RoPE]`` named by
  ``csrc/common/params.h:12-15`` (ModelType::V32) and specified by the
  FlashMLA interface docstring (vLLM ``third_party/flashmla/
  flash_mla_interface.py:95-101``); same dequant order as MODEL1.
* ``sparse_decode_reference``   follows ``tests/reference.py:82-132``:
  -1 / out-of-range index -> zero K row (logit 0, not -inf), positions
  >= max(topk_length, 1) -> -inf, natural-log LSE, fp32 softmax and P.V,
  sink scales the output by 1/(1+exp(sink-lse)) and is folded into the
  returned LSE as logaddexp(lse, sink).

Extension not present in the reference oracle (parity unpinned by the
reference's tests): the SWA sidecar ``extra_*`` arguments follow the
reference kernel (``csrc/sm120/decode/sparse_decode_kernel.cuh:226-233,
346-352``): the extra tokens join the same softmax, their length is
clamped to [0, extra_topk] (not to >= 1), invalid extra indices give a
zero row.

Pinning: ``tests/test_oracle.py`` checks this module against golden
vectors produced by running the reference's own ``tests/reference.py``
(``tests/golden/make_golden.py``).
"""
from __future__ import annotations

from typing import Optional, Tuple

import numpy as np

# ---------------------------------------------------------------- layouts
# MODEL1 (DeepSeek-V4-Flash): tests/reference.py:28-37
M1_NOPE = 448
M1_ROPE = 64
M1_DQK = M1_NOPE + M1_ROPE          # 512
M1_TILE = 64
M1_NSCALE = M1_NOPE // M1_TILE      # 7
M1_SCALE_SLOTS = 8
M1_NOPE_ROPE_BYTES = M1_NOPE + 2 * M1_ROPE   # 576
M1_BYTES_PER_TOKEN = M1_NOPE_ROPE_BYTES + M1_SCALE_SLOTS  # 584

# V32 (DeepSeek-V3.2 FP8 sparse): 656 B per token, token-contiguous
V32_NOPE = 512
V32_ROPE = 64
V32_DQK = V32_NOPE + V32_ROPE       # 576
V32_TILE = 128
V32_NSCALE = V32_NOPE // V32_TILE   # 4
V32_BYTES_PER_TOKEN = V32_NOPE + 4 * V32_NSCALE + 2 * V32_ROPE  # 656

D_V = 512


# ------------------------------------------------------------- bf16 / fp8
def _e4m3fn_table() -> np.ndarray:
    """float32 value of every float8_e4m3fn byte (OCP FP8 E4M3, no inf,
    0x7f/0xff = NaN), built from the format definition."""
    t = np.zeros(256, dtype=np.float32)
    for b in range(256):
        s = -1.0 if b & 0x80 else 1.0
        e = (b >> 3) & 0xF
        m = b & 0x7
        if e == 0xF and m == 0x7:
            t[b] = np.nan
        elif e == 0:
            t[b] = s * (m / 8.0) * 2.0 ** -6
        else:
            t[b] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return t


E4M3_TO_F32 = _e4m3fn_table()


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16, returned as uint16 bits."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u >> 16) & 1) + np.uint32(0x7FFF)
    out = ((u + r) >> 16).astype(np.uint16)
    out = np.where(nan, np.uint16(0x7FC0), out)
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def ue8m0_to_scale(b: np.ndarray) -> np.ndarray:
    """2**(b-127) in fp32 (tests/reference.py:40-42).  b=0 is the
    subnormal 2**-127, b=255 overflows to +inf as torch.pow does."""
    b = np.asarray(b, dtype=np.uint32)
    bits = np.where(b == 0, np.uint32(0x00400000), b << 23)
    return bits.astype(np.uint32).view(np.float32)


# ------------------------------------------------------------------ unpack
def unpack_model1_rows(kv_pages: np.ndarray, page_block: int,
                       rows: np.ndarray) -> np.ndarray:
    """Dequantise the given flat token rows of a MODEL1 page arena into
    bf16-valued float32 [len(rows), 512] (tests/reference.py:45-79).

    kv_pages: uint8 [num_blocks, >= page_block*584] (per-page arena:
    page_block x 576 B nope|rope rows, then page_block x 8 B scales)."""
    rows = np.asarray(rows, dtype=np.int64)
    page = rows // page_block
    off = rows % page_block
    arena = kv_pages.reshape(kv_pages.shape[0], -1)
    nr = np.ascontiguousarray(arena[page[:, None], off[:, None] * M1_NOPE_ROPE_BYTES
                                    + np.arange(M1_NOPE_ROPE_BYTES)[None, :]])
    sc = arena[page[:, None], page_block * M1_NOPE_ROPE_BYTES
               + off[:, None] * M1_SCALE_SLOTS + np.arange(M1_NSCALE)[None, :]]
    nope = E4M3_TO_F32[nr[:, :M1_NOPE]].reshape(-1, M1_NSCALE, M1_TILE)
    scale = ue8m0_to_scale(sc)[:, :, None]
    nope = round_bf16((nope * scale).astype(np.float32).reshape(-1, M1_NOPE))
    rope = bf16_bits_to_f32(
        np.ascontiguousarray(nr[:, M1_NOPE:]).view(np.uint16).reshape(-1, M1_ROPE))
    return np.concatenate([nope, rope], axis=-1)


def unpack_v32_rows(kv: np.ndarray, page_block: int, rows: np.ndarray,
                    stride_block: Optional[int] = None) -> np.ndarray:
    """Dequantise flat token rows of a V32 cache into bf16-valued float32
    [len(rows), 576].  kv: uint8 [num_blocks, page_block, 1, 656] (or any
    view whose per-page bytes are page_block consecutive 656-B records)."""
    rows = np.asarray(rows, dtype=np.int64)
    flat = kv.reshape(kv.shape[0], -1)
    page = rows // page_block
    off = rows % page_block
    rec = flat[page[:, None], off[:, None] * V32_BYTES_PER_TOKEN
               + np.arange(V32_BYTES_PER_TOKEN)[None, :]]
    rec = np.ascontiguousarray(rec)
    nope = E4M3_TO_F32[rec[:, :V32_NOPE]].reshape(-1, V32_NSCALE, V32_TILE)
    scale = rec[:, V32_NOPE:V32_NOPE + 16].copy().view(np.float32)[:, :, None]
    nope = round_bf16((nope * scale).astype(np.float32).reshape(-1, V32_NOPE))
    rope = bf16_bits_to_f32(rec[:, V32_NOPE + 16:].copy().view(np.uint16))
    return np.concatenate([nope, rope], axis=-1)


def unpack_rows(layout: str, kv: np.ndarray, page_block: int,
                rows: np.ndarray) -> np.ndarray:
    if layout == "model1":
        return unpack_model1_rows(kv, page_block, rows)
    if layout == "v32":
        return unpack_v32_rows(kv, page_block, rows)
    raise ValueError(f"unknown layout {layout!r}")


def num_tokens(layout: str, kv: np.ndarray, page_block: int) -> int:
    return int(kv.shape[0]) * page_block


def gather_rows(layout: str, kv: np.ndarray, page_block: int,
                idx: np.ndarray) -> np.ndarray:
    """K rows for a vector of flat indices; -1 or >= num_tokens give a zero
    row (tests/reference.py:110-114)."""
    n = num_tokens(layout, kv, page_block)
    idx = np.asarray(idx, dtype=np.int64)
    valid = (idx >= 0) & (idx < n)
    d = M1_DQK if layout == "model1" else V32_DQK
    k = np.zeros((idx.shape[0], d), dtype=np.float32)
    if valid.any():
        k[valid] = unpack_rows(layout, kv, page_block, idx[valid])
    return k


# ------------------------------------------------------------------ decode
def sparse_decode_reference(
    q: np.ndarray,                    # float32 [b, s_q, h_q, d_qk] (bf16 values)
    kv: np.ndarray,                   # uint8 cache (layout dependent)
    indices: np.ndarray,              # int32 [b, s_q, topk]
    topk_length: Optional[np.ndarray],  # int32 [b] or None
    attn_sink: Optional[np.ndarray],  # float32 [h_q] or None
    sm_scale: float,
    page_block: int,
    layout: str = "model1",
    extra_kv: Optional[np.ndarray] = None,
    extra_indices: Optional[np.ndarray] = None,
    extra_topk_length: Optional[np.ndarray] = None,
    extra_page_block: Optional[int] = None,
    lse_includes_sink: bool = True,
) -> Tuple[np.ndarray, np.ndarray]:
    """Returns (out float32 [b, s_q, h_q, 512] holding bf16 values,
    lse float32 [b, s_q, h_q]), as tests/reference.py:82-132."""
    b, s_q, h_q, d_qk = q.shape
    topk = indices.shape[-1]
    want = M1_DQK if layout == "model1" else V32_DQK
    assert d_qk == want, (d_qk, want)
    out = np.zeros((b, s_q, h_q, D_V), dtype=np.float32)
    lse_out = np.zeros((b, s_q, h_q), dtype=np.float32)
    for bi in range(b):
        for si in range(s_q):
            idx = indices[bi, si].astype(np.int64)
            length = int(topk_length[bi]) if topk_length is not None else topk
            length = max(length, 1)
            k = gather_rows(layout, kv, page_block, idx)
            mask = np.arange(topk) < length
            if extra_kv is not None:
                eidx = extra_indices[bi, si].astype(np.int64)
                etopk = eidx.shape[0]
                elen = etopk
                if extra_topk_length is not None:
                    elen = min(etopk, int(extra_topk_length[bi]))
                elen = max(elen, 0)
                ek = gather_rows(layout, extra_kv, extra_page_block, eidx)
                k = np.concatenate([k, ek], axis=0)
                mask = np.concatenate([mask, np.arange(etopk) < elen])
            qf = q[bi, si].astype(np.float32)
            logits = (qf @ k.T).astype(np.float32) * np.float32(sm_scale)
            logits = np.where(mask[None, :], logits, np.float32(-np.inf))
            mx = logits.max(axis=-1, keepdims=True)
            e = np.exp(logits - mx)
            ssum = e.sum(axis=-1, keepdims=True)
            lse = (np.log(ssum) + mx)[:, 0]
            p = e / ssum
            o = p @ k[:, :D_V]
            if attn_sink is not None:
                sink = attn_sink.astype(np.float32)
                o = o * (1.0 / (1.0 + np.exp(sink - lse)))[:, None]
                if lse_includes_sink:
                    m = np.maximum(lse, sink)
                    lse = m + np.log(np.exp(lse - m) + np.exp(sink - m))
            out[bi, si] = round_bf16(o.astype(np.float32))
            lse_out[bi, si] = lse
    return out, lse_out
