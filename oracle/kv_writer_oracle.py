"""CPU oracle for the KV-cache writer (numpy restatement).

TEST INFRASTRUCTURE ONLY.  Nothing in the shipped package imports this
module; only ``tests/`` (and ``bench.py``'s CPU-baseline leg) use it, as
the checker.

What it restates: the producer of the cache bytes that the decode path
reads.  The reference names SGLang's ``quant_k_cache_v4`` as that producer
(``tests/reference.py:45-49``) but ships no quantiser: its fake batches
write random e4m3 bytes and random exponents (``tests/reference.py:
135-200``).  The byte formats are the reference's unpack
(``tests/reference.py:40-79``, MODEL1) and the FlashMLA FP8 record
(vLLM ``v1/attention/backends/mla/flashmla_sparse.py:70-92``, V32).  The
quantisation rules follow vLLM 0.22's writers for the same formats:

* MODEL1: ``quantize_and_insert_k_kernel`` (vLLM ``models/deepseek_v4/
  common/ops/cache_utils.py:23-140``): per 64 NoPE columns
  ``amax = max(max|x|, 1e-4)``, ``e = ceil(log2(amax / 448))``,
  ``q = e4m3(clamp(x / 2^e, +-448))``, scale byte ``e + 127``, 8th byte 0;
  RoPE copied as bf16; token row at ``offset * 576`` in its page, scale
  bytes at ``P * 576 + offset * 8``.
* V32: ``concat_and_cache_mla(..., kv_cache_dtype="fp8_ds_mla")`` (vLLM
  ``_custom_ops.py:2613-2623``; compiled, its source is not in the image,
  so the rule was read off its outputs on a B200: every scale equals the
  correctly rounded fp32 ``amax / 448``, an all-zero tile stores FLT_MIN
  and zero bytes, and the quantised bytes equal ``e4m3(x / scale)``):
  per 128 latent columns ``scale = max(amax / 448, FLT_MIN)`` stored as
  fp32, ``q = e4m3(clamp(x / scale, +-448))``.

For bf16 inputs ``amax / 448`` is either an exact power of two or at least
2^-7 (relative) away from one, so ``ceil(log2(.))`` here (numpy's log2)
and the kernel's exponent-bit reading agree exactly.

``f32_to_e4m3`` is this module's own round-to-nearest-even e4m3 encoder
(checked against torch's cast over every bf16 value by the CPU tests).

Pinning: ``tests/golden/make_kv_writer_golden.py`` quantises seeded tokens
with this module and runs the reference's own unpack on the bytes; the
fixture stores both, so the CPU tests hold the format to the reference.
The GPU tests compare the CUDA writer with this module byte for byte and
with vLLM's writers when vLLM is importable.
"""
from __future__ import annotations

import numpy as np

FP8_MAX = 448.0
AMAX_FLOOR = np.float32(1e-4)          # MODEL1
FLT_MIN = np.float32(1.17549435e-38)   # V32: scale of an all-zero tile
V32_RECORD = 656
MODEL1_ROW = 576
MODEL1_SCALE_BYTES = 8


def bf16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << 16).view(np.float32)


def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3 (fn) bytes, nearest even.  |x| must be <= 448 or NaN.

    e4m3: 1 sign, 4 exponent (bias 7), 3 mantissa bits; normals
    [2^-6, 448], subnormals k * 2^-9 (k = 1..7), NaN 0x7F / 0xFF."""
    x = np.asarray(x, dtype=np.float32)
    sign = np.signbit(x).astype(np.uint8) << 7
    a = np.abs(x).astype(np.float64)
    nan = np.isnan(a)
    a = np.where(nan, 0.0, a)
    _, ex = np.frexp(a)                      # a = m * 2^ex, m in [0.5, 1)
    e = np.maximum(ex - 1, -6)               # binade; subnormals share 2^-6's quantum
    quantum = np.ldexp(1.0, e - 3)
    k = np.rint(a / quantum)                 # exact division; rint = half to even
    v = k * quantum                          # rounded magnitude (may step up a binade)
    _, ev = np.frexp(v)
    ev = ev - 1
    normal = v >= 2.0 ** -6
    mant = np.where(normal, v / np.ldexp(1.0, np.where(normal, ev, 0) - 3) - 8, v / 2.0 ** -9)
    expf = np.where(normal, ev + 7, 0)
    bits = (expf.astype(np.int64) << 3) | mant.astype(np.int64)
    out = bits.astype(np.uint8) | sign
    return np.where(nan, np.uint8(0x7F) | sign, out).astype(np.uint8)


def _clamp(x: np.ndarray) -> np.ndarray:
    # NaN passes through, as torch.clamp does
    return np.where(x > FP8_MAX, np.float32(FP8_MAX), np.where(x < -FP8_MAX, np.float32(-FP8_MAX), x))


def quantize_v32_rows(latent_bf16: np.ndarray, rope_bf16: np.ndarray) -> np.ndarray:
    """latent uint16 (bf16 bits) [n, 512], rope uint16 [n, 64] -> uint8 [n, 656]."""
    n = latent_bf16.shape[0]
    x = bf16_bits_to_f32(latent_bf16).reshape(n, 4, 128)
    amax = np.abs(x).max(axis=-1)
    scale = np.maximum((amax / np.float32(FP8_MAX)).astype(np.float32), FLT_MIN)       # [n, 4]
    q = f32_to_e4m3(_clamp((x / scale[..., None]).astype(np.float32))).reshape(n, 512)
    out = np.empty((n, V32_RECORD), np.uint8)
    out[:, :512] = q
    out[:, 512:528] = scale.view(np.uint8).reshape(n, 16)
    out[:, 528:] = np.ascontiguousarray(rope_bf16, dtype=np.uint16).view(np.uint8).reshape(n, 128)
    return out


def quantize_model1_rows(nope_bf16: np.ndarray, rope_bf16: np.ndarray):
    """nope uint16 [n, 448], rope uint16 [n, 64] -> (rows uint8 [n, 576], scales uint8 [n, 8])."""
    n = nope_bf16.shape[0]
    x = bf16_bits_to_f32(nope_bf16).reshape(n, 7, 64)
    amax = np.maximum(np.abs(x).max(axis=-1), AMAX_FLOOR)
    e = np.ceil(np.log2((amax / np.float32(FP8_MAX)).astype(np.float32))).astype(np.int32)   # [n, 7]
    inv = np.ldexp(np.float32(1.0), -e).astype(np.float32)
    q = f32_to_e4m3(_clamp((x * inv[..., None]).astype(np.float32))).reshape(n, 448)
    rows = np.empty((n, MODEL1_ROW), np.uint8)
    rows[:, :448] = q
    rows[:, 448:] = np.ascontiguousarray(rope_bf16, dtype=np.uint16).view(np.uint8).reshape(n, 128)
    scales = np.zeros((n, MODEL1_SCALE_BYTES), np.uint8)
    scales[:, :7] = (e + 127).astype(np.uint8)
    return rows, scales


def kv_cache_write(layout: str, arena: np.ndarray, page_block: int, nope_bf16: np.ndarray,
                   rope_bf16: np.ndarray, slots: np.ndarray, stride_row: int = V32_RECORD) -> np.ndarray:
    """Scatter the quantised tokens into ``arena`` (uint8 [num_blocks,
    stride_block], modified in place and returned).  Slots < 0 or past the
    cache are skipped; later tokens overwrite earlier ones on equal slots."""
    num_blocks = arena.shape[0]
    cache_tokens = num_blocks * page_block
    slots = np.asarray(slots, dtype=np.int64)
    keep = np.nonzero((slots >= 0) & (slots < cache_tokens))[0]
    if keep.size == 0:
        return arena
    pg, off = slots[keep] // page_block, slots[keep] % page_block
    if layout == "v32":
        rec = quantize_v32_rows(nope_bf16[keep], rope_bf16[keep])
        cols = off[:, None] * stride_row + np.arange(V32_RECORD)[None, :]
        arena[pg[:, None], cols] = rec
    else:
        rows, scales = quantize_model1_rows(nope_bf16[keep], rope_bf16[keep])
        arena[pg[:, None], off[:, None] * MODEL1_ROW + np.arange(MODEL1_ROW)[None, :]] = rows
        base = page_block * MODEL1_ROW
        arena[pg[:, None], base + off[:, None] * MODEL1_SCALE_BYTES + np.arange(8)[None, :]] = scales
    return arena
