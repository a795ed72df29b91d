"""CPU oracle for the indexer logits, fp8_paged_mqa_logits (numpy).

TEST INFRASTRUCTURE ONLY: used by tests/ and bench.py's CPU-baseline leg.

Restates DeepGEMM's published torch statement of the op as vLLM 0.22
carries it (``v1/attention/ops/rocm_aiter_mla_sparse.py:256-300``, "taken
from DeepGEMM tests/test_attention.py"), next_n == 1 branch: per request b
the first ceil(ctx_b / P) pages of its block table are read, each page
holding P x d e4m3 values then P x fp32 scales;
``score[t, h] = relu(k[t] . q[b, h])``, ``logit[t] = sum_h score[t, h] *
w[b, h] * k_scale[t]`` for t < ctx_b, -inf elsewhere.  For next_n > 1 the
same page layout is used with DeepGEMM's causal rule
(``rocm_aiter_mla_sparse.py:301-345``): row i of request b sees
t < ctx_b and t <= ctx_b - next_n + i.  That branch of the torch statement
reads the cache token-interleaved instead of page-sectioned, so it is not
run; the rule is restated here on the page-sectioned layout vLLM's indexer
cache writer produces.

Computed in float64 (the tensor cores accumulate in fp32 in another order;
tests compare with a relative tolerance).

Pinning: ``tests/golden/make_mqa_logits_golden.py`` runs vLLM's torch
statement on seeded inputs (next_n = 1) and stores inputs and logits;
``tests/test_mqa_logits_oracle.py`` holds this module to them.
"""
from __future__ import annotations

import numpy as np

from .sparse_decode_oracle import E4M3_TO_F32


def fp8_paged_mqa_logits(q_u8: np.ndarray, kv_pages: np.ndarray, weights: np.ndarray, context_lens: np.ndarray,
                         block_table: np.ndarray, page_block: int, max_model_len: int,
                         clean_logits: bool = True) -> np.ndarray:
    """q_u8 uint8 e4m3 [B, next_n, H, D]; kv_pages uint8 [num_blocks, >= P*(D+4)];
    weights fp32 [B*next_n, H]; context_lens int [B]; block_table int [B, *].
    Returns fp32 [B*next_n, max_model_len]; positions not computed are NaN
    when clean_logits is False (the caller must not read them)."""
    B, nn, H, D = q_u8.shape
    P = page_block
    q = E4M3_TO_F32[q_u8].astype(np.float64)
    out = np.full((B * nn, max_model_len), -np.inf if clean_logits else np.nan, np.float64)
    for b in range(B):
        ctx = int(context_lens[b])
        if ctx <= 0:
            if not clean_logits:
                out[b * nn:(b + 1) * nn, :] = np.nan
            continue
        npages = -(-ctx // P)
        pages = np.asarray(block_table[b, :npages], dtype=np.int64)
        arena = kv_pages[pages]
        vals = E4M3_TO_F32[arena[:, :P * D].reshape(npages * P, D)].astype(np.float64)
        scale = np.ascontiguousarray(arena[:, P * D:P * D + 4 * P]).view(np.float32).reshape(npages * P)
        tiles_end = min(-(-ctx // 128) * 128, max_model_len)
        for i in range(nn):
            s = vals[:ctx] @ q[b, i].T                       # [ctx, H]
            logit = (np.maximum(s, 0.0) * weights[b * nn + i][None, :].astype(np.float64)).sum(1)
            logit = logit * scale[:ctx].astype(np.float64)
            t = np.arange(ctx)
            ok = t <= ctx - nn + i
            row = out[b * nn + i]
            row[:tiles_end] = -np.inf
            lim = min(ctx, max_model_len)
            row[:lim] = np.where(ok[:lim], logit[:lim], -np.inf)
    return out.astype(np.float32)
