"""CPU oracle for the sparse prefill (``flash_mla_sparse_fwd``).  TEST
INFRASTRUCTURE: only tests/ and __graft_entry__.smoke() use it, as the
checker; the product path never calls it.

The reference repository has no prefill (its decode kernel flattens s_q
into the batch, csrc/sm120/decode/sparse_decode_kernel.cuh:38-40); the op
is FlashMLA's, as vLLM 0.22 ships it (third-party, compiled:
``vllm/third_party/flashmla/flash_mla_interface.py:180-217``, docstring
semantics).  This restates those published semantics in numpy, float64:

    s[h, j]   = sm_scale * q[h] . kv[indices[j]]          (d_qk columns)
    valid j   : 0 <= indices[j] < s_kv and j < topk_length
    max_logits[h] = max_j valid s[h, j]           (-inf if none valid)
    lse[h]        = log sum_j valid exp(s[h, j])  (+inf if none valid)
    out[h]        = sum_j valid exp(s[h, j] - lse[h]) kv[indices[j], :512]
                    * 1 / (1 + exp(attn_sink[h] - lse[h]))   (if a sink)
    (no valid position: out = 0)

Pinned against the library kernel itself: tests/golden/prefill/*.npz hold
vLLM's outputs on B200 for seeded inputs (tests/golden/
make_prefill_golden.py), and tests/test_sparse_prefill_oracle.py checks
this restatement against them.
"""
from __future__ import annotations

import numpy as np


def sparse_prefill_reference(q, kv, indices, sm_scale, topk_length=None, attn_sink=None, d_v=512):
    """q float [s_q, h_q, d_qk]; kv float [s_kv, d_qk] (or [s_kv, 1, d_qk]);
    indices int [s_q, topk] (or [s_q, 1, topk]) -> (out [s_q, h_q, d_v],
    max_logits [s_q, h_q], lse [s_q, h_q]) as float64."""
    q = np.asarray(q, dtype=np.float64)
    kv = np.asarray(kv, dtype=np.float64)
    if kv.ndim == 3:
        kv = kv[:, 0]
    idx = np.asarray(indices)
    if idx.ndim == 3:
        idx = idx[:, 0]
    s_q, h_q, _ = q.shape
    s_kv = kv.shape[0]
    topk = idx.shape[1]
    out = np.zeros((s_q, h_q, d_v))
    mx = np.full((s_q, h_q), -np.inf)
    lse = np.full((s_q, h_q), np.inf)
    for i in range(s_q):
        n = topk if topk_length is None else int(topk_length[i])
        ids = idx[i].astype(np.int64)
        ok = (ids >= 0) & (ids < s_kv) & (np.arange(topk) < n)
        if not ok.any():
            continue
        k = kv[ids[ok]]
        s = (q[i] @ k.T) * sm_scale            # [h_q, valid]
        m = s.max(axis=1)
        e = np.exp(s - m[:, None])
        tot = e.sum(axis=1)
        mx[i] = m
        lse[i] = m + np.log(tot)
        o = (e / tot[:, None]) @ k[:, :d_v]
        if attn_sink is not None:
            sk = np.asarray(attn_sink, dtype=np.float64)
            with np.errstate(over="ignore"):
                o = o * (1.0 / (1.0 + np.exp(sk - lse[i])))[:, None]
        out[i] = o
    return out, mx, lse
