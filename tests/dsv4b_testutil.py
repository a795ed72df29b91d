"""Helpers shared by the GPU parity tests: run the oracle on a Batch."""
from __future__ import annotations

import numpy as np
import torch

from oracle import sparse_decode_oracle as O


def bf16_to_f32_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def oracle_for(q, kv, indices, topk_length, attn_sink, sm_scale, layout, extra=None,
               lse_includes_sink=True):
    """Run the numpy oracle on torch inputs (any device).  `kv` is the 4-D
    cache; for MODEL1 the oracle reads the page arena behind the view."""
    qn = bf16_to_f32_np(q)
    kvn = kv.detach().cpu().contiguous().view(torch.uint8).numpy()
    page = kv.shape[1]
    if layout == "model1":
        kvn = kvn.reshape(kv.shape[0], -1)
    idx = indices.detach().cpu().numpy()
    tk = None if topk_length is None else topk_length.detach().cpu().numpy()
    sk = None if attn_sink is None else attn_sink.detach().cpu().numpy()
    kw = {}
    if extra is not None:
        ekv, eidx, etk = extra
        ekvn = ekv.detach().cpu().contiguous().view(torch.uint8).numpy()
        if layout == "model1":
            ekvn = ekvn.reshape(ekv.shape[0], -1)
        kw = dict(extra_kv=ekvn, extra_indices=eidx.detach().cpu().numpy(),
                  extra_topk_length=None if etk is None else etk.detach().cpu().numpy(),
                  extra_page_block=ekv.shape[1])
    return O.sparse_decode_reference(qn, kvn, idx, tk, sk, sm_scale, page, layout=layout,
                                     lse_includes_sink=lse_includes_sink, **kw)


# Tolerances stated by the north star: bf16 output max-abs err <= 2e-2 at
# rtol 1e-2; LSE within 1e-3.
OUT_ATOL, OUT_RTOL = 2e-2, 1e-2
LSE_ATOL, LSE_RTOL = 1e-3, 1e-3


def assert_matches(out, lse, ref_out, ref_lse):
    """out [b,s,h,512] bf16 torch; lse [b,h,s] torch; ref_* numpy with the
    oracle's [b,s,h] LSE layout."""
    o = out.float().cpu().numpy()
    l = lse.float().cpu().numpy().transpose(0, 2, 1)
    np.testing.assert_allclose(o, ref_out, atol=OUT_ATOL, rtol=OUT_RTOL)
    np.testing.assert_allclose(l, ref_lse, atol=LSE_ATOL, rtol=LSE_RTOL)


def oracle_rows_v32(bt, rows):
    """Oracle output for selected query rows of a full-size V32 batch
    without copying the whole cache to the host: the rows' referenced cache
    records are gathered on the device into a compact cache (one token per
    page) and the indices remapped to it.  `rows` are (b, s) pairs.
    Returns (out [n, h_q, 512], lse [n, h_q]) as numpy."""
    kv_flat = bt.kv.view(-1, 656)
    n_tok = kv_flat.shape[0]
    idx = torch.stack([bt.indices[b_, s_] for b_, s_ in rows]).long()      # [n, topk]
    valid = (idx >= 0) & (idx < n_tok)
    uniq, inv = torch.unique(torch.where(valid, idx, torch.zeros_like(idx)), return_inverse=True)
    compact = kv_flat[uniq].contiguous().view(-1, 1, 1, 656)
    remap = torch.where(valid, inv, torch.full_like(inv, -1)).to(torch.int32)
    q = torch.stack([bt.q[b_, s_] for b_, s_ in rows]).unsqueeze(1)         # [n, 1, h_q, 576]
    out, lse = oracle_for(q, compact, remap.unsqueeze(1), None, bt.attn_sink, bt.sm_scale, "v32")
    return out[:, 0], lse[:, 0]


def assert_rows_match(out, lse, bt, rows):
    """Checks selected (b, s) rows of a decode result against oracle_rows_v32."""
    ref_out, ref_lse = oracle_rows_v32(bt, rows)
    o = np.stack([out[b_, s_].float().cpu().numpy() for b_, s_ in rows])
    l = np.stack([lse[b_, :, s_].float().cpu().numpy() for b_, s_ in rows])
    np.testing.assert_allclose(o, ref_out, atol=OUT_ATOL, rtol=OUT_RTOL)
    np.testing.assert_allclose(l, ref_lse, atol=LSE_ATOL, rtol=LSE_RTOL)
