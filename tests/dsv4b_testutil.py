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
