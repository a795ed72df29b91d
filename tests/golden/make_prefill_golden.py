"""Golden vectors for the sparse prefill, from the library kernel itself.

The reference repository has no prefill; the op it would run next to its
decode is FlashMLA's ``flash_mla_sparse_fwd`` as vLLM 0.22 ships it
(compiled, ``vllm/third_party/flashmla/flash_mla_interface.py:180-217``).
Run on a B200 box of this image (vLLM is installed there):

    python tests/golden/make_prefill_golden.py [--out DIR]

It builds seeded inputs, runs vLLM's kernel and writes inputs + outputs to
``tests/golden/prefill/*.npz`` (bf16 tensors as uint16 bit patterns).  The
tests only read these files: tests/test_sparse_prefill_oracle.py pins the
numpy oracle to them on the CPU; the GPU tests compare our kernel with
them and with the oracle.
"""
from __future__ import annotations

import math
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "prefill")

# name: (s_q, h_q, d_qk, s_kv, topk, with topk_length, sink kind, seed)
CASES = {
    "d576_h64_ragged": (4, 64, 576, 256, 192, True, "normal", 1),
    "d512_h128": (3, 128, 512, 200, 128, False, None, 2),
    "d576_h64_sink_inf": (2, 64, 576, 400, 384, True, "inf", 3),
}


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def make(out_dir, name, s_q, h_q, d, s_kv, topk, with_tl, sink_kind, seed):
    from vllm.third_party.flashmla.flash_mla_interface import flash_mla_sparse_fwd
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(s_q, h_q, d, generator=g).to(torch.bfloat16)
    kv = torch.randn(s_kv, 1, d, generator=g).to(torch.bfloat16)
    idx = torch.randint(0, s_kv, (s_q, 1, topk), generator=g, dtype=torch.int32)
    idx[0, 0, 3:40] = -1                       # padding
    idx[-1, 0, 7:19] = s_kv + 5                # out of range
    if s_q > 2:
        idx[1, 0, :] = -1                      # a token with no valid position
    tl = None
    if with_tl:
        tl = torch.randint(topk // 2, topk + 1, (s_q,), generator=g, dtype=torch.int32)
        if s_q > 3:
            tl[2] = 0                          # topk_length 0
    sink = None
    if sink_kind == "normal":
        sink = torch.randn(h_q, generator=g)
    elif sink_kind == "inf":
        sink = torch.randn(h_q, generator=g)
        sink[0], sink[1] = float("inf"), float("-inf")
    sm_scale = 1.0 / math.sqrt(d)
    o, m, l = flash_mla_sparse_fwd(q.cuda(), kv.cuda(), idx.cuda(), sm_scale, 512,
                                   None if sink is None else sink.cuda(), None if tl is None else tl.cuda())
    torch.cuda.synchronize()
    np.savez_compressed(
        os.path.join(out_dir, f"{name}.npz"),
        q=bits(q), kv=bits(kv), indices=idx.numpy(), sm_scale=np.float64(sm_scale),
        topk_length=np.zeros(0, np.int32) if tl is None else tl.numpy(),
        attn_sink=np.zeros(0, np.float32) if sink is None else sink.numpy(),
        out=bits(o), max_logits=m.cpu().numpy(), lse=l.cpu().numpy())


def main():
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=OUT, help="output directory (default tests/golden/prefill)")
    out_dir = ap.parse_args().out
    os.makedirs(out_dir, exist_ok=True)
    for name, spec in CASES.items():
        make(out_dir, name, *spec)
        print("wrote", name)


if __name__ == "__main__":
    main()
