"""Generate the indexer-logits fixtures (tests/golden/mqa_logits/*.npz).

    python tests/golden/make_mqa_logits_golden.py

Runs DeepGEMM's published torch statement of fp8_paged_mqa_logits, as
vLLM 0.22 carries it (vllm/v1/attention/ops/rocm_aiter_mla_sparse.py:
256-300, importable on CPU), on seeded inputs with next_n = 1 (the branch
that reads the page-sectioned cache layout) and stores inputs and logits.
The cache pages hold valid e4m3 values (no NaN codes) and positive scales;
some context lengths are not multiples of the page or of 128.
"""
from __future__ import annotations

import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "mqa_logits")


def make(name, B, H, P, ctx, num_blocks, max_model_len, seed):
    from vllm.v1.attention.ops.rocm_aiter_mla_sparse import fp8_paged_mqa_logits_torch
    g = torch.Generator().manual_seed(seed)
    D = 128
    q = (torch.randn(B, 1, H, D, generator=g) * 2).to(torch.float8_e4m3fn)
    vals = (torch.randn(num_blocks, P * D, generator=g) * 2).to(torch.float8_e4m3fn).view(torch.uint8)
    scales = (torch.rand(num_blocks, P, generator=g) * 0.1 + 0.01).contiguous()
    kv = torch.cat([vals, scales.view(torch.uint8).view(num_blocks, P * 4)], dim=1).contiguous()
    w = torch.randn(B, H, generator=g)
    ctx_t = torch.tensor(ctx, dtype=torch.int32)
    max_pages = max(-(-c // P) for c in ctx)
    bt = torch.stack([torch.randperm(num_blocks, generator=g)[:max_pages] for _ in range(B)]).to(torch.int32)
    logits = fp8_paged_mqa_logits_torch(q, kv.view(num_blocks, P, 1, D + 4), w, ctx_t, bt, max_model_len)
    np.savez_compressed(os.path.join(OUT_DIR, f"{name}.npz"), q=q.view(torch.uint8).numpy(), kv=kv.numpy(),
                        weights=w.numpy(), context_lens=ctx_t.numpy(), block_table=bt.numpy(), page_block=P,
                        max_model_len=max_model_len, logits=logits.numpy())
    print("wrote", name, tuple(q.shape), "ctx", ctx)


def main():
    os.makedirs(OUT_DIR, exist_ok=True)
    make("h64_p64", B=3, H=64, P=64, ctx=[1, 300, 640], num_blocks=24, max_model_len=768, seed=1)
    make("h64_p32", B=2, H=64, P=32, ctx=[129, 257], num_blocks=20, max_model_len=320, seed=2)
    make("h32_p128", B=2, H=32, P=128, ctx=[500, 128], num_blocks=8, max_model_len=512, seed=3)


if __name__ == "__main__":
    main()
