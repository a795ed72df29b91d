"""Generate golden vectors by running the reference's own CPU oracle.

Run in a container that holds the reference checkout (read-only):

    python tests/golden/make_golden.py --reference /path/to/deepseek-v4-flash-sm120

It imports the reference's unmodified ``tests/reference.py``
(``make_fake_batch`` at :135-199, ``sparse_decode_reference`` at :82-132),
builds MODEL1 batches on the CPU with fixed seeds, runs the oracle and
writes inputs + outputs to ``tests/golden/*.npz``.  The GPU box does not
have the reference; the tests only read these files.

Cases: the shapes of the reference's ``tests/test_sparse_decode.py``
(``test_matches_reference`` :27-49 and ``test_topk_length_mask`` :52-67),
plus edge cases those tests do not cover: attn_sink, guaranteed -1 and
out-of-range indices, topk_length = 0 and > topk.
"""
from __future__ import annotations

import argparse
import importlib.util
import math
import os

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _load_reference(ref_root: str):
    path = os.path.join(ref_root, "tests", "reference.py")
    spec = importlib.util.spec_from_file_location("dsv4_reference_oracle", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _save(name, q, kv_pages, idx, tk, sink, sm_scale, page_block, out, lse):
    np.savez_compressed(
        os.path.join(HERE, f"{name}.npz"),
        q_bf16=_bf16_bits(q),
        kv_pages=kv_pages.numpy(),
        indices=idx.numpy().astype(np.int32),
        topk_length=(tk.numpy().astype(np.int32) if tk is not None
                     else np.zeros(0, np.int32)),
        has_topk_length=np.array(tk is not None),
        attn_sink=(sink.numpy().astype(np.float32) if sink is not None
                   else np.zeros(0, np.float32)),
        has_sink=np.array(sink is not None),
        sm_scale=np.array(sm_scale, dtype=np.float64),
        page_block=np.array(page_block),
        out_bf16=_bf16_bits(out),
        lse=lse.numpy().astype(np.float32),
    )
    print("wrote", name, tuple(q.shape), "topk", idx.shape[-1])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("DSV4_REFERENCE_ROOT", ""))
    args = ap.parse_args()
    ref = _load_reference(args.reference)
    torch.set_num_threads(max(1, os.cpu_count() or 1))

    def run(name, b, h_q, num_blocks, page_block, topk, seed, tk=None,
            sink=False, force_invalid=False):
        torch.manual_seed(seed)
        q, kv_pages, _kv_view, idx = ref.make_fake_batch(
            b=b, h_q=h_q, num_blocks=num_blocks, page_block=page_block,
            topk=topk, seed=seed, device="cpu")
        if force_invalid:
            n = num_blocks * page_block
            idx = idx.clone()
            idx[:, :, -16:] = -1          # -1 padding tail
            idx[:, :, 3] = n              # first out-of-range value
            idx[:, :, 5] = n + 1000       # far out of range
            idx[:, :, 7] = -1
        sink_t = None
        if sink:
            g = torch.Generator().manual_seed(seed + 100)
            sink_t = torch.randn(h_q, generator=g, dtype=torch.float32)
        tk_t = None if tk is None else torch.tensor(tk, dtype=torch.int32)
        sm_scale = 1.0 / math.sqrt(512)
        out, lse = ref.sparse_decode_reference(
            q, kv_pages, idx, topk_length=tk_t, attn_sink=sink_t,
            sm_scale=sm_scale, page_block=page_block)
        _save(name, q, kv_pages, idx, tk_t, sink_t, sm_scale, page_block, out, lse)

    # tests/test_sparse_decode.py:27-49 shapes (b=2, 8 pages of 64 tokens)
    run("m1_h64_topk64", 2, 64, 8, 64, 64, 0)
    run("m1_h64_topk2048", 2, 64, 8, 64, 2048, 0)
    run("m1_h128_topk256", 2, 128, 8, 64, 256, 0)
    # tests/test_sparse_decode.py:52-67 (topk_length mask)
    run("m1_topk_length", 2, 64, 4, 64, 512, 1, tk=[64, 32])
    # edge cases the reference tests do not cover
    run("m1_sink", 2, 64, 8, 64, 256, 2, sink=True)
    run("m1_invalid_idx", 2, 16, 8, 64, 192, 3, force_invalid=True)
    run("m1_len0_and_over", 2, 16, 8, 64, 160, 4, tk=[0, 100000], sink=True)


if __name__ == "__main__":
    main()
