"""Generate the KV-cache writer fixtures (tests/golden/kv_writer/*.npz).

Run in a container that holds the reference checkout (read-only):

    python tests/golden/make_kv_writer_golden.py --reference /path/to/deepseek-v4-flash-sm120

Seeded bf16 tokens (mixed magnitudes, all-zero tiles, tiles whose
max |x| is exactly 448 * 2^j, negative zeros, tiny subnormal-range values)
are quantised and scattered into a paged cache by the CPU oracle
(``oracle/kv_writer_oracle.py``) with some slots -1 or past the cache; every other cache byte starts as
0xA5 (FILL) and must stay so.

MODEL1 fixtures also store the reference's own unpack of the written pages
(``tests/reference.py:61-79`` ``_pages_to_bf16``, imported unmodified), so
the CPU tests hold the writer's bytes to the reference's reading of them.
The reference has no V32 unpack; the V32 fixture carries the oracle's
bytes only (held to vLLM's writer by the GPU tests).
"""
from __future__ import annotations

import argparse
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
OUT_DIR = os.path.join(HERE, "kv_writer")
FILL = 0xA5
sys.path.insert(0, ROOT)

from oracle import kv_writer_oracle as KW  # noqa: E402


def _load_reference(ref_root: str):
    path = os.path.join(ref_root, "tests", "reference.py")
    spec = importlib.util.spec_from_file_location("dsv4_reference_oracle", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def tokens(n: int, cols: int, seed: int) -> np.ndarray:
    """bf16 bits [n, cols] with the edge tiles described above (tile = 64
    columns; V32 scales over 128, so its edges cover both halves)."""
    g = torch.Generator().manual_seed(seed)
    mag = torch.exp(torch.empty(n, 1).uniform_(-12.0, 12.0, generator=g))
    x = (torch.randn(n, cols, generator=g) * mag).to(torch.bfloat16)
    w = min(cols, 128)
    x[0, :w] = 0.0                                     # all-zero tiles -> 1e-4 floor
    x[1, :w] = -0.0
    x[2, :] = (torch.randn(cols, generator=g) * 1e-38).to(torch.bfloat16)  # tiny values
    x[3, :w] = (torch.rand(w, generator=g) * 448.0).to(torch.bfloat16)
    x[3, 5] = 448.0                                    # amax / 448 exactly 2^0
    x[4, :w] = (torch.rand(w, generator=g) * 0.875).to(torch.bfloat16)
    x[4, w - 3] = -0.875                                  # amax / 448 = 2^-9
    x[5, :] = (torch.randn(cols, generator=g) * 1e30).to(torch.bfloat16)  # huge values
    return x.view(torch.int16).numpy().view(np.uint16)


def slots_for(n: int, cache_tokens: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    s = rng.permutation(cache_tokens)[:n].astype(np.int64)
    s[rng.choice(n, size=max(1, n // 16), replace=False)] = -1
    s[n // 3] = cache_tokens          # past the cache: skipped
    s[n // 2] = cache_tokens + 1000
    return s


def make_model1(ref, name: str, n: int, page_block: int, num_blocks: int, seed: int):
    nope = tokens(n, 448, seed)
    rope = tokens(n, 64, seed + 1)
    slots = slots_for(n, num_blocks * page_block, seed + 2)
    arena = np.full((num_blocks, page_block * 584), FILL, np.uint8)
    KW.kv_cache_write("model1", arena, page_block, nope, rope, slots)
    deq = ref._pages_to_bf16(torch.from_numpy(arena.copy()), page_block)   # [cache tokens, 512] bf16
    written = np.nonzero((slots >= 0) & (slots < num_blocks * page_block))[0]
    deq_bits = deq[torch.from_numpy(slots[written])].contiguous().view(torch.int16).numpy().view(np.uint16)
    np.savez_compressed(os.path.join(OUT_DIR, f"{name}.npz"), layout="model1", nope=nope, rope=rope,
                        slots=slots, page_block=page_block, arena_after=arena,
                        ref_dequant_tokens=written, ref_dequant=deq_bits)
    print("wrote", name, n, "tokens", num_blocks, "pages of", page_block)


def make_v32(name: str, n: int, page_block: int, num_blocks: int, seed: int):
    nope = tokens(n, 512, seed)
    rope = tokens(n, 64, seed + 1)
    slots = slots_for(n, num_blocks * page_block, seed + 2)
    arena = np.full((num_blocks, page_block * 656), FILL, np.uint8)
    KW.kv_cache_write("v32", arena, page_block, nope, rope, slots)
    np.savez_compressed(os.path.join(OUT_DIR, f"{name}.npz"), layout="v32", nope=nope, rope=rope,
                        slots=slots, page_block=page_block, arena_after=arena)
    print("wrote", name, n, "tokens", num_blocks, "pages of", page_block)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    ref = _load_reference(args.reference)
    os.makedirs(OUT_DIR, exist_ok=True)
    make_model1(ref, "model1_p64", n=200, page_block=64, num_blocks=5, seed=11)
    make_model1(ref, "model1_p256", n=300, page_block=256, num_blocks=2, seed=12)
    make_v32("v32_p64", n=200, page_block=64, num_blocks=5, seed=13)


if __name__ == "__main__":
    main()
