"""KV-cache byte formats: quantisers and seeded synthetic batches.

Quantisers write the two page formats the decode kernel reads:

* V32 (DeepSeek-V3.2, FlashMLA FP8 sparse; vLLM flash_mla_interface.py:95-101):
  656 B per token, token-contiguous: 512 x e4m3 (latent / scale of its
  128-column tile), 4 x fp32 scales (max(amax / 448, FLT_MIN) per 128
  columns, vLLM's fp8_ds_mla rule), 64 x bf16 RoPE.  Pages are
  [page_block, 1, 656].
* MODEL1 (DeepSeek-V4-Flash; reference tests/reference.py:7-19): per page
  page_block x 576 B rows [448 x e4m3 | 64 x bf16 RoPE], then page_block x
  8 B of UE8M0 exponents (7 used: 2^e per 64 columns, + 1 pad).

``make_batch`` builds the synthetic inputs the benchmark configurations
describe (seeded): q ~ N(0,1) bf16, latent ~ N(0,1) quantised as above,
RoPE ~ N(0,1) bf16, per-request block tables that are random page
permutations, and distinct top-k positions per query row (optional -1
tail, optional overlap between the s_q draft rows).
"""
from __future__ import annotations

import dataclasses
import math
from typing import Optional

import torch

FP8_MAX = 448.0
AMAX_FLOOR = 1e-4  # MODEL1: an all-zero tile gets scale 2^ceil(log2(1e-4/448))
FLT_MIN = 1.17549435e-38  # V32: an all-zero tile gets scale FLT_MIN


def _to_e4m3_bytes(x: torch.Tensor) -> torch.Tensor:
    return x.clamp(-FP8_MAX, FP8_MAX).to(torch.float8_e4m3fn).view(torch.uint8)


def quantize_v32(latent: torch.Tensor, rope: torch.Tensor) -> torch.Tensor:
    """latent [N, 512] float, rope [N, 64] bf16 -> uint8 [N, 656]."""
    n = latent.shape[0]
    lt = latent.to(torch.bfloat16).float().view(n, 4, 128)
    amax = lt.abs().amax(dim=-1)
    # divide by a tensor: torch's CUDA division by a Python scalar multiplies
    # by the reciprocal, which is not the correctly rounded quotient
    scale = (amax / torch.full_like(amax, FP8_MAX)).clamp_min(FLT_MIN)     # [N, 4] fp32
    q8 = _to_e4m3_bytes(lt / scale.unsqueeze(-1)).view(n, 512)
    sc = scale.contiguous().view(torch.uint8).view(n, 16)
    rp = rope.to(torch.bfloat16).contiguous().view(torch.uint8).view(n, 128)
    return torch.cat([q8, sc, rp], dim=-1).contiguous()


def quantize_model1_pages(nope: torch.Tensor, rope: torch.Tensor, page_block: int) -> torch.Tensor:
    """nope [N, 448] float, rope [N, 64] bf16 (N = pages * page_block) ->
    uint8 page arena [pages, page_block * 584]."""
    n = nope.shape[0]
    assert n % page_block == 0
    pages = n // page_block
    nt = nope.float().view(n, 7, 64)
    amax = nt.abs().amax(dim=-1).clamp_min(AMAX_FLOOR)
    e = torch.ceil(torch.log2(amax / FP8_MAX)).clamp(-127, 127)            # power-of-two scale
    q8 = _to_e4m3_bytes(nt / torch.pow(2.0, e).unsqueeze(-1)).view(n, 448)
    ebytes = (e + 127).to(torch.uint8)
    sc = torch.cat([ebytes, torch.zeros(n, 1, dtype=torch.uint8, device=nope.device)], dim=-1)
    rp = rope.to(torch.bfloat16).contiguous().view(torch.uint8).view(n, 128)
    rows = torch.cat([q8, rp], dim=-1).view(pages, page_block * 576)
    return torch.cat([rows, sc.view(pages, page_block * 8)], dim=-1).contiguous()


@dataclasses.dataclass
class BatchSpec:
    b: int
    s_q: int
    h_q: int
    topk: int
    ctx: int                      # logical context length per request
    page_block: int = 256
    layout: str = "v32"           # "v32" | "model1"
    cache_ctx: Optional[int] = None  # tokens allocated per request (>= ctx)
    invalid_tail: int = 0         # last N indices of every row set to -1
    draft_overlap: float = 0.0    # fraction of row s>0 indices shared with row 0
    with_sink: bool = True
    seed: int = 0


@dataclasses.dataclass
class Batch:
    q: torch.Tensor               # bf16 [b, s_q, h_q, d_qk]
    kv: torch.Tensor              # uint8 [num_blocks, page_block, 1, bytes]
    indices: torch.Tensor         # int32 [b, s_q, topk] flat page*P + offset
    attn_sink: Optional[torch.Tensor]
    sm_scale: float
    spec: BatchSpec

    @property
    def d_qk(self) -> int:
        return self.q.shape[-1]


def make_batch(spec: BatchSpec, device="cuda", chunk_tokens: int = 1 << 20) -> Batch:
    g = torch.Generator(device=device).manual_seed(spec.seed)
    d_qk = 576 if spec.layout == "v32" else 512
    cache_ctx = spec.cache_ctx or spec.ctx
    pages_per_req = -(-cache_ctx // spec.page_block)
    num_blocks = spec.b * pages_per_req
    n_tok = num_blocks * spec.page_block
    q = torch.randn(spec.b, spec.s_q, spec.h_q, d_qk, generator=g, device=device).to(torch.bfloat16)

    # cache, generated and quantised in chunks of whole pages
    step = max(spec.page_block, (chunk_tokens // spec.page_block) * spec.page_block)
    if spec.layout == "v32":
        kv = torch.empty(n_tok, 656, dtype=torch.uint8, device=device)
        for s in range(0, n_tok, step):
            e = min(n_tok, s + step)
            lat = torch.randn(e - s, 512, generator=g, device=device)
            rope = torch.randn(e - s, 64, generator=g, device=device).to(torch.bfloat16)
            kv[s:e] = quantize_v32(lat, rope)
        kv = kv.view(num_blocks, spec.page_block, 1, 656)
    else:
        arena = torch.empty(num_blocks, spec.page_block * 584, dtype=torch.uint8, device=device)
        pstep = step // spec.page_block
        for s in range(0, num_blocks, pstep):
            e = min(num_blocks, s + pstep)
            nt = (e - s) * spec.page_block
            nope = torch.randn(nt, 448, generator=g, device=device)
            rope = torch.randn(nt, 64, generator=g, device=device).to(torch.bfloat16)
            arena[s:e] = quantize_model1_pages(nope, rope, spec.page_block)
        kv = arena.view(num_blocks, spec.page_block, 1, 584)

    # block tables: request r owns a random permutation of pages
    perm = torch.randperm(num_blocks, generator=g, device=device).view(spec.b, pages_per_req)
    idx = torch.empty(spec.b, spec.s_q, spec.topk, dtype=torch.int64, device=device)
    for bi in range(spec.b):
        base = torch.randperm(spec.ctx, generator=g, device=device)[: spec.topk]
        idx[bi, 0] = base
        for si in range(1, spec.s_q):
            fresh = torch.randperm(spec.ctx, generator=g, device=device)[: spec.topk]
            n_share = int(round(spec.draft_overlap * spec.topk))
            row = fresh.clone()
            if n_share:
                # keep n_share of row 0's positions, fill the rest with positions not in row 0
                mask = torch.ones(spec.ctx, dtype=torch.bool, device=device)
                mask[base] = False
                pool = torch.nonzero(mask).squeeze(1)
                pick = pool[torch.randperm(pool.numel(), generator=g, device=device)[: spec.topk - n_share]]
                row = torch.cat([base[:n_share], pick])
                row = row[torch.randperm(spec.topk, generator=g, device=device)]
            idx[bi, si] = row
    page = perm.gather(1, (idx // spec.page_block).view(spec.b, -1)).view_as(idx)
    flat = (page * spec.page_block + idx % spec.page_block).to(torch.int32)
    if spec.invalid_tail:
        flat[..., -spec.invalid_tail:] = -1
    sink = torch.randn(spec.h_q, generator=g, device=device) if spec.with_sink else None
    return Batch(q=q, kv=kv, indices=flat.contiguous(), attn_sink=sink,
                 sm_scale=1.0 / math.sqrt(d_qk), spec=spec)


def _request_indices(spec: BatchSpec, g: torch.Generator, device) -> torch.Tensor:
    """Logical top-k positions [s_q, topk] of one request: distinct uniform
    positions in [0, ctx) per draft row, row s > 0 sharing
    round(draft_overlap * topk) of row 0's positions."""
    idx = torch.empty(spec.s_q, spec.topk, dtype=torch.int64, device=device)
    base = torch.randperm(spec.ctx, generator=g, device=device)[: spec.topk]
    idx[0] = base
    n_share = int(round(spec.draft_overlap * spec.topk))
    for si in range(1, spec.s_q):
        if n_share:
            mask = torch.ones(spec.ctx, dtype=torch.bool, device=device)
            mask[base] = False
            pool = torch.nonzero(mask).squeeze(1)
            pick = pool[torch.randperm(pool.numel(), generator=g, device=device)[: spec.topk - n_share]]
            row = torch.cat([base[:n_share], pick])
            idx[si] = row[torch.randperm(spec.topk, generator=g, device=device)]
        else:
            idx[si] = torch.randperm(spec.ctx, generator=g, device=device)[: spec.topk]
    return idx


def make_batch_shard(spec: BatchSpec, lo: int, hi: int, device="cuda") -> Batch:
    """Requests [lo, hi) of the global batch `spec` (spec.b requests), built
    so that any rank can build its own shard alone: request r's q, cache
    rows and top-k positions come from a generator seeded by (spec.seed, r)
    only, so the rows of a request are the same bytes in every shard that
    holds it (and in the unsharded batch, lo = 0, hi = spec.b).  The shard's
    cache holds only its requests' pages, placed by a random permutation of
    the shard's pages (the block tables are random page permutations, as in
    make_batch).  attn_sink is seeded by spec.seed alone (one per model)."""
    if not 0 <= lo < hi <= spec.b:
        raise ValueError(f"bad request range [{lo}, {hi}) of {spec.b}")
    nreq = hi - lo
    d_qk = 576 if spec.layout == "v32" else 512
    bpt = 656 if spec.layout == "v32" else 584
    cache_ctx = spec.cache_ctx or spec.ctx
    P = spec.page_block
    ppr = -(-cache_ctx // P)
    num_blocks = nreq * ppr
    g_place = torch.Generator(device=device).manual_seed(spec.seed * 7919 + lo * 104729 + hi)
    perm = torch.randperm(num_blocks, generator=g_place, device=device).view(nreq, ppr)
    q = torch.empty(nreq, spec.s_q, spec.h_q, d_qk, dtype=torch.bfloat16, device=device)
    idx = torch.empty(nreq, spec.s_q, spec.topk, dtype=torch.int64, device=device)
    if spec.layout == "v32":
        kv = torch.empty(num_blocks, P, 656, dtype=torch.uint8, device=device)
    else:
        kv = torch.empty(num_blocks, P * 584, dtype=torch.uint8, device=device)
    for i, r in enumerate(range(lo, hi)):
        g = torch.Generator(device=device).manual_seed(spec.seed * 1000003 + r)
        q[i] = torch.randn(spec.s_q, spec.h_q, d_qk, generator=g, device=device).to(torch.bfloat16)
        n = ppr * P
        if spec.layout == "v32":
            rows = quantize_v32(torch.randn(n, 512, generator=g, device=device),
                                torch.randn(n, 64, generator=g, device=device).to(torch.bfloat16))
            kv[perm[i]] = rows.view(ppr, P, 656)
        else:
            kv[perm[i]] = quantize_model1_pages(torch.randn(n, 448, generator=g, device=device),
                                                torch.randn(n, 64, generator=g, device=device).to(torch.bfloat16),
                                                P)
        idx[i] = _request_indices(spec, g, device)
    page = perm.gather(1, (idx // P).view(nreq, -1)).view_as(idx)
    flat = (page * P + idx % P).to(torch.int32)
    if spec.invalid_tail:
        flat[..., -spec.invalid_tail:] = -1
    g_sink = torch.Generator(device=device).manual_seed(spec.seed)
    sink = torch.randn(spec.h_q, generator=g_sink, device=device) if spec.with_sink else None
    shard_spec = BatchSpec(**{**spec.__dict__, "b": nreq})
    return Batch(q=q, kv=kv.view(num_blocks, P, 1, bpt), indices=flat.contiguous(), attn_sink=sink,
                 sm_scale=1.0 / math.sqrt(d_qk), spec=shard_spec)


# The benchmark configurations (BASELINE.json "configs"), as BatchSpecs.
CONFIGS = {
    0: BatchSpec(b=1, s_q=1, h_q=16, topk=128, ctx=4096, page_block=256, invalid_tail=16),
    1: BatchSpec(b=32, s_q=1, h_q=64, topk=2048, ctx=131072, page_block=256),
    2: BatchSpec(b=8, s_q=2, h_q=128, topk=2048, ctx=300000, cache_ctx=393216, page_block=256,
                 draft_overlap=0.5),
    4: BatchSpec(b=256, s_q=1, h_q=128, topk=2048, ctx=65536, page_block=256),
}


def sweep_spec(b: int, ctx: int) -> BatchSpec:
    """Configuration 3 (CUDA-graph batch sweep): h_q 64, top-k 2048."""
    return BatchSpec(b=b, s_q=1, h_q=64, topk=2048, ctx=ctx, page_block=256)
