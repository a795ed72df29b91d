"""Multi-GPU partition layer, tested on CPU with gloo (world size 2).

Sparse decode shards with no data-path collective: query rows
(batch sharding) or query heads (head sharding over a replicated cache)
are independent.  Each rank here builds its own shard the way the
benchmark does (batch: only its requests and their pages), runs the CPU
oracle on it, the
shards are reassembled with the same all-gather helpers the GPU path
uses (NCCL there, gloo here), and the result is compared with the
unsharded oracle on every rank.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dsv4b_testutil import OUT_ATOL, OUT_RTOL, oracle_for


def _free_port() -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_even_ranges_cover_and_balance():
    from deepseek_v4_kernel import partition
    for n in (0, 1, 7, 32, 257):
        for world in (1, 2, 3, 8):
            spans = [partition.even_range(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1


def test_head_range_requires_even_split():
    from deepseek_v4_kernel import partition
    assert partition.head_range(128, 3, 4) == (96, 128)
    with pytest.raises(ValueError):
        partition.head_range(64, 0, 3)
    with pytest.raises(ValueError):
        partition.even_range(8, 2, 2)


@pytest.mark.parametrize("layout", ["v32", "model1"])
def test_batch_shards_hold_the_unsharded_requests(layout):
    """make_batch_shard: the requests of a shard are byte-identical to the
    same requests of the unsharded batch (q, gathered cache rows, -1
    padding), whatever the page placement."""
    from deepseek_v4_kernel import kvcache
    spec = kvcache.BatchSpec(b=7, s_q=2, h_q=16, topk=96, ctx=700, page_block=64, layout=layout,
                             draft_overlap=0.5, invalid_tail=5, seed=11)
    full = kvcache.make_batch_shard(spec, 0, spec.b, device="cpu")

    def rows(bt):
        if layout == "v32":
            flat = bt.kv.view(-1, 656)
            g = flat[bt.indices.clamp_min(0).long()]
        else:  # MODEL1: [576-B row | 8-B scales] per token, from the page arena
            arena = bt.kv.view(bt.kv.shape[0], -1)
            P = bt.kv.shape[1]
            i = bt.indices.clamp_min(0).long()
            pg, off = i // P, i % P
            r = arena[pg.unsqueeze(-1), off.unsqueeze(-1) * 576 + torch.arange(576)]
            s = arena[pg.unsqueeze(-1), P * 576 + off.unsqueeze(-1) * 8 + torch.arange(8)]
            g = torch.cat([r, s], -1)
        return torch.where((bt.indices >= 0).unsqueeze(-1), g, torch.zeros_like(g))

    parts = [kvcache.make_batch_shard(spec, lo, hi, device="cpu") for lo, hi in ((0, 3), (3, 4), (4, 7))]
    assert torch.equal(full.q, torch.cat([s.q for s in parts]))
    assert torch.equal(rows(full), torch.cat([rows(s) for s in parts]))
    assert torch.equal(full.indices < 0, torch.cat([s.indices < 0 for s in parts]))
    assert all(s.kv.shape[0] == (hi - lo) * 11 for s, (lo, hi) in zip(parts, ((0, 3), (3, 4), (4, 7))))


def _worker(rank, world, port, mode):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from deepseek_v4_kernel import kvcache, partition
        torch.set_num_threads(1)
        spec = kvcache.BatchSpec(b=5, s_q=1, h_q=16, topk=96, ctx=512, page_block=64,
                                 invalid_tail=7, seed=5)
        bt = kvcache.make_batch_shard(spec, 0, spec.b, device="cpu")
        ref_out, _ = oracle_for(bt.q, bt.kv, bt.indices, None, bt.attn_sink, bt.sm_scale, "v32")
        if mode == "batch":
            # as the benchmark does: the rank builds only its own requests
            # (and their pages) of the global batch
            lo, hi = partition.batch_range(spec.b, rank, world)
            sh = kvcache.make_batch_shard(spec, lo, hi, device="cpu")
            out, _ = oracle_for(sh.q, sh.kv, sh.indices, None, sh.attn_sink, sh.sm_scale, "v32")
            full = partition.all_gather_batch(torch.from_numpy(out), spec.b, world)
        else:
            q, sink, (lo, hi) = partition.shard_heads(bt.q, bt.attn_sink, rank, world)
            out, _ = oracle_for(q, bt.kv, bt.indices, None, sink, bt.sm_scale, "v32")
            full = partition.all_gather_heads(torch.from_numpy(out), world)
        # the shard's products are blocked differently by numpy's BLAS, so a
        # few outputs can round to the neighbouring bf16 value
        np.testing.assert_allclose(full.numpy(), ref_out, rtol=OUT_RTOL, atol=OUT_ATOL)
        assert np.mean(full.numpy() != ref_out) < 1e-3
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["batch", "head"])
def test_sharded_oracle_matches_unsharded_gloo_world2(mode):
    mp.spawn(_worker, args=(2, _free_port(), mode), nprocs=2, join=True)
