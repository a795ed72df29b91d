"""Indexer logits on the GPU (dsv4b_fp8_paged_mqa_logits via indexer.py).

Against the fixtures from DeepGEMM's torch statement (as vLLM carries it),
against the CPU oracle on random batches (head counts 32/64/128, next_n
1/2/4, page sizes 32/64/128, context lengths around page and tile edges,
empty requests, padded page stride, clean_logits off), the device schedule
against its restatement, CUDA-graph capture, and BASELINE config 1's size
(b 32, 131,072 positions) on sampled rows.

Tolerance: q and k are e4m3, products are exact in fp32, the tensor core
and the oracle (float64) sum them in different orders: |got - want| <=
1e-4 * (|want| + max |row|) per row.
"""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import mqa_logits_oracle as M

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "mqa_logits")
FIXTURES = sorted(os.path.splitext(os.path.basename(p))[0] for p in glob.glob(os.path.join(GOLDEN, "*.npz")))


def assert_logits_close(got: np.ndarray, want: np.ndarray, computed_only=False):
    if not computed_only:
        np.testing.assert_array_equal(np.isneginf(got), np.isneginf(want))
    fin = np.isfinite(want)
    for r in range(want.shape[0]):
        f = fin[r]
        if not f.any():
            continue
        scale = np.abs(want[r, f]).max()
        err = np.abs(got[r, f] - want[r, f])
        assert np.all(err <= 1e-4 * (np.abs(want[r, f]) + scale)), (r, err.max(), scale)


def make_case(B, nn, H, P, ctx, seed, pad_page=0, spare_pages=3):
    g = torch.Generator().manual_seed(seed)
    D = 128
    pages = [-(-c // P) for c in ctx]
    nb = sum(pages) + spare_pages
    q = (torch.randn(B, nn, H, D, generator=g) * 2).to(torch.float8_e4m3fn)
    stride = P * (D + 4) + pad_page
    arena = torch.zeros(nb, stride, dtype=torch.uint8)
    arena[:, :P * D] = (torch.randn(nb, P * D, generator=g) * 2).to(torch.float8_e4m3fn).view(torch.uint8)
    arena[:, P * D:P * (D + 4)] = (torch.rand(nb, P, generator=g) * 0.1 + 0.01).view(torch.uint8).view(nb, P * 4)
    w = torch.randn(B * nn, H, generator=g)
    perm = torch.randperm(nb, generator=g)
    bt = torch.zeros(B, max(max(pages), 1) + 2, dtype=torch.int32)
    o = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[o:o + pages[b]]
        o += pages[b]
    return q, arena, w, torch.tensor(ctx, dtype=torch.int32), bt, P


def run_gpu(q, arena, w, ctx, bt, P, max_model_len, clean=True, num_sms=148):
    from deepseek_v4_kernel import indexer
    nb = arena.size(0)
    kv = arena.cuda().as_strided((nb, P, 1, 132), (arena.size(1), 132, 132, 1))
    ctx_d = ctx.cuda()
    sched = indexer.get_paged_mqa_logits_metadata(ctx_d, P, num_sms)
    out = indexer.fp8_paged_mqa_logits(q.cuda(), kv, w.cuda(), ctx_d, bt.cuda(), sched, max_model_len, clean)
    torch.cuda.synchronize()
    return out.cpu().numpy(), sched.cpu().numpy()


def run_oracle(q, arena, w, ctx, bt, P, max_model_len, clean=True):
    return M.fp8_paged_mqa_logits(q.view(torch.uint8).numpy(), arena.numpy(), w.numpy(), ctx.numpy(), bt.numpy(),
                                  P, max_model_len, clean)


@pytest.mark.parametrize("name", FIXTURES)
def test_fixtures(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    P = int(z["page_block"])
    q = torch.from_numpy(z["q"]).view(torch.float8_e4m3fn)
    got, _ = run_gpu(q, torch.from_numpy(z["kv"]), torch.from_numpy(z["weights"]),
                     torch.from_numpy(z["context_lens"]), torch.from_numpy(z["block_table"]), P,
                     int(z["max_model_len"]))
    assert_logits_close(got, z["logits"])


@pytest.mark.parametrize("B,nn,H,P,ctx,pad", [
    (5, 1, 64, 64, [0, 1, 127, 128, 129], 0),
    (4, 1, 64, 64, [5000, 64, 0, 2049], 16),
    (3, 2, 64, 64, [300, 1, 1000], 0),
    (2, 1, 128, 32, [777, 1500], 0),
    (3, 1, 32, 128, [256, 1000, 3], 0),
    (2, 4, 64, 64, [640, 130], 0),
    (3, 2, 128, 64, [400, 900, 1], 0),
])
def test_random_vs_oracle(B, nn, H, P, ctx, pad):
    case = make_case(B, nn, H, P, ctx, seed=B * 100 + H + P + nn, pad_page=pad)
    mml = max(ctx) + 200
    got, _ = run_gpu(*case, mml)
    assert_logits_close(got, run_oracle(*case, mml))


def test_unclean_writes_only_computed_tiles():
    case = make_case(2, 1, 64, 64, [100, 300], seed=5)
    mml = 1024
    from deepseek_v4_kernel import indexer
    q, arena, w, ctx, bt, P = case
    nb = arena.size(0)
    kv = arena.cuda().view(nb, P, 1, 132)
    sched = indexer.get_paged_mqa_logits_metadata(ctx.cuda(), P, 148)
    out = torch.full((2, mml), 7.0, device="cuda")
    indexer.fp8_paged_mqa_logits(q.cuda(), kv, w.cuda(), ctx.cuda(), bt.cuda(), sched, mml, False, out=out)
    got = out.cpu().numpy()
    want = run_oracle(*case, mml)
    assert_logits_close(got[:, :384], want[:, :384], computed_only=True)
    assert np.isneginf(got[0, 100:128]).all() and (got[0, 128:] == 7.0).all()   # tile tail masked, rest untouched
    assert (got[1, 384:] == 7.0).all()


@pytest.mark.parametrize("num_sms", [1, 7, 148, 300])
def test_schedule_restatement(num_sms):
    ctx = [0, 5, 128, 129, 0, 0, 4096, 1, 70000, 0]
    from deepseek_v4_kernel import indexer
    sched = indexer.get_paged_mqa_logits_metadata(torch.tensor(ctx, dtype=torch.int32, device="cuda"), 64,
                                                  num_sms).cpu().numpy()
    tiles = [-(-c // 128) for c in ctx]
    prefix = np.concatenate([[0], np.cumsum(tiles)])
    T = prefix[-1]
    for i in range(num_sms + 1):
        target = T * i // num_sms
        if target >= T:
            want = (len(ctx), 0)
        else:
            b = int(np.searchsorted(prefix, target, side="right") - 1)
            want = (b, int(target - prefix[b]))
        assert tuple(sched[i]) == want, (i, tuple(sched[i]), want)
    # any CTA count gives the same logits
    case = make_case(len(ctx), 1, 64, 64, [min(c, 3000) for c in ctx], seed=9)
    a, _ = run_gpu(*case, 3100, num_sms=num_sms)
    b, _ = run_gpu(*case, 3100, num_sms=148)
    np.testing.assert_array_equal(a, b)


def test_graph_capture_and_status():
    from deepseek_v4_kernel import indexer
    q, arena, w, ctx, bt, P = make_case(3, 1, 64, 64, [1000, 2000, 64], seed=11)
    nb = arena.size(0)
    kv = arena.cuda().view(nb, P, 1, 132)
    qd, wd, cd, bd = q.cuda(), w.cuda(), ctx.cuda(), bt.cuda()
    sched = indexer.get_paged_mqa_logits_metadata(cd, P, 148)
    eager = indexer.fp8_paged_mqa_logits(qd, kv, wd, cd, bd, sched, 2048)
    out = torch.zeros_like(eager)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        indexer.fp8_paged_mqa_logits(qd, kv, wd, cd, bd, sched, 2048, out=out)
    torch.cuda.current_stream().wait_stream(s)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    assert indexer.mqa_logits_status() == 0


def test_config1_size_sampled_rows():
    """b 32 x 131,072 positions (BASELINE config 1's contexts), P 64,
    554 MB of index cache; two rows checked in full against the oracle."""
    from deepseek_v4_kernel import indexer
    B, H, P, ctx_len = 32, 64, 64, 131072
    pages = ctx_len // P
    nb = B * pages
    g = torch.Generator(device="cuda").manual_seed(3)
    arena = torch.empty(nb, P * 132, dtype=torch.uint8, device="cuda")
    arena[:, :P * 128] = (torch.randn(nb, P * 128, generator=g, device="cuda") * 2).to(torch.float8_e4m3fn).view(torch.uint8)
    arena[:, P * 128:] = (torch.rand(nb, P, generator=g, device="cuda") * 0.1 + 0.01).view(torch.uint8).view(nb, P * 4)
    q = (torch.randn(B, 1, H, 128, generator=g, device="cuda") * 2).to(torch.float8_e4m3fn)
    w = torch.randn(B, H, generator=g, device="cuda")
    ctx = torch.full((B,), ctx_len, dtype=torch.int32, device="cuda")
    bt = torch.randperm(nb, generator=g, device="cuda").view(B, pages).int()
    sched = indexer.get_paged_mqa_logits_metadata(ctx, P, 148)
    out = indexer.fp8_paged_mqa_logits(q, arena.view(nb, P, 1, 132), w, ctx, bt, sched, ctx_len)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    for b in (0, 31):
        rows = bt[b].cpu().numpy()
        sub = arena[torch.from_numpy(rows).cuda().long()].cpu().numpy()
        want = M.fp8_paged_mqa_logits(q[b:b + 1].view(torch.uint8).cpu().numpy(), sub, w[b:b + 1].cpu().numpy(),
                                      np.array([ctx_len]), np.arange(pages)[None, :], P, ctx_len)
        assert_logits_close(out[b:b + 1].cpu().numpy(), want)
