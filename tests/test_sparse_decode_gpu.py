"""GPU parity tests: the sm_100a path against the CPU oracle and against
the reference's own golden vectors.  Tolerances (written here and in
dsv4b_testutil): output max-abs 2e-2 at rtol 1e-2, LSE 1e-3; the gather /
dequantisation is compared bit for bit."""
import math

import numpy as np
import pytest
import torch

from dsv4b_testutil import LSE_ATOL, LSE_RTOL, OUT_ATOL, OUT_RTOL, assert_matches, assert_rows_match, oracle_for
from golden_io import golden_names, load_golden
from oracle import schedule_oracle as SO
from oracle import sparse_decode_oracle as O

pytestmark = pytest.mark.gpu



def _kc():
    from deepseek_v4_kernel import kvcache
    return kvcache


def _params(batch, topk_length=None, extra=None):
    from deepseek_v4_kernel import ops
    q = batch.q
    b, s_q, h_q, d_qk = q.shape
    o = torch.empty(b, s_q, h_q, 512, dtype=torch.bfloat16, device=q.device)
    l = torch.empty(b, h_q, s_q, dtype=torch.float32, device=q.device)
    return ops.build_params(q, batch.kv, batch.indices, topk_length, batch.attn_sink,
                            *(extra if extra else (None, None, None)), 512, batch.sm_scale, o, l)


def _run(batch, topk_length=None, parts=None, extra=None, out=None):
    from deepseek_v4_kernel import ops
    q, kv, idx = batch.q, batch.kv, batch.indices
    tsm = ns = None
    if parts is not None:
        tsm, ns = ops.get_mla_metadata_tensors(_params(batch, topk_length, extra), q.device, parts)
    ekv, eidx, etk = extra if extra else (None, None, None)
    return ops.sparse_decode_fwd(q, kv, idx, topk_length, batch.attn_sink, tsm, ns, ekv, eidx, etk,
                                 512, batch.sm_scale, out=out)


@pytest.fixture(scope="module", autouse=True)
def _device():
    torch.cuda.set_device(0)
    from deepseek_v4_kernel import _lib
    assert _lib.lib.dsv4b_check_device(0) == 0, "not an sm_100 device"
    yield
    from deepseek_v4_kernel import ops
    assert ops.read_kernel_status() == 0, "a kernel wait timed out"


# ---------------------------------------------------------------- gather
@pytest.mark.parametrize("layout", ["v32", "model1"])
def test_gather_dequant_bit_exact(layout):
    from deepseek_v4_kernel import ops
    spec = _kc().BatchSpec(b=2, s_q=1, h_q=16, topk=300, ctx=2048, page_block=64, layout=layout,
                           seed=11)
    bt = _kc().make_batch(spec)
    n_tok = bt.kv.shape[0] * bt.kv.shape[1]
    idx = bt.indices.reshape(-1)[:512].clone()
    idx[::17] = -1
    idx[5] = n_tok
    idx[9] = n_tok + 12345
    got = ops.gather_dequant(bt.kv, idx)
    kvn = bt.kv.cpu().view(torch.uint8).numpy()
    if layout == "model1":
        kvn = kvn.reshape(bt.kv.shape[0], -1)
    want = O.gather_rows(layout, kvn, bt.kv.shape[1], idx.cpu().numpy())
    got_bits = got.cpu().view(torch.int16).numpy().view(np.uint16)
    want_bits = O.f32_to_bf16_bits(want)
    assert np.array_equal(got_bits, want_bits)


def test_gather_dequant_subnormal_and_extreme_scales():
    """fp8 subnormals, UE8M0 exponents 0/1/254 (MODEL1), tiny / huge fp32
    scales (V32) decode exactly like the oracle."""
    from deepseek_v4_kernel import ops
    rng = np.random.default_rng(3)
    # V32: 8 tokens, one page
    rec = rng.integers(0, 256, size=(8, 656), dtype=np.uint8)
    rec[:, :512] &= 0xF7                      # clear bit 3 -> no NaN encodings (0x7F/0xFF)
    rec[:, :64] = rng.integers(0, 8, size=(8, 64), dtype=np.uint8)  # subnormals
    scales = np.array([[1e-30, 3e20, 1.0 / 3.0, 7.1e-3]] * 8, np.float32)
    rec[:, 512:528] = scales.view(np.uint8)
    rec[:, 528:] = rng.integers(0, 256, size=(8, 128), dtype=np.uint8) & 0x7F
    kv = torch.from_numpy(rec).view(1, 8, 1, 656).cuda()
    idx = torch.arange(8, dtype=torch.int32, device="cuda")
    got = ops.gather_dequant(kv, idx).cpu().view(torch.int16).numpy().view(np.uint16)
    want = O.f32_to_bf16_bits(O.gather_rows("v32", rec.reshape(1, 8, 1, 656), 8, np.arange(8)))
    assert np.array_equal(got, want)
    # MODEL1: 4 tokens, one page of 4
    arena = np.zeros((1, 4 * 584), np.uint8)
    nr = rng.integers(0, 256, size=(4, 576), dtype=np.uint8)
    nr[:, :448] &= 0xF7
    nr[:, 448:] &= 0x7F
    arena[0, :4 * 576] = nr.reshape(-1)
    sc = np.array([[0, 1, 254, 127, 120, 135, 2, 0]] * 4, np.uint8)
    arena[0, 4 * 576:] = sc.reshape(-1)
    kvm = torch.from_numpy(arena).view(1, 4, 1, 584).cuda()
    got = ops.gather_dequant(kvm, torch.arange(4, dtype=torch.int32, device="cuda"))
    got = got.cpu().view(torch.int16).numpy().view(np.uint16)
    want = O.f32_to_bf16_bits(O.gather_rows("model1", arena, 4, np.arange(4)))
    assert np.array_equal(got, want)


# ---------------------------------------------------------------- golden (reference outputs)
@pytest.mark.parametrize("name", golden_names())
def test_matches_reference_golden(name):
    from deepseek_v4_kernel import sparse_decode_fwd
    g = load_golden(name)
    P = g["page_block"]
    q = torch.from_numpy(g["q_bf16"].view(np.int16)).view(torch.bfloat16).cuda()
    kv = torch.from_numpy(g["kv_pages"]).cuda()
    kv_view = kv.view(kv.shape[0], P, 1, 584)
    idx = torch.from_numpy(g["indices"]).cuda()
    tk = None if g["topk_length"] is None else torch.from_numpy(g["topk_length"]).cuda()
    sink = None if g["attn_sink"] is None else torch.from_numpy(g["attn_sink"]).cuda()
    out, lse, _, _ = sparse_decode_fwd(q, kv_view, idx, tk, sink, None, None, None, None, None,
                                       512, g["sm_scale"])
    assert_matches(out, lse, g["out_f32"], g["lse"])


# ---------------------------------------------------------------- V32 vs oracle
V32_CASES = [
    # b, s_q, h_q, topk, ctx, page, invalid_tail, with_sink
    (1, 1, 16, 128, 4096, 256, 16, True),
    (2, 1, 64, 64, 512, 64, 0, False),
    (2, 1, 64, 2048, 4096, 64, 0, True),
    (2, 1, 128, 256, 1024, 64, 3, True),
    (3, 2, 64, 300, 2048, 256, 7, True),       # s_q = 2, ragged topk
    (1, 1, 32, 1, 64, 64, 0, True),            # topk = 1
    (1, 1, 80, 200, 1000, 64, 0, False),       # h_q not a multiple of 64
]


@pytest.mark.parametrize("case", V32_CASES, ids=lambda c: "b{}s{}h{}k{}".format(*c[:4]))
def test_v32_matches_oracle(case):
    b, s_q, h_q, topk, ctx, page, tail, sink = case
    spec = _kc().BatchSpec(b=b, s_q=s_q, h_q=h_q, topk=topk, ctx=ctx, page_block=page,
                           invalid_tail=tail, with_sink=sink, seed=b * 131 + topk)
    bt = _kc().make_batch(spec)
    out, lse, _, _ = _run(bt)
    ref_out, ref_lse = oracle_for(bt.q, bt.kv, bt.indices, None, bt.attn_sink, bt.sm_scale, "v32")
    assert_matches(out, lse, ref_out, ref_lse)


def test_topk_length_and_zero_length():
    spec = _kc().BatchSpec(b=4, s_q=1, h_q=64, topk=512, ctx=4096, page_block=64, seed=5)
    bt = _kc().make_batch(spec)
    tk = torch.tensor([64, 32, 0, 100000], dtype=torch.int32, device="cuda")
    out, lse, _, _ = _run(bt, topk_length=tk)
    ref_out, ref_lse = oracle_for(bt.q, bt.kv, bt.indices, tk, bt.attn_sink, bt.sm_scale, "v32")
    assert_matches(out, lse, ref_out, ref_lse)


@pytest.mark.parametrize("parts", [1, 3, 7, 148, 300])
def test_split_counts_agree(parts):
    """Any scheduler part count gives the oracle's answer: contiguous plan
    + combine (1 part), row-aligned + combine (3), clusters of 2 (7) and
    8 (148, 300) merged in distributed shared memory."""
    spec = _kc().BatchSpec(b=3, s_q=1, h_q=64, topk=1000, ctx=8192, page_block=64,
                           invalid_tail=5, seed=21)
    bt = _kc().make_batch(spec)
    tk = torch.tensor([1000, 130, 257], dtype=torch.int32, device="cuda")
    out, lse, tsm, ns = _run(bt, topk_length=tk, parts=parts)
    ref_out, ref_lse = oracle_for(bt.q, bt.kv, bt.indices, tk, bt.attn_sink, bt.sm_scale, "v32")
    assert_matches(out, lse, ref_out, ref_lse)
    from deepseek_v4_kernel import ops
    c = ops.plan_cluster_size(_params(bt, tk), parts)
    recs, want_ns = SO.plan(SO.row_tiles(3, 1, 1000, tk.tolist()), parts, c)
    assert tsm.cpu().tolist() == recs
    assert ns.cpu().tolist() == want_ns


@pytest.mark.parametrize("b,s_q,topk,parts", [(2, 1, 64, 148), (2, 1, 256, 74), (32, 1, 2048, 148),
                                              (3, 1, 1000, 7), (5, 3, 900, 148), (200, 1, 512, 148),
                                              (1, 1, 4096, 148), (20, 1, 512, 8), (33, 1, 256, 148)])
def test_scheduler_records_match_oracle(b, s_q, topk, parts):
    """The device scheduler's records equal the restated plan, in both the
    row-aligned (rows <= parts) and the contiguous mode, including row
    counts whose shared-memory tables start at odd offsets, on both sides of
    the single-warp scheduler's 32-row limit."""
    from deepseek_v4_kernel import ops
    spec = _kc().BatchSpec(b=b, s_q=s_q, h_q=64, topk=topk, ctx=8192, page_block=64, seed=3)
    bt = _kc().make_batch(spec)
    out = torch.empty(b, s_q, 64, 512, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(b, 64, s_q, dtype=torch.float32, device="cuda")
    p = ops.build_params(bt.q, bt.kv, bt.indices, None, None, None, None, None, 512, bt.sm_scale, out, lse)
    tsm, ns = ops.get_mla_metadata_tensors(p, torch.device("cuda", 0), parts)
    c = ops.plan_cluster_size(p, parts)
    recs, want_ns = SO.plan(SO.row_tiles(b, s_q, topk, None), parts, c)
    assert ns.cpu().tolist() == want_ns
    assert tsm.cpu().tolist() == recs


def test_extra_kv_sidecar():
    kc = _kc()
    spec = kc.BatchSpec(b=2, s_q=1, h_q=64, topk=256, ctx=2048, page_block=64, seed=8)
    bt = kc.make_batch(spec)
    ex = kc.make_batch(kc.BatchSpec(b=2, s_q=1, h_q=64, topk=192, ctx=512, page_block=64, seed=9))
    etk = torch.tensor([192, 70], dtype=torch.int32, device="cuda")
    extra = (ex.kv, ex.indices, etk)
    out, lse, _, _ = _run(bt, extra=extra, parts=5)
    ref_out, ref_lse = oracle_for(bt.q, bt.kv, bt.indices, None, bt.attn_sink, bt.sm_scale, "v32",
                                  extra=extra)
    assert_matches(out, lse, ref_out, ref_lse)


def test_model1_matches_oracle_multi_split():
    spec = _kc().BatchSpec(b=2, s_q=2, h_q=128, topk=700, ctx=4096, page_block=64, layout="model1",
                           invalid_tail=9, seed=4)
    bt = _kc().make_batch(spec)
    out, lse, _, _ = _run(bt, parts=11)
    ref_out, ref_lse = oracle_for(bt.q, bt.kv, bt.indices, None, bt.attn_sink, bt.sm_scale, "model1")
    assert_matches(out, lse, ref_out, ref_lse)


# ---------------------------------------------------------------- full size (config 1)
def test_config1_full_size_properties():
    """BASELINE config 1 at full size: rows checked against the oracle, and
    size-independent properties (index order and -1 padding invariance)."""
    kc = _kc()
    bt = kc.make_batch(kc.CONFIGS[1])
    out, lse, tsm, ns = _run(bt)
    # eight rows; in the cluster plan every row is split over the 4 ranks of
    # its cluster, so each row checks the cross-rank merge of all 512 dims
    assert_rows_match(out, lse, bt, [(r, 0) for r in (0, 5, 9, 13, 17, 22, 26, 31)])
    # permuting the top-k order changes nothing but summation order
    perm = torch.randperm(bt.indices.shape[-1], device="cuda")
    out2, lse2, _, _ = _run(kc.Batch(bt.q, bt.kv, bt.indices[..., perm].contiguous(), bt.attn_sink,
                                     bt.sm_scale, bt.spec))
    torch.testing.assert_close(out2.float(), out.float(), atol=2e-3, rtol=1e-2)
    torch.testing.assert_close(lse2, lse, atol=1e-4, rtol=1e-4)
    # appending -1 pads adds exactly one exp(0 - lse) term per pad to the LSE
    pad = torch.full((32, 1, 128), -1, dtype=torch.int32, device="cuda")
    idx3 = torch.cat([bt.indices, pad], dim=-1).contiguous()
    _, lse3, _, _ = _run(kc.Batch(bt.q, bt.kv, idx3, None, bt.sm_scale, bt.spec))
    _, lse_ns, _, _ = _run(kc.Batch(bt.q, bt.kv, bt.indices, None, bt.sm_scale, bt.spec))
    want = torch.logaddexp(lse_ns, torch.full_like(lse_ns, math.log(128.0)))
    torch.testing.assert_close(lse3, want, atol=2e-4, rtol=1e-4)


def test_config2_full_size_matches_oracle():
    """BASELINE config 2 exactly (b 8, s_q 2, h_q 128, top-k 2048, 50 %
    overlap between the two draft rows, 393,216-token cache per request):
    every query row against the oracle, both head groups."""
    kc = _kc()
    bt = kc.make_batch(kc.CONFIGS[2])
    out, lse, _, _ = _run(bt)
    assert_rows_match(out, lse, bt, [(b_, s_) for b_ in range(8) for s_ in range(2)])


def test_config4_full_size_sampled_rows():
    """BASELINE config 4 on one GPU (b 256, h_q 128, top-k 2048, 64K
    contexts, an 11 GB cache): the contiguous split plan with the combine
    kernel.  Sixteen rows, including the rows that hold part boundaries of
    the schedule (split rows merged by the combine), against the oracle."""
    from deepseek_v4_kernel import ops
    kc = _kc()
    bt = kc.make_batch(kc.CONFIGS[4])
    out, lse, tsm, ns = _run(bt)
    splits = ns.cpu().numpy()
    split_rows = [r for r in range(256) if splits[r + 1] - splits[r] > 1]
    assert split_rows, "config 4 is expected to split rows across parts"
    pick = sorted(set(split_rows[:6] + split_rows[-4:] + [0, 1, 100, 128, 200, 255]))[:16]
    assert_rows_match(out, lse, bt, [(r, 0) for r in pick])


# ---------------------------------------------------------------- graphs + interface
def test_cuda_graph_replay():
    from deepseek_v4_kernel import ops
    kc = _kc()
    bt = kc.make_batch(kc.BatchSpec(b=4, s_q=1, h_q=64, topk=2048, ctx=32768, page_block=256, seed=2))
    out_ref, lse_ref, tsm, ns = _run(bt)
    out = torch.empty_like(out_ref)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ops.sparse_decode_fwd(bt.q, bt.kv, bt.indices, None, bt.attn_sink, tsm, ns, None, None, None,
                              512, bt.sm_scale, out=out)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        _, lse_g, _, _ = ops.sparse_decode_fwd(bt.q, bt.kv, bt.indices, None, bt.attn_sink, tsm, ns,
                                               None, None, None, 512, bt.sm_scale, out=out)
    out.zero_()
    g.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(out, out_ref, atol=0, rtol=0)
    torch.testing.assert_close(lse_g, lse_ref, atol=0, rtol=0)


def test_flash_mla_interface_schedmeta_reuse():
    import deepseek_v4_kernel as dk_
    kc = _kc()
    bt = kc.make_batch(kc.BatchSpec(b=2, s_q=1, h_q=64, topk=512, ctx=4096, page_block=64, seed=6))
    meta, none = dk_.get_mla_metadata()
    assert none is None and not meta.have_initialized
    o1, l1 = dk_.flash_mla_with_kvcache(bt.q, bt.kv, None, None, 512, meta, is_fp8_kvcache=True,
                                        indices=bt.indices, attn_sink=bt.attn_sink)
    assert meta.have_initialized and meta.config.topk == 512 and meta.tile_scheduler_metadata is not None
    o2, l2 = dk_.flash_mla_with_kvcache(bt.q, bt.kv, None, None, 512, meta, is_fp8_kvcache=True,
                                        indices=bt.indices, attn_sink=bt.attn_sink)
    torch.testing.assert_close(o1, o2, atol=0, rtol=0)
    assert l1.shape == (2, 64, 1)
    ref_out, ref_lse = oracle_for(bt.q, bt.kv, bt.indices, None, bt.attn_sink,
                                  1.0 / math.sqrt(576), "v32")
    assert_matches(o1, l1, ref_out, ref_lse)


def test_patch_wrapper_routes_sparse_to_b200():
    from deepseek_v4_kernel import _patch, interface
    import types
    calls = []
    fake = types.SimpleNamespace(FlashMLASchedMeta=interface.FlashMLASchedMeta)

    def upstream(**kw):
        calls.append(kw)
        return "upstream"

    fake.flash_mla_with_kvcache = upstream
    assert _patch.patch_module(fake)
    kc = _kc()
    bt = kc.make_batch(kc.BatchSpec(b=1, s_q=1, h_q=64, topk=256, ctx=1024, page_block=64, seed=1))
    meta = interface.FlashMLASchedMeta()
    o, l = fake.flash_mla_with_kvcache(bt.q, bt.kv, None, None, 512, meta, is_fp8_kvcache=True,
                                       indices=bt.indices)
    assert not calls and o.shape == (1, 1, 64, 512)
    assert fake.flash_mla_with_kvcache(bt.q, bt.kv, None, None, 512, meta, is_fp8_kvcache=False,
                                       indices=None) == "upstream"
    assert len(calls) == 1


@pytest.mark.parametrize("mode", ["batch", "head"])
def test_partition_shards_match_full_decode(mode):
    """The multi-GPU partition decodes each shard independently (no data-path
    collective); on one GPU the reassembled shards equal the full decode."""
    from deepseek_v4_kernel import partition
    spec = _kc().BatchSpec(b=6, s_q=1, h_q=128, topk=640, ctx=4096, page_block=64, seed=23)
    bt = _kc().make_batch(spec)
    full_out, full_lse, _, _ = _run(bt)
    world = 2
    outs = []
    for rank in range(world):
        if mode == "batch":
            q, idx, _, (lo, hi) = partition.shard_batch(bt.q, bt.indices, None, rank, world)
            shard = _kc().Batch(q=q, kv=bt.kv, indices=idx, attn_sink=bt.attn_sink, sm_scale=bt.sm_scale,
                                spec=spec)
        else:
            q, sink, (lo, hi) = partition.shard_heads(bt.q, bt.attn_sink, rank, world)
            shard = _kc().Batch(q=q, kv=bt.kv, indices=bt.indices, attn_sink=sink, sm_scale=bt.sm_scale,
                                spec=spec)
        o, l, _, _ = _run(shard)
        outs.append((o, l))
    # shards get their own split plans, so only the accumulation order differs
    got = torch.cat([o for o, _ in outs], dim=0 if mode == "batch" else 2)
    got_lse = torch.cat([l for _, l in outs], dim=0 if mode == "batch" else 1)
    torch.testing.assert_close(got.float(), full_out.float(), atol=OUT_ATOL, rtol=OUT_RTOL)
    torch.testing.assert_close(got_lse, full_lse, atol=LSE_ATOL, rtol=LSE_RTOL)


@pytest.mark.parametrize("b,topk", [(1, 2048), (4, 1024), (33, 512), (200, 256)])
def test_cuda_graph_capture_and_replay(b, topk):
    """The whole step (flash_mla_with_kvcache with a reused FlashMLASchedMeta)
    is captured once in a CUDA graph and replayed with new q / indices in the
    same buffers, as SGLang's decode graphs do; each replay matches the
    oracle.  The first call (workspace, scheduler, cluster set-up) runs
    before capture."""
    import deepseek_v4_kernel as dk
    kc = _kc()
    spec = kc.BatchSpec(b=b, s_q=1, h_q=64, topk=topk, ctx=4096, page_block=64, invalid_tail=3, seed=51)
    bt = kc.make_batch(spec)
    q_buf, idx_buf = bt.q.clone(), bt.indices.clone()
    sched, _ = dk.get_mla_metadata()

    def step():
        return dk.flash_mla_with_kvcache(q_buf, bt.kv, None, None, 512, sched, softmax_scale=bt.sm_scale,
                                         is_fp8_kvcache=True, indices=idx_buf, attn_sink=bt.attn_sink)

    step()
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out_g, lse_g = step()
    for seed in (52, 53):
        other = kc.make_batch(kc.BatchSpec(**{**spec.__dict__, "seed": seed}))
        q_buf.copy_(other.q)
        idx_buf.copy_(other.indices)  # same cache geometry, so valid rows of bt.kv
        g.replay()
        torch.cuda.synchronize()
        ref_out, ref_lse = oracle_for(q_buf, bt.kv, idx_buf, None, bt.attn_sink, bt.sm_scale, "v32")
        assert_matches(out_g, lse_g, ref_out, ref_lse)


@pytest.mark.parametrize("layout,b,s_q,h_q,topk,cluster", [
    ("v32", 32, 1, 64, 2048, True),      # config-1 shape: clusters of 4
    ("model1", 32, 1, 64, 1024, True),   # MODEL1 under the cluster plan
    ("v32", 8, 2, 128, 1024, True),      # s_q 2, two head groups, clusters
    ("v32", 5, 1, 96, 700, False),       # h_q not a multiple of 64, clusters off
    ("model1", 3, 2, 16, 333, False),    # small head count, ragged top-k
])
def test_plans_and_layouts_match_oracle(layout, b, s_q, h_q, topk, cluster):
    """Every plan the scheduler can pick (cluster merge or split + combine)
    gives the oracle's answer for both layouts, with a -1 tail, sinks and
    topk_length."""
    from deepseek_v4_kernel import ops
    spec = _kc().BatchSpec(b=b, s_q=s_q, h_q=h_q, topk=topk, ctx=8192, page_block=64, layout=layout,
                           invalid_tail=11, seed=61)
    bt = _kc().make_batch(spec)
    tk = torch.randint(1, topk + 1, (b,), dtype=torch.int32, device="cuda")
    parts = ops.num_sm_parts(torch.device("cuda", 0), h_q)
    c = ops.plan_cluster_size(_params(bt, tk), parts)
    assert (c > 1) == cluster, c
    out, lse, _, _ = _run(bt, topk_length=tk)
    ref_out, ref_lse = oracle_for(bt.q, bt.kv, bt.indices, tk, bt.attn_sink, bt.sm_scale, layout)
    assert_matches(out, lse, ref_out, ref_lse)


def test_extra_kv_sidecar_cluster_plan():
    """The SWA sidecar under the default (cluster) plan: the extra tiles join
    the split of each row."""
    kc = _kc()
    spec = kc.BatchSpec(b=16, s_q=1, h_q=64, topk=1024, ctx=4096, page_block=64, seed=71)
    bt = kc.make_batch(spec)
    ex = kc.make_batch(kc.BatchSpec(b=16, s_q=1, h_q=64, topk=256, ctx=1024, page_block=64, seed=72))
    etk = torch.randint(0, 257, (16,), dtype=torch.int32, device="cuda")
    extra = (ex.kv, ex.indices, etk)
    out, lse, _, _ = _run(bt, extra=extra)
    ref_out, ref_lse = oracle_for(bt.q, bt.kv, bt.indices, None, bt.attn_sink, bt.sm_scale, "v32",
                                  extra=extra)
    assert_matches(out, lse, ref_out, ref_lse)


@pytest.mark.gpu
def test_mma_rate_probe_reports_every_shape():
    """dsv4b_mma_rate_probe (the measurement behind the decode kernel's
    tensor-core roofline) runs each shape's chain and reports its MMA
    count and a positive cycle count per CTA."""
    import torch
    from deepseek_v4_kernel import _lib
    torch.cuda.set_device(0)
    out = torch.zeros(2 * 4, dtype=torch.int64, device="cuda")
    for shape, mmas in ((0, 36), (1, 32), (2, 16), (3, 8), (4, 36), (5, 32)):
        rc = _lib.lib.dsv4b_mma_rate_probe(shape, 4, out.data_ptr(), torch.cuda.current_stream().cuda_stream)
        assert rc == 0, _lib.STATUS.get(rc, rc)
        torch.cuda.synchronize()
        v = out.view(4, 2).cpu()
        assert (v[:, 1] == mmas).all(), v
        assert (v[:, 0] > 0).all(), v
    assert _lib.lib.dsv4b_mma_rate_probe(6, 4, out.data_ptr(), None) == -1


@pytest.mark.gpu
def test_gather_rate_probe_runs_both_mechanisms():
    """dsv4b_gather_rate_probe (the measurement behind the gather ceiling)
    gathers rows with both mechanisms, its bounded waits all complete, and
    it refuses bad arguments."""
    import torch
    from deepseek_v4_kernel import _lib
    torch.cuda.set_device(0)
    kv = torch.randint(0, 255, (4096 * 656,), dtype=torch.uint8, device="cuda")
    rows = torch.randint(0, 4096, (3000,), dtype=torch.int32, device="cuda")
    scratch = torch.zeros(148 * 256 + 4, dtype=torch.int32, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    for mech in (0, 1):
        rc = _lib.lib.dsv4b_gather_rate_probe(mech, kv.data_ptr(), 656, 656, rows.data_ptr(), 3000,
                                              scratch.data_ptr(), scratch.numel() * 4, s)
        assert rc == 0, _lib.STATUS.get(rc, rc)
    torch.cuda.synchronize()
    assert int(scratch[-4].item()) == 0
    assert _lib.lib.dsv4b_gather_rate_probe(2, kv.data_ptr(), 656, 656, rows.data_ptr(), 3000,
                                            scratch.data_ptr(), scratch.numel() * 4, s) == -1
    assert _lib.lib.dsv4b_gather_rate_probe(0, kv.data_ptr(), 656, 650, rows.data_ptr(), 3000,
                                            scratch.data_ptr(), scratch.numel() * 4, s) == -1
