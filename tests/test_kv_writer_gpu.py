"""KV-cache writer on the GPU (dsv4b_kv_cache_write via cache_ops).

Bit-exact against the CPU oracle (oracle/kv_writer_oracle.py) and the
committed fixtures; bit-exact against vLLM's own writers for the same
formats when vLLM is importable (it is part of the image); a write ->
sparse-decode round trip; and, at the benchmark's full size, properties
(idempotence, sampled rows against the oracle).
"""
import glob
import os

import numpy as np
import pytest
import torch

from dsv4b_testutil import LSE_ATOL, LSE_RTOL, OUT_ATOL, OUT_RTOL, oracle_for
from oracle import kv_writer_oracle as KW

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "kv_writer")
FIXTURES = sorted(os.path.splitext(os.path.basename(p))[0] for p in glob.glob(os.path.join(GOLDEN, "*.npz")))
FILL = 0xA5


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _from_bits(a: np.ndarray, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16).to(device)


def _tokens(n, cols, seed, device="cuda", spread=3.0):
    """bf16 rows with per-row magnitudes exp(N(0, spread^2))."""
    g = torch.Generator(device=device).manual_seed(seed)
    mag = torch.exp(torch.randn(n, 1, generator=g, device=device) * spread)
    x = (torch.randn(n, cols, generator=g, device=device) * mag).to(torch.bfloat16)
    x[:3] = 0.0            # all-zero tiles (1e-4 floor)
    if n > 3:
        x[3, 7] = 448.0    # amax / 448 an exact power of two
    return x


def _slots(n, cache_tokens, seed, dtype=torch.int64):
    g = torch.Generator().manual_seed(seed)
    s = torch.randperm(cache_tokens, generator=g)[:n].to(dtype)
    s[torch.randperm(n, generator=g)[: n // 20]] = -1
    return s.cuda()


@pytest.mark.parametrize("slot_dtype", [torch.int64, torch.int32])
@pytest.mark.parametrize("name", FIXTURES)
def test_fixture_bytes(name, slot_dtype):
    from deepseek_v4_kernel import cache_ops
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    page = int(z["page_block"])
    want = z["arena_after"]
    arena = torch.full(want.shape, FILL, dtype=torch.uint8, device="cuda")
    nope, rope = _from_bits(z["nope"]), _from_bits(z["rope"])
    slots = torch.from_numpy(z["slots"]).to(slot_dtype).cuda()
    if str(z["layout"]) == "model1":
        cache_ops.quantize_and_insert_k_cache(torch.cat([nope, rope], 1), arena, slots, block_size=page)
    else:
        cache_ops.concat_and_cache_mla(nope, rope, arena.view(arena.shape[0], page, 656), slots)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(arena.cpu().numpy(), want)


@pytest.mark.parametrize("layout", ["v32", "model1"])
@pytest.mark.parametrize("row_pad", [0, 16])
def test_random_strided_inputs_vs_oracle(layout, row_pad):
    """Inputs are column slices of a wider buffer; V32 records may sit at a
    padded row stride; MODEL1 pages at a padded page stride."""
    from deepseek_v4_kernel import _lib, cache_ops
    n, page, nb = 20000, 256, 100
    base = _tokens(n, 640, seed=5 + row_pad)
    ncol = 512 if layout == "v32" else 448
    nope, rope = base[:, :ncol], base[:, 576:640]
    slots = _slots(n, nb * page, seed=6)
    if layout == "v32":
        rec = 656 + row_pad
        cache = torch.full((nb, page, 1, rec), FILL, dtype=torch.uint8, device="cuda")
        view = cache[..., :656]
        cache_ops.kv_cache_write(_lib.LAYOUT_V32, nope, rope, slots, view)
        arena = np.full((nb, page * rec), FILL, np.uint8)
        KW.kv_cache_write("v32", arena, page, _bits(nope), _bits(rope), slots.cpu().numpy(), stride_row=rec)
    else:
        stride = page * 584 + row_pad * 64
        cache = torch.full((nb, stride), FILL, dtype=torch.uint8, device="cuda")
        cache_ops.kv_cache_write(_lib.LAYOUT_MODEL1, nope, rope, slots, cache, block_size=page)
        arena = np.full((nb, stride), FILL, np.uint8)
        KW.kv_cache_write("model1", arena, page, _bits(nope), _bits(rope), slots.cpu().numpy())
    torch.cuda.synchronize()
    got = cache.cpu().numpy().reshape(nb, -1)
    bad = np.count_nonzero(got != arena)
    assert bad == 0, f"{bad} bytes differ"


def test_cuda_graph_capture_and_status():
    """The writer captures in a CUDA graph (no host sync, no allocation);
    replaying writes the same bytes; the status word stays clean."""
    from deepseek_v4_kernel import cache_ops
    n, page, nb = 1000, 64, 40
    k = _tokens(n, 512, 61)
    slots = _slots(n, nb * page, 62)
    eager = torch.full((nb, page * 584), FILL, dtype=torch.uint8, device="cuda")
    cache_ops.quantize_and_insert_k_cache(k, eager, slots, block_size=page)
    graphed = torch.full_like(eager, FILL)
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        cache_ops.quantize_and_insert_k_cache(k, graphed, slots, block_size=page)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    assert bool((graphed == FILL).all())          # capture ran nothing
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(graphed, eager)
    assert cache_ops.kv_cache_write_status() == 0


@pytest.mark.parametrize("n", [1, 31, 32, 33, 148 * 32 + 5])
def test_chunk_edges(n):
    """Token counts around the 32-token chunk and the one-CTA-per-SM grid."""
    from deepseek_v4_kernel import _lib, cache_ops
    page, nb = 64, 200
    nope, rope = _tokens(n, 512, 70 + n % 7), _tokens(n, 64, 71)
    slots = _slots(n, nb * page, 72) if n > 20 else torch.arange(n, device="cuda") * 3
    cache = torch.full((nb, page, 656), FILL, dtype=torch.uint8, device="cuda")
    cache_ops.kv_cache_write(_lib.LAYOUT_V32, nope, rope, slots, cache)
    arena = np.full((nb, page * 656), FILL, np.uint8)
    KW.kv_cache_write("v32", arena, page, _bits(nope), _bits(rope), slots.cpu().numpy())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(cache.cpu().numpy().reshape(nb, -1), arena)


def test_quotient_selftest():
    """The V32 writer's quotient (reciprocal + FMA refinement) against the
    hardware division: every finite bf16 numerator x 20,000 scales, e4m3
    bytes and fp32 bits."""
    import ctypes
    from deepseek_v4_kernel import _lib
    g = torch.Generator(device="cuda").manual_seed(81)
    amax = torch.exp(torch.empty(16000, device="cuda").uniform_(-80.0, 40.0, generator=g))
    amax = amax.to(torch.bfloat16).float()                       # the writer's amax is a bf16 value
    edge = torch.tensor([1e-4, 448.0, 1.0, 3.0e38, 2.0 ** -20, 7.0, 0.875, 0.0, 1e-30, 1e-39, 2.0 ** -52,
                         2.0 ** -51 * 1.5], device="cuda")
    rnd = torch.exp(torch.empty(4000 - edge.numel(), device="cuda").uniform_(-30.0, 30.0, generator=g))
    f448 = lambda t: torch.clamp(t / torch.full_like(t, 448.0), min=1.17549435e-38)  # the V32 scale rule
    scales = torch.cat([f448(amax), f448(edge), rnd]).contiguous()
    mism = torch.zeros(2, dtype=torch.int64, device="cuda")
    rc = _lib.lib.dsv4b_kv_write_selftest(scales.data_ptr(), scales.numel(), mism.data_ptr(),
                                          torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert mism.tolist() == [0, 0]


def test_empty_and_all_skipped():
    from deepseek_v4_kernel import cache_ops
    cache = torch.full((2, 64 * 584), FILL, dtype=torch.uint8, device="cuda")
    k = _tokens(8, 512, 1)
    cache_ops.quantize_and_insert_k_cache(k[:0], cache, torch.empty(0, dtype=torch.int64, device="cuda"))
    cache_ops.quantize_and_insert_k_cache(k, cache, torch.tensor([-1, -5, 128, 10**6] * 2, device="cuda"))
    torch.cuda.synchronize()
    assert bool((cache == FILL).all())


@pytest.mark.parametrize("layout", ["v32", "model1"])
def test_write_then_decode(layout):
    """A cache written by the writer decodes like the oracle says."""
    from deepseek_v4_kernel import _lib, cache_ops, ops
    b, h_q, topk, page, nb = 4, 64, 512, 64, 64
    toks = nb * page
    ncol, d_qk = (512, 576) if layout == "v32" else (448, 512)
    # unit-scale tokens, like real latents (a row spread of e^(+-9) makes
    # softmax degenerate and says nothing about the cache bytes)
    nope, rope = _tokens(toks, ncol, 21, spread=0.0), _tokens(toks, 64, 22, spread=0.0)
    slots = torch.randperm(toks, generator=torch.Generator().manual_seed(3)).cuda()
    if layout == "v32":
        kv = torch.zeros(nb, page, 1, 656, dtype=torch.uint8, device="cuda")
        cache_ops.kv_cache_write(_lib.LAYOUT_V32, nope, rope, slots, kv)
    else:
        arena = torch.zeros(nb, page * 584, dtype=torch.uint8, device="cuda")
        cache_ops.kv_cache_write(_lib.LAYOUT_MODEL1, nope, rope, slots, arena, block_size=page)
        kv = arena.view(nb, page, 1, 584)
    g = torch.Generator(device="cuda").manual_seed(4)
    q = torch.randn(b, 1, h_q, d_qk, generator=g, device="cuda").to(torch.bfloat16)
    idx = torch.stack([torch.randperm(toks, device="cuda")[:topk] for _ in range(b)]).view(b, 1, topk).int()
    sink = torch.randn(h_q, device="cuda")
    scale = d_qk ** -0.5
    out, lse, _, _ = ops.sparse_decode_fwd(q, kv, idx, None, sink, None, None, None, None, None, 512, scale)
    want_out, want_lse = oracle_for(q, kv, idx, None, sink, scale, layout)
    np.testing.assert_allclose(out.float().cpu().numpy(), want_out, atol=OUT_ATOL, rtol=OUT_RTOL)
    np.testing.assert_allclose(lse.cpu().numpy(), np.transpose(want_lse, (0, 2, 1)), atol=LSE_ATOL, rtol=LSE_RTOL)


def test_model1_matches_vllm_writer():
    """Byte for byte against vLLM 0.22's quantize_and_insert_k_cache
    (Triton; vllm/models/deepseek_v4/common/ops/cache_utils.py)."""
    try:
        from vllm.models.deepseek_v4.common.ops.cache_utils import quantize_and_insert_k_cache as vllm_write
    except Exception as e:  # pragma: no cover - depends on the image
        pytest.skip(f"vLLM writer not importable: {e}")
    from deepseek_v4_kernel import cache_ops
    n, page, nb = 6000, 64, 120
    stride = 65 * 576                       # vLLM pads a 64-token page to a multiple of 576 B
    k = _tokens(n, 512, 31)
    slots = _slots(n, nb * page, 32)
    a = torch.full((nb, stride), FILL, dtype=torch.uint8, device="cuda")
    b = a.clone()
    vllm_write(k, a, slots, block_size=page, is_ue8m0=True)
    cache_ops.quantize_and_insert_k_cache(k, b, slots, block_size=page)
    torch.cuda.synchronize()
    diff = (a != b)
    assert int(diff.sum()) == 0, f"{int(diff.sum())} bytes differ from vLLM's writer"


def test_v32_matches_vllm_concat_and_cache_mla():
    """Byte for byte against vLLM's concat_and_cache_mla(kv_cache_dtype=
    "fp8_ds_mla"), all-zero tiles and tiles of tiny values included."""
    try:
        from vllm import _custom_ops as vops
        op = vops.concat_and_cache_mla
    except Exception as e:  # pragma: no cover
        pytest.skip(f"vLLM concat_and_cache_mla not importable: {e}")
    from deepseek_v4_kernel import cache_ops
    n, page, nb = 6000, 64, 120
    kv_c, k_pe = _tokens(n, 512, 41, spread=4.0), _tokens(n, 64, 42)
    kv_c[10, :128] = 1e-30                  # tiny tiles: scale far below 2^-60
    kv_c[11, 128:256] = (torch.randn(128, device="cuda") * 1e-39).to(torch.bfloat16)   # subnormal values
    slots = _slots(n, nb * page, 43)
    a = torch.full((nb, page, 656), FILL, dtype=torch.uint8, device="cuda")
    b = a.clone()
    op(kv_c, k_pe, a, slots, "fp8_ds_mla", torch.ones(1, device="cuda"))
    cache_ops.concat_and_cache_mla(kv_c, k_pe, b, slots)
    torch.cuda.synchronize()
    diff = (a != b)
    nbad = int(diff.sum())
    if nbad:
        where = diff.view(-1, 656).any(0).nonzero().flatten().tolist()
        pytest.fail(f"{nbad} bytes differ from vLLM's fp8_ds_mla writer at record offsets "
                    f"{where[:8]}{'...' if len(where) > 8 else ''}")


def test_synthetic_generator_matches_writer():
    """The package's synthetic-cache quantiser (kvcache.quantize_v32, run
    on the GPU) and the CUDA writer produce the same records."""
    from deepseek_v4_kernel import _lib, cache_ops, kvcache
    n = 3000
    lat, rope = _tokens(n, 512, 91), _tokens(n, 64, 92)
    want = kvcache.quantize_v32(lat, rope)
    cache = torch.zeros(1, n, 656, dtype=torch.uint8, device="cuda")
    cache_ops.kv_cache_write(_lib.LAYOUT_V32, lat, rope, torch.arange(n, device="cuda"), cache)
    torch.cuda.synchronize()
    assert torch.equal(cache[0], want)


def test_full_size_properties():
    """BASELINE config 1's cache (131,072-token context x 32 requests, V32,
    2.75 GB): write 131,072 tokens at random slots.  Writing twice gives the
    same bytes; 4,096 sampled rows equal the oracle's quantisation."""
    from deepseek_v4_kernel import _lib, cache_ops
    page, nb, n = 256, 16384, 131072
    cache = torch.zeros(nb, page, 1, 656, dtype=torch.uint8, device="cuda")
    nope, rope = _tokens(n, 512, 51), _tokens(n, 64, 52)
    slots = torch.randperm(nb * page, device="cuda")[:n]
    cache_ops.kv_cache_write(_lib.LAYOUT_V32, nope, rope, slots, cache)
    sums1 = cache.view(torch.int64).view(nb, -1).sum(1)   # wrapping word sums per page
    cache_ops.kv_cache_write(_lib.LAYOUT_V32, nope, rope, slots, cache)
    sums2 = cache.view(torch.int64).view(nb, -1).sum(1)
    assert torch.equal(sums1, sums2)
    pick = torch.randperm(n, generator=torch.Generator().manual_seed(9))[:4096].cuda()
    s = slots[pick]
    got = cache.view(-1, 656)[s].cpu().numpy()
    want = KW.quantize_v32_rows(_bits(nope[pick]), _bits(rope[pick]))
    np.testing.assert_array_equal(got, want)
