"""CPU checks of the KV-cache writer oracle (oracle/kv_writer_oracle.py).

* its e4m3 encoder against torch's float8_e4m3fn cast (every finite bf16
  value, random fp32, every e4m3 code round-tripped);
* the committed fixtures (tests/golden/kv_writer/): the oracle reproduces
  their bytes, and for MODEL1 the reference's own unpack of those bytes
  (stored in the fixture) equals the decode oracle's unpack and the input
  tokens within the e4m3 rounding bound -- the format pin;
* the oracle agrees with the package's torch quantisers that build the
  synthetic caches (deepseek_v4_kernel/kvcache.py);
* the Python writer's argument checks (no GPU needed to reach them).
"""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import kv_writer_oracle as KW
from oracle import sparse_decode_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "kv_writer")
FIXTURES = sorted(os.path.splitext(os.path.basename(p))[0] for p in glob.glob(os.path.join(GOLDEN, "*.npz")))
FILL = 0xA5


def load_fixture(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    return {k: z[k] for k in z.files}


def test_fixtures_present():
    assert {"model1_p64", "model1_p256", "v32_p64"} <= set(FIXTURES)


def test_e4m3_encoder_matches_torch_on_every_bf16():
    u = np.arange(1 << 16, dtype=np.uint32)
    f = (u << 16).view(np.float32)
    f = np.clip(f[np.isfinite(f)], -448, 448).astype(np.float32)
    want = torch.from_numpy(f).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(KW.f32_to_e4m3(f), want)


def test_e4m3_encoder_matches_torch_random_fp32():
    rng = np.random.default_rng(3)
    g = (rng.standard_normal(500_000) * np.exp(rng.uniform(-25, 7, 500_000))).astype(np.float32)
    g = np.clip(g, -448, 448)
    want = torch.from_numpy(g).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(KW.f32_to_e4m3(g), want)


def test_e4m3_encoder_round_trips_every_code():
    codes = np.array([c for c in range(256) if c not in (0x7F, 0xFF)], np.uint8)
    vals = O.E4M3_TO_F32[codes]
    got = KW.f32_to_e4m3(vals)
    # +0 and -0 are distinct codes and must stay distinct
    np.testing.assert_array_equal(got, codes)


@pytest.mark.parametrize("name", FIXTURES)
def test_oracle_reproduces_fixture_bytes(name):
    d = load_fixture(name)
    layout = str(d["layout"])
    arena = np.full_like(d["arena_after"], FILL)
    KW.kv_cache_write(layout, arena, int(d["page_block"]), d["nope"], d["rope"], d["slots"])
    np.testing.assert_array_equal(arena, d["arena_after"])


@pytest.mark.parametrize("name", [n for n in FIXTURES if n.startswith("model1")])
def test_reference_unpack_of_written_pages(name):
    """The reference's unpack (tests/reference.py:61-79, run by the fixture
    generator) reads the written tokens back as the decode oracle does, and
    within e4m3 rounding of the bf16 inputs."""
    d = load_fixture(name)
    page = int(d["page_block"])
    toks = d["ref_dequant_tokens"]
    slots = d["slots"][toks]
    ref = O.bf16_bits_to_f32(d["ref_dequant"])
    ours = O.unpack_model1_rows(d["arena_after"], page, slots)
    np.testing.assert_array_equal(ref.view(np.uint32), ours.view(np.uint32))
    x = KW.bf16_bits_to_f32(np.concatenate([d["nope"][toks], d["rope"][toks]], axis=1))
    np.testing.assert_array_equal(ref[:, 448:], x[:, 448:])          # RoPE copied exactly
    nope, deq = x[:, :448].reshape(-1, 7, 64), ref[:, :448].reshape(-1, 7, 64)
    amax = np.maximum(np.abs(nope).max(-1, keepdims=True), 1e-4)
    scale = 2.0 ** np.ceil(np.log2(amax / 448.0))
    # e4m3 half-ulp (1/16 relative; 2^-10 * scale in the subnormal range)
    # plus the bf16 rounding of the dequantised value
    bound = np.abs(nope) / 16 + scale * 2.0 ** -10 + np.abs(nope) * 2.0 ** -8 + 1e-45
    assert np.all(np.abs(deq - nope) <= bound)


@pytest.mark.parametrize("name", FIXTURES)
def test_fixture_untouched_bytes_and_skipped_slots(name):
    d = load_fixture(name)
    page = int(d["page_block"])
    arena = d["arena_after"]
    nb = arena.shape[0]
    written = {int(s) for s in d["slots"] if 0 <= s < nb * page}
    assert len(written) < len(d["slots"])                 # the fixture has skipped slots
    untouched = [t for t in range(nb * page) if t not in written]
    rec = 656 if str(d["layout"]) == "v32" else 576
    for t in untouched[:50]:
        p, o = divmod(t, page)
        assert np.all(arena[p, o * rec:(o + 1) * rec] == FILL)


def _bf16_tokens(n, cols, seed):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(n, cols, generator=g) * torch.exp(torch.randn(n, 1, generator=g) * 3)).to(torch.bfloat16)
    return x


def test_oracle_matches_synthetic_cache_quantisers():
    from deepseek_v4_kernel import kvcache
    lat, rope = _bf16_tokens(96, 512, 1), _bf16_tokens(96, 64, 2)
    want = kvcache.quantize_v32(lat, rope).numpy()
    got = KW.quantize_v32_rows(lat.view(torch.int16).numpy().view(np.uint16),
                               rope.view(torch.int16).numpy().view(np.uint16))
    np.testing.assert_array_equal(got, want)
    nope, rope = _bf16_tokens(128, 448, 3), _bf16_tokens(128, 64, 4)
    pages = kvcache.quantize_model1_pages(nope, rope, 64).numpy()
    arena = np.zeros_like(pages)
    KW.kv_cache_write("model1", arena, 64, nope.view(torch.int16).numpy().view(np.uint16),
                      rope.view(torch.int16).numpy().view(np.uint16), np.arange(128))
    np.testing.assert_array_equal(arena, pages)


def test_writer_argument_checks_on_host():
    from deepseek_v4_kernel import cache_ops
    k = torch.zeros(4, 512, dtype=torch.bfloat16)
    cache = torch.zeros(2, 64 * 584, dtype=torch.uint8)
    slots = torch.arange(4)
    with pytest.raises(RuntimeError):
        cache_ops.quantize_and_insert_k_cache(k.float(), cache, slots)      # not bf16
    with pytest.raises(RuntimeError):
        cache_ops.quantize_and_insert_k_cache(k[:, :448], cache, slots)     # wrong width
    with pytest.raises(RuntimeError):
        cache_ops.quantize_and_insert_k_cache(k, cache, slots.float())      # slot dtype
    with pytest.raises(RuntimeError):
        cache_ops.quantize_and_insert_k_cache(k, cache, slots, is_ue8m0=False)
    with pytest.raises(RuntimeError):
        cache_ops.quantize_and_insert_k_cache(k, cache, slots)              # CPU tensors
    with pytest.raises(RuntimeError):
        cache_ops.concat_and_cache_mla(k, k[:, :64], torch.zeros(2, 64, 656, dtype=torch.uint8), slots,
                                       kv_cache_dtype="auto")
