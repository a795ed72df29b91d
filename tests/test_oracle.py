"""CPU: pin the numpy oracle against the reference's own outputs
(golden vectors from tests/reference.py) and against known answers."""
import math

import numpy as np
import pytest

from golden_io import golden_names, load_golden
from oracle import sparse_decode_oracle as O


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_reference_golden(name):
    g = load_golden(name)
    out, lse = O.sparse_decode_reference(
        g["q_f32"], g["kv_pages"], g["indices"], g["topk_length"],
        g["attn_sink"], g["sm_scale"], g["page_block"], layout="model1")
    # both are fp32 paths; differences come only from summation order
    np.testing.assert_allclose(out, g["out_f32"], atol=2e-3, rtol=1e-2)
    ulp = np.abs(out.view(np.uint32).astype(np.int64)
                 - g["out_f32"].view(np.uint32).astype(np.int64))
    assert (ulp <= 1).mean() > 0.99
    np.testing.assert_allclose(lse, g["lse"], atol=1e-5, rtol=1e-5)


def test_e4m3_table_known_values():
    t = O.E4M3_TO_F32
    assert t[0x00] == 0.0 and t[0x38] == 1.0 and t[0x7E] == 448.0
    assert t[0xFE] == -448.0 and t[0x01] == 2.0 ** -9 and np.isnan(t[0x7F])
    assert t[0x08] == 2.0 ** -6 and t[0x40] == 2.0


def test_ue8m0_scale():
    s = O.ue8m0_to_scale(np.array([127, 128, 125, 0, 1, 254, 255], np.uint8))
    assert list(s[:3]) == [1.0, 2.0, 0.25]
    assert s[3] == np.float32(2.0 ** -127) and s[4] == np.float32(2.0 ** -126)
    assert s[5] == np.float32(2.0 ** 127) and np.isinf(s[6])


def test_bf16_rounding_ties_to_even():
    x = np.array([1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, -1.0 - 2 ** -8], np.float32)
    r = O.round_bf16(x)
    assert list(r) == [1.0, 1.0 + 2 ** -6, -1.0]


def _v32_record(fp8_bytes, scales, rope_bits):
    rec = np.zeros(656, np.uint8)
    rec[:512] = fp8_bytes
    rec[512:528] = np.asarray(scales, np.float32).view(np.uint8)
    rec[528:] = np.asarray(rope_bits, np.uint16).view(np.uint8)
    return rec


def test_v32_unpack_known_answer():
    fp8 = np.full(512, 0x38, np.uint8)                  # 1.0 everywhere
    fp8[128:256] = 0x40                                 # 2.0
    fp8[256] = 0xB8                                     # -1.0
    fp8[300] = 0x01                                     # 2**-9 (subnormal)
    scales = [0.5, 3.0, 1.0 / 3.0, 1e-3]
    rope = np.full(64, 0x3F80, np.uint16)               # bf16 1.0
    rope[5] = 0xC000                                    # -2.0
    kv = np.zeros((2, 4, 1, 656), np.uint8)
    kv[1, 2, 0] = _v32_record(fp8, scales, rope)
    row = O.unpack_v32_rows(kv, 4, np.array([1 * 4 + 2]))[0]
    assert row.shape == (576,)
    assert np.all(row[:128] == 0.5) and np.all(row[129:256] == 6.0)
    third = np.float32(1.0) / np.float32(3.0)
    assert row[256] == O.round_bf16(np.array([-third], np.float32))[0]
    assert row[300] == O.round_bf16(np.array([np.float32(2.0 ** -9) * third], np.float32))[0]
    assert row[400] == O.round_bf16(np.array([np.float32(1e-3)], np.float32))[0]
    assert row[512] == 1.0 and row[517] == -2.0


def test_invalid_rows_are_zero_and_give_logit_zero():
    rng = np.random.default_rng(0)
    kv = rng.integers(0, 256, size=(2, 4, 1, 656), dtype=np.uint8)
    kv[..., 512:528] = np.frombuffer(np.full(4, 0.01, np.float32).tobytes(), np.uint8)
    kv = kv & np.where(np.arange(656) < 512, 0x77, 0xFF).astype(np.uint8)  # no NaN bytes
    kv[..., 528:] = 0
    idx = np.array([[[0, -1, 8, 100]]], np.int32)       # 8 tokens total
    k = O.gather_rows("v32", kv, 4, idx[0, 0])
    assert np.all(k[1:] == 0)
    q = np.ones((1, 1, 2, 576), np.float32)
    out, lse = O.sparse_decode_reference(q, kv, idx, None, None, 0.1, 4, layout="v32")
    logit0 = 0.1 * k[0].sum()
    want = np.log(np.exp(logit0) + 3.0)                 # three zero logits
    np.testing.assert_allclose(lse[0, 0], [want, want], rtol=1e-5)


def test_topk_length_clamps_to_one():
    rng = np.random.default_rng(1)
    kv = np.zeros((1, 8, 1, 656), np.uint8)
    kv[..., :512] = rng.integers(0, 0x70, size=(1, 8, 1, 512), dtype=np.uint8)
    kv[..., 512:528] = np.frombuffer(np.full(4, 1.0, np.float32).tobytes(), np.uint8)
    idx = np.array([[[3, 4, 5]]], np.int32)
    q = rng.standard_normal((1, 1, 4, 576)).astype(np.float32)
    o0, l0 = O.sparse_decode_reference(q, kv, idx, np.array([0], np.int32), None,
                                       1 / math.sqrt(576), 8, layout="v32")
    o1, l1 = O.sparse_decode_reference(q, kv, idx[..., :1], None, None,
                                       1 / math.sqrt(576), 8, layout="v32")
    np.testing.assert_array_equal(o0, o1)
    np.testing.assert_allclose(l0, l1, rtol=1e-6)
