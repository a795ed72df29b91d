"""CPU: the sparse-prefill oracle (oracle/sparse_prefill_oracle.py) against
the golden vectors of the library kernel it restates (vLLM 0.22's FlashMLA
flash_mla_sparse_fwd, run on a B200 by tests/golden/make_prefill_golden.py):
outputs, max_logits and lse, including the tokens with no valid position
(lse +inf, max -inf, output 0), -1 / out-of-range indices, topk_length and
an attention sink with +-inf entries."""
import glob
import os

import numpy as np
import pytest

from oracle import sparse_prefill_oracle as SP

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "prefill")
FIXTURES = sorted(os.path.splitext(os.path.basename(p))[0] for p in glob.glob(os.path.join(GOLDEN, "*.npz")))


def bf16(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def test_fixtures_present():
    assert len(FIXTURES) >= 3


@pytest.mark.parametrize("name", FIXTURES)
def test_oracle_matches_library_golden(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    tl = z["topk_length"] if z["topk_length"].size else None
    sink = z["attn_sink"] if z["attn_sink"].size else None
    out, mx, lse = SP.sparse_prefill_reference(bf16(z["q"]), bf16(z["kv"]), z["indices"], float(z["sm_scale"]),
                                               tl, sink)
    np.testing.assert_allclose(out, bf16(z["out"]), atol=1e-2, rtol=1e-2)
    np.testing.assert_allclose(mx, z["max_logits"], atol=1e-4, rtol=1e-5)
    np.testing.assert_allclose(lse, z["lse"], atol=1e-4, rtol=1e-5)
    # the conventions for a token with no valid position are the library's
    empty = ~np.isfinite(z["lse"])
    if empty.any():
        assert np.all(z["lse"][empty] == np.inf) and np.all(z["max_logits"][empty] == -np.inf)
        assert np.all(bf16(z["out"])[empty.any(axis=1)] == 0)


def test_oracle_edge_cases():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((3, 4, 576))
    kv = rng.standard_normal((50, 576))
    idx = rng.integers(0, 50, (3, 16))
    idx[1] = -1
    out, mx, lse = SP.sparse_prefill_reference(q, kv, idx, 0.05, topk_length=np.array([16, 16, 0]))
    assert np.all(lse[1] == np.inf) and np.all(lse[2] == np.inf) and np.all(mx[1:] == -np.inf)
    assert np.all(out[1:] == 0)
    # one valid position: softmax weight 1
    idx2 = np.full((1, 8), -1)
    idx2[0, 5] = 7
    out, mx, lse = SP.sparse_prefill_reference(q[:1], kv, idx2, 0.05)
    np.testing.assert_allclose(out[0], np.broadcast_to(kv[7, :512], (4, 512)))
    np.testing.assert_allclose(lse[0], mx[0])
