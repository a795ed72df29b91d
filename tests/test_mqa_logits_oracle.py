"""CPU checks of the indexer-logits oracle (oracle/mqa_logits_oracle.py)
against the fixtures made by running DeepGEMM's torch statement as vLLM
carries it (tests/golden/make_mqa_logits_golden.py), plus the schedule
rule and the Python layer's argument checks."""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import mqa_logits_oracle as M

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "mqa_logits")
FIXTURES = sorted(os.path.splitext(os.path.basename(p))[0] for p in glob.glob(os.path.join(GOLDEN, "*.npz")))


def load(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    return {k: z[k] for k in z.files}


def test_fixtures_present():
    assert len(FIXTURES) >= 3


@pytest.mark.parametrize("name", FIXTURES)
def test_oracle_matches_deepgemm_torch_statement(name):
    d = load(name)
    got = M.fp8_paged_mqa_logits(d["q"], d["kv"], d["weights"], d["context_lens"], d["block_table"],
                                 int(d["page_block"]), int(d["max_model_len"]))
    want = d["logits"]
    np.testing.assert_array_equal(np.isinf(got), np.isinf(want))
    fin = np.isfinite(want)
    np.testing.assert_allclose(got[fin], want[fin], rtol=1e-4, atol=1e-3)


def test_causal_rule_next_n():
    """next_n = 2: row i sees t <= ctx - 2 + i; row 1 equals a next_n = 1
    call on the same data, row 0 drops the last position."""
    rng = np.random.default_rng(0)
    P, D, H = 64, 128, 64
    kv = rng.integers(0, 0x70, (4, P * (D + 4)), dtype=np.uint8)
    kv[:, P * D:] = np.full((4, P), 0.5, np.float32).view(np.uint8)
    q = rng.integers(0, 0x70, (1, 2, H, D), dtype=np.uint8)
    w = rng.standard_normal((2, H)).astype(np.float32)
    bt = np.array([[2, 0, 3, 1]], np.int32)
    two = M.fp8_paged_mqa_logits(q, kv, w, np.array([200]), bt, P, 256)
    one = M.fp8_paged_mqa_logits(q[:, 1:], kv, w[1:], np.array([200]), bt, P, 256)
    np.testing.assert_array_equal(two[1], one[0])
    assert np.isneginf(two[0, 199]) and np.isfinite(two[0, 198]) and np.isfinite(two[1, 199])


def test_argument_checks_on_host():
    from deepseek_v4_kernel import indexer
    q = torch.zeros(2, 1, 64, 128, dtype=torch.float8_e4m3fn)
    kv = torch.zeros(4, 64, 1, 132, dtype=torch.uint8)
    w = torch.zeros(2, 64)
    ctx = torch.tensor([10, 20], dtype=torch.int32)
    bt = torch.zeros(2, 4, dtype=torch.int32)
    sched = torch.zeros(149, 2, dtype=torch.int32)
    with pytest.raises(RuntimeError):
        indexer.fp8_paged_mqa_logits(q.float(), kv, w, ctx, bt, sched, 64)            # q dtype
    with pytest.raises(RuntimeError):
        indexer.fp8_paged_mqa_logits((q, torch.ones(1)), kv, w, ctx, bt, sched, 64)   # FP4 path
    with pytest.raises(RuntimeError):
        indexer.fp8_paged_mqa_logits(q, kv[..., :130], w, ctx, bt, sched, 64)         # bad page row
    with pytest.raises(RuntimeError):
        indexer.fp8_paged_mqa_logits(q, kv, w[:1], ctx, bt, sched, 64)                # weights shape
    with pytest.raises(RuntimeError):
        indexer.fp8_paged_mqa_logits(q, kv, w, ctx.long(), bt, sched, 64)             # ctx dtype
    with pytest.raises(RuntimeError):
        indexer.get_paged_mqa_logits_metadata(ctx, 48, 148)                           # page size
