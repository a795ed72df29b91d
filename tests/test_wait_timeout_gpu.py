"""GPU test of the decode kernel's failure path: a bounded mbarrier wait
that runs out of time.

Every mbarrier wait of the decode kernel gives up after a time limit
(4e9 SM cycles, about 2 s).  The CTA then raises its abort flag, every role
leaves its loop (the softmax threads all together, through a vote on their
named barrier), the MMA issuer waits for the tensor-core work it issued,
TMEM is freed and the workspace status word gets bit 0 (kErrWaitTimeout).
The kernel returns normally, so the CUDA context stays usable.

The test makes a wait run out without any fault, through the test hook
dsv4b_set_test_stall: one producer thread per CTA withholds its
first arrival on the Q barrier (a barrier nothing else completes), so the
MMA issuer's first wait gives up and the CTA aborts.  It checks the status
word, checks that DSV4B_CHECK_STATUS mode raises DSV4B_ERR_KERNEL_TIMEOUT,
clears the hook, and checks that the next call on the same context
matches the oracle and leaves the status word clear.  Both decode plans
are covered: split partials + combine kernel (b = 4) and the
thread-block-cluster merge (b = 32).  Each stalled call takes about the
wait limit (2-4 s).
"""
import pytest
import torch

from dsv4b_testutil import assert_matches, oracle_for

pytestmark = pytest.mark.gpu


def _run(bt):
    from deepseek_v4_kernel import ops
    out, lse, _, _ = ops.sparse_decode_fwd(bt.q, bt.kv, bt.indices, None, bt.attn_sink, None, None,
                                           None, None, None, 512, bt.sm_scale)
    torch.cuda.synchronize()
    return out, lse


@pytest.mark.parametrize("b", [4, 32])
def test_wait_timeout_sets_status_then_recovers(b, monkeypatch):
    from deepseek_v4_kernel import _lib, kvcache, ops
    torch.cuda.set_device(0)
    lib = _lib.lib
    bt = kvcache.make_batch(kvcache.BatchSpec(b=b, s_q=1, h_q=64, topk=2048, ctx=4096,
                                              page_block=64, seed=71 + b))
    _run(bt)  # module loaded, workspace sized, status clear
    assert ops.read_kernel_status() == 0
    try:
        assert lib.dsv4b_set_test_stall(_lib.STALL_DECODE) == 0
        _run(bt)
        assert ops.read_kernel_status() & 1, "the withheld arrival did not make a wait run out"
        # DSV4B_CHECK_STATUS mode turns the status into an exception
        monkeypatch.setattr(ops, "CHECK_STATUS", True)
        with pytest.raises(_lib.DSV4BError) as ei:
            _run(bt)
        assert ei.value.status == -6
        monkeypatch.setattr(ops, "CHECK_STATUS", False)
    finally:
        assert lib.dsv4b_set_test_stall(0) == 0
    ops.read_kernel_status()  # clear whatever the aborted calls left
    out, lse = _run(bt)
    assert ops.read_kernel_status() == 0
    ref_out, ref_lse = oracle_for(bt.q, bt.kv, bt.indices, None, bt.attn_sink, bt.sm_scale, "v32")
    assert_matches(out, lse, ref_out, ref_lse)


def test_kv_writer_wait_timeout_then_recovers():
    """KV-cache writer: the producer skips its first chunk's copies, the
    consumers' first wait runs out, the writer status word gets bit 0; after
    the hook is cleared the same write produces the same bytes as before."""
    from deepseek_v4_kernel import _lib, cache_ops
    torch.cuda.set_device(0)
    lib = _lib.lib
    n, page, nb = 4096, 64, 80
    g = torch.Generator(device="cuda").manual_seed(5)
    nope = torch.randn(n, 512, generator=g, device="cuda").to(torch.bfloat16)
    rope = torch.randn(n, 64, generator=g, device="cuda").to(torch.bfloat16)
    slots = torch.randperm(nb * page, device="cuda")[:n].to(torch.int64)

    def write():
        cache = torch.zeros(nb, page, 656, dtype=torch.uint8, device="cuda")
        cache_ops.concat_and_cache_mla(nope, rope, cache, slots)
        torch.cuda.synchronize()
        return cache

    want = write()
    assert cache_ops.kv_cache_write_status() == 0
    try:
        assert lib.dsv4b_set_test_stall(_lib.STALL_KV_WRITE) == 0
        write()
        assert cache_ops.kv_cache_write_status() & 1, "the withheld chunk did not make a wait run out"
    finally:
        assert lib.dsv4b_set_test_stall(0) == 0
    cache_ops.kv_cache_write_status()
    assert torch.equal(write(), want)
    assert cache_ops.kv_cache_write_status() == 0


def test_mqa_logits_wait_timeout_then_recovers():
    """Indexer logits: the page-id warp withholds its first batch, the
    producer's first wait runs out, the indexer status word gets bit 0;
    after the hook is cleared the next call matches the oracle."""
    from deepseek_v4_kernel import _lib, indexer
    from test_mqa_logits_gpu import assert_logits_close, make_case, run_gpu, run_oracle
    torch.cuda.set_device(0)
    lib = _lib.lib
    case = make_case(4, 1, 64, 64, [5000, 777, 12000, 64], seed=9)
    run_gpu(*case, max_model_len=12288)
    assert indexer.mqa_logits_status() == 0
    try:
        assert lib.dsv4b_set_test_stall(_lib.STALL_MQA_LOGITS) == 0
        run_gpu(*case, max_model_len=12288)
        assert indexer.mqa_logits_status() & 1, "the withheld page-id batch did not make a wait run out"
    finally:
        assert lib.dsv4b_set_test_stall(0) == 0
    indexer.mqa_logits_status()
    got, _ = run_gpu(*case, max_model_len=12288)
    assert indexer.mqa_logits_status() == 0
    assert_logits_close(got, run_oracle(*case, max_model_len=12288))


def test_set_test_stall_rejects_unknown_bits():
    from deepseek_v4_kernel import _lib
    assert _lib.lib.dsv4b_set_test_stall(8) == -1
    assert _lib.lib.dsv4b_set_test_stall(0) == 0
