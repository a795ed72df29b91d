"""The reference's own SM120 kernel, built for sm_100a, as a second checker
and as the GPU bar to beat.

``oracle/Makefile.ref`` compiles the reference's unmodified
``csrc/sm120/decode/sparse_decode_instantiation.cu`` (with
``sparse_decode_kernel.cuh``) plus a small harness into
``oracle/_ref/libref_sm120.so``.  The reference kernel supports only the
MODEL1 layout with s_q = 1 and no split-KV.  Inputs here stay inside what
it handles: no out-of-range indices (it does no upper-bound check), no
``topk_length`` (its clamp differs from the reference's own oracle).

1. The reference kernel agrees with this repo's CPU oracle (pinning the
   oracle to the reference's real kernel as well as to its Python oracle).
2. This build's kernel agrees with the reference kernel.
3. On the MODEL1 twin of BASELINE config 1 (b 32, h 64, top-k 2048, 128K
   contexts) this build's kernel is faster than the reference kernel on the
   same B200; both times are printed.
"""
import ctypes
import os
import statistics

import numpy as np
import pytest
import torch

from dsv4b_testutil import LSE_ATOL, LSE_RTOL, OUT_ATOL, OUT_RTOL, oracle_for

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_LIB = os.path.join(ROOT, "oracle", "_ref", "libref_sm120.so")


def _ref_lib():
    if not os.path.exists(REF_LIB):
        pytest.skip("oracle/_ref/libref_sm120.so not built (needs the reference checkout)")
    lib = ctypes.CDLL(REF_LIB)
    vp = ctypes.c_void_p
    lib.ref_sm120_sparse_decode.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, vp, vp,
                                            ctypes.c_int, ctypes.c_int, vp, vp, vp, vp, vp]
    return lib


def _ref_run(lib, bt, out, lse):
    b, s_q, h_q, _ = bt.q.shape
    assert s_q == 1
    rc = lib.ref_sm120_sparse_decode(
        b, h_q, bt.indices.shape[-1], bt.sm_scale, bt.q.data_ptr(), bt.kv.data_ptr(), bt.kv.shape[0],
        bt.kv.shape[1], bt.indices.data_ptr(),
        bt.attn_sink.data_ptr() if bt.attn_sink is not None else None, out.data_ptr(), lse.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    assert rc == 0


@pytest.mark.parametrize("h_q,topk", [(64, 256), (128, 2048)])
def test_reference_kernel_vs_oracle_and_ours(h_q, topk):
    from deepseek_v4_kernel import kvcache, ops
    lib = _ref_lib()
    torch.cuda.set_device(0)
    spec = kvcache.BatchSpec(b=3, s_q=1, h_q=h_q, topk=topk, ctx=8192, page_block=64, layout="model1",
                             invalid_tail=9, seed=41)
    bt = kvcache.make_batch(spec)
    out_ref = torch.empty(3, 1, h_q, 512, dtype=torch.bfloat16, device="cuda")
    lse_ref = torch.empty(3, 1, h_q, dtype=torch.float32, device="cuda")
    _ref_run(lib, bt, out_ref, lse_ref)
    torch.cuda.synchronize()
    want_out, want_lse = oracle_for(bt.q, bt.kv, bt.indices, None, bt.attn_sink, bt.sm_scale, "model1")
    np.testing.assert_allclose(out_ref.float().cpu().numpy(), want_out, atol=OUT_ATOL, rtol=OUT_RTOL)
    np.testing.assert_allclose(lse_ref.cpu().numpy(), want_lse, atol=LSE_ATOL, rtol=LSE_RTOL)
    out, lse, _, _ = ops.sparse_decode_fwd(bt.q, bt.kv, bt.indices, None, bt.attn_sink, None, None, None,
                                           None, None, 512, bt.sm_scale)
    torch.testing.assert_close(out.float(), out_ref.float(), atol=OUT_ATOL, rtol=OUT_RTOL)
    torch.testing.assert_close(lse[:, :, 0], lse_ref[:, 0, :], atol=LSE_ATOL, rtol=LSE_RTOL)


def test_faster_than_reference_kernel_config1_model1():
    from deepseek_v4_kernel import kvcache, ops
    lib = _ref_lib()
    torch.cuda.set_device(0)
    spec = kvcache.BatchSpec(b=32, s_q=1, h_q=64, topk=2048, ctx=131072, page_block=256, layout="model1", seed=7)
    bt = kvcache.make_batch(spec)
    out_ref = torch.empty(32, 1, 64, 512, dtype=torch.bfloat16, device="cuda")
    lse_ref = torch.empty(32, 1, 64, dtype=torch.float32, device="cuda")
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    sched, _ = __import__("deepseek_v4_kernel").get_mla_metadata()

    def ours():
        ops.sparse_decode_fwd(bt.q, bt.kv, bt.indices, None, bt.attn_sink, None, None, None, None, None,
                              512, bt.sm_scale)

    def ref():
        _ref_run(lib, bt, out_ref, lse_ref)

    def timed(fn, n=10):
        for _ in range(3):
            flush.zero_()
            fn()
        ts = []
        for _ in range(n):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ts.append(a.elapsed_time(b) * 1e3)
        return statistics.median(ts)

    t_ours, t_ref = timed(ours), timed(ref)
    print(f"\nconfig 1 MODEL1 twin: this build {t_ours:.1f} us/step, reference SM120 kernel on sm_100a "
          f"{t_ref:.1f} us/step ({t_ref / t_ours:.1f}x)")
    assert t_ours < t_ref
