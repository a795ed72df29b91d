"""GPU test of dsv4b_sparse_decode_noalloc, the entry point that allocates
nothing.

Some callers cannot allocate device memory when they run a decode step: a
serving engine that has already given all free HBM to its KV-cache pool, or
a C / FFI caller with no caching allocator that must not call cudaMalloc
mid-step.  For them the library keeps a fixed 32 MiB scratch per GPU and
this entry point uses it in place of a caller workspace.  The test calls it
through the C ABI twice in a row (on two different batches, so stale
scratch contents from the first call cannot leak into the second) and
checks each result against the workspace entry point dsv4b_sparse_decode
on the same inputs, within the tolerances the other GPU tests use, that
the free device memory does not change across a repeated call, and that the
noalloc status word (read with dsv4b_read_kernel_status(NULL, 0, ...)) is
clear after each call.  It also checks that an oversized request is
refused before any launch.

The file name makes pytest collect it last, so a run stopped by a failure
here has already run every other test; it also passes alone in a fresh
process.
"""
import ctypes

import pytest
import torch

from dsv4b_testutil import LSE_ATOL, LSE_RTOL, OUT_ATOL, OUT_RTOL

pytestmark = pytest.mark.gpu


def _both_paths(bt):
    from deepseek_v4_kernel import _lib, ops
    lib = _lib.lib
    q = bt.q
    b, s_q, h_q, _ = q.shape
    dev = q.device
    outs = {}
    for name in ("workspace", "noalloc"):
        out = torch.full((b, s_q, h_q, 512), float("nan"), dtype=torch.bfloat16, device=dev)
        lse = torch.full((b, h_q, s_q), float("nan"), dtype=torch.float32, device=dev)
        p = ops.build_params(q, bt.kv, bt.indices, None, bt.attn_sink, None, None, None, 512,
                             bt.sm_scale, out, lse)
        tsm, ns = ops.get_mla_metadata_tensors(p, dev)
        parts = tsm.size(0)
        stream = torch.cuda.current_stream(dev).cuda_stream
        if name == "workspace":
            nbytes = lib.dsv4b_workspace_bytes(b, s_q, h_q, parts)
            ws = ops.workspace(dev, nbytes)
            rc = lib.dsv4b_sparse_decode(ctypes.byref(p), tsm.data_ptr(), ns.data_ptr(), parts,
                                         ws.data_ptr(), ws.numel(), stream)
        else:
            # Twice: the first call of a process may still load code lazily
            # (the documented reason to make it before sizing a KV pool);
            # the second must leave the free device memory unchanged.
            for call in range(2):
                torch.cuda.synchronize()
                free0 = torch.cuda.mem_get_info(dev)[0]
                rc = lib.dsv4b_sparse_decode_noalloc(ctypes.byref(p), tsm.data_ptr(), ns.data_ptr(),
                                                     parts, stream)
                torch.cuda.synchronize()
                free1 = torch.cuda.mem_get_info(dev)[0]
                if call == 1:
                    assert free1 == free0, f"a repeated noalloc call changed free memory by {free0 - free1} B"
                flags = ctypes.c_int(-1)
                assert lib.dsv4b_read_kernel_status(None, 0, ctypes.byref(flags), stream) == 0
                assert flags.value == 0, "a wait of the noalloc call timed out"
        assert rc == 0, _lib.STATUS.get(rc, rc)
        torch.cuda.synchronize()
        outs[name] = (out, lse)
    return outs


def test_noalloc_matches_workspace_entry_point_twice():
    from deepseek_v4_kernel import kvcache
    torch.cuda.set_device(0)
    # different batches, each split over several scheduler parts
    specs = [
        kvcache.BatchSpec(b=4, s_q=1, h_q=64, topk=2048, ctx=32768, page_block=256, seed=31),
        kvcache.BatchSpec(b=3, s_q=2, h_q=128, topk=1000, ctx=8192, page_block=64,
                          invalid_tail=9, seed=32),
        # 32 rows: the rows are merged inside thread-block clusters
        kvcache.BatchSpec(b=32, s_q=1, h_q=64, topk=2048, ctx=8192, page_block=64, seed=33),
    ]
    for spec in specs:
        outs = _both_paths(kvcache.make_batch(spec))
        (o_ws, l_ws), (o_na, l_na) = outs["workspace"], outs["noalloc"]
        assert not torch.isnan(o_na.float()).any() and not torch.isnan(l_na).any()
        torch.testing.assert_close(o_na.float(), o_ws.float(), atol=OUT_ATOL, rtol=OUT_RTOL)
        torch.testing.assert_close(l_na, l_ws, atol=LSE_ATOL, rtol=LSE_RTOL)


def test_noalloc_refuses_requests_beyond_its_scratch():
    from deepseek_v4_kernel import _lib, ops
    torch.cuda.set_device(0)
    lib = _lib.lib
    b, h_q = 512, 128           # workspace ~ (512 + parts) x 128 x 2 KB >> 32 MiB
    assert lib.dsv4b_workspace_bytes(b, 1, h_q, 74) > _lib.NOALLOC_SCRATCH_BYTES
    q = torch.zeros(b, 1, h_q, 576, dtype=torch.bfloat16, device="cuda")
    kv = torch.zeros(1, 64, 1, 656, dtype=torch.uint8, device="cuda")
    idx = torch.zeros(b, 1, 128, dtype=torch.int32, device="cuda")
    out = torch.empty(b, 1, h_q, 512, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(b, h_q, 1, dtype=torch.float32, device="cuda")
    p = ops.build_params(q, kv, idx, None, None, None, None, None, 512, 0.04, out, lse)
    tsm = torch.zeros(74, 8, dtype=torch.int32, device="cuda")
    ns = torch.zeros(b + 1, dtype=torch.int32, device="cuda")
    rc = lib.dsv4b_sparse_decode_noalloc(ctypes.byref(p), tsm.data_ptr(), ns.data_ptr(), 74,
                                         torch.cuda.current_stream().cuda_stream)
    assert rc == -7, _lib.STATUS.get(rc, rc)
    assert b"32 MiB" in lib.dsv4b_status_string(rc)
