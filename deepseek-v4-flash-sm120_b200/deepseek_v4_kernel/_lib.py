"""ctypes binding of the C ABI in include/dsv4b.h (libdsv4b.so).

The library is loaded from this package directory at import; a missing or
unloadable library raises ImportError (there is no fallback path).
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("DSV4B_LIBRARY", os.path.join(_HERE, "libdsv4b.so"))

LAYOUT_V32 = 0
LAYOUT_MODEL1 = 1
LAYOUT_BF16_576 = 2   # sparse prefill (bf16 KV rows)
LAYOUT_BF16_512 = 3

STATUS = {
    0: "DSV4B_OK",
    -1: "DSV4B_ERR_INVALID_ARGUMENT",
    -2: "DSV4B_ERR_UNSUPPORTED",
    -3: "DSV4B_ERR_CUDA",
    -4: "DSV4B_ERR_WORKSPACE",
    -5: "DSV4B_ERR_ARCH",
    -6: "DSV4B_ERR_KERNEL_TIMEOUT",
    -7: "DSV4B_ERR_SCRATCH_LIMIT",
}

# Every symbol include/dsv4b.h declares (checked by tests/test_abi.py).
EXPORTED = (
    "dsv4b_version", "dsv4b_status_string", "dsv4b_check_device",
    "dsv4b_num_sm_parts", "dsv4b_workspace_bytes", "dsv4b_get_mla_metadata",
    "dsv4b_sparse_decode", "dsv4b_combine", "dsv4b_sparse_decode_partial",
    "dsv4b_gather_dequant", "dsv4b_read_kernel_status", "dsv4b_sparse_decode_noalloc",
    "dsv4b_plan_cluster_size", "dsv4b_kv_cache_write",
    "dsv4b_kv_cache_write_status", "dsv4b_kv_write_selftest",
    "dsv4b_mqa_logits_metadata", "dsv4b_fp8_paged_mqa_logits", "dsv4b_mqa_logits_status",
    "dsv4b_set_test_stall", "dsv4b_prefill_workspace_bytes", "dsv4b_sparse_prefill",
    "dsv4b_mma_rate_probe", "dsv4b_gather_rate_probe",
)

NOALLOC_SCRATCH_BYTES = 32 * 1024 * 1024

# dsv4b_set_test_stall bits
STALL_DECODE, STALL_KV_WRITE, STALL_MQA_LOGITS = 1, 2, 4

_i32, _i64, _f32, _vp = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p


class SchedMeta(ctypes.Structure):
    """dsv4b_sched_meta (32 bytes, DecodingSchedMeta field order)."""
    _fields_ = [
        ("begin_req_idx", _i32), ("end_req_idx", _i32),
        ("begin_block_idx", _i32), ("end_block_idx", _i32),
        ("begin_split_idx", _i32), ("is_first_req_splitted", _i32),
        ("is_last_req_splitted", _i32), ("num_tiles", _i32),
    ]


class DecodeParams(ctypes.Structure):
    """dsv4b_decode_params; field order and types must match dsv4b.h."""
    _fields_ = [
        ("layout", _i32), ("b", _i32), ("s_q", _i32), ("h_q", _i32),
        ("d_qk", _i32), ("d_v", _i32), ("topk", _i32), ("sm_scale", _f32),
        ("lse_includes_sink", _i32),
        ("q", _vp), ("stride_q_b", _i64), ("stride_q_s", _i64), ("stride_q_h", _i64),
        ("kv", _vp), ("num_blocks", _i32), ("page_block_size", _i32),
        ("stride_kv_block", _i64), ("stride_kv_row", _i64),
        ("indices", _vp), ("stride_idx_b", _i64), ("stride_idx_s", _i64),
        ("topk_length", _vp), ("attn_sink", _vp),
        ("extra_kv", _vp), ("extra_num_blocks", _i32), ("extra_page_block_size", _i32),
        ("extra_topk", _i32), ("stride_extra_kv_block", _i64), ("stride_extra_kv_row", _i64),
        ("extra_indices", _vp), ("stride_extra_idx_b", _i64), ("stride_extra_idx_s", _i64),
        ("extra_topk_length", _vp),
        ("out", _vp), ("stride_o_b", _i64), ("stride_o_s", _i64), ("stride_o_h", _i64),
        ("lse", _vp),
        ("prefill", _i32), ("max_logits", _vp),
    ]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"deepseek_v4_kernel: {LIB_PATH} is not built; run "
            "`python deepseek-v4-flash-sm120_b200/build.py` (nvcc, sm_100a)")
    lib = ctypes.CDLL(LIB_PATH)
    lib.dsv4b_version.restype = ctypes.c_int
    lib.dsv4b_status_string.restype = ctypes.c_char_p
    lib.dsv4b_status_string.argtypes = [ctypes.c_int]
    lib.dsv4b_check_device.argtypes = [ctypes.c_int]
    lib.dsv4b_num_sm_parts.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.POINTER(_i32)]
    lib.dsv4b_workspace_bytes.restype = ctypes.c_size_t
    lib.dsv4b_workspace_bytes.argtypes = [ctypes.c_int] * 4
    P = ctypes.POINTER(DecodeParams)
    lib.dsv4b_get_mla_metadata.argtypes = [P, ctypes.c_int, _vp, _vp, _vp]
    lib.dsv4b_plan_cluster_size.argtypes = [P, ctypes.c_int, ctypes.POINTER(_i32)]
    for fn in (lib.dsv4b_sparse_decode, lib.dsv4b_sparse_decode_partial):
        fn.argtypes = [P, _vp, _vp, ctypes.c_int, _vp, ctypes.c_size_t, _vp]
    lib.dsv4b_combine.argtypes = [P, _vp, ctypes.c_int, _vp, ctypes.c_size_t, _vp]
    lib.dsv4b_gather_dequant.argtypes = [ctypes.c_int, _vp, ctypes.c_int, ctypes.c_int,
                                         _i64, _i64, _vp, ctypes.c_int, _vp, _vp]
    lib.dsv4b_kv_cache_write.argtypes = [ctypes.c_int, _vp, _i64, _vp, _i64, _vp, ctypes.c_int, _i64,
                                         _vp, ctypes.c_int, ctypes.c_int, _i64, _i64, _vp]
    lib.dsv4b_mqa_logits_metadata.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp]
    lib.dsv4b_fp8_paged_mqa_logits.argtypes = [_vp, _vp, ctypes.c_int, _vp]
    lib.dsv4b_mqa_logits_status.argtypes = [ctypes.POINTER(ctypes.c_int), _vp]
    lib.dsv4b_kv_write_selftest.argtypes = [_vp, ctypes.c_int, _vp, _vp]
    lib.dsv4b_kv_cache_write_status.argtypes = [ctypes.POINTER(ctypes.c_int), _vp]
    lib.dsv4b_sparse_decode_noalloc.argtypes = [P, _vp, _vp, ctypes.c_int, _vp]
    lib.dsv4b_read_kernel_status.argtypes = [_vp, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int), _vp]
    lib.dsv4b_set_test_stall.argtypes = [ctypes.c_int]
    lib.dsv4b_gather_rate_probe.restype = ctypes.c_int
    lib.dsv4b_gather_rate_probe.argtypes = [ctypes.c_int, _vp, _i64, ctypes.c_int, _vp, ctypes.c_int, _vp,
                                            ctypes.c_size_t, _vp]
    lib.dsv4b_mma_rate_probe.restype = ctypes.c_int
    lib.dsv4b_mma_rate_probe.argtypes = [ctypes.c_int, ctypes.c_int, _vp, _vp]
    lib.dsv4b_prefill_workspace_bytes.restype = ctypes.c_size_t
    lib.dsv4b_prefill_workspace_bytes.argtypes = [ctypes.c_int]
    lib.dsv4b_sparse_prefill.argtypes = [P, _vp, ctypes.c_size_t, _vp]
    return lib


lib = _load()


class DSV4BError(RuntimeError):
    """A C-ABI call returned a non-zero dsv4b_status."""

    def __init__(self, fn: str, status: int):
        self.status = status
        msg = lib.dsv4b_status_string(status).decode()
        super().__init__(f"{fn} failed: {STATUS.get(status, status)} ({msg})")


def check(fn: str, status: int) -> None:
    if status != 0:
        raise DSV4BError(fn, status)
