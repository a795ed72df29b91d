// C ABI entry points (include/dsv4b.h): argument validation, workspace
// carving, and the launch sequence.  Replaces the ATen host wrapper of the
// reference (csrc/api/sparse_decode.cpp:29-172): same checks, but status
// codes instead of TORCH_CHECK / abort(), no per-call
// cudaGetDeviceProperties, no output transpose copy.
#include <climits>
#include <cstdint>
#include <cstdio>
#include <cstdlib>

#include "dsv4b.h"
#include "dsv4b_kernels.h"

namespace {

constexpr size_t kStatusBytes = 256;

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

struct WsLayout {
  size_t lse_off, o_off, total;
};

// Workspace: [status word | lse_accum [splits][h_q] | o_accum [splits][h_q]
// [512]]; a query row split over k parts adds k - 1 splits, so b*s_q +
// parts bounds the split count.
inline WsLayout ws_layout(int b, int s_q, int h_q, int parts) {
  const size_t max_splits = (size_t)b * s_q + (size_t)parts;
  WsLayout w;
  w.lse_off = kStatusBytes;
  w.o_off = align_up(w.lse_off + max_splits * h_q * sizeof(float), 256);
  w.total = align_up(w.o_off + max_splits * (size_t)h_q * 512 * sizeof(float), 256);
  return w;
}

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int check_cache(int layout, const void* kv, int num_blocks, int page, int64_t stride_block,
                int64_t stride_row) {
  if (!kv || num_blocks <= 0 || page <= 0) return DSV4B_ERR_INVALID_ARGUMENT;
  if ((int64_t)num_blocks * page > INT_MAX) return DSV4B_ERR_INVALID_ARGUMENT;
  if (!aligned(kv, 16) || stride_block % 16 != 0) return DSV4B_ERR_INVALID_ARGUMENT;
  if (layout == DSV4B_LAYOUT_V32) {
    if (stride_row < 656 || stride_row % 16 != 0) return DSV4B_ERR_INVALID_ARGUMENT;
    if (stride_block < (int64_t)(page - 1) * stride_row + 656) return DSV4B_ERR_INVALID_ARGUMENT;
  } else {
    if (stride_block < (int64_t)page * 584) return DSV4B_ERR_INVALID_ARGUMENT;
  }
  return DSV4B_OK;
}

int check_params(const dsv4b_decode_params* p) {
  if (!p) return DSV4B_ERR_INVALID_ARGUMENT;
  if (p->layout != DSV4B_LAYOUT_V32 && p->layout != DSV4B_LAYOUT_MODEL1) return DSV4B_ERR_INVALID_ARGUMENT;
  if (p->prefill || p->max_logits) return DSV4B_ERR_INVALID_ARGUMENT;  // dsv4b_sparse_prefill's fields
  if (p->b <= 0 || p->s_q <= 0 || p->h_q <= 0 || p->topk <= 0) return DSV4B_ERR_INVALID_ARGUMENT;
  if ((int64_t)p->b * p->s_q > dsv4b::kMaxSchedRows) return DSV4B_ERR_UNSUPPORTED;
  if (p->d_v != 512) return DSV4B_ERR_UNSUPPORTED;
  if (p->d_qk != (p->layout == DSV4B_LAYOUT_V32 ? 576 : 512)) return DSV4B_ERR_INVALID_ARGUMENT;
  if (!p->q || !p->indices || !p->out || !p->lse) return DSV4B_ERR_INVALID_ARGUMENT;
  if (!aligned(p->q, 16) || p->stride_q_b % 8 || p->stride_q_s % 8 || p->stride_q_h % 8)
    return DSV4B_ERR_INVALID_ARGUMENT;
  if (!aligned(p->out, 16) || p->stride_o_b % 8 || p->stride_o_s % 8 || p->stride_o_h % 8)
    return DSV4B_ERR_INVALID_ARGUMENT;
  if (!aligned(p->lse, 4) || !aligned(p->indices, 4)) return DSV4B_ERR_INVALID_ARGUMENT;
  int rc = check_cache(p->layout, p->kv, p->num_blocks, p->page_block_size, p->stride_kv_block,
                       p->stride_kv_row);
  if (rc) return rc;
  if (p->extra_kv) {
    if (!p->extra_indices || p->extra_topk < 0) return DSV4B_ERR_INVALID_ARGUMENT;
    rc = check_cache(p->layout, p->extra_kv, p->extra_num_blocks, p->extra_page_block_size,
                     p->stride_extra_kv_block, p->stride_extra_kv_row);
    if (rc) return rc;
  }
  return DSV4B_OK;
}

// Sparse prefill: workspace = [status word | schedule records [rows] |
// num_splits [rows + 1]].
inline size_t prefill_ws_bytes(int rows) {
  return align_up(kStatusBytes + (size_t)rows * sizeof(dsv4b_sched_meta) + ((size_t)rows + 1) * 4, 256);
}

constexpr int kMaxPrefillRows = 1 << 24;

int check_prefill_params(const dsv4b_decode_params* p) {
  if (!p) return DSV4B_ERR_INVALID_ARGUMENT;
  if (p->layout != DSV4B_LAYOUT_BF16_576 && p->layout != DSV4B_LAYOUT_BF16_512) return DSV4B_ERR_INVALID_ARGUMENT;
  if (p->prefill != 1 || p->lse_includes_sink != 0 || p->extra_kv) return DSV4B_ERR_INVALID_ARGUMENT;
  if (p->b <= 0 || p->s_q != 1 || p->h_q <= 0 || p->topk <= 0) return DSV4B_ERR_INVALID_ARGUMENT;
  if (p->b > kMaxPrefillRows || p->h_q > 65535 * 64) return DSV4B_ERR_UNSUPPORTED;
  // one grid column of tokens x 64-head groups
  if ((int64_t)p->b * ((p->h_q + 63) / 64) > 2147483647) return DSV4B_ERR_UNSUPPORTED;
  if (p->d_v != 512) return DSV4B_ERR_UNSUPPORTED;
  if (p->d_qk != (p->layout == DSV4B_LAYOUT_BF16_576 ? 576 : 512)) return DSV4B_ERR_INVALID_ARGUMENT;
  if (!p->q || !p->indices || !p->out || !p->lse || !p->kv) return DSV4B_ERR_INVALID_ARGUMENT;
  if (!aligned(p->q, 16) || p->stride_q_b % 8 || p->stride_q_h % 8) return DSV4B_ERR_INVALID_ARGUMENT;
  if (!aligned(p->out, 16) || p->stride_o_b % 8 || p->stride_o_h % 8) return DSV4B_ERR_INVALID_ARGUMENT;
  if (!aligned(p->lse, 4) || !aligned(p->indices, 4) || (p->max_logits && !aligned(p->max_logits, 4)))
    return DSV4B_ERR_INVALID_ARGUMENT;
  // KV rows: 16-byte aligned base and row stride (16-byte loads), a whole d_qk row each.
  if (!aligned(p->kv, 16) || p->num_blocks <= 0 || p->page_block_size != 1) return DSV4B_ERR_INVALID_ARGUMENT;
  if (p->stride_kv_block % 16 != 0 || p->stride_kv_block < (int64_t)p->d_qk * 2) return DSV4B_ERR_INVALID_ARGUMENT;
  return DSV4B_OK;
}

struct DevInfo {
  bool init = false;
  int major = 0, minor = 0, sms = 0;
};
DevInfo g_dev[64];

int dev_info(int device, DevInfo** out) {
  if (device < 0 || device >= 64) return DSV4B_ERR_INVALID_ARGUMENT;
  DevInfo& d = g_dev[device];
  if (!d.init) {
    if (cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
      return DSV4B_ERR_CUDA;
    d.init = true;
  }
  *out = &d;
  return DSV4B_OK;
}

int current_arch_ok() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return DSV4B_ERR_CUDA;
  return dsv4b_check_device(dev);
}

int cuda_rc(cudaError_t e) {
  if (e == cudaSuccess) return DSV4B_OK;
  if (getenv("DSV4B_VERBOSE")) fprintf(stderr, "dsv4b: CUDA error %s\n", cudaGetErrorString(e));
  return DSV4B_ERR_CUDA;
}

int check_workspace(const dsv4b_decode_params* p, int parts, void* ws, size_t ws_bytes,
                    WsLayout* w) {
  if (parts <= 0 || parts > 65535) return DSV4B_ERR_INVALID_ARGUMENT;
  *w = ws_layout(p->b, p->s_q, p->h_q, parts);
  if (!ws || !aligned(ws, 256) || ws_bytes < w->total) return DSV4B_ERR_WORKSPACE;
  return DSV4B_OK;
}

// Built-in scratch for dsv4b_sparse_decode_noalloc: a __device__ array of
// the library's module, so each device holds DSV4B_NOALLOC_SCRATCH_BYTES of
// it from the moment the module is loaded on that device (with lazy module
// loading, the CUDA default, that is the first call that touches the
// module there) until the context is destroyed.  In host code the name is
// only a host-side stand-in; the device address comes from
// cudaGetSymbolAddress with the device current.
static __device__ __align__(256) unsigned char g_noalloc_scratch[DSV4B_NOALLOC_SCRATCH_BYTES];

// Device address of the current device's scratch.  Looked up on every call
// (a runtime table lookup, no allocation once the module is loaded): a
// cached address would go stale when the context is reset and recreated.
int noalloc_scratch(void** out) {
  void* ptr = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (e != cudaSuccess || !ptr) return cuda_rc(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
  *out = ptr;
  return DSV4B_OK;
}

}  // namespace

extern "C" {

int dsv4b_version(void) { return 100; }

const char* dsv4b_status_string(int status) {
  switch (status) {
    case DSV4B_OK: return "ok";
    case DSV4B_ERR_INVALID_ARGUMENT: return "invalid argument";
    case DSV4B_ERR_UNSUPPORTED: return "unsupported configuration";
    case DSV4B_ERR_CUDA: return "CUDA runtime error";
    case DSV4B_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case DSV4B_ERR_ARCH: return "device is not an sm_100 (B200-class) GPU";
    case DSV4B_ERR_KERNEL_TIMEOUT: return "a kernel wait hit its time limit";
    case DSV4B_ERR_SCRATCH_LIMIT:
      return "request exceeds the fixed 32 MiB no-allocation scratch (use dsv4b_sparse_decode)";
    default: return "unknown status";
  }
}

int dsv4b_check_device(int device) {
  DevInfo* d = nullptr;
  const int rc = dev_info(device, &d);
  if (rc) return rc;
  return (d->major == 10 && d->minor == 0) ? DSV4B_OK : DSV4B_ERR_ARCH;
}

int dsv4b_num_sm_parts(int device, int h_q, int32_t* num_sm_parts) {
  if (!num_sm_parts || h_q <= 0) return DSV4B_ERR_INVALID_ARGUMENT;
  DevInfo* d = nullptr;
  const int rc = dev_info(device, &d);
  if (rc) return rc;
  const int groups = (h_q + dsv4b::kHeadsPerCtaPublic - 1) / dsv4b::kHeadsPerCtaPublic;
  const int parts = d->sms / groups;
  *num_sm_parts = parts > 0 ? parts : 1;
  return DSV4B_OK;
}

size_t dsv4b_workspace_bytes(int b, int s_q, int h_q, int num_sm_parts) {
  if (b <= 0 || s_q <= 0 || h_q <= 0 || num_sm_parts <= 0) return 0;
  return ws_layout(b, s_q, h_q, num_sm_parts).total;
}

int dsv4b_get_mla_metadata(const dsv4b_decode_params* p, int num_sm_parts,
                           dsv4b_sched_meta* sched_meta, int32_t* num_splits, void* stream) {
  int rc = check_params(p);
  if (rc) return rc;
  if (num_sm_parts <= 0 || num_sm_parts > 65535 || !sched_meta || !num_splits)
    return DSV4B_ERR_INVALID_ARGUMENT;
  if ((rc = current_arch_ok())) return rc;
  return cuda_rc(dsv4b::launch_sched_meta(*p, num_sm_parts, sched_meta, num_splits,
                                          static_cast<cudaStream_t>(stream)));
}

int dsv4b_plan_cluster_size(const dsv4b_decode_params* p, int num_sm_parts, int32_t* cluster_size) {
  int rc = check_params(p);
  if (rc) return rc;
  if (num_sm_parts <= 0 || num_sm_parts > 65535 || !cluster_size) return DSV4B_ERR_INVALID_ARGUMENT;
  if ((rc = current_arch_ok())) return rc;
  *cluster_size = dsv4b::plan_cluster_size(*p, num_sm_parts);
  return DSV4B_OK;
}

int dsv4b_sparse_decode_partial(const dsv4b_decode_params* p, const dsv4b_sched_meta* sched_meta,
                                const int32_t* num_splits, int num_sm_parts, void* workspace,
                                size_t workspace_bytes, void* stream) {
  int rc = check_params(p);
  if (rc) return rc;
  if (!sched_meta || !num_splits) return DSV4B_ERR_INVALID_ARGUMENT;
  WsLayout w;
  if ((rc = check_workspace(p, num_sm_parts, workspace, workspace_bytes, &w))) return rc;
  if ((rc = current_arch_ok())) return rc;
  char* ws = static_cast<char*>(workspace);
  return cuda_rc(dsv4b::launch_sparse_decode(
      *p, sched_meta, num_splits, num_sm_parts, reinterpret_cast<float*>(ws + w.lse_off),
      reinterpret_cast<float*>(ws + w.o_off), reinterpret_cast<int*>(ws),
      static_cast<cudaStream_t>(stream)));
}

int dsv4b_combine(const dsv4b_decode_params* p, const int32_t* num_splits, int num_sm_parts,
                  void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_params(p);
  if (rc) return rc;
  if (!num_splits) return DSV4B_ERR_INVALID_ARGUMENT;
  WsLayout w;
  if ((rc = check_workspace(p, num_sm_parts, workspace, workspace_bytes, &w))) return rc;
  if ((rc = current_arch_ok())) return rc;
  if (dsv4b::plan_cluster_size(*p, num_sm_parts) > 1) return DSV4B_OK;  // merged in the clusters
  char* ws = static_cast<char*>(workspace);
  return cuda_rc(dsv4b::launch_combine(*p, num_splits, reinterpret_cast<const float*>(ws + w.lse_off),
                                       reinterpret_cast<const float*>(ws + w.o_off),
                                       static_cast<cudaStream_t>(stream)));
}

int dsv4b_sparse_decode(const dsv4b_decode_params* p, const dsv4b_sched_meta* sched_meta,
                        const int32_t* num_splits, int num_sm_parts, void* workspace,
                        size_t workspace_bytes, void* stream) {
  const int rc = dsv4b_sparse_decode_partial(p, sched_meta, num_splits, num_sm_parts, workspace,
                                             workspace_bytes, stream);
  if (rc) return rc;
  return dsv4b_combine(p, num_splits, num_sm_parts, workspace, workspace_bytes, stream);
}

int dsv4b_gather_dequant(int layout, const void* kv, int num_blocks, int page_block_size,
                         int64_t stride_kv_block, int64_t stride_kv_row, const int32_t* indices,
                         int n, void* out_bf16, void* stream) {
  if (layout != DSV4B_LAYOUT_V32 && layout != DSV4B_LAYOUT_MODEL1) return DSV4B_ERR_INVALID_ARGUMENT;
  int rc = check_cache(layout, kv, num_blocks, page_block_size, stride_kv_block, stride_kv_row);
  if (rc) return rc;
  if (n < 0 || (n > 0 && (!indices || !out_bf16 || !aligned(out_bf16, 16))))
    return DSV4B_ERR_INVALID_ARGUMENT;
  if (n == 0) return DSV4B_OK;
  if ((rc = current_arch_ok())) return rc;
  return cuda_rc(dsv4b::launch_gather_dequant(layout, kv, num_blocks, page_block_size, stride_kv_block,
                                              stride_kv_row, indices, n, out_bf16,
                                              static_cast<cudaStream_t>(stream)));
}

int dsv4b_mma_rate_probe(int shape, int ctas, long long* out, void* stream) {
  if (shape < 0 || shape > 5 || ctas <= 0 || ctas > 65535 || !out || !aligned(out, 16))
    return DSV4B_ERR_INVALID_ARGUMENT;
  int rc = current_arch_ok();
  if (rc) return rc;
  return cuda_rc(dsv4b::launch_mma_probe(shape, ctas, out, static_cast<cudaStream_t>(stream)));
}

int dsv4b_gather_rate_probe(int mechanism, const void* kv, int64_t row_stride, int row_bytes,
                            const int32_t* rows, int n, void* scratch, size_t scratch_bytes, void* stream) {
  if (mechanism < 0 || mechanism > 1 || !kv || !rows || n <= 0 || row_bytes <= 0 || row_bytes % 16 ||
      row_bytes > 1536 || row_stride < row_bytes || row_stride % 16 || !aligned(kv, 16) || !scratch ||
      scratch_bytes < (size_t)(148 * 256 + 4) * 4 || !aligned(scratch, 16))
    return DSV4B_ERR_INVALID_ARGUMENT;
  int rc = current_arch_ok();
  if (rc) return rc;
  uint32_t* sink = static_cast<uint32_t*>(scratch);
  int* err = reinterpret_cast<int*>(sink + 148 * 256);
  return cuda_rc(dsv4b::launch_gather_rate(mechanism, kv, row_stride, row_bytes, rows, n, sink, err,
                                           static_cast<cudaStream_t>(stream)));
}

int dsv4b_kv_cache_write(int layout, const void* nope, int64_t stride_nope, const void* rope,
                         int64_t stride_rope, const void* slot_mapping, int slot_bytes, int64_t n,
                         void* kv, int num_blocks, int page_block_size, int64_t stride_kv_block,
                         int64_t stride_kv_row, void* stream) {
  if (layout != DSV4B_LAYOUT_V32 && layout != DSV4B_LAYOUT_MODEL1) return DSV4B_ERR_INVALID_ARGUMENT;
  int rc = check_cache(layout, kv, num_blocks, page_block_size, stride_kv_block, stride_kv_row);
  if (rc) return rc;
  if (n < 0 || n > (int64_t)INT_MAX || (slot_bytes != 4 && slot_bytes != 8)) return DSV4B_ERR_INVALID_ARGUMENT;
  if (n == 0) return DSV4B_OK;
  const int64_t nope_cols = layout == DSV4B_LAYOUT_V32 ? 512 : 448;
  if (!nope || !rope || !slot_mapping || !aligned(nope, 16) || !aligned(rope, 16) ||
      !aligned(slot_mapping, slot_bytes))
    return DSV4B_ERR_INVALID_ARGUMENT;
  if (stride_nope % 8 || stride_rope % 8 || (n > 1 && (stride_nope < nope_cols || stride_rope < 64)))
    return DSV4B_ERR_INVALID_ARGUMENT;
  if ((rc = current_arch_ok())) return rc;
  return cuda_rc(dsv4b::launch_kv_cache_write(layout, nope, stride_nope, rope, stride_rope, slot_mapping,
                                              slot_bytes, n, kv, num_blocks, page_block_size,
                                              stride_kv_block, stride_kv_row,
                                              static_cast<cudaStream_t>(stream)));
}

int dsv4b_kv_cache_write_status(int* flags, void* stream) {
  if (!flags) return DSV4B_ERR_INVALID_ARGUMENT;
  return cuda_rc(dsv4b::read_kv_write_status(flags, static_cast<cudaStream_t>(stream)));
}

int dsv4b_kv_write_selftest(const float* scales, int n_scales, unsigned long long* mismatches,
                            void* stream) {
  if (!scales || n_scales <= 0 || !mismatches) return DSV4B_ERR_INVALID_ARGUMENT;
  int rc = current_arch_ok();
  if (rc) return rc;
  return cuda_rc(dsv4b::launch_div_selftest(scales, n_scales, mismatches, static_cast<cudaStream_t>(stream)));
}

int dsv4b_mqa_logits_metadata(const int32_t* context_lens, int b, int num_sms, int32_t* sched, void* stream) {
  if (!context_lens || !sched || b <= 0 || b > dsv4b::kMaxMqaRequests || num_sms <= 0 || num_sms > 65535)
    return DSV4B_ERR_INVALID_ARGUMENT;
  int rc = current_arch_ok();
  if (rc) return rc;
  return cuda_rc(dsv4b::launch_mqa_metadata(context_lens, b, num_sms, sched, static_cast<cudaStream_t>(stream)));
}

int dsv4b_fp8_paged_mqa_logits(const dsv4b_mqa_logits_params* p, const int32_t* sched, int num_sms,
                               void* stream) {
  if (!p || !sched || num_sms <= 0 || num_sms > 65535) return DSV4B_ERR_INVALID_ARGUMENT;
  if (p->b <= 0 || p->b > dsv4b::kMaxMqaRequests || p->next_n <= 0 || p->d != 128) return DSV4B_ERR_INVALID_ARGUMENT;
  if (p->h != 32 && p->h != 64 && p->h != 128) return DSV4B_ERR_UNSUPPORTED;
  const int n = p->next_n * p->h;
  if (n != 32 && n != 64 && n != 128 && n != 256) return DSV4B_ERR_UNSUPPORTED;
  const int P = p->page_block_size;
  if (P != 32 && P != 64 && P != 128) return DSV4B_ERR_UNSUPPORTED;
  if (!p->q || !p->kv || !p->weights || !p->context_lens || !p->block_table || !p->logits)
    return DSV4B_ERR_INVALID_ARGUMENT;
  if (!aligned(p->q, 16) || !aligned(p->kv, 16) || !aligned(p->weights, 16) || !aligned(p->logits, 4))
    return DSV4B_ERR_INVALID_ARGUMENT;
  if (p->num_blocks <= 0 || p->stride_kv_block % 16 || p->stride_kv_block < (int64_t)P * 132)
    return DSV4B_ERR_INVALID_ARGUMENT;
  if (p->max_model_len < 0 || p->stride_logits < p->max_model_len || p->stride_block_table < 0)
    return DSV4B_ERR_INVALID_ARGUMENT;
  int rc = current_arch_ok();
  if (rc) return rc;
  int bad = 0;
  const cudaError_t e = dsv4b::launch_mqa_logits(*p, sched, num_sms, static_cast<cudaStream_t>(stream), &bad);
  if (bad) return DSV4B_ERR_INVALID_ARGUMENT;
  return cuda_rc(e);
}

int dsv4b_mqa_logits_status(int* flags, void* stream) {
  if (!flags) return DSV4B_ERR_INVALID_ARGUMENT;
  return cuda_rc(dsv4b::read_mqa_status(flags, static_cast<cudaStream_t>(stream)));
}

int dsv4b_sparse_decode_noalloc(const dsv4b_decode_params* p, const dsv4b_sched_meta* sched_meta,
                                const int32_t* num_splits, int num_sm_parts, void* stream) {
  int rc = check_params(p);
  if (rc) return rc;
  if (!sched_meta || !num_splits || num_sm_parts <= 0 || num_sm_parts > 65535)
    return DSV4B_ERR_INVALID_ARGUMENT;
  const WsLayout w = ws_layout(p->b, p->s_q, p->h_q, num_sm_parts);
  if (w.total > (size_t)DSV4B_NOALLOC_SCRATCH_BYTES) return DSV4B_ERR_SCRATCH_LIMIT;
  if ((rc = current_arch_ok())) return rc;
  void* scratch = nullptr;
  if ((rc = noalloc_scratch(&scratch))) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(scratch);
  // The status word must start at zero; the partials are fully written
  // before they are read, so nothing else needs clearing.
  if ((rc = cuda_rc(cudaMemsetAsync(ws, 0, kStatusBytes, s)))) return rc;
  if ((rc = cuda_rc(dsv4b::launch_sparse_decode(*p, sched_meta, num_splits, num_sm_parts,
                                                reinterpret_cast<float*>(ws + w.lse_off),
                                                reinterpret_cast<float*>(ws + w.o_off),
                                                reinterpret_cast<int*>(ws), s))))
    return rc;
  if (dsv4b::plan_cluster_size(*p, num_sm_parts) > 1) return DSV4B_OK;  // merged in the clusters
  return cuda_rc(dsv4b::launch_combine(*p, num_splits, reinterpret_cast<const float*>(ws + w.lse_off),
                                       reinterpret_cast<const float*>(ws + w.o_off), s));
}

int dsv4b_set_test_stall(int kernels) {
  if (kernels & ~(DSV4B_STALL_DECODE | DSV4B_STALL_KV_WRITE | DSV4B_STALL_MQA_LOGITS))
    return DSV4B_ERR_INVALID_ARGUMENT;
  int rc = current_arch_ok();
  if (rc) return rc;
  if ((rc = cuda_rc(dsv4b::set_decode_test_stall((kernels & DSV4B_STALL_DECODE) != 0)))) return rc;
  if ((rc = cuda_rc(dsv4b::set_kv_write_test_stall((kernels & DSV4B_STALL_KV_WRITE) != 0)))) return rc;
  return cuda_rc(dsv4b::set_mqa_test_stall((kernels & DSV4B_STALL_MQA_LOGITS) != 0));
}

int dsv4b_read_kernel_status(void* workspace, size_t workspace_bytes, int* flags, void* stream) {
  if (!flags) return DSV4B_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc;
  if (!workspace && workspace_bytes == 0) {  // the status word of dsv4b_sparse_decode_noalloc
    if ((rc = current_arch_ok())) return rc;
    if ((rc = noalloc_scratch(&workspace))) return rc;
    workspace_bytes = kStatusBytes;
  }
  if (!workspace || workspace_bytes < kStatusBytes) return DSV4B_ERR_INVALID_ARGUMENT;
  if ((rc = cuda_rc(cudaMemcpyAsync(flags, workspace, sizeof(int), cudaMemcpyDeviceToHost, s)))) return rc;
  if ((rc = cuda_rc(cudaStreamSynchronize(s)))) return rc;
  return cuda_rc(cudaMemsetAsync(workspace, 0, sizeof(int), s));
}

size_t dsv4b_prefill_workspace_bytes(int rows) {
  return rows <= 0 || rows > kMaxPrefillRows ? 0 : prefill_ws_bytes(rows);
}

int dsv4b_sparse_prefill(const dsv4b_decode_params* p, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_prefill_params(p);
  if (rc) return rc;
  const int rows = p->b;
  if (!workspace || !aligned(workspace, 256) || workspace_bytes < prefill_ws_bytes(rows)) return DSV4B_ERR_WORKSPACE;
  if ((rc = current_arch_ok())) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  char* ws = static_cast<char*>(workspace);
  auto* sched = reinterpret_cast<dsv4b_sched_meta*>(ws + kStatusBytes);
  auto* num_splits = reinterpret_cast<int32_t*>(ws + kStatusBytes + (size_t)rows * sizeof(dsv4b_sched_meta));
  if ((rc = cuda_rc(cudaMemsetAsync(ws, 0, kStatusBytes, s)))) return rc;
  return cuda_rc(dsv4b::run_sparse_prefill(*p, sched, num_splits, reinterpret_cast<int*>(ws), s));
}

}  // extern "C"
