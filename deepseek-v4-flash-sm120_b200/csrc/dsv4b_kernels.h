// Host-side launch functions of the device kernels (internal to the
// library; the public surface is include/dsv4b.h).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include "dsv4b.h"

namespace dsv4b {

// Largest b * s_q the on-device scheduler accepts (its per-row tables
// live in shared memory).
constexpr int kMaxSchedRows = 16384;

// Query heads handled by one decode CTA (UMMA N).
constexpr int kHeadsPerCtaPublic = 64;

cudaError_t launch_sparse_decode(const dsv4b_decode_params& p, const dsv4b_sched_meta* sched,
                                 const int32_t* num_splits, int num_sm_parts, float* lse_accum,
                                 float* o_accum, int* err, cudaStream_t stream);

int decode_smem_bytes(int layout);

// cuTensorMapEncodeTiled from the driver (csrc/mqa_logits.cu).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn();

// Sparse prefill (csrc/sparse_prefill.cu, csrc/sparse_decode_sm100a.cu):
// the one-part-per-token schedule, then the decode kernel's bf16 layout.
cudaError_t launch_sparse_prefill(const dsv4b_decode_params& p, const dsv4b_sched_meta* sched,
                                  const int32_t* num_splits, int* err, cudaStream_t stream);
cudaError_t run_sparse_prefill(const dsv4b_decode_params& p, dsv4b_sched_meta* sched, int32_t* num_splits,
                               int* err, cudaStream_t stream);

// Test hook: whether the decode kernel's producers withhold their first
// Q^T arrival on the current device (stall != 0), so that a wait runs out.
cudaError_t set_decode_test_stall(int stall);

// Cluster size of the split plan for this batch (1 = no cluster: split
// partials go through the combine kernel).  The scheduler, the decode
// launch and the C ABI all decide with this one function.
int plan_cluster_size(const dsv4b_decode_params& p, int num_sm_parts);

// Measurement: per CTA, the best-of-six cycles of one decode MMA shape's
// chain and its MMA count (out[2 i], out[2 i + 1]; cycles -1 after a wait
// gave up).  Shapes: 0 QK^T, 1 PV, 2 QK^T A with N 128, 3 with N 256,
// 4 and 5: 0 and 1 from precomputed descriptors.
cudaError_t launch_mma_probe(int shape, int ctas, long long* out, cudaStream_t stream);

// Measurement: gather n random rows (row numbers in `rows`) of row_bytes
// each with one mechanism (0 register loads, 1 per-row bulk copies) on 148
// CTAs; sink takes 148 x 256 words, err the timeout status.
cudaError_t launch_gather_rate(int mechanism, const void* kv, int64_t row_stride, int row_bytes,
                               const int32_t* rows, int n, uint32_t* sink, int* err, cudaStream_t stream);

cudaError_t launch_sched_meta(const dsv4b_decode_params& p, int num_sm_parts,
                              dsv4b_sched_meta* sched, int32_t* num_splits, cudaStream_t stream);

cudaError_t launch_combine(const dsv4b_decode_params& p, const int32_t* num_splits,
                           const float* lse_accum, const float* o_accum, cudaStream_t stream);

cudaError_t launch_gather_dequant(int layout, const void* kv, int num_blocks, int page_block_size,
                                  int64_t stride_kv_block, int64_t stride_kv_row,
                                  const int32_t* indices, int n, void* out_bf16,
                                  cudaStream_t stream);

cudaError_t launch_kv_cache_write(int layout, const void* nope, int64_t stride_nope, const void* rope,
                                  int64_t stride_rope, const void* slots, int slot_bytes, int64_t n,
                                  void* kv, int num_blocks, int page, int64_t stride_block,
                                  int64_t stride_row, cudaStream_t stream);

cudaError_t read_kv_write_status(int* flags, cudaStream_t stream);
cudaError_t set_kv_write_test_stall(int stall);  // test hook, see dsv4b_set_test_stall
cudaError_t launch_div_selftest(const float* scales, int n_scales, unsigned long long* mismatches,
                                cudaStream_t stream);

// Indexer logits (csrc/mqa_logits.cu).
constexpr int kMaxMqaRequests = 16384;
cudaError_t launch_mqa_metadata(const int32_t* ctx, int b, int num_sms, int32_t* sched, cudaStream_t stream);
cudaError_t launch_mqa_logits(const dsv4b_mqa_logits_params& p, const int32_t* sched, int num_sms,
                              cudaStream_t stream, int* bad_arg);
cudaError_t read_mqa_status(int* flags, cudaStream_t stream);
cudaError_t set_mqa_test_stall(int stall);  // test hook, see dsv4b_set_test_stall

}  // namespace dsv4b
