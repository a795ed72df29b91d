// Sparse prefill host side: the one-part-per-token tile schedule, then the
// decode kernel's bf16 layout instantiation (csrc/sparse_decode_sm100a.cu,
// run_producer_bf16).
//
// Semantics are FlashMLA's flash_mla_sparse_fwd (vLLM
// third_party/flashmla/flash_mla_interface.py:180-217): q [s_q, h_q, d_qk]
// bf16 against a bf16 KV tensor [s_kv, d_qk] through per-token top-k row
// numbers.  A prefill batch has thousands of query tokens, so each token
// is one CTA per 64 heads over all of its top-k tiles: no split-KV, no
// combine.
#include <cuda_runtime.h>

#include "dsv4b_internal.cuh"
#include "dsv4b_kernels.h"

namespace dsv4b {
namespace {

// Part r = query token r, all of its tiles (counted as the decode kernel's
// cursor counts them: ceil(max(len, 1) / 128)); num_splits = 0..rows.
__global__ void prefill_sched_kernel(const dsv4b_decode_params p, int rows, dsv4b_sched_meta* sched,
                                     int32_t* num_splits) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r > rows) return;
  num_splits[r] = r;
  if (r == rows) return;
  const ReqInfo ri = req_info(p, r);
  dsv4b_sched_meta m;
  m.begin_req_idx = r;
  m.end_req_idx = r;
  m.begin_block_idx = 0;
  m.end_block_idx = ri.nt;
  m.begin_split_idx = r;
  m.is_first_req_splitted = 0;
  m.is_last_req_splitted = 0;
  m.num_tiles = ri.nt;
  sched[r] = m;
}

}  // namespace

cudaError_t run_sparse_prefill(const dsv4b_decode_params& p, dsv4b_sched_meta* sched, int32_t* num_splits,
                               int* err, cudaStream_t stream) {
  const int rows = p.b * p.s_q;
  prefill_sched_kernel<<<(rows + 1 + 255) / 256, 256, 0, stream>>>(p, rows, sched, num_splits);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_sparse_prefill(p, sched, num_splits, err, stream);
}

}  // namespace dsv4b
