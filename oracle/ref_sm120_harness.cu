// TEST INFRASTRUCTURE ONLY: a C entry point around the reference's own
// SM120 sparse-decode kernel, compiled for sm_100a from the reference's
// sources where they lie (see oracle/Makefile.ref).  It fills the
// reference's SparseAttnDecodeParams for contiguous MODEL1 tensors exactly
// as its host wrapper does (csrc/api/sparse_decode.cpp:93-145, s_q = 1,
// no scheduler) and calls sm120::launch_dsv4_sparse_decode_v32
// (csrc/sm120/decode/sparse_decode_instantiation.cu:10-23).  Used by the
// GPU tests to pin the oracle against the reference kernel's output and to
// time the reference kernel beside this build's kernel.
#include <cuda_runtime.h>

#include "common/params.h"
#include "sm120/decode/sparse_decode.h"

extern "C" int ref_sm120_sparse_decode(int b, int h_q, int topk, float sm_scale, const void* q,
                                       const void* kv, int num_blocks, int page_block,
                                       const int* indices, const float* attn_sink, void* out,
                                       float* lse, void* stream) {
  using namespace dsv4_kernel;
  SparseAttnDecodeParams p{};
  p.b = b;
  p.s_q = 1;
  p.h_q = h_q;
  p.h_kv = 1;
  p.d_qk = 512;
  p.d_v = 512;
  p.sm_scale = sm_scale;
  p.sm_scale_div_log2 = sm_scale * 1.4426950408889634f;
  p.num_blocks = num_blocks;
  p.page_block_size = page_block;
  p.topk = topk;
  p.model_type = ModelType::V32;  // the reference's own label for its MODEL1 launch
  p.q = reinterpret_cast<cutlass::bfloat16_t*>(const_cast<void*>(q));
  p.kv = reinterpret_cast<cutlass::bfloat16_t*>(const_cast<void*>(kv));
  p.indices = const_cast<int*>(indices);
  p.topk_length = nullptr;
  p.attn_sink = const_cast<float*>(attn_sink);
  p.lse = lse;
  p.out = reinterpret_cast<cutlass::bfloat16_t*>(out);
  // contiguous [b, 1, h_q, 512] q / out, [num_blocks, P, 1, 584] kv (bytes),
  // [b, 1, topk] indices, [b, 1, h_q] lse
  p.stride_q_b = h_q * 512;
  p.stride_q_s_q = h_q * 512;
  p.stride_q_h_q = 512;
  p.stride_kv_block = page_block * 584;
  p.stride_kv_row = 584;
  p.stride_indices_b = topk;
  p.stride_indices_s_q = topk;
  p.stride_lse_b = h_q;
  p.stride_lse_s_q = h_q;
  p.stride_o_b = h_q * 512;
  p.stride_o_s_q = h_q * 512;
  p.stride_o_h_q = 512;
  p.stream = static_cast<cudaStream_t>(stream);
  p.num_sm_parts = 1;
  sm120::launch_dsv4_sparse_decode_v32(p);
  return static_cast<int>(cudaGetLastError());
}
