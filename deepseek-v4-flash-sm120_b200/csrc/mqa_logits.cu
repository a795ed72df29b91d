// Indexer logits, fp8_paged_mqa_logits, on the tcgen05 tensor cores.
//
// For query row (b, i) and cache position t (see include/dsv4b.h):
//   logits[b*next_n+i][t] = k_scale[t] * sum_h w[b*next_n+i][h] *
//                           relu(sum_d q[b][i][h][d] * k[t][d])
// masked to -inf outside t < ctx_b, t <= ctx_b - next_n + i.  The contract
// is DeepGEMM's fp8_paged_mqa_logits as vLLM binds it (utils/deep_gemm.py:
// 386-460); vLLM carries DeepGEMM's torch statement of it
// (v1/attention/ops/rocm_aiter_mla_sparse.py:256-300).  The cache layout is
// vLLM's indexer K cache: per page P x 128 e4m3 values, then P x fp32
// scales.
//
// Design.  A tile is 128 consecutive cache positions of one request
// (128 / P pages); per tile the work is one 128 x N x 128 fp8 GEMM
// (M = positions, N = next_n * h query heads, K = d) and an epilogue that
// reduces the N accumulators of each position to next_n logits.  It is
// HBM-bound (132 B per position against 2 * N * 128 FLOPs):
//   * persistent grid, one 256-thread CTA per SM; the tiles of all
//     requests are split evenly over the CTAs by a device-side schedule
//     (mqa_meta_kernel, DeepGEMM's get_paged_mqa_logits_metadata);
//   * warp 0 / lane 0 streams pages with TMA tiled loads (3-D tensor map
//     over [pages][P][128 B], SWIZZLE_128B, straight into the UMMA K-major
//     layout) into an 8-stage ring, and each request's Q block (2-D map)
//     into one of two Q buffers;
//   * warp 1 / lane 0 issues the four K = 32 kind::f8f6f4 MMAs of a tile
//     into one of two TMEM accumulators (2 x N columns) and commits them
//     to the ring slot and the accumulator;
//   * warps 4-7 (TMEM lanes 0-127 = the tile's positions) read the
//     accumulator, apply relu, the head weights and the page scale, and
//     store the logits (consecutive threads, consecutive positions).
// All waits are bounded (status word g_mqa_status); no multicast.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>

#include "dsv4b.h"
#include "dsv4b_kernels.h"
#include "dsv4b_ptx.cuh"

namespace dsv4b {

__device__ int g_mqa_status;  // kErr* bits of the logits kernel on this device

namespace {

constexpr int kTileTok = 128;
constexpr int kDim = 128;
constexpr int kStages = 8;
constexpr int kMqaThreads = 256;
constexpr int kStageBytes = kTileTok * kDim;  // 16 KB of e4m3
constexpr int kMetaThreads = 1024;

struct MqaArgs {
  int b, next_n, h;
  const uint8_t* kv;
  int num_blocks, page;
  int64_t stride_block;
  const float* weights;
  const int32_t* ctx;
  const int32_t* block_table;
  int64_t stride_bt;
  float* logits;
  int64_t stride_logits;
  int max_model_len;
  int clean;
};

__device__ __forceinline__ int tiles_of(const int32_t* ctx, int b) {
  const int c = __ldg(ctx + b);
  return c > 0 ? (c + kTileTok - 1) / kTileTok : 0;
}

// Next (request, tile) in the flattened order, skipping empty requests.
__device__ __forceinline__ void advance(int& b, int& j, const int32_t* ctx, int B) {
  if (++j < tiles_of(ctx, b)) return;
  j = 0;
  do {
    ++b;
  } while (b < B && tiles_of(ctx, b) == 0);
}

// ------------------------------------------------------------------ schedule
// sched[i] = first (request, tile) of CTA i, sched[G] = (B, 0): CTA i owns
// the flattened tiles [floor(i T / G), floor((i+1) T / G)).
__global__ void __launch_bounds__(kMetaThreads) mqa_meta_kernel(const int32_t* __restrict__ ctx, int B, int G,
                                                                int32_t* __restrict__ sched) {
  extern __shared__ int prefix[];  // [B + 1] + [kMetaThreads] scratch
  int* part = prefix + B + 1;
  const int tid = threadIdx.x;
  const int per = (B + kMetaThreads - 1) / kMetaThreads;
  const int lo = min(B, tid * per), hi = min(B, lo + per);
  int s = 0;
  for (int b = lo; b < hi; ++b) s += tiles_of(ctx, b);
  part[tid] = s;
  __syncthreads();
  // inclusive scan of the per-thread sums (Hillis-Steele, 10 steps)
  for (int o = 1; o < kMetaThreads; o <<= 1) {
    const int v = tid >= o ? part[tid - o] : 0;
    __syncthreads();
    part[tid] += v;
    __syncthreads();
  }
  int run = tid ? part[tid - 1] : 0;
  for (int b = lo; b < hi; ++b) {
    prefix[b] = run;
    run += tiles_of(ctx, b);
  }
  if (tid == kMetaThreads - 1) prefix[B] = part[kMetaThreads - 1];
  __syncthreads();
  const long long T = prefix[B];
  for (int i = tid; i <= G; i += kMetaThreads) {
    const long long target = T * i / G;
    int b = B, j = 0;
    if (target < T) {
      int l = 0, r = B;  // largest b with prefix[b] <= target (then prefix[b+1] > target)
      while (r - l > 1) {
        const int m = (l + r) >> 1;
        if (prefix[m] <= target) l = m;
        else r = m;
      }
      while (l + 1 <= B && prefix[l + 1] <= target) ++l;  // skip empty requests
      b = l;
      j = (int)(target - prefix[l]);
    }
    sched[2 * i] = b;
    sched[2 * i + 1] = j;
  }
}

// ------------------------------------------------------------------ logits
template <int N>
__global__ void __launch_bounds__(kMqaThreads, 1)
mqa_logits_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                  const MqaArgs a, const int32_t* __restrict__ sched) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t ring = smem_u32(smem);
  const uint32_t qbuf = ring + kStages * kStageBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes + 2 * N * kDim);
  uint64_t* full = bars;
  uint64_t* empty = full + kStages;
  uint64_t* qfull = empty + kStages;
  uint64_t* qempty = qfull + 2;
  uint64_t* tfull = qempty + 2;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(done + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 2);
  constexpr uint32_t kTmemCols = 2 * N;  // 64 / 128 / 256 / 512: a power of two

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qfull[i], 1);
      mbar_init(&qempty[i], 1);
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int B = a.b;
  const int b0 = sched[2 * blockIdx.x], j0 = sched[2 * blockIdx.x + 1];
  const int b1 = sched[2 * blockIdx.x + 2], j1 = sched[2 * blockIdx.x + 3];
  auto before_end = [&](int b, int j) { return b < b1 || (b == b1 && j < j1); };
  const int ppt = kTileTok / a.page;  // pages per tile

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int k = 0, rq = -1, prev_b = -1;
    for (int b = b0, j = j0; b < B && before_end(b, j); advance(b, j, a.ctx, B), ++k) {
      if (b != prev_b) {
        ++rq;
        const int qb = rq & 1;
        if (rq >= 2 && !mbar_wait(&qempty[qb], ((rq >> 1) - 1) & 1, abort_flag, &g_mqa_status)) break;
        mbar_arrive_expect_tx(&qfull[qb], N * kDim);
        tma_load_2d(qbuf + qb * N * kDim, &tmq, 0, b * N, &qfull[qb]);
        prev_b = b;
      }
      const int s = k % kStages;
      if (k >= kStages && !mbar_wait(&empty[s], ((k / kStages) - 1) & 1, abort_flag, &g_mqa_status)) break;
      const int ctx = __ldg(a.ctx + b);
      int needed = 0;
      for (int p = 0; p < ppt; ++p) needed += (j * ppt + p) * a.page < ctx;
      mbar_arrive_expect_tx(&full[s], (uint32_t)(needed * a.page * kDim));
      const int32_t* bt = a.block_table + (int64_t)b * a.stride_bt;
      for (int p = 0; p < needed; ++p) {
        const int phys = __ldg(bt + j * ppt + p);
        // an out-of-range page id reads zeros (TMA fills outside the map)
        tma_load_3d(ring + s * kStageBytes + p * a.page * kDim, &tmk, 0, 0, phys, &full[s]);
      }
    }
    if (*abort_flag) {  // let this CTA's copies land before it exits
      for (int kk = k - 1; kk >= 0 && kk >= k - kStages; --kk) {
        const long long t0 = clock64();
        while (!mbar_try_wait(smem_u32(&full[kk % kStages]), (kk / kStages) & 1, 1000u) &&
               clock64() - t0 < kWaitLimitCycles) {
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA
    constexpr uint32_t idesc = idesc_e4m3_f32(128, N);
    int k = 0, rq = -1, prev_b = -1;
    for (int b = b0, j = j0; b < B && before_end(b, j); advance(b, j, a.ctx, B), ++k) {
      if (b != prev_b) {
        if (rq >= 0) umma_commit(&qempty[rq & 1]);  // the previous request's Q is free once its MMAs finish
        ++rq;
        if (!mbar_wait(&qfull[rq & 1], (rq >> 1) & 1, abort_flag, &g_mqa_status)) break;
        prev_b = b;
      }
      const int s = k % kStages, acc = k & 1;
      if (!mbar_wait(&full[s], (k / kStages) & 1, abort_flag, &g_mqa_status)) break;
      if (k >= 2 && !mbar_wait(&tempty[acc], ((k >> 1) - 1) & 1, abort_flag, &g_mqa_status)) break;
      tc_fence_after();
      const uint32_t a_s = ring + s * kStageBytes, b_s = qbuf + (rq & 1) * N * kDim;
#pragma unroll
      for (int kk = 0; kk < kDim / 32; ++kk)
        umma_f8_ss(tmem + acc * N, sdesc_sw128(a_s + kk * 32, 16, 1024), sdesc_sw128(b_s + kk * 32, 16, 1024), idesc,
                   kk > 0);
      umma_commit(&empty[s]);
      umma_commit(&tfull[acc]);
    }
    // every MMA has completed before the accumulators are freed
    umma_commit(done);
    const long long t0 = clock64();
    while (!mbar_try_wait(smem_u32(done), 0, 1000u) && clock64() - t0 < kWaitLimitCycles) {
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int r = (warp - 4) * 32 + lane;  // TMEM lane = position within the tile
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const int nn = a.next_n, H = a.h;
    int k = 0;
    for (int b = b0, j = j0; b < B && before_end(b, j); advance(b, j, a.ctx, B), ++k) {
      const int acc = k & 1;
      const int ctx = __ldg(a.ctx + b);
      const int t = j * kTileTok + r;
      float scale = 0.f;
      if (t < ctx) {
        const int phys = __ldg(a.block_table + (int64_t)b * a.stride_bt + t / a.page);
        if (phys >= 0 && phys < a.num_blocks)
          scale = __ldg(reinterpret_cast<const float*>(a.kv + (int64_t)phys * a.stride_block +
                                                       (int64_t)a.page * kDim) + t % a.page);
      }
      if (!mbar_wait(&tfull[acc], (k >> 1) & 1, abort_flag, &g_mqa_status)) break;
      tc_fence_after();
      float res[N / 32];  // next_n <= N / 32
      for (int i = 0; i < nn; ++i) {
        const float4* w = reinterpret_cast<const float4*>(a.weights + ((int64_t)b * nn + i) * H);
        float sum = 0.f;
        for (int c = 0; c < H / 32; ++c) {
          float v[32];
          tmem_ld32(tmem + lane_base + acc * N + i * H + 32 * c, v);
          tc_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const float4 wv = __ldg(w + (32 * c + e) / 4);
            sum = fmaf(fmaxf(v[e], 0.f), wv.x, sum);
            sum = fmaf(fmaxf(v[e + 1], 0.f), wv.y, sum);
            sum = fmaf(fmaxf(v[e + 2], 0.f), wv.z, sum);
            sum = fmaf(fmaxf(v[e + 3], 0.f), wv.w, sum);
          }
        }
        res[i] = sum * scale;
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (t < a.max_model_len) {
        for (int i = 0; i < nn; ++i) {
          const bool ok = t < ctx && t <= ctx - nn + i;
          a.logits[((int64_t)b * nn + i) * a.stride_logits + t] = ok ? res[i] : -INFINITY;
        }
      }
    }
    if (a.clean && !*abort_flag) {
      // positions past each request's last tile: -inf (requests split over CTAs round-robin)
      for (int b = blockIdx.x; b < B; b += gridDim.x) {
        const int from = tiles_of(a.ctx, b) * kTileTok;
        for (int i = 0; i < nn; ++i) {
          float* row = a.logits + ((int64_t)b * nn + i) * a.stride_logits;
          for (int t = from + r; t < a.max_model_len; t += 128) row[t] = -INFINITY;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

template <int N>
cudaError_t launch_logits(const CUtensorMap& tmq, const CUtensorMap& tmk, const MqaArgs& a, const int32_t* sched,
                          int grid, cudaStream_t stream) {
  constexpr int smem = 1024 + kStages * kStageBytes + 2 * N * kDim + 256;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    e = cudaFuncSetAttribute(mqa_logits_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr_done[dev] = true;
  }
  mqa_logits_kernel<N><<<grid, kMqaThreads, smem, stream>>>(tmq, tmk, a, sched);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_mqa_metadata(const int32_t* ctx, int b, int num_sms, int32_t* sched, cudaStream_t stream) {
  const int smem = (b + 1 + kMetaThreads) * (int)sizeof(int);
  static bool attr_done[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    e = cudaFuncSetAttribute(mqa_meta_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (kMaxMqaRequests + 1 + kMetaThreads) * (int)sizeof(int));
    if (e != cudaSuccess) return e;
    attr_done[dev] = true;
  }
  mqa_meta_kernel<<<1, kMetaThreads, smem, stream>>>(ctx, b, num_sms, sched);
  return cudaGetLastError();
}

cudaError_t launch_mqa_logits(const dsv4b_mqa_logits_params& p, const int32_t* sched, int num_sms,
                              cudaStream_t stream, int* bad_arg) {
  *bad_arg = 0;
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  const int N = p.next_n * p.h;
  CUtensorMap tmq, tmk;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)kDim, (cuuint64_t)p.b * N};
    const cuuint64_t strides[1] = {(cuuint64_t)kDim};
    const cuuint32_t box[2] = {(cuuint32_t)kDim, (cuuint32_t)N};
    const cuuint32_t es[2] = {1, 1};
    if (enc(&tmq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(p.q), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      *bad_arg = 1;
      return cudaErrorInvalidValue;
    }
  }
  {
    const cuuint64_t dims[3] = {(cuuint64_t)kDim, (cuuint64_t)p.page_block_size, (cuuint64_t)p.num_blocks};
    const cuuint64_t strides[2] = {(cuuint64_t)kDim, (cuuint64_t)p.stride_kv_block};
    const cuuint32_t box[3] = {(cuuint32_t)kDim, (cuuint32_t)p.page_block_size, 1};
    const cuuint32_t es[3] = {1, 1, 1};
    if (enc(&tmk, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(p.kv), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      *bad_arg = 1;
      return cudaErrorInvalidValue;
    }
  }
  MqaArgs a;
  a.b = p.b;
  a.next_n = p.next_n;
  a.h = p.h;
  a.kv = static_cast<const uint8_t*>(p.kv);
  a.num_blocks = p.num_blocks;
  a.page = p.page_block_size;
  a.stride_block = p.stride_kv_block;
  a.weights = p.weights;
  a.ctx = p.context_lens;
  a.block_table = p.block_table;
  a.stride_bt = p.stride_block_table;
  a.logits = p.logits;
  a.stride_logits = p.stride_logits;
  a.max_model_len = p.max_model_len;
  a.clean = p.clean_logits;
  switch (N) {
    case 32: return launch_logits<32>(tmq, tmk, a, sched, num_sms, stream);
    case 64: return launch_logits<64>(tmq, tmk, a, sched, num_sms, stream);
    case 128: return launch_logits<128>(tmq, tmk, a, sched, num_sms, stream);
    case 256: return launch_logits<256>(tmq, tmk, a, sched, num_sms, stream);
    default: *bad_arg = 1; return cudaErrorInvalidValue;
  }
}

cudaError_t read_mqa_status(int* flags, cudaStream_t stream) {
  cudaError_t e = cudaMemcpyFromSymbolAsync(flags, g_mqa_status, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return e;
  if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
  static const int zero = 0;
  return cudaMemcpyToSymbolAsync(g_mqa_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
}

}  // namespace dsv4b
