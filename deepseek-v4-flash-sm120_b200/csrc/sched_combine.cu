// K2 get_mla_metadata (split-KV tile scheduler), K3 split combine, and the
// debug row gather.
//
// K2 replaces the reference's placeholder scheduler tensors
// (csrc/api/sparse_decode.cpp:147-158, num_sm_parts = 1) with a real
// plan: every query row r = b*s_q + s owns ceil(len/128) main tiles plus
// ceil(extra_len/128) extra tiles.  When clusters of C >= 2 CTAs fit
// (plan_cluster_size), row r owns the C parts of cluster r, which merge
// the row in distributed shared memory.  Else, with no more rows than
// parts, the plan
// is row-aligned: t* is the smallest per-part tile cap with
// sum_r ceil(tiles_r / t*) <= parts and row r is shared evenly by
// ceil(tiles_r / t*) parts, so no CTA switches rows (one Q load and one
// epilogue each).  Otherwise the concatenated tile list is cut into
// min(num_sm_parts, total tiles) contiguous, equal (+-1 tile) ranges, one
// per decode CTA column.  A row cut by a range boundary becomes several
// splits whose partial (O, LSE) the combine kernel merges.  Everything
// runs on the device (one CTA), so a captured CUDA graph replays it.
//
// K3 merges splits: lse = log sum_i exp(lse_i), O = sum_i exp(lse_i - lse)
// O_i, then the sink epilogue of tests/reference.py:124-129.  One CTA per
// (query row, head) or per (query row, four heads) by batch size; rows with
// a single split were written by K1 directly.
#include <cuda_bf16.h>

#include "dsv4b_internal.cuh"
#include "dsv4b_kernels.h"

namespace dsv4b {

namespace {

// One CTA; 1024 threads, or a single warp when there are at most 32 query
// rows (every scan is then a shuffle scan with no block barrier, which is
// what a small batch's graph-captured step waits on).
constexpr int kSchedThreads = 1024;

// Exclusive scan of v over the NT threads of the block; returns the prefix
// for this thread and writes the block total to *total.
template <int NT>
__device__ int block_exclusive_scan(int v, int* scratch, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if constexpr (NT == 32) {
    *total = __shfl_sync(0xffffffffu, x, 31);
    return x - v;
  }
  if (lane == 31) scratch[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < NT / 32 ? scratch[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    scratch[lane] = w;  // inclusive per-warp totals
  }
  __syncthreads();
  const int warp_prefix = warp > 0 ? scratch[warp - 1] : 0;
  *total = scratch[31];
  __syncthreads();
  return warp_prefix + x - v;
}

// Part that owns global tile t when T tiles are split into P ranges
// [floor(pT/P), floor((p+1)T/P)): the largest p with floor(pT/P) <= t.
__device__ __forceinline__ int part_of_tile(long long t, long long T, long long P) {
  return (int)(((t + 1) * P + T - 1) / T) - 1;
}

__device__ __forceinline__ dsv4b_sched_meta empty_record() {
  dsv4b_sched_meta m;
  m.begin_req_idx = 0;
  m.end_req_idx = -1;
  m.begin_block_idx = m.end_block_idx = 0;
  m.begin_split_idx = 0;
  m.is_first_req_splitted = m.is_last_req_splitted = 0;
  m.num_tiles = 0;
  return m;
}

template <int NT>
__global__ void __launch_bounds__(NT)
    sched_meta_kernel(const dsv4b_decode_params p, int num_sm_parts, int cluster_c,
                      dsv4b_sched_meta* sched, int32_t* num_splits) {
  // scratch first: its base stays 16-byte aligned whatever R is, so the
  // 32-entry reductions over it may be read as vectors.
  extern __shared__ __align__(16) int sh[];
  // The decode grid that follows may launch now (its CTAs set up on-chip
  // state, then wait in griddepcontrol.wait for this grid to complete).
  asm volatile("griddepcontrol.launch_dependents;");
  const int R = p.b * p.s_q;
  int* scratch = sh;                // [32]
  int* tile_off = sh + 32;          // [R + 1]
  int* part_off = sh + 32 + R + 1;  // [R + 1] (row-aligned plan)

  // 1. tiles per query row -> exclusive prefix
  int carry = 0;
  for (int base = 0; base < R; base += NT) {
    const int r = base + threadIdx.x;
    const int n = r < R ? req_info(p, r).nt : 0;
    int tot;
    const int ex = block_exclusive_scan<NT>(n, scratch, &tot);
    if (r < R) tile_off[r] = carry + ex;
    carry += tot;
  }
  if (threadIdx.x == 0) tile_off[R] = carry;
  __syncthreads();
  const long long T = tile_off[R];
  const int P_eff = (int)min((long long)num_sm_parts, T);

  if (cluster_c > 1) {
    // Cluster plan: row r owns parts r*C .. r*C+C-1 (one cluster), its
    // tiles shared evenly; the cluster merges the row itself, so every row
    // counts as one split for the combine kernel.
    for (int r = threadIdx.x; r <= R; r += NT) num_splits[r] = r;
    for (int part = threadIdx.x; part < num_sm_parts; part += NT) {
      dsv4b_sched_meta m = empty_record();
      const int r = part / cluster_c, j = part - r * cluster_c;
      if (r < R) {
        const int n = tile_off[r + 1] - tile_off[r];
        const int b0 = j * n / cluster_c, b1 = (j + 1) * n / cluster_c;
        if (b1 > b0) {
          m.begin_req_idx = m.end_req_idx = r;
          m.begin_block_idx = b0;
          m.end_block_idx = b1;
          m.begin_split_idx = r;
          m.is_first_req_splitted = b0 > 0;
          m.is_last_req_splitted = b1 < n;
          m.num_tiles = b1 - b0;
        }
      }
      sched[part] = m;
    }
    return;
  }

  if (R <= num_sm_parts) {
    // Row-aligned plan.  t* by bisection over [1, max_r tiles_r] (the
    // upper end always fits since R <= parts); every step is uniform
    // across the block.
    int max_t = 0;
    for (int r = threadIdx.x; r < R; r += NT) max_t = max(max_t, tile_off[r + 1] - tile_off[r]);
    for (int o = 16; o > 0; o >>= 1) max_t = max(max_t, __shfl_xor_sync(0xffffffffu, max_t, o));
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = max_t;
    __syncthreads();
    int hi = 0;
    for (int w = 0; w < NT / 32; ++w) hi = max(hi, scratch[w]);
    int lo = 1;
    __syncthreads();
    while (lo < hi) {
      const int mid = (lo + hi) / 2;
      int tot_parts = 0;
      for (int base = 0; base < R; base += NT) {
        const int r = base + threadIdx.x;
        const int n = r < R ? (tile_off[r + 1] - tile_off[r] + mid - 1) / mid : 0;
        int tot;
        block_exclusive_scan<NT>(n, scratch, &tot);
        tot_parts += tot;
      }
      if (tot_parts <= num_sm_parts) hi = mid; else lo = mid + 1;
    }
    const int tcap = lo;
    carry = 0;
    for (int base = 0; base < R; base += NT) {
      const int r = base + threadIdx.x;
      const int k = r < R ? (tile_off[r + 1] - tile_off[r] + tcap - 1) / tcap : 0;
      int tot;
      const int ex = block_exclusive_scan<NT>(k, scratch, &tot);
      if (r < R) part_off[r] = num_splits[r] = carry + ex;
      carry += tot;
    }
    if (threadIdx.x == 0) part_off[R] = num_splits[R] = carry;
    __syncthreads();
    for (int part = threadIdx.x; part < num_sm_parts; part += NT) {
      dsv4b_sched_meta m = empty_record();
      if (part < part_off[R]) {
        int a = 0, z = R - 1;  // the row r with part_off[r] <= part < part_off[r + 1]
        while (a < z) {
          const int mid = (a + z + 1) >> 1;
          if (part_off[mid] <= part) a = mid; else z = mid - 1;
        }
        const int r = a, j = part - part_off[r], k = part_off[r + 1] - part_off[r];
        const int n = tile_off[r + 1] - tile_off[r];
        m.begin_req_idx = m.end_req_idx = r;
        m.begin_block_idx = (int)((long long)j * n / k);
        m.end_block_idx = (int)((long long)(j + 1) * n / k);
        m.begin_split_idx = part_off[r] + j;
        m.is_first_req_splitted = m.begin_block_idx > 0;
        m.is_last_req_splitted = m.end_block_idx < n;
        m.num_tiles = m.end_block_idx - m.begin_block_idx;
      }
      sched[part] = m;
    }
    return;
  }

  // 2. splits per row -> exclusive prefix = num_splits
  carry = 0;
  for (int base = 0; base < R; base += NT) {
    const int r = base + threadIdx.x;
    int n = 0;
    if (r < R) {
      const int first = part_of_tile(tile_off[r], T, P_eff);
      const int last = part_of_tile(tile_off[r + 1] - 1, T, P_eff);
      n = last - first + 1;
    }
    int tot;
    const int ex = block_exclusive_scan<NT>(n, scratch, &tot);
    if (r < R) num_splits[r] = carry + ex;
    carry += tot;
  }
  if (threadIdx.x == 0) {
    num_splits[R] = carry;
  }
  __syncthreads();

  // 3. one record per part
  for (int part = threadIdx.x; part < num_sm_parts; part += NT) {
    dsv4b_sched_meta m = empty_record();
    if (part < P_eff) {
      const long long t0 = (long long)part * T / P_eff;
      const long long t1 = (long long)(part + 1) * T / P_eff;  // exclusive, > t0
      // row containing tile x: largest r with tile_off[r] <= x
      auto row_of = [&](long long x) {
        int lo = 0, hi = R - 1;
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (tile_off[mid] <= x) lo = mid; else hi = mid - 1;
        }
        return lo;
      };
      const int br = row_of(t0), er = row_of(t1 - 1);
      m.begin_req_idx = br;
      m.end_req_idx = er;
      m.begin_block_idx = (int)(t0 - tile_off[br]);
      m.end_block_idx = (int)(t1 - tile_off[er]);
      m.begin_split_idx = num_splits[br] + (part - part_of_tile(tile_off[br], T, P_eff));
      m.is_first_req_splitted = m.begin_block_idx > 0;
      m.is_last_req_splitted = (tile_off[er] + m.end_block_idx) < tile_off[er + 1];
      m.num_tiles = (int)(t1 - t0);
    }
    sched[part] = m;
  }
}

// ------------------------------------------------------------- combine
// One 128-thread CTA per (query row, head); thread t owns dims 4t..4t+3.
// The decode kernel leaves split partials o_accum[split][h_q][512] (already
// divided by the split's own row sum) and lse_accum[split][h_q].
constexpr int kCombineThreads = kDv / 4;  // 128 per head
// Two shapes, chosen per launch by the number of query rows (with 148
// scheduler parts, few rows mean many splits per row):
//  * few rows: one head per CTA, up to 16 splits held in registers
//    (127 registers, every split's load in flight at once);
//  * 16 rows or more (<= ~10 splits per row): four heads per CTA and 8
//    splits in registers (64 registers, twice the resident warps), which
//    measured 376 vs 390 us at config 4 and 35.8 vs 37.9 us at 16 rows, but
//    2-4 us slower at 1-8 rows.
constexpr int kCombineRowsForWide = 16;

// Launched (outside CUDA-graph capture) as a programmatic dependent of the
// decode kernel: the CTAs start while the decode grid drains and wait here
// for its completion (and the visibility of its partials) instead of paying
// a full launch gap.
template <int kCombineHeads, int kCombineRegSplits>
__global__ void __launch_bounds__(kCombineThreads * kCombineHeads)
    combine_kernel(const dsv4b_decode_params p, const int32_t* __restrict__ num_splits,
                   const float* __restrict__ lse_accum, const float* __restrict__ o_accum) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int r = blockIdx.x, t = threadIdx.x % kCombineThreads;
  const int head = blockIdx.y * kCombineHeads + threadIdx.x / kCombineThreads;
  const int s0 = __ldg(num_splits + r), s1 = __ldg(num_splits + r + 1);
  const int n = s1 - s0;
  if (n <= 1 || head >= p.h_q) return;  // n <= 1: written by the decode kernel
  constexpr float kLog2e = 1.4426950408889634f;
  const float* lse_col = lse_accum + (int64_t)s0 * p.h_q + head;
  const float4* src = reinterpret_cast<const float4*>(o_accum + ((int64_t)s0 * p.h_q + head) * kDv) + t;
  const int64_t step = (int64_t)p.h_q * (kDv / 4);  // float4s between splits

  // The first kCombineRegSplits partial rows and all their LSEs are loaded
  // before any arithmetic, so the kernel waits on memory once (the weights
  // depend on the LSEs, the loads of the rows do not); more splits loop.
  float4 v[kCombineRegSplits];
  float l2[kCombineRegSplits];
#pragma unroll
  for (int i = 0; i < kCombineRegSplits; ++i) {
    v[i] = i < n ? __ldg(src + i * step) : make_float4(0.f, 0.f, 0.f, 0.f);
    l2[i] = i < n ? __ldg(lse_col + (int64_t)i * p.h_q) * kLog2e : -INFINITY;
  }
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < kCombineRegSplits; ++i) mx = fmaxf(mx, l2[i]);
  for (int i = kCombineRegSplits; i < n; ++i) mx = fmaxf(mx, __ldg(lse_col + (int64_t)i * p.h_q) * kLog2e);
  float sum = 0.0f;
#pragma unroll
  for (int i = 0; i < kCombineRegSplits; ++i) {
    l2[i] = i < n ? exp2f(l2[i] - mx) : 0.0f;
    sum += l2[i];
  }
  for (int i = kCombineRegSplits; i < n; ++i) sum += exp2f(__ldg(lse_col + (int64_t)i * p.h_q) * kLog2e - mx);
  const float inv = 1.0f / sum;
  const float lse = (mx + log2f(sum)) / kLog2e;

  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
  for (int i = 0; i < kCombineRegSplits; ++i) {
    const float wi = l2[i] * inv;  // 0 past n
    acc.x = fmaf(wi, v[i].x, acc.x);
    acc.y = fmaf(wi, v[i].y, acc.y);
    acc.z = fmaf(wi, v[i].z, acc.z);
    acc.w = fmaf(wi, v[i].w, acc.w);
  }
  for (int i = kCombineRegSplits; i < n; ++i) {
    const float4 vi = __ldg(src + i * step);
    const float wi = exp2f(__ldg(lse_col + (int64_t)i * p.h_q) * kLog2e - mx) * inv;
    acc.x = fmaf(wi, vi.x, acc.x);
    acc.y = fmaf(wi, vi.y, acc.y);
    acc.z = fmaf(wi, vi.z, acc.z);
    acc.w = fmaf(wi, vi.w, acc.w);
  }
  float scale = 1.0f, lse_out = lse;
  if (p.attn_sink) {
    const float sink = __ldg(p.attn_sink + head);
    scale = 1.0f / (1.0f + expf(sink - lse));
    if (p.lse_includes_sink) {
      const float m = fmaxf(lse, sink);
      lse_out = m + logf(expf(lse - m) + expf(sink - m));
    }
  }
  const int b = r / p.s_q, s = r - b * p.s_q;
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out) + (int64_t)b * p.stride_o_b +
                       (int64_t)s * p.stride_o_s + (int64_t)head * p.stride_o_h + 4 * t;
  const __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x * scale, acc.y * scale);
  const __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z * scale, acc.w * scale);
  uint2 o;
  o.x = *reinterpret_cast<const uint32_t*>(&lo);
  o.y = *reinterpret_cast<const uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(out) = o;
  if (t == 0) p.lse[((int64_t)b * p.h_q + head) * p.s_q + s] = lse_out;
}

// ------------------------------------------------------------- debug gather
// One thread per (row, half): the exact producer path of K1 (same loads,
// same dq16), written to a plain row-major [n, d_qk] bf16 array.
template <int L>
__global__ void gather_dequant_kernel(const uint8_t* kv, int num_blocks, int page,
                                      int64_t stride_block, int64_t stride_row,
                                      const int32_t* __restrict__ idx, int n,
                                      __nv_bfloat16* __restrict__ out) {
  using LT = LayoutT<L>;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int row = t >> 1, half = t & 1;
  if (row >= n) return;
  const RowSrc r = row_src<L>(kv, page, stride_block, stride_row, num_blocks * page, __ldg(idx + row), true);
  const uint4 sc = load_scales<L>(r);
  uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)row * LT::kDqk);
  for (int c = 0; c < LT::kFp8Chunks; ++c) {
    uint4 a, b, o0, o1, o2, o3;
    load_fp8_half<L>(r, c, half, a, b);
    const float s = chunk_scale<L>(sc, c);
    dq16(a, s, o0, o1);
    dq16(b, s, o2, o3);
    uint4* d = dst + c * 8 + half * 4;
    d[0] = o0; d[1] = o1; d[2] = o2; d[3] = o3;
  }
  uint4 rope[4];
  load_rope_half<L>(r, half, rope);
  uint4* d = dst + LT::kFp8Chunks * 8 + half * 4;
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] = rope[i];
}

}  // namespace

cudaError_t launch_sched_meta(const dsv4b_decode_params& p, int num_sm_parts,
                              dsv4b_sched_meta* sched, int32_t* num_splits, cudaStream_t stream) {
  const int R = p.b * p.s_q;
  const size_t smem = (size_t)(32 + 2 * (R + 1)) * sizeof(int);
  static bool attr_done[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    e = cudaFuncSetAttribute(sched_meta_kernel<kSchedThreads>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)((32 + 2 * (kMaxSchedRows + 1)) * sizeof(int)));
    if (e != cudaSuccess) return e;
    attr_done[dev] = true;
  }
  const int cc = plan_cluster_size(p, num_sm_parts);
  if (R <= 32)
    sched_meta_kernel<32><<<1, 32, smem, stream>>>(p, num_sm_parts, cc, sched, num_splits);
  else
    sched_meta_kernel<kSchedThreads><<<1, kSchedThreads, smem, stream>>>(p, num_sm_parts, cc, sched, num_splits);
  return cudaGetLastError();
}

cudaError_t launch_combine(const dsv4b_decode_params& p, const int32_t* num_splits,
                           const float* lse_accum, const float* o_accum, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  const bool wide = p.b * p.s_q >= kCombineRowsForWide;
  const int heads = wide ? 4 : 1;
  cfg.gridDim = dim3(p.b * p.s_q, (p.h_q + heads - 1) / heads, 1);
  cfg.blockDim = dim3(kCombineThreads * heads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  // Stream launches: a programmatic dependent of the decode kernel, so its
  // launch overlaps the decode's tail.  Inside a CUDA graph the kernel
  // boundary is already cheap and the programmatic edge measured slower, so
  // captured launches are plain (griddepcontrol.wait is then a no-op).
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  cudaError_t e = cudaStreamIsCapturing(stream, &cap);
  if (e != cudaSuccess) return e;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = cap == cudaStreamCaptureStatusNone ? 1 : 0;
  return wide ? cudaLaunchKernelEx(&cfg, combine_kernel<4, 8>, p, num_splits, lse_accum, o_accum)
              : cudaLaunchKernelEx(&cfg, combine_kernel<1, 16>, p, num_splits, lse_accum, o_accum);
}

cudaError_t launch_gather_dequant(int layout, const void* kv, int num_blocks, int page_block_size,
                                  int64_t stride_kv_block, int64_t stride_kv_row,
                                  const int32_t* indices, int n, void* out_bf16,
                                  cudaStream_t stream) {
  const int threads = 256;
  const int blocks = (2 * n + threads - 1) / threads;
  if (layout == DSV4B_LAYOUT_V32)
    gather_dequant_kernel<DSV4B_LAYOUT_V32><<<blocks, threads, 0, stream>>>(
        static_cast<const uint8_t*>(kv), num_blocks, page_block_size, stride_kv_block, stride_kv_row,
        indices, n, static_cast<__nv_bfloat16*>(out_bf16));
  else
    gather_dequant_kernel<DSV4B_LAYOUT_MODEL1><<<blocks, threads, 0, stream>>>(
        static_cast<const uint8_t*>(kv), num_blocks, page_block_size, stride_kv_block, stride_kv_row,
        indices, n, static_cast<__nv_bfloat16*>(out_bf16));
  return cudaGetLastError();
}

}  // namespace dsv4b
