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
//   * persistent grid, one 384-thread CTA per SM; the tiles of all
//     requests are split evenly over the CTAs by a device-side schedule
//     (mqa_meta_kernel, DeepGEMM's get_paged_mqa_logits_metadata);
//   * warp 2 reads the block table ahead, 32 entries per parallel batch,
//     into a double buffer in shared memory;
//   * warp 0 streams pages with TMA tiled loads (3-D tensor map over
//     [pages][P][128 B], SWIZZLE_128B, straight into the UMMA K-major
//     layout) into an 8-stage ring, four tiles per step with one page per
//     lane (a single issuing thread capped the stream near 3 TB/s);
//   * warp 1 / lane 0 loads each request's Q block (2-D map, one request
//     ahead into the other of two buffers) and issues the four K = 32
//     kind::f8f6f4 MMAs of a tile into one of two TMEM accumulators
//     (2 x N columns), committing them to the ring slot and the
//     accumulator;
//     The producer also bulk-copies each page's scale section into the
//     stage, so the epilogue never waits on a dependent global load;
//   * two epilogue groups, warps 4-7 and 8-11 (TMEM lanes 0-127 = the
//     tile's positions), take alternate tiles (and so one accumulator
//     each): they read the accumulator, apply relu, the head weights
//     (staged in shared memory once per request) and the page scale,
//     release the stage, and store the logits (consecutive threads,
//     consecutive positions).
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
// Test hook (dsv4b_set_test_stall): when set, the page-id warp of every
// CTA withholds its first arrival, so the producer's first wait runs out.
__device__ int g_mqa_test_stall = 0;

// cuTensorMapEncodeTiled from the driver (no link-time libcuda dependency);
// nullptr if the driver does not provide it.
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

namespace {

constexpr int kTileTok = 128;
constexpr int kDim = 128;
constexpr int kMqaThreads = 384;  // producer, MMA, 2 idle, two 4-warp epilogue groups
constexpr int kStageBytes = kTileTok * kDim;  // 16 KB of e4m3
constexpr int kScaleBytes = kTileTok * 4;     // the tile's page scales
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

// A walk over one CTA's tiles that keeps the current request's context
// length in registers: a global load only when the request changes (a
// reload per tile put a dependent load latency on every producer step).
struct TileCursor {
  const int32_t* ctx_lens;
  int B, b, j, ctx, tiles, b_end, j_end;
  __device__ __forceinline__ void load_req() {
    ctx = b < B ? __ldg(ctx_lens + b) : 0;
    tiles = ctx > 0 ? (ctx + kTileTok - 1) / kTileTok : 0;
  }
  __device__ __forceinline__ void init(const int32_t* c, int nb, int b0, int j0, int b1, int j1) {
    ctx_lens = c;
    B = nb;
    b = b0;
    j = j0;
    b_end = b1;
    j_end = j1;
    load_req();
  }
  __device__ __forceinline__ bool valid() const { return b < B && (b < b_end || (b == b_end && j < j_end)); }
  __device__ __forceinline__ void next() {
    if (++j < tiles) return;
    j = 0;
    do {
      ++b;
      load_req();
    } while (b < B && tiles == 0);
  }
};

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
struct MqaRing {
  // ring depth: as many 16 KB stages as fit beside the Q buffers
  static constexpr int kStages = 8;  // deeper rings (10-12) measured no faster
};

template <int N>
__global__ void __launch_bounds__(kMqaThreads, 1)
mqa_logits_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                  const MqaArgs a, const int32_t* __restrict__ sched) {
  constexpr int kStages = MqaRing<N>::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t ring = smem_u32(smem);
  const uint32_t qbuf = ring + kStages * kStageBytes;
  float* scales = reinterpret_cast<float*>(smem + kStages * kStageBytes + 2 * N * kDim);  // [kStages][128]
  float* wbuf = scales + kStages * kTileTok;                                                 // [2 groups][2][N] head weights
  uint64_t* bars = reinterpret_cast<uint64_t*>(wbuf + 4 * N);
  uint64_t* full = bars;
  uint64_t* empty = full + kStages;
  uint64_t* qfull = empty + kStages;
  uint64_t* qempty = qfull + 2;
  uint64_t* tfull = qempty + 2;
  uint64_t* tempty = tfull + 2;
  uint64_t* done = tempty + 2;
  uint64_t* btfull = done + 1;
  uint64_t* btempty = btfull + 2;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(btempty + 2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(btempty + 3);
  int* bt_buf = reinterpret_cast<int*>(btempty + 4);  // [2][32] page ids, filled by warp 2
  constexpr uint32_t kTmemCols = 2 * N;  // 64 / 128 / 256 / 512: a power of two

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + 4);  // the MMA commit + one arrive per epilogue warp (after the scales)
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qfull[i], 1);
      mbar_init(&qempty[i], 1);
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 128);
    }
    mbar_init(done, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&btfull[i], 1);
      mbar_init(&btempty[i], 1);
    }
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
  const int ppt = kTileTok / a.page;  // pages per tile
  const int tpb = 32 / ppt;           // tiles per 32-entry page-id batch

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // One step covers kBatch tiles, one page per lane: lane l takes page
    // l % ppt of tile k0 + l / ppt.  A single issuing thread needed about
    // 1,300 SM cycles per tile (cursor, page ids, expect_tx, four copy
    // issues in sequence), which capped the stream near 3 TB/s; the lanes
    // issue their copies together.
    constexpr int kBatch = 4;
    const int my_t = lane / ppt, p = lane % ppt;
    const bool active = my_t < kBatch;
    TileCursor cur;
    cur.init(a.ctx, B, b0, j0, b1, j1);
    for (int i = 0; i < my_t && cur.valid(); ++i) cur.next();
    int k0 = 0;
    for (;; k0 += kBatch) {
      const bool live = active && cur.valid();
      if (!__any_sync(0xffffffffu, live)) break;
      const int q = k0 / tpb, slot = q & 1;
      bool ok = true;
      if (k0 % tpb == 0) ok = mbar_wait(&btfull[slot], (q >> 1) & 1, abort_flag, &g_mqa_status);
      const int k = k0 + my_t, s = k % kStages;
      const bool needed = live && (cur.j * ppt + p) * a.page < cur.ctx;
      const int phys = needed ? bt_buf[slot * 32 + (k % tpb) * ppt + p] : -1;
      const bool in_range = needed && phys >= 0 && phys < a.num_blocks;
      __syncwarp();
      if ((k0 + kBatch) % tpb == 0 && lane == 0) mbar_arrive(&btempty[slot]);  // the batch is read
      if (ok && live && p == 0 && k >= kStages)
        ok = mbar_wait(&empty[s], ((k / kStages) - 1) & 1, abort_flag, &g_mqa_status);
      if (!__all_sync(0xffffffffu, ok)) break;
      if (needed && !in_range)  // an out-of-range page id: values read as zeros (TMA fill), scales 0
        for (int e = 0; e < a.page; ++e) scales[s * kTileTok + p * a.page + e] = 0.f;
      const unsigned nmask = __ballot_sync(0xffffffffu, needed);
      const unsigned vmask = __ballot_sync(0xffffffffu, in_range);
      __syncwarp();  // the zeroed scales are ordered before the arrive below
      if (live && p == 0) {
        const unsigned tile_mask = ((1u << ppt) - 1u) << (my_t * ppt);
        mbar_arrive_expect_tx(&full[s], (uint32_t)(__popc(nmask & tile_mask) * a.page * kDim +
                                                   __popc(vmask & tile_mask) * a.page * 4));
      }
      __syncwarp();
      if (needed) tma_load_3d(ring + s * kStageBytes + p * a.page * kDim, &tmk, 0, 0, phys, &full[s]);
      if (in_range)
        bulk_g2s(smem_u32(scales + s * kTileTok + p * a.page),
                 a.kv + (int64_t)phys * a.stride_block + (int64_t)a.page * kDim, a.page * 4, &full[s]);
      for (int i = 0; i < kBatch && cur.valid(); ++i) cur.next();
    }
    if (*abort_flag && lane == 0) {  // let this CTA's copies land before it exits
      // Both loop exits come before batch k0's copies are issued: the
      // stages in flight are those of tiles k0 - kStages .. k0 - 1.
      for (int kk = k0 - 1; kk >= 0 && kk >= k0 - kStages; --kk) {
        const long long t0 = clock64();
        while (!mbar_try_wait(smem_u32(&full[kk % kStages]), (kk / kStages) & 1, 1000u) &&
               clock64() - t0 < kWaitLimitCycles) {
        }
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ page ids
    // Batches of 32 block-table entries (tpb tiles), one per lane, loaded
    // in parallel into a double buffer ahead of the producer: the
    // producer's per-tile critical path never waits on a global load.
    // Test hook: withhold the first batch's arrival, so the producer's
    // first wait can only run out.
    const bool withhold_first = g_mqa_test_stall != 0;
    TileCursor cur;  // this lane's cursor: tile q * tpb + lane / ppt
    cur.init(a.ctx, B, b0, j0, b1, j1);
    for (int i = 0; i < lane / ppt && cur.valid(); ++i) cur.next();
    for (int q = 0;; ++q) {
      const int slot = q & 1;
      const bool live = cur.valid();
      if (!__any_sync(0xffffffffu, live)) break;
      if (q >= 2 && !mbar_wait(&btempty[slot], ((q >> 1) - 1) & 1, abort_flag, &g_mqa_status)) break;
      int phys = -1;
      if (live) {
        const int lp = cur.j * ppt + lane % ppt;
        if (lp * a.page < cur.ctx) phys = __ldg(a.block_table + (int64_t)cur.b * a.stride_bt + lp);
      }
      bt_buf[slot * 32 + lane] = phys;
      __syncwarp();
      if (lane == 0 && !(withhold_first && q == 0)) mbar_arrive(&btfull[slot]);
      for (int i = 0; i < tpb && cur.valid(); ++i) cur.next();
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA
    constexpr uint32_t idesc = idesc_e4m3_f32(128, N);
    // The MMA lane also loads Q: request r goes to buffer r & 1; when r
    // starts, r + 1's Q is loaded into the other buffer once the MMAs of
    // r - 1 (its previous user) have completed.
    auto next_request = [&](int b) {
      int nb = b + 1;
      while (nb < B && tiles_of(a.ctx, nb) == 0) ++nb;
      return (nb < b1 || (nb == b1 && j1 > 0)) ? nb : -1;
    };
    int q_loads0 = 0, q_loads1 = 0;  // Q loads issued into buffer 0 / 1 (scalars: no local memory)
    auto load_q = [&](int b, int slot) {
      mbar_arrive_expect_tx(&qfull[slot], N * kDim);
      tma_load_2d(qbuf + slot * N * kDim, &tmq, 0, b * N, &qfull[slot]);
      if (slot) ++q_loads1; else ++q_loads0;
    };
    int k = 0, rq = -1, prev_b = -1;
    TileCursor cur;
    for (cur.init(a.ctx, B, b0, j0, b1, j1); cur.valid(); cur.next(), ++k) {
      const int b = cur.b;
      if (b != prev_b) {
        if (rq >= 0) umma_commit(&qempty[rq & 1]);  // request rq's Q is free once its MMAs finish
        ++rq;
        if (rq == 0) load_q(b, 0);
        const int nb = next_request(b);
        if (nb >= 0) {
          const int ns = (rq + 1) & 1;
          if (rq >= 1 && !mbar_wait(&qempty[ns], ((rq - 1) >> 1) & 1, abort_flag, &g_mqa_status)) break;
          load_q(nb, ns);
        }
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
    // after an abort, the last Q load of each buffer may still be in
    // flight: it lands before the CTA's shared memory goes away
    if (*abort_flag) {
      for (int i = 0; i < 2; ++i) {
        const int nq = i ? q_loads1 : q_loads0;
        if (nq == 0) continue;
        const long long t1 = clock64();
        while (!mbar_try_wait(smem_u32(&qfull[i]), (nq - 1) & 1, 1000u) &&
               clock64() - t1 < kWaitLimitCycles) {
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    // Group g (warps 4-7 or 8-11) takes the tiles with k % 2 == g and so
    // always the same TMEM accumulator.
    const int g = (warp - 4) >> 2;
    const int r = ((warp - 4) & 3) * 32 + lane;  // TMEM lane = position within the tile
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const int nn = a.next_n, H = a.h;
    // One query row of 64 heads (the DeepSeek indexer shape): the row's
    // weights live in registers for the whole request, so the per-tile sum
    // is register arithmetic only.
    const bool w_in_regs = N == 64 && nn == 1;
    float wr[N == 64 ? 64 : 1];
    // After a failed wait a warp stops working but keeps walking its tiles:
    // its group's named barrier (at each request change) still counts on
    // it, and a wait can give up in one warp while the barrier completes
    // for another, so leaving the loop could strand the group's others.
    // The lanes of a warp poll their waits in lockstep (nothing before them
    // diverges), so they give up together; a per-tile warp vote to enforce
    // that measured 7% slower on B200 at b = 32 x 131,072 positions.
    bool dead = false;
    int k = 0, rq = -1, prev_b = -1;
    TileCursor cur;
    for (cur.init(a.ctx, B, b0, j0, b1, j1); cur.valid(); cur.next(), ++k) {
      if ((k & 1) != g) continue;
      const int b = cur.b, j = cur.j;
      const int acc = g, s = k % kStages;
      if (b != prev_b) {  // this request's head weights into shared memory
        ++rq;
        prev_b = b;
        float* wb = wbuf + (g * 2 + (rq & 1)) * N;
        for (int e = r; e < N; e += 128) wb[e] = __ldg(a.weights + (int64_t)b * N + e);
        named_bar_sync(1 + g, 128);
        if constexpr (N == 64) {
          if (w_in_regs) {
#pragma unroll
            for (int e = 0; e < 64; e += 4) {
              const float4 wv = reinterpret_cast<const float4*>(wb)[e / 4];
              wr[e] = wv.x;
              wr[e + 1] = wv.y;
              wr[e + 2] = wv.z;
              wr[e + 3] = wv.w;
            }
          }
        }
      }
      if (dead) continue;
      const float* wb = wbuf + (g * 2 + (rq & 1)) * N;
      const int ctx = cur.ctx;
      const int t = j * kTileTok + r;
      if (!mbar_wait(&tfull[acc], (k >> 1) & 1, abort_flag, &g_mqa_status)) {
        dead = true;
        continue;
      }
      tc_fence_after();
      if (!mbar_wait(&full[s], (k / kStages) & 1, abort_flag, &g_mqa_status)) {
        dead = true;
        continue;
      }
      const float scale = scales[s * kTileTok + r];
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      float res[N / 32];  // next_n <= N / 32
      bool done_sum = false;
      if constexpr (N == 64) {
        if (w_in_regs) {
          float v[64];
          tmem_ld64(tmem + lane_base + acc * N, v);
          tc_wait_ld();
          // Accumulators (s0, s1) and (s2, s3) as packed f32x2 pairs: one
          // fma.rn.f32x2 per two heads (each lane an ordinary fp32 FMA, so
          // the sums are bit-identical to four scalar accumulators).
          uint64_t s01 = 0, s23 = 0;
#pragma unroll
          for (int e = 0; e < 64; e += 4) {
            uint64_t x01, x23, w01, w23;
            asm("mov.b64 %0, {%1, %2};" : "=l"(x01) : "f"(fmaxf(v[e], 0.f)), "f"(fmaxf(v[e + 1], 0.f)));
            asm("mov.b64 %0, {%1, %2};" : "=l"(x23) : "f"(fmaxf(v[e + 2], 0.f)), "f"(fmaxf(v[e + 3], 0.f)));
            asm("mov.b64 %0, {%1, %2};" : "=l"(w01) : "f"(wr[e]), "f"(wr[e + 1]));
            asm("mov.b64 %0, {%1, %2};" : "=l"(w23) : "f"(wr[e + 2]), "f"(wr[e + 3]));
            asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(s01) : "l"(x01), "l"(w01));
            asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(s23) : "l"(x23), "l"(w23));
          }
          float s0, s1, s2, s3;
          asm("mov.b64 {%0, %1}, %2;" : "=f"(s0), "=f"(s1) : "l"(s01));
          asm("mov.b64 {%0, %1}, %2;" : "=f"(s2), "=f"(s3) : "l"(s23));
          res[0] = ((s0 + s1) + (s2 + s3)) * scale;
          done_sum = true;
        }
      }
      for (int i = 0; i < nn && !done_sum; ++i) {
        const float4* w = reinterpret_cast<const float4*>(wb + i * H);
        float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
        for (int c = 0; c < H / 32; c += 2) {
          float v[64];
          if (c + 1 < H / 32) {
            tmem_ld64(tmem + lane_base + acc * N + i * H + 32 * c, v);
          } else {
            tmem_ld32(tmem + lane_base + acc * N + i * H + 32 * c, *reinterpret_cast<float(*)[32]>(&v[0]));
          }
          tc_wait_ld();
          const int ne = c + 1 < H / 32 ? 64 : 32;
#pragma unroll
          for (int e = 0; e < 64; e += 4) {
            if (e < ne) {
              const float4 wv = w[(32 * c + e) / 4];
              s0 = fmaf(fmaxf(v[e], 0.f), wv.x, s0);
              s1 = fmaf(fmaxf(v[e + 1], 0.f), wv.y, s1);
              s2 = fmaf(fmaxf(v[e + 2], 0.f), wv.z, s2);
              s3 = fmaf(fmaxf(v[e + 3], 0.f), wv.w, s3);
            }
          }
        }
        res[i] = ((s0 + s1) + (s2 + s3)) * scale;
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
    if (a.clean && !*abort_flag && g == 0) {
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

template <int N>
cudaError_t launch_logits(const CUtensorMap& tmq, const CUtensorMap& tmk, const MqaArgs& a, const int32_t* sched,
                          int grid, cudaStream_t stream) {
  constexpr int kStages = MqaRing<N>::kStages;
  // mbarriers: full/empty per stage; qfull, qempty, tfull, tempty, btfull,
  // btempty (2 each); done.  Then the abort flag, the TMEM slot and the
  // [2][32] page-id buffer.
  constexpr int kNumBars = 2 * kStages + 6 * 2 + 1;
  constexpr int kBarBytes = kNumBars * 8 + 16 + 2 * 32 * 4;
  constexpr int smem = 1024 + kStages * kStageBytes + 2 * N * kDim + kStages * kScaleBytes + 4 * N * 4 + kBarBytes;
  static_assert(smem <= 227 * 1024, "logits kernel shared memory");
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

cudaError_t set_mqa_test_stall(int stall) {
  return cudaMemcpyToSymbol(g_mqa_test_stall, &stall, sizeof(stall));
}

cudaError_t read_mqa_status(int* flags, cudaStream_t stream) {
  cudaError_t e = cudaMemcpyFromSymbolAsync(flags, g_mqa_status, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return e;
  if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
  static const int zero = 0;
  return cudaMemcpyToSymbolAsync(g_mqa_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
}

}  // namespace dsv4b
