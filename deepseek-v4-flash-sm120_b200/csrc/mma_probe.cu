// Measurement kernel: the issue-to-completion time of the decode kernel's
// tcgen05.mma shapes with resident shared-memory operands (no loads, no
// other warps), so the tensor-core side of K1's roofline can be read off
// the machine instead of assumed.  Each CTA issues one shape's MMA chain
// from one thread, commits, waits (bounded) and keeps the best of six
// repetitions in SM cycles.  Used by `bench.py --op mma_rates`.
#include <cuda_runtime.h>

#include "dsv4b_internal.cuh"
#include "dsv4b_kernels.h"

namespace dsv4b {
namespace {

constexpr int kProbeA = 9 * 16384;  // a V32 K tile: nine 128 x 64 bf16 SW128 chunk slots
constexpr int kProbeB = 9 * 8192;   // Q^T of 64 heads (or up to 256 B rows for the wide shapes)
constexpr int kProbeSmem = kProbeA + kProbeB + 1024;

__device__ bool probe_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  const long long t0 = clock64();
  while (clock64() - t0 < kWaitLimitCycles)
    if (mbar_try_wait(a, parity, 1000u)) return true;
  return false;
}

// shape 0: QK^T as K1 issues it (M 128 tokens, N 64 heads, A and B K-major,
//          9 chunks x 4 K-steps into one accumulator)
// shape 1: PV as K1 issues it (M 128 dims, N 64 heads, A and B MN-major,
//          4 M-blocks x 8 K-steps)
// shape 2: the QK^T A operand with N 128 (4 chunks x 4 K-steps)
// shape 3: the QK^T A operand with N 256 (2 chunks x 4 K-steps)
// shapes 4, 5: shapes 0, 1 issued from precomputed descriptors (one 64-bit
//          add per MMA instead of building each descriptor), to separate
//          the issuing thread's cost from the tensor core's
__global__ void __launch_bounds__(128) mma_probe_kernel(int shape, long long* out) {
  extern __shared__ uint8_t raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar;
  __shared__ uint32_t tbase;
  __shared__ int stop;
  const uint32_t a_s = smem_u32(sm), b_s = a_s + kProbeA;
  // bf16 1.0 / 0 patterns: finite operands, the values do not matter
  for (int i = threadIdx.x; i < (kProbeA + kProbeB) / 16; i += 128)
    sts_v4(a_s + i * 16, make_uint4(0x3F803F80u, 0u, 0x3F803F80u, 0u));
  fence_proxy_async_smem();
  if (threadIdx.x < 32) tmem_alloc(&tbase, 512);
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    stop = 0;
  }
  fence_mbarrier_init();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tbase;
  long long best = -1;
  int n = 0;
  for (int rep = 0; rep < 6; ++rep) {
    if (threadIdx.x == 0) {
      const long long t0 = clock64();
      n = 0;
      if (shape == 0) {
        constexpr uint32_t id = idesc_bf16_f32(128, 64, false, false);
        for (int c = 0; c < 9; ++c)
          for (int kk = 0; kk < 4; ++kk, ++n)
            umma_bf16_ss(tm, sdesc_sw128(a_s + c * 16384 + kk * 32, 16, 1024),
                         sdesc_sw128(b_s + c * 8192 + kk * 32, 16, 1024), id, (c | kk) != 0);
      } else if (shape == 1) {
        constexpr uint32_t id = idesc_bf16_f32(128, 64, true, true);
        for (int m = 0; m < 4; ++m)
          for (int kk = 0; kk < 8; ++kk, ++n)
            umma_bf16_ss(tm + 64 + 64 * m, sdesc_sw128(a_s + 2 * m * 16384 + kk * 2048, 16384, 1024),
                         sdesc_sw128(b_s + kk * 2048, 8192, 1024), id, kk != 0);
      } else if (shape == 4) {  // shape 0 issued from precomputed descriptors (one add each)
        constexpr uint32_t id = idesc_bf16_f32(128, 64, false, false);
        const uint64_t ad0 = sdesc_sw128(a_s, 16, 1024), bd0 = sdesc_sw128(b_s, 16, 1024);
        umma_bf16_ss(tm, ad0, bd0, id, 0u);
#pragma unroll
        for (int i = 1; i < 36; ++i) {
          const int c = i >> 2, kk = i & 3;
          umma_bf16_acc(tm, ad0 + (uint64_t)((c * 16384 + kk * 32) >> 4), bd0 + (uint64_t)((c * 8192 + kk * 32) >> 4), id);
        }
        n = 36;
      } else if (shape == 5) {  // shape 1 issued from precomputed descriptors
        constexpr uint32_t id = idesc_bf16_f32(128, 64, true, true);
        const uint64_t ad0 = sdesc_sw128(a_s, 16384, 1024), bd0 = sdesc_sw128(b_s, 8192, 1024);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int m = i >> 3, kk = i & 7;
          const uint64_t ad = ad0 + (uint64_t)((2 * m * 16384 + kk * 2048) >> 4), bd = bd0 + (uint64_t)((kk * 2048) >> 4);
          if (kk == 0) umma_bf16_ss(tm + 64 + 64 * m, ad, bd, id, 0u);
          else umma_bf16_acc(tm + 64 + 64 * m, ad, bd, id);
        }
        n = 32;
      } else {
        const int nn = shape == 2 ? 128 : 256, chunks = shape == 2 ? 4 : 2;
        const uint32_t id = shape == 2 ? idesc_bf16_f32(128, 128, false, false) : idesc_bf16_f32(128, 256, false, false);
        for (int c = 0; c < chunks; ++c)
          for (int kk = 0; kk < 4; ++kk, ++n)
            umma_bf16_ss(tm, sdesc_sw128(a_s + c * 16384 + kk * 32, 16, 1024),
                         sdesc_sw128(b_s + c * nn * 128 + kk * 32, 16, 1024), id, (c | kk) != 0);
      }
      umma_commit(&bar);
      const bool ok = probe_wait(&bar, rep & 1);
      const long long dt = clock64() - t0;
      if (!ok) {
        best = -1;
        stop = 1;
      } else if (n > 0 && (best < 0 || dt < best)) {
        best = dt;
      }
    }
    __syncthreads();
    if (stop) break;  // a wait gave up: every thread leaves together
  }
  if (threadIdx.x == 0) {
    out[2 * blockIdx.x] = best;
    out[2 * blockIdx.x + 1] = n;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc(tm, 512);
}

}  // namespace

cudaError_t launch_mma_probe(int shape, int ctas, long long* out, cudaStream_t stream) {
  static bool attr_done[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_done[dev]) {
    e = cudaFuncSetAttribute(mma_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kProbeSmem);
    if (e != cudaSuccess) return e;
    attr_done[dev] = true;
  }
  mma_probe_kernel<<<ctas, 128, kProbeSmem, stream>>>(shape, out);
  return cudaGetLastError();
}

}  // namespace dsv4b

// ------------------------------------------------------------- gather rate
// Measurement kernel: how fast one mechanism gathers random whole cache
// rows (the decode kernel's access pattern) into an SM, with nothing else
// running.  Each CTA takes a contiguous share of the n row numbers.
//  mechanism 0: 16-byte ld.global.nc by all 256 threads with the decode
//               kernel's lane mapping (12 loads in flight per thread),
//               folded into registers;
//  mechanism 1: one cp.async.bulk per row into shared memory, issued by
//               lane 0 of each of the 8 warps into its own 4-stage ring of
//               4 rows, completing on mbarriers (bounded waits).
// Rows are row_bytes long (a multiple of 16) at kv + row * row_stride.
namespace dsv4b {
namespace {

constexpr int kGatherThreads = 256;
constexpr int kGatherStages = 4, kGatherRowsPerStage = 4;

__global__ void __launch_bounds__(kGatherThreads)
    gather_rate_kernel(int mechanism, const uint8_t* __restrict__ kv, int64_t row_stride, int row_bytes,
                       const int32_t* __restrict__ rows, int n, uint32_t* __restrict__ sink, int* err) {
  extern __shared__ __align__(128) uint8_t gsm[];
  const int per = (n + gridDim.x - 1) / gridDim.x;
  const int r0 = blockIdx.x * per, r1 = min(n, r0 + per);
  if (r0 >= r1) return;
  uint32_t x = 0;
  if (mechanism == 0) {
    // K1's mapping: a warp takes 4 rows per pass, lane q = lane & 7 reads
    // the 16-byte pieces q, q + 8, ... of row lane >> 3 (a warp load covers
    // 4 rows x 128 contiguous bytes); two passes (8 rows, up to 12 loads per
    // thread) are in flight before any is used, their row numbers loaded
    // one step ahead.
    const int pieces = row_bytes / 16;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, q = lane & 7, sub = lane >> 3;
    int ra = r0 + warp * 8 + sub, rb = ra + 4;
    int ia = ra < r1 ? __ldg(rows + ra) : -1, ib = rb < r1 ? __ldg(rows + rb) : -1;
    for (int base = r0 + warp * 8; base < r1; base += 8 * 8) {
      const int nra = base + 64 + sub, nrb = nra + 4;
      const int nia = nra < r1 ? __ldg(rows + nra) : -1, nib = nrb < r1 ? __ldg(rows + nrb) : -1;
      uint4 v[12];
#pragma unroll
      for (int u = 0; u < 6; ++u) {
        const int pc = q + 8 * u;
        v[u] = (ia >= 0 && pc < pieces) ? ldg_nc_v4(kv + (int64_t)ia * row_stride + 16 * pc) : make_uint4(0, 0, 0, 0);
        v[6 + u] = (ib >= 0 && pc < pieces) ? ldg_nc_v4(kv + (int64_t)ib * row_stride + 16 * pc) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 12; ++u) x ^= v[u].x ^ v[u].y ^ v[u].z ^ v[u].w;
      ia = nia;
      ib = nib;
    }
  } else {
    __shared__ uint64_t bars[8][kGatherStages];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0)
      for (int s = 0; s < kGatherStages; ++s) mbar_init(&bars[warp][s], 1);
    fence_mbarrier_init();
    __syncwarp();
    const uint32_t ring = smem_u32(gsm) + (uint32_t)warp * kGatherStages * kGatherRowsPerStage * row_bytes;
    if (lane == 0) {
      int j = 0;
      bool ok = true;
      for (int r = r0 + warp * kGatherRowsPerStage; r < r1 && ok; r += 8 * kGatherRowsPerStage, ++j) {
        const int s = j % kGatherStages;
        if (j >= kGatherStages) {  // the stage's previous rows have landed
          const long long t0 = clock64();
          while (!mbar_try_wait(smem_u32(&bars[warp][s]), ((j / kGatherStages) - 1) & 1, 1000u))
            if (clock64() - t0 > kWaitLimitCycles) {
              ok = false;
              atomicOr(err, kErrWaitTimeout);
              break;
            }
        }
        if (!ok) break;
        const int nr = min(kGatherRowsPerStage, r1 - r);
        mbar_arrive_expect_tx(&bars[warp][s], (uint32_t)(nr * row_bytes));
        for (int q = 0; q < nr; ++q)
          bulk_g2s(ring + (uint32_t)((s * kGatherRowsPerStage + q) * row_bytes),
                   kv + (int64_t)__ldg(rows + r + q) * row_stride, (uint32_t)row_bytes, &bars[warp][s]);
      }
      // drain: every stage still in flight lands before the CTA exits (the
      // last chunk c that used stage s is waited for)
      for (int s = 0; s < kGatherStages && s < j; ++s) {
        const int c = s + kGatherStages * ((j - 1 - s) / kGatherStages);
        const long long t0 = clock64();
        while (!mbar_try_wait(smem_u32(&bars[warp][s]), (c / kGatherStages) & 1, 1000u))
          if (clock64() - t0 > kWaitLimitCycles) {
            atomicOr(err, kErrWaitTimeout);
            break;
          }
      }
      x = *reinterpret_cast<const uint32_t*>(gsm + (size_t)warp * kGatherStages * kGatherRowsPerStage * row_bytes);
    }
  }
  sink[blockIdx.x * kGatherThreads + threadIdx.x] = x;
}

}  // namespace

cudaError_t launch_gather_rate(int mechanism, const void* kv, int64_t row_stride, int row_bytes,
                               const int32_t* rows, int n, uint32_t* sink, int* err, cudaStream_t stream) {
  const int ctas = 148;
  const size_t smem = mechanism == 1 ? (size_t)8 * kGatherStages * kGatherRowsPerStage * row_bytes : 0;
  static bool attr_done[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_done[dev]) {
    e = cudaFuncSetAttribute(gather_rate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    attr_done[dev] = true;
  }
  gather_rate_kernel<<<ctas, kGatherThreads, smem, stream>>>(mechanism, static_cast<const uint8_t*>(kv),
                                                            row_stride, row_bytes, rows, n, sink, err);
  return cudaGetLastError();
}

}  // namespace dsv4b
