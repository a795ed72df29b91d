// KV-cache writer: quantise bf16 tokens into the FP8 page formats the decode
// kernel reads, scattered into the paged cache by a slot mapping.
//
// This is the producer side of the decode path's cache -- SGLang's
// quant_k_cache_v4 named by the reference (tests/reference.py:45-58 unpacks
// its output) and vLLM's writers for the same bytes:
// quantize_and_insert_k_cache (MODEL1, vllm/models/deepseek_v4/common/ops/
// cache_utils.py:23-140) and concat_and_cache_mla with kv_cache_dtype
// "fp8_ds_mla" (V32, vllm/_custom_ops.py:2613-2623; record format at
// vllm/v1/attention/backends/mla/flashmla_sparse.py:70-92).
//
// Per token:
//   V32    reads 1024 B latent + 128 B RoPE, writes one 656 B record
//          [512 e4m3 | 4 fp32 scales | 64 bf16 RoPE];
//          scale = max(amax / 448, FLT_MIN) per 128 columns (an all-zero
//          tile gets FLT_MIN), q = e4m3(x / scale) -- vLLM's fp8_ds_mla rule.
//   MODEL1 reads 896 B NoPE + 128 B RoPE, writes a 576 B row
//          [448 e4m3 | 64 bf16 RoPE] and 8 scale bytes in the page's scale
//          section; scale = 2^ceil(log2(max(amax, 1e-4) / 448)) per 64
//          columns, stored as the biased exponent (UE8M0), 8th byte 0.
// e4m3 conversion rounds to nearest even after clamping to +-448.  Tokens
// whose slot is negative or past the cache are skipped (vLLM skips -1).
//
// Design (HBM-bound byte work): a persistent grid, one CTA per SM.  Tokens
// are cut into chunks of kChunkTok consecutive tokens; CTA c takes chunks
// c, c + grid, ...  A producer warp streams each chunk's input rows into a
// kStages-deep shared-memory ring with untiled bulk copies (completion
// counted on the stage's "full" mbarrier), keeping about 220 KB of reads in
// flight per SM.  Dense inputs take one copy per chunk (NoPE and RoPE
// adjacent in one row tensor, e.g. a [n, 576] / [n, 512] k) or two (two
// dense tensors); other strides take two copies per token.  Small copies
// are what limits a bulk-copy stream (about 60 SM cycles each), so the
// chunk copies matter; 24 consumer warps take one
// token at a time from the ring (each LDS instruction of a warp reads 512
// contiguous bytes: no bank conflicts), reduce the tile maxima with warp
// shuffles and store the quantised bytes straight to the cache with
// coalesced 8/16-byte stores.  Every mbarrier wait is bounded; a timeout
// leaves kErrWaitTimeout in a per-device status word
// (dsv4b_kv_cache_write_status) and the CTA drains its copies and exits.
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "dsv4b.h"
#include "dsv4b_kernels.h"
#include "dsv4b_ptx.cuh"

// Probe builds only (never the shipped library): 1 = consumers skip the
// quantise and the stores, 2 = every token is stored to slot 0.
#ifndef DSV4B_KVW_PROBE
#define DSV4B_KVW_PROBE 0
#endif

namespace dsv4b {

__device__ int g_kv_write_status;  // kErr* bits of the writer kernels on this device
// Test hook (dsv4b_set_test_stall): when set, the producer of every CTA
// skips its first chunk's copies and arrival, so the consumers' first wait
// runs out.
__device__ int g_kv_write_test_stall = 0;

namespace {

constexpr int kChunkTok = 48;            // tokens per ring stage
constexpr int kStages = 4;
constexpr int kConsumerWarps = 24;
constexpr int kWriterThreads = (kConsumerWarps + 1) * 32;  // + producer warp
constexpr int kInRow = 1152;             // smem bytes per token: V32 1024 + 128 (MODEL1 uses 1024)
constexpr int kStageBytes = kChunkTok * kInRow;
constexpr int kRingBytes = kStages * kStageBytes;
constexpr int kSmemBytes = kRingBytes + 2 * kStages * 8 + 16;
static_assert(kChunkTok % kConsumerWarps == 0, "whole tokens per consumer warp");
static_assert(kSmemBytes <= 227 * 1024, "ring fits one CTA's shared memory");
constexpr float kFp8Max = 448.0f;
constexpr float kAmaxFloor = 1e-4f;       // MODEL1
constexpr float kFltMin = 1.17549435e-38f; // V32: smallest scale (all-zero tile)

// Stage layouts of the input ring.
enum : int {
  kCopyRows = 0,      // one copy per chunk: token j at j * (nope + 128) bytes, RoPE after NoPE
  kCopyBlocks = 1,    // two copies per chunk: NoPE j at j * nope, RoPE j at kChunkTok * nope + 128 j
  kCopyPerToken = 2,  // kCopyBlocks layout, two copies per token
};

template <int L>
struct WriterT;
template <>
struct WriterT<DSV4B_LAYOUT_V32> {
  static constexpr int kNopeBytes = 1024;
};
template <>
struct WriterT<DSV4B_LAYOUT_MODEL1> {
  static constexpr int kNopeBytes = 896;
};

__device__ __forceinline__ uint4 lds_v4(uint32_t saddr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(saddr));
  return v;
}

// 8 bf16 (one uint4) -> 8 floats (exact).
__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// Round to e4m3, nearest even, saturating: a finite value beyond +-448
// becomes +-448 (448 is the largest e4m3fn value, and everything from 448
// up to the overflow threshold 464 rounds to it anyway), so this equals
// clamp(x, -448, 448) followed by the cast; NaN stays NaN.
__device__ __forceinline__ uint32_t e4m3x4(float a, float b, float c, float d) {
  const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return (lo & 0xffffu) | (hi << 16);
}

__device__ __forceinline__ float abs_max8(const float* f) {
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(f[i]));
  return m;
}

// Maximum over aligned groups of `width` lanes (width a power of two <= 16).
template <int W>
__device__ __forceinline__ float group_max(float v) {
#pragma unroll
  for (int o = 1; o < W; o <<= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// a / b correctly rounded (round to nearest even), given y = RN(1/b), for
// the quotients the writer rounds to e4m3 (no overflow; an underflowed
// residual only occurs for quotients far below e4m3's smallest value).
// Markstein's FMA refinement (P. Markstein, "Computation of elementary
// functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1),
// 1990): q0 = RN(a y) is within 2 ulp of a/b; each step takes the exact
// residual r = a - b q with one FMA and corrects q by RN(q + r y).  The
// first step brings q within one ulp, the second returns RN(a/b).
// dsv4b_kv_write_selftest compares it with the hardware division.
// The residual is kept negated (r = b q - a, then q - r y): the same
// values, but a zero numerator keeps its sign (-0 / b = -0).
__device__ __forceinline__ float div_markstein(float a, float b, float y) {
  float q = a * y;
  float r = fmaf(b, q, -a);
  q = fmaf(r, -y, q);
  r = fmaf(b, q, -a);
  return fmaf(r, -y, q);
}

// The same refinement on two numerators at once with Blackwell's packed
// f32x2 multiply / FMA (each lane of the pair is an ordinary IEEE fp32
// operation, so the results equal div_markstein's).
__device__ __forceinline__ uint64_t pack2(float lo, float hi) {
  uint64_t v;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(lo), "f"(hi));
  return v;
}
__device__ __forceinline__ void unpack2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ void div_markstein2(float& a0, float& a1, uint64_t b2, uint64_t y2, uint64_t ny2) {
  const uint64_t a = pack2(a0, a1);
  const uint64_t na = a ^ 0x8000000080000000ull;
  uint64_t q = mul2(a, y2);
  uint64_t r = fma2(b2, q, na);
  q = fma2(r, ny2, q);
  r = fma2(b2, q, na);
  q = fma2(r, ny2, q);
  unpack2(q, a0, a1);
}

// x / scale as the writer computes it: the refinement, except for scales
// below 2^-60 (tiles of tiny values), where its residual could underflow
// and the division itself is used.  (For the self-test: it also checks that
// the packed and scalar forms agree, returning a NaN if they do not.)
constexpr float kMinRefinedScale = 0x1p-60f;
__device__ __forceinline__ float writer_quotient(float a, float b) {
  if (!(b >= kMinRefinedScale)) return a / b;
  const float y = __frcp_rn(b);
  float q0 = a, q1 = a;  // the packed path the writer runs
  div_markstein2(q0, q1, pack2(b, b), pack2(y, y), pack2(-y, -y));
  const float q = div_markstein(a, b, y);
  return __float_as_uint(q0) == __float_as_uint(q) && __float_as_uint(q1) == __float_as_uint(q) ? q : __int_as_float(0x7fc00001);
}

__device__ __forceinline__ uint2 quant8_div(const float* f, float scale) {
  float q[8];
  if (scale >= kMinRefinedScale) {
    const float y = __frcp_rn(scale);
    const uint64_t b2 = pack2(scale, scale), y2 = pack2(y, y), ny2 = pack2(-y, -y);
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
      q[i] = f[i];
      q[i + 1] = f[i + 1];
      div_markstein2(q[i], q[i + 1], b2, y2, ny2);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = f[i] / scale;
  }
  return make_uint2(e4m3x4(q[0], q[1], q[2], q[3]), e4m3x4(q[4], q[5], q[6], q[7]));
}

// 8 values times an exact power of two -> 8 e4m3 bytes.
__device__ __forceinline__ uint2 quant8_mul(const float* f, float inv) {
  return make_uint2(e4m3x4(f[0] * inv, f[1] * inv, f[2] * inv, f[3] * inv),
                    e4m3x4(f[4] * inv, f[5] * inv, f[6] * inv, f[7] * inv));
}

// ceil(log2(r)) for a positive normal fp32 r, read off its bits: the
// unbiased exponent, plus one when any mantissa bit is set.
__device__ __forceinline__ int ceil_log2_normal(float r) {
  const uint32_t u = __float_as_uint(r);
  return (int)((u >> 23) & 0xffu) - 127 + ((u & 0x7fffffu) != 0u);
}

__device__ __forceinline__ void stg_v2(void* p, uint2 v) { *reinterpret_cast<uint2*>(p) = v; }
__device__ __forceinline__ void stg_v4(void* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }

struct WriterArgs {
  const uint8_t* nope;    // bf16 rows, byte stride below
  int64_t stride_nope;    // bytes
  const uint8_t* rope;
  int64_t stride_rope;    // bytes
  const void* slots;
  int64_t n;
  uint8_t* kv;
  int64_t cache_tokens;
  int page;
  int64_t stride_block;
  int64_t stride_row;     // V32 only
  int copy_mode;          // kCopy*
};

// One V32 token: 1024 B latent at snope, 128 B RoPE at srope -> 656 B
// record.  Lane l holds latent columns [8l, 8l+8) (tile l/16) and
// [256+8l, 256+8l+8) (tile 2 + l/16).
__device__ __forceinline__ void write_v32_token(uint32_t snope, uint32_t srope, uint8_t* rec, int lane) {
  float f0[8], f1[8];
  bf16x8_to_f32(lds_v4(snope + 16 * lane), f0);
  bf16x8_to_f32(lds_v4(snope + 512 + 16 * lane), f1);
  uint4 r = make_uint4(0, 0, 0, 0);
  if (lane < 8) r = lds_v4(srope + 16 * lane);
  const float s0 = fmaxf(group_max<16>(abs_max8(f0)) / kFp8Max, kFltMin);
  const float s1 = fmaxf(group_max<16>(abs_max8(f1)) / kFp8Max, kFltMin);
  stg_v2(rec + 8 * lane, quant8_div(f0, s0));
  stg_v2(rec + 256 + 8 * lane, quant8_div(f1, s1));
  const float t1 = __shfl_sync(0xffffffffu, s0, 16);
  const float t3 = __shfl_sync(0xffffffffu, s1, 16);
  if (lane == 0)
    stg_v4(rec + 512, make_uint4(__float_as_uint(s0), __float_as_uint(t1), __float_as_uint(s1), __float_as_uint(t3)));
  if (lane < 8) stg_v4(rec + 528 + 16 * lane, r);
}

// One MODEL1 token: 896 B NoPE at snope, 128 B RoPE at srope -> 576 B row
// + 8 scale bytes.  Lane l holds NoPE columns [8l, 8l+8) (tile l/8); lanes
// 0..23 also [256+8l, +8) (tile 4 + l/8); lanes 24..31 hold RoPE columns
// [8(l-24), +8).
__device__ __forceinline__ void write_model1_token(uint32_t snope, uint32_t srope, uint8_t* row, uint8_t* scl,
                                                   int lane) {
  float f0[8], f1[8];
  bf16x8_to_f32(lds_v4(snope + 16 * lane), f0);
  const uint4 u1 = lds_v4(lane < 24 ? snope + 512 + 16 * lane : srope + 16 * (lane - 24));
  bf16x8_to_f32(u1, f1);
  const bool nope2 = lane < 24;
  const int e0 = ceil_log2_normal(fmaxf(group_max<8>(abs_max8(f0)), kAmaxFloor) / kFp8Max);
  const int e1 = ceil_log2_normal(fmaxf(group_max<8>(abs_max8(f1)), kAmaxFloor) / kFp8Max);
  stg_v2(row + 8 * lane, quant8_mul(f0, __uint_as_float((uint32_t)(127 - e0) << 23)));
  if (nope2) stg_v2(row + 256 + 8 * lane, quant8_mul(f1, __uint_as_float((uint32_t)(127 - e1) << 23)));
  else stg_v4(row + 448 + 16 * (lane - 24), u1);
  // UE8M0 bytes: tiles 0..3 from e0 of lanes 0, 8, 16, 24; tiles 4..6 from
  // e1 of lanes 0, 8, 16
  uint32_t w0 = 0, w1 = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) w0 |= (uint32_t)(__shfl_sync(0xffffffffu, e0, 8 * k) + 127) << (8 * k);
#pragma unroll
  for (int k = 0; k < 3; ++k) w1 |= (uint32_t)(__shfl_sync(0xffffffffu, e1, 8 * k) + 127) << (8 * k);
  if (lane == 0) stg_v2(scl, make_uint2(w0, w1));
}

template <int L, typename SlotT>
__global__ void __launch_bounds__(kWriterThreads, 1) kv_write_kernel(const WriterArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kRingBytes);
  uint64_t* empty = full + kStages;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kStages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kNope = WriterT<L>::kNopeBytes;
  constexpr int kRowBytes = kNope + 128;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();

  const int64_t chunks = (a.n + kChunkTok - 1) / kChunkTok;
  const uint32_t ring = smem_u32(smem);
  const SlotT* slots = static_cast<const SlotT*>(a.slots);

  if (warp == kConsumerWarps) {
    // ---------------------------------------------------------- producer
    const bool withhold_first = g_kv_write_test_stall != 0;
    int k = 0;
    for (int64_t c = blockIdx.x; c < chunks; c += gridDim.x, ++k) {
      const int s = k % kStages;
      if (k >= kStages && !mbar_wait(&empty[s], ((k / kStages) - 1) & 1, abort_flag, &g_kv_write_status)) break;
      if (withhold_first && k == 0) continue;
      const int64_t t0 = c * kChunkTok;
      const int ntok = a.n - t0 < kChunkTok ? (int)(a.n - t0) : kChunkTok;
      const uint32_t stage = ring + s * kStageBytes;
      if (lane == 0) {
        mbar_arrive_expect_tx(&full[s], (uint32_t)(ntok * kRowBytes));
        if (a.copy_mode == kCopyRows) {
          bulk_g2s(stage, a.nope + t0 * a.stride_nope, (uint32_t)(ntok * kRowBytes), &full[s]);
        } else if (a.copy_mode == kCopyBlocks) {
          bulk_g2s(stage, a.nope + t0 * a.stride_nope, (uint32_t)(ntok * kNope), &full[s]);
          bulk_g2s(stage + kChunkTok * kNope, a.rope + t0 * a.stride_rope, (uint32_t)(ntok * 128), &full[s]);
        }
      }
      __syncwarp();
      if (a.copy_mode == kCopyPerToken) {
        for (int j = lane; j < ntok; j += 32) {
          const int64_t t = t0 + j;
          bulk_g2s(stage + j * kNope, a.nope + t * a.stride_nope, kNope, &full[s]);
          bulk_g2s(stage + kChunkTok * kNope + j * 128, a.rope + t * a.stride_rope, 128, &full[s]);
        }
      }
    }
    // On an abort, wait (bounded) for this CTA's copies still in flight
    // before the CTA's shared memory goes away.
    if (*abort_flag && lane == 0) {
      for (int j = k - 1; j >= 0 && j >= k - kStages; --j) {
        if (withhold_first && j == 0) continue;  // nothing was issued for it
        const uint32_t fa = smem_u32(&full[j % kStages]);
        const long long t0 = clock64();
        while (!mbar_try_wait(fa, (j / kStages) & 1, 1000u) && clock64() - t0 < kWaitLimitCycles) {
        }
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  // Each warp takes tokens warp, warp + 24 of every chunk.  The slots of
  // the next chunk are loaded while the current one is quantised.
  constexpr int kPerWarp = kChunkTok / kConsumerWarps;
  auto load_slots = [&](int64_t c, int64_t (&sl)[kPerWarp]) {
#pragma unroll
    for (int i = 0; i < kPerWarp; ++i) {
      const int64_t t = c * kChunkTok + warp + i * kConsumerWarps;
      sl[i] = (c < chunks && t < a.n) ? (int64_t)__ldg(slots + t) : -1;
    }
  };
  int64_t slot[kPerWarp], next[kPerWarp];
  load_slots(blockIdx.x, slot);
  int k = 0;
  for (int64_t c = blockIdx.x; c < chunks; c += gridDim.x, ++k) {
    const int s = k % kStages;
    load_slots(c + gridDim.x, next);
    if (!mbar_wait(&full[s], (k / kStages) & 1, abort_flag, &g_kv_write_status)) break;
#pragma unroll
    for (int i = 0; i < kPerWarp; ++i) {
      const int j = warp + i * kConsumerWarps;
      int64_t sl = slot[i];
      if (sl < 0 || sl >= a.cache_tokens) continue;  // warp-uniform
#if DSV4B_KVW_PROBE == 1
      continue;  // probe build: stream the inputs only
#elif DSV4B_KVW_PROBE == 2
      sl = 0;    // probe build: every token overwrites slot 0 (no DRAM writes)
#endif
      const uint32_t stage = ring + s * kStageBytes;
      const uint32_t snope = a.copy_mode == kCopyRows ? stage + j * kRowBytes : stage + j * kNope;
      const uint32_t srope = a.copy_mode == kCopyRows ? snope + kNope : stage + kChunkTok * kNope + j * 128;
      uint8_t* page_base = a.kv + (sl / a.page) * a.stride_block;
      const int64_t pos = sl % a.page;
      if constexpr (L == DSV4B_LAYOUT_V32) {
        write_v32_token(snope, srope, page_base + pos * a.stride_row, lane);
      } else {
        write_model1_token(snope, srope, page_base + pos * 576, page_base + (int64_t)a.page * 576 + pos * 8, lane);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
    for (int i = 0; i < kPerWarp; ++i) slot[i] = next[i];
  }
}

// Self-test of writer_quotient against the hardware division over the
// writer's domain (|a| <= 448 b, so no quotient overflows): every finite
// bf16 a (blockIdx.y selects the high byte) against n_scales scales b.
// mismatches[0] += e4m3 bytes that differ (what the writer stores);
// mismatches[1] += fp32 quotients with |a/b| >= 2^-20 whose bits differ.
__global__ void div_selftest_kernel(const float* __restrict__ scales, int n_scales,
                                    unsigned long long* mismatches) {
  const uint32_t bits = (blockIdx.y << 8) | (threadIdx.x & 0xffu);
  const float a = __uint_as_float(bits << 16);
  if (!isfinite(a)) return;
  unsigned int bad8 = 0, bad32 = 0;
  for (int j = blockIdx.x * (blockDim.x >> 8) + (threadIdx.x >> 8); j < n_scales; j += gridDim.x * (blockDim.x >> 8)) {
    const float b = scales[j];
    if (!(fabsf(a) <= 448.0f * b)) continue;
    const float got = writer_quotient(a, b);
    const float want = a / b;
    bad8 += (e4m3x4(got, 0.f, 0.f, 0.f) & 0xffu) != (e4m3x4(want, 0.f, 0.f, 0.f) & 0xffu);
    bad32 += fabsf(want) >= 0x1p-20f && __float_as_uint(got) != __float_as_uint(want);
  }
  if (bad8) atomicAdd(&mismatches[0], (unsigned long long)bad8);
  if (bad32) atomicAdd(&mismatches[1], (unsigned long long)bad32);
}

template <int L, typename SlotT>
cudaError_t launch_writer(const WriterArgs& a, cudaStream_t stream) {
  static bool attr_done[64] = {};
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && !attr_done[dev]) {
    e = cudaFuncSetAttribute(kv_write_kernel<L, SlotT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done[dev] = true;
  }
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const int64_t chunks = (a.n + kChunkTok - 1) / kChunkTok;
  const unsigned grid = (unsigned)(chunks < sms ? chunks : sms);
  kv_write_kernel<L, SlotT><<<grid, kWriterThreads, kSmemBytes, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_kv_cache_write(int layout, const void* nope, int64_t stride_nope, const void* rope,
                                  int64_t stride_rope, const void* slots, int slot_bytes, int64_t n,
                                  void* kv, int num_blocks, int page, int64_t stride_block,
                                  int64_t stride_row, cudaStream_t stream) {
  WriterArgs a;
  a.nope = static_cast<const uint8_t*>(nope);
  a.stride_nope = stride_nope * 2;
  a.rope = static_cast<const uint8_t*>(rope);
  a.stride_rope = stride_rope * 2;
  a.slots = slots;
  a.n = n;
  a.kv = static_cast<uint8_t*>(kv);
  a.cache_tokens = (int64_t)num_blocks * page;
  a.page = page;
  a.stride_block = stride_block;
  a.stride_row = stride_row;
  const int64_t nope_bytes = layout == DSV4B_LAYOUT_V32 ? 1024 : 896;
  if (a.stride_nope == nope_bytes + 128 && a.stride_rope == a.stride_nope && a.rope == a.nope + nope_bytes)
    a.copy_mode = kCopyRows;
  else if (a.stride_nope == nope_bytes && a.stride_rope == 128)
    a.copy_mode = kCopyBlocks;
  else
    a.copy_mode = kCopyPerToken;
  if (layout == DSV4B_LAYOUT_V32)
    return slot_bytes == 8 ? launch_writer<DSV4B_LAYOUT_V32, int64_t>(a, stream)
                           : launch_writer<DSV4B_LAYOUT_V32, int32_t>(a, stream);
  return slot_bytes == 8 ? launch_writer<DSV4B_LAYOUT_MODEL1, int64_t>(a, stream)
                         : launch_writer<DSV4B_LAYOUT_MODEL1, int32_t>(a, stream);
}

cudaError_t launch_div_selftest(const float* scales, int n_scales, unsigned long long* mismatches,
                                cudaStream_t stream) {
  div_selftest_kernel<<<dim3(64, 256), 1024, 0, stream>>>(scales, n_scales, mismatches);
  return cudaGetLastError();
}

cudaError_t set_kv_write_test_stall(int stall) {
  return cudaMemcpyToSymbol(g_kv_write_test_stall, &stall, sizeof(stall));
}

cudaError_t read_kv_write_status(int* flags, cudaStream_t stream) {
  cudaError_t e = cudaMemcpyFromSymbolAsync(flags, g_kv_write_status, sizeof(int), 0, cudaMemcpyDeviceToHost, stream);
  if (e != cudaSuccess) return e;
  if ((e = cudaStreamSynchronize(stream)) != cudaSuccess) return e;
  static const int zero = 0;
  return cudaMemcpyToSymbolAsync(g_kv_write_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream);
}

}  // namespace dsv4b
