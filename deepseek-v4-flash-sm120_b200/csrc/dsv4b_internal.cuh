// Device-side pieces shared by the decode, scheduler, combine and debug
// gather kernels: layout traits, the split-KV tile walk, and the FP8 row
// decoder (gather + dequantise one 16-byte unit at a time).
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "dsv4b.h"
#include "dsv4b_ptx.cuh"

namespace dsv4b {

constexpr int kTileTokens = 128;  // top-k positions per tile (UMMA M)
constexpr int kHeadsPerCta = 64;  // query heads per CTA (UMMA N)
constexpr int kDv = 512;

// Per-layout constants.  A "chunk" is 64 d_qk columns = one 128-byte
// SWIZZLE_128B atom column of the bf16 K tile.
template <int L>
struct LayoutT;

// DeepSeek-V3.2: [512 e4m3 | 4 fp32 scales (one per 128) | 64 bf16 RoPE].
template <>
struct LayoutT<DSV4B_LAYOUT_V32> {
  static constexpr int kDqk = 576;
  static constexpr int kChunks = 9;       // 8 FP8 chunks + RoPE chunk
  static constexpr int kFp8Chunks = 8;
  static constexpr int kRecordBytes = 656;
  static constexpr int kScaleOffset = 512;
  static constexpr int kRopeOffset = 528;
  static constexpr bool kPInRopeSlot = true;  // V excludes RoPE: reuse its slot for P
};

// DeepSeek-V4-Flash MODEL1: per page P x [448 e4m3 | 64 bf16 RoPE] rows
// then P x 8 UE8M0 scale bytes (one per 64 elements).  V = the full row.
template <>
struct LayoutT<DSV4B_LAYOUT_MODEL1> {
  static constexpr int kDqk = 512;
  static constexpr int kChunks = 8;       // 7 FP8 chunks + RoPE chunk
  static constexpr int kFp8Chunks = 7;
  static constexpr int kRowBytes = 576;
  static constexpr int kScaleBytes = 8;
  static constexpr int kRopeOffset = 448;
  static constexpr bool kPInRopeSlot = false;
};

// Sparse prefill: a bf16 [s_kv, d_qk] KV tensor; rows are copied into the
// K tile without dequantisation.  Same chunk structure as V32 (576: the
// RoPE chunk's slot doubles as P^T) and MODEL1 (512).
template <>
struct LayoutT<DSV4B_LAYOUT_BF16_576> {
  static constexpr int kDqk = 576;
  static constexpr int kChunks = 9;
  static constexpr bool kPInRopeSlot = true;
};
template <>
struct LayoutT<DSV4B_LAYOUT_BF16_512> {
  static constexpr int kDqk = 512;
  static constexpr int kChunks = 8;
  static constexpr bool kPInRopeSlot = false;
};

__host__ __device__ constexpr bool is_bf16_layout(int L) {
  return L == DSV4B_LAYOUT_BF16_576 || L == DSV4B_LAYOUT_BF16_512;
}

// ------------------------------------------------------------- schedule
struct ReqInfo {
  int b, s;
  int len_main;   // attended main positions, clamped to [1, topk]
  int len_valid;  // the same, clamped to [0, topk] (prefill masks rows past it)
  int ntm;        // main tiles
  int len_extra;  // attended extra positions, clamped to [0, extra_topk]
  int nt;         // total tiles (main then extra)
};

// Per query row ("req" r = b * s_q + s).  Main length follows
// tests/reference.py:107-109 (length = max(topk_length[b], 1), capped at
// topk); the extra length follows the reference kernel
// (csrc/sm120/decode/sparse_decode_kernel.cuh:226-233: clamp to >= 0).
__device__ __forceinline__ ReqInfo req_info(const dsv4b_decode_params& p, int r) {
  ReqInfo ri;
  ri.b = r / p.s_q;
  ri.s = r - ri.b * p.s_q;
  int len = p.topk;
  if (p.topk_length) len = min(len, __ldg(p.topk_length + ri.b));
  ri.len_main = max(len, 1);
  ri.len_valid = max(len, 0);
  ri.ntm = (ri.len_main + kTileTokens - 1) / kTileTokens;
  int el = 0;
  if (p.extra_kv) {
    el = p.extra_topk;
    if (p.extra_topk_length) el = min(el, __ldg(p.extra_topk_length + ri.b));
    el = max(el, 0);
  }
  ri.len_extra = el;
  ri.nt = ri.ntm + (el + kTileTokens - 1) / kTileTokens;
  return ri;
}

// Walks the (req, tile) pairs one scheduler part owns, in order.
struct TileCursor {
  bool valid;
  int req, t, t_lo, t_hi;
  ReqInfo ri;
};

__device__ __forceinline__ void cursor_enter_req(const dsv4b_decode_params& p,
                                                 const dsv4b_sched_meta& sm, int req,
                                                 TileCursor& c) {
  c.req = req;
  c.ri = req_info(p, req);
  c.t_lo = (req == sm.begin_req_idx) ? sm.begin_block_idx : 0;
  c.t_hi = (req == sm.end_req_idx) ? sm.end_block_idx : c.ri.nt;
  c.t = c.t_lo;
}

__device__ __forceinline__ TileCursor cursor_begin(const dsv4b_decode_params& p,
                                                   const dsv4b_sched_meta& sm) {
  TileCursor c;
  c.valid = sm.end_req_idx >= sm.begin_req_idx;
  if (!c.valid) return c;
  int req = sm.begin_req_idx;
  cursor_enter_req(p, sm, req, c);
  while (c.t >= c.t_hi) {  // skip empty head/tail ranges
    if (++req > sm.end_req_idx) { c.valid = false; return c; }
    cursor_enter_req(p, sm, req, c);
  }
  return c;
}

__device__ __forceinline__ TileCursor cursor_next(const dsv4b_decode_params& p,
                                                  const dsv4b_sched_meta& sm, TileCursor c) {
  if (!c.valid) return c;
  if (c.t + 1 < c.t_hi) { ++c.t; return c; }
  int req = c.req;
  do {
    if (++req > sm.end_req_idx) { c.valid = false; return c; }
    cursor_enter_req(p, sm, req, c);
  } while (c.t >= c.t_hi);
  return c;
}

// Where a tile's positions live: main (indices) or extra (extra_indices).
struct TileSpan {
  const int32_t* idx;   // index row of this query, already offset to the tile
  int npos;             // valid positions in this tile (1..128)
  const uint8_t* kv;
  int num_tokens;       // num_blocks * page_block_size of that cache
  int page;             // page_block_size
  int64_t stride_block, stride_row;
};

__device__ __forceinline__ TileSpan tile_span(const dsv4b_decode_params& p, const TileCursor& c) {
  TileSpan ts;
  const bool extra = c.t >= c.ri.ntm;
  const int tt = extra ? c.t - c.ri.ntm : c.t;
  const int len = extra ? c.ri.len_extra : c.ri.len_main;
  ts.npos = min(kTileTokens, len - tt * kTileTokens);
  if (!extra) {
    ts.idx = p.indices + (int64_t)c.ri.b * p.stride_idx_b + (int64_t)c.ri.s * p.stride_idx_s +
             (int64_t)tt * kTileTokens;
    ts.kv = static_cast<const uint8_t*>(p.kv);
    ts.num_tokens = p.num_blocks * p.page_block_size;
    ts.page = p.page_block_size;
    ts.stride_block = p.stride_kv_block;
    ts.stride_row = p.stride_kv_row;
  } else {
    ts.idx = p.extra_indices + (int64_t)c.ri.b * p.stride_extra_idx_b +
             (int64_t)c.ri.s * p.stride_extra_idx_s + (int64_t)tt * kTileTokens;
    ts.kv = static_cast<const uint8_t*>(p.extra_kv);
    ts.num_tokens = p.extra_num_blocks * p.extra_page_block_size;
    ts.page = p.extra_page_block_size;
    ts.stride_block = p.stride_extra_kv_block;
    ts.stride_row = p.stride_extra_kv_row;
  }
  return ts;
}

// ------------------------------------------------------------- row decoder
// Address of one cache row.  rec = first byte of the token's record (V32)
// or of its nope|rope row (MODEL1); scl = its scale bytes.  Invalid rows
// (index -1, index >= number of cached tokens, or a masked position) get
// valid = false and decode to zeros, as tests/reference.py:110-114 zeroes
// them (logit 0, zero V row).
struct RowSrc {
  const uint8_t* rec;
  const uint8_t* scl;
  bool valid;
};

template <int L>
__device__ __forceinline__ RowSrc row_src(const uint8_t* kv, int page, int64_t stride_block,
                                          int64_t stride_row, int num_tokens, int idx,
                                          bool in_range) {
  RowSrc r;
  r.valid = in_range && idx >= 0 && idx < num_tokens;
  const int i = r.valid ? idx : 0;
  const int pg = i / page, off = i - pg * page;
  const uint8_t* base = kv + (int64_t)pg * stride_block;
  if constexpr (L == DSV4B_LAYOUT_V32) {
    r.rec = base + (int64_t)off * stride_row;
    r.scl = r.rec + LayoutT<L>::kScaleOffset;
  } else {
    r.rec = base + (int64_t)off * LayoutT<L>::kRowBytes;
    r.scl = base + (int64_t)page * LayoutT<L>::kRowBytes + (int64_t)off * LayoutT<L>::kScaleBytes;
  }
  return r;
}

// UE8M0 byte -> fp32 2^(b-127), built from the exponent bits (exact; b = 0
// is the subnormal 2^-127, b = 255 is +inf), tests/reference.py:40-42.
__device__ __forceinline__ float ue8m0_to_f32(uint32_t b) {
  return __uint_as_float(b == 0 ? 0x00400000u : (b << 23));
}

// Two e4m3 (low byte first) -> two bf16 = RN_bf16(fp32(e4m3) * scale):
// e4m3 -> f16 is exact, f16 -> f32 is exact, one fp32 RN multiply, one RN
// round to bf16; the order of tests/reference.py:53-56.  The scale comes
// pre-packed as {s, s}, so the two fp32 multiplies are one packed f32x2
// multiply (Blackwell; each lane an ordinary IEEE fp32 RN multiply).
__device__ __forceinline__ uint32_t dq_pair2(uint32_t two, uint64_t ss) {
  const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)two, __NV_E4M3);
  __half2 h;
  *reinterpret_cast<__half2_raw*>(&h) = hr;
  const float2 f = __half22float2(h);
  uint64_t a, d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(f.x), "f"(f.y));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(ss));
  float x, y;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(x), "=f"(y) : "l"(d));
  const __nv_bfloat162 o = __floats2bfloat162_rn(x, y);
  return *reinterpret_cast<const uint32_t*>(&o);
}

// 16 e4m3 -> 16 bf16 (two 16-byte units), one scale.
__device__ __forceinline__ void dq16(uint4 in, float s, uint4& lo, uint4& hi) {
  uint64_t ss;
  asm("mov.b64 %0, {%1, %1};" : "=l"(ss) : "f"(s));
  lo.x = dq_pair2(in.x & 0xFFFFu, ss);
  lo.y = dq_pair2(in.x >> 16, ss);
  lo.z = dq_pair2(in.y & 0xFFFFu, ss);
  lo.w = dq_pair2(in.y >> 16, ss);
  hi.x = dq_pair2(in.z & 0xFFFFu, ss);
  hi.y = dq_pair2(in.z >> 16, ss);
  hi.z = dq_pair2(in.w & 0xFFFFu, ss);
  hi.w = dq_pair2(in.w >> 16, ss);
}

// Scale of FP8 chunk c (64 columns) of a row, from the raw scale bytes.
template <int L>
__device__ __forceinline__ float chunk_scale(const uint4& sc, int c) {
  if constexpr (L == DSV4B_LAYOUT_V32) {
    const uint32_t w = (c >> 1) == 0 ? sc.x : (c >> 1) == 1 ? sc.y : (c >> 1) == 2 ? sc.z : sc.w;
    return __uint_as_float(w);
  } else {
    const uint32_t w = c < 4 ? sc.x : sc.y;
    return ue8m0_to_f32((w >> (8 * (c & 3))) & 0xFFu);
  }
}

template <int L>
__device__ __forceinline__ uint4 load_scales(const RowSrc& r) {
  if (!r.valid) return make_uint4(0, 0, 0, 0);
  if constexpr (L == DSV4B_LAYOUT_V32) {
    return ldg_nc_v4(r.scl);
  } else {
    const uint2 v = ldg_nc_v2(r.scl);
    return make_uint4(v.x, v.y, 0, 0);
  }
}

// Raw bytes one producer thread owns for FP8 chunk c of its row: the
// thread's half (0/1) of the chunk = 32 e4m3 = two 16-byte loads.
template <int L>
__device__ __forceinline__ void load_fp8_half(const RowSrc& r, int c, int half, uint4& a,
                                              uint4& b) {
  if (!r.valid) {
    a = b = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint8_t* src = r.rec + c * 64 + half * 32;
  a = ldg_nc_v4(src);
  b = ldg_nc_v4(src + 16);
}

// The thread's half of the RoPE chunk: 32 bf16 = four 16-byte loads.
template <int L>
__device__ __forceinline__ void load_rope_half(const RowSrc& r, int half, uint4 (&v)[4]) {
  if (!r.valid) {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint8_t* src = r.rec + LayoutT<L>::kRopeOffset + half * 64;
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = ldg_nc_v4(src + 16 * i);
}

// Byte offset of 16-byte unit u of row r inside a SWIZZLE_128B tile whose
// rows are 128 bytes (tile base 1024-byte aligned).
__device__ __forceinline__ uint32_t sw128_off(int r, int u) {
  return (uint32_t)(r * 128 + ((u ^ (r & 7)) << 4));
}

}  // namespace dsv4b
