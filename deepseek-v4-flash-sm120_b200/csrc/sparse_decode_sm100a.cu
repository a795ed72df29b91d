// K1: sparse FP8 MLA decode for sm_100a (tcgen05 / TMEM).
//
// Replaces the reference's CUDA-core kernel
// (csrc/sm120/decode/sparse_decode_kernel.cuh:202-403).  Same math
// (tests/reference.py:105-131): gather top-k rows by flat index, dequantise
// FP8 to bf16, S = Q K^T * scale, softmax over the positions, O = P V,
// sink epilogue.  Different machine mapping:
//
//  * One CTA = one scheduler part (a run of 128-position tiles of one or
//    more query rows, from get_mla_metadata) x one group of 64 heads.
//  * S is computed transposed, S^T[tok, head] = K_tile . Q^T, so the 128
//    tokens of a tile are the UMMA M dimension (M = 128, full tensor rate)
//    and the 64 heads are N.  O is computed transposed as well,
//    O^T[dim, head] += V^T . P^T, with V^T read MN-major straight out of
//    the same bf16 K tile (4 M-blocks of 128 dims).
//  * TMEM (512 columns): S^T [0,64), O^T [64,320), softmax row sums
//    [320,384) (ones[64 x 128] . P^T on the tensor core).
//  * Shared memory: Q^T (64 heads x d_qk bf16, 72 KB for V32) and a ring of
//    d_qk/64 chunk slots, each a 128-token x 64-column bf16 SWIZZLE_128B
//    tile (16 KB).  PV M-block m releases slots 2m, 2m+1, so the next
//    tile's dequant overlaps the current PV.  V32 writes P^T into the RoPE
//    slot (RoPE is not part of V); MODEL1 has a separate P^T buffer.
//
// Warp roles (384 threads):
//   warps 0-7   producers: per tile, each thread owns four token rows and a
//               16-byte column unit of every 128-column chunk pair; loads
//               raw FP8 / scales / RoPE with 16-byte loads one tile ahead,
//               dequantises, stores swizzled bf16; also loads Q^T at each
//               query-row change.
//   warps 8-11  softmax + epilogue: thread = token row = TMEM lane;
//               column max via redux.sync + a 4-warp exchange, lazy
//               rescaling (only when a head's max grows by > 2^8), P^T to
//               shared memory, final normalisation, sink, LSE and the
//               output / split-partial store (or the cluster merge).
//               Warp 8 allocates TMEM and its lane 0 issues every
//               tcgen05.mma, between its softmax passes.
//
// All mbarrier waits are bounded (dsv4b_ptx.cuh: mbar_wait); on a timeout
// the CTA raises an abort flag, every role leaves its loop, TMEM is freed
// and the workspace status word records kErrWaitTimeout.
#include <cuda_bf16.h>

#include <cstddef>
#include <cstdlib>

#include "dsv4b_internal.cuh"
#include "dsv4b_kernels.h"

namespace dsv4b {

// Test hook (dsv4b_set_test_stall): when set, producer thread 0 of
// every CTA withholds its first Q^T arrival, so the MMA issuer's first wait
// can only run out.  The waits themselves keep the compile-time limit
// kWaitLimitCycles: reading a limit from device memory inside them, even
// only on their slow path, measured 2 us slower per decode call on B200.
__device__ int g_decode_test_stall = 0;

#ifdef DSV4B_TRACE
// Debug-build phase trace (never in the shipped library).  The recording
// thread of each role writes (clock64 | event | arg) words with plain
// global stores for the first kTraceCtas CTAs of head group 0; the log is
// read back with dsv4b_debug_trace_read().
constexpr int kTraceCtas = 8;
__device__ unsigned long long g_trace[kTraceCtas * 3 * 128];
__shared__ unsigned long long* s_trace_base;
__shared__ int s_trace_n[3];
// Per-producer-warp log (lane 0 of warps 0-7): 64 words per warp.
__device__ unsigned long long g_trace_w[kTraceCtas * 8 * 64];
__shared__ int s_trace_wn[8];
#define DSV4B_TR_WARP(ev, a)                                                                   \
  do {                                                                                         \
    const int w_ = threadIdx.x >> 5;                                                           \
    if ((threadIdx.x & 31) == 0 && w_ < 8 && blockIdx.x < kTraceCtas && blockIdx.y == 0) {     \
      const int k_ = s_trace_wn[w_]++;                                                         \
      if (k_ < 64)                                                                             \
        g_trace_w[(blockIdx.x * 8 + w_) * 64 + k_] =                                           \
            ((unsigned long long)clock64() << 24) | ((ev) << 16) | ((unsigned)(a) & 0xFFFFu);  \
    }                                                                                          \
  } while (0)
#define DSV4B_TR_ROLE(role, ev, a)                                                        \
  do {                                                                                    \
    const int k_ = s_trace_n[role]++;                                                     \
    if (s_trace_base && k_ < 128)                                                         \
      s_trace_base[(role) * 128 + k_] =                                                   \
          ((unsigned long long)clock64() << 24) | ((ev) << 16) | ((unsigned)(a) & 0xFFFFu); \
  } while (0)
#else
#define DSV4B_TR_ROLE(role, ev, a) \
  do {                             \
  } while (0)
#define DSV4B_TR_WARP(ev, a) \
  do {                       \
  } while (0)
#endif

namespace {

constexpr int kProducerWarps = 8;
constexpr int kSoftmaxWarps = 4;
// 384 threads = 3 x 128: the register allocator then grants 168 per thread
// (a 416-thread block is allocated as 512 threads and capped at 128).
constexpr int kThreads = (kProducerWarps + kSoftmaxWarps) * 32;  // 384
constexpr int kProducerThreads = kProducerWarps * 32;
constexpr int kSoftmaxThreads = kSoftmaxWarps * 32;
constexpr int kMmaWarp = kProducerWarps;  // lane 0 of the first softmax warp issues the MMAs
// Named barriers of the cluster merge: its 256 worker threads, then each
// half's 128 (one staging tile per half).
constexpr uint32_t kMergeBar = 3;

constexpr int kQChunkBytes = kHeadsPerCta * 128;       // 8 KB
constexpr int kSlotBytes = kTileTokens * 128;          // 16 KB
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0, kColO = 64, kColL = 320;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct Misc {
  // Epilogue transpose tile (8 KB).  Between epilogues it holds bf16 ones:
  // the A operand of the row-sum UMMA (ones[64 x 128 tok] . P^T), so it
  // sits at offset 0, 1024-byte aligned like every SW128 operand.
  __nv_bfloat16 stage[32][128];
  uint64_t full[9];
  uint64_t empty[5];
  uint64_t s_full, p_full, q_full, q_empty, o_full;
  uint64_t drain;  // end of the MMA issuer's tcgen05 work (abort path)
  uint32_t tmem_base;
  int abort;
  uint32_t cl_live;    // cluster epilogue: bit i = cluster rank i holds a partial
  int q_loads;         // Q^T loads issued (thread 0); the abort path waits for the last
  alignas(16) float red[4][64];
  alignas(16) float m_use[64];    // read as float4
  alignas(16) float alpha[64];
  alignas(16) float scale_o[64];
};
static_assert(offsetof(Misc, red) % 16 == 0 && offsetof(Misc, m_use) % 16 == 0 &&
                  offsetof(Misc, alpha) % 16 == 0 && offsetof(Misc, scale_o) % 16 == 0,
              "Misc float arrays must be 16-byte aligned (vector shared-memory loads)");
static_assert(offsetof(Misc, stage) == 0, "stage must start Misc (SW128 operand)");
static_assert(sizeof(Misc) % 16 == 0, "Misc size");

template <int L>
struct SmemPlan {
  static constexpr int kChunks = LayoutT<L>::kChunks;
  static constexpr int kQOff = 0;
  static constexpr int kSlotOff = kChunks * kQChunkBytes;
  static constexpr int kPOff = LayoutT<L>::kPInRopeSlot ? kSlotOff + (kChunks - 1) * kSlotBytes
                                                        : kSlotOff + kChunks * kSlotBytes;
  static constexpr int kMiscOff =
      kSlotOff + kChunks * kSlotBytes + (LayoutT<L>::kPInRopeSlot ? 0 : kSlotBytes);
  static constexpr int kBytes = kMiscOff + (int)sizeof(Misc) + 1024;  // + alignment slack
};

static_assert(SmemPlan<DSV4B_LAYOUT_V32>::kMiscOff % 1024 == 0 &&
                  SmemPlan<DSV4B_LAYOUT_MODEL1>::kMiscOff % 1024 == 0,
              "Misc must be 1024-byte aligned");
// The cluster merge receives 512 dims x 64 heads fp32 (128 KB) in the K slots.
static_assert(SmemPlan<DSV4B_LAYOUT_V32>::kMiscOff - SmemPlan<DSV4B_LAYOUT_V32>::kSlotOff >= 131072 &&
                  SmemPlan<DSV4B_LAYOUT_MODEL1>::kMiscOff - SmemPlan<DSV4B_LAYOUT_MODEL1>::kSlotOff >= 131072,
              "cluster receive area");
static_assert(SmemPlan<DSV4B_LAYOUT_V32>::kBytes <= 232448, "V32 smem plan too large");
static_assert(SmemPlan<DSV4B_LAYOUT_MODEL1>::kBytes <= 232448, "MODEL1 smem plan too large");

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  const __nv_bfloat162 o = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&o);
}

// Empty barrier guarding chunk slot c.
template <int L>
__device__ __forceinline__ int empty_of(int c) {
  return (LayoutT<L>::kPInRopeSlot && c == LayoutT<L>::kChunks - 1) ? 4 : (c >> 1);
}

// ------------------------------------------------------------- Q^T load
// Q^T of query row (b, s), head group g: NCH TMA tile loads (64 columns x
// 64 heads, SWIZZLE_128B, straight into the chunk's 1024-byte-aligned
// slot) from the 4-D q tensor map [b][s][h][d_qk], completing on q_full.
// Issued by one thread: a TMA load bypasses the load/store path the row
// gather saturates (a cp.async Q^T load shared it and delayed the first
// tile by ~2 us).  Heads past h_q read as zeros (out of the tensor).
template <int NCH>
__device__ __forceinline__ void load_q_tma(const CUtensorMap* q_map, uint32_t q_s, int g, const TileCursor& c,
                                           Misc& M) {
  mbar_arrive_expect_tx_relaxed(&M.q_full, NCH * kQChunkBytes);
#pragma unroll
  for (int ch = 0; ch < NCH; ++ch)
    tma_load_4d(q_s + ch * kQChunkBytes, q_map, ch * 64, g * kHeadsPerCta, c.ri.s, c.ri.b, &M.q_full);
  ++M.q_loads;
}

// ------------------------------------------------------------- producers
// Gather mapping.  Producer warp w owns tile rows 16w..16w+15 and handles
// four of them per pass: in pass k lane l works on row 16w + 4k + (l >> 3)
// and on the 16-byte column q = l & 7 of a 128-byte block of that row.  A
// warp load instruction therefore reads four rows x 128 contiguous bytes
// (whole 32-byte sectors), and the unit of work is a "chunk pair": 128
// columns = two 64-column SW128 chunk slots = one V32 scale tile = the slot
// pair one PV M-block releases.
//
// Loads are pipelined pair by pair: right after a thread has stored chunk
// pair m of tile t, it issues the loads of pair m of tile t+1 into the same
// registers, so every load has about a whole tile period to land and the
// load-store path sees a steady trickle instead of one burst per tile.  An
// mbarrier arrive does not wait for the thread's loads in flight (measured
// on B200: a release arrive with 24 loads outstanding takes ~100 cycles),
// so the hand-offs are not delayed by them.  The scales of tile t+1 are
// loaded once pair 3 of tile t (their last user) is stored, the V32 RoPE
// chunk once its slot has been filled, and the indices of tile t+2 last.
constexpr int kRowsPerThread = 4;

template <int L>
struct ProdRegs {
  RowSrc rs[kRowsPerThread];
  uint4 f[4][kRowsPerThread];  // chunk pairs 0-3 (MODEL1 pair 3: fp8 or RoPE part 0)
  uint4 sc[kRowsPerThread];    // V32: 4 fp32 scales; MODEL1: 8 UE8M0 bytes in .x/.y
  uint4 rp[kRowsPerThread];    // V32 RoPE; MODEL1 RoPE part 1
};

// Flat cache index of tile row r, or -1 for padding (>= the row's attended
// length), which decodes to a zero row.
__device__ __forceinline__ int producer_index(const dsv4b_decode_params& p, const TileCursor& c,
                                              int r) {
  const TileSpan ts = tile_span(p, c);
  return r < ts.npos ? __ldg(ts.idx + r) : -1;
}

__device__ __forceinline__ uint4 ldg_or_zero(bool ok, const uint8_t* ptr) {
  return ok ? ldg_nc_v4(ptr) : make_uint4(0, 0, 0, 0);
}

template <int L>
__device__ __forceinline__ void rows_of(const dsv4b_decode_params& p, const TileCursor& c,
                                        const int (&idx)[kRowsPerThread], ProdRegs<L>& R) {
  const TileSpan ts = tile_span(p, c);
#pragma unroll
  for (int k = 0; k < kRowsPerThread; ++k)
    R.rs[k] = row_src<L>(ts.kv, ts.page, ts.stride_block, ts.stride_row, ts.num_tokens, idx[k], true);
}

// Lane q's 16 bytes of chunk pair m of each of its rows (MODEL1 pair 3,
// lanes 4-7: the 64 bf16 RoPE columns, 32 bytes per lane).
template <int L>
__device__ __forceinline__ void load_pair(int m, int q, ProdRegs<L>& R) {
#pragma unroll
  for (int k = 0; k < kRowsPerThread; ++k) {
    const RowSrc& r = R.rs[k];
    if (L == DSV4B_LAYOUT_MODEL1 && m == 3 && q >= 4) {
      R.f[3][k] = ldg_or_zero(r.valid, r.rec + LayoutT<L>::kRopeOffset + 32 * (q - 4));
      R.rp[k] = ldg_or_zero(r.valid, r.rec + LayoutT<L>::kRopeOffset + 32 * (q - 4) + 16);
    } else {
      R.f[m][k] = ldg_or_zero(r.valid, r.rec + 128 * m + 16 * q);
    }
  }
}

template <int L>
__device__ __forceinline__ void load_scales_all(ProdRegs<L>& R) {
#pragma unroll
  for (int k = 0; k < kRowsPerThread; ++k) R.sc[k] = load_scales<L>(R.rs[k]);
}

template <int L>
__device__ __forceinline__ void load_rope_v32(int q, ProdRegs<L>& R) {
#pragma unroll
  for (int k = 0; k < kRowsPerThread; ++k)
    R.rp[k] = ldg_or_zero(R.rs[k].valid, R.rs[k].rec + LayoutT<L>::kRopeOffset + 16 * q);
}

// Scale of the 16 columns lane q holds in chunk pair m.
template <int L>
__device__ __forceinline__ float pair_scale(const uint4& sc, int m, int q) {
  if constexpr (L == DSV4B_LAYOUT_V32) {
    return __uint_as_float(m == 0 ? sc.x : m == 1 ? sc.y : m == 2 ? sc.z : sc.w);
  } else {
    const int byte = 2 * m + (q >> 2);  // 64-column UE8M0 tiles
    const uint32_t w = byte < 4 ? sc.x : sc.y;
    return ue8m0_to_f32((w >> (8 * (byte & 3))) & 0xFFu);
  }
}

// Dequantises lane q's 16 e4m3 of chunk pair m of one row into its two
// 16-byte units of chunk slot 2m + q/4.  Lanes 4-7 (the second slot) store
// their high unit first, so each store instruction covers all eight
// 16-byte granules of a row (no bank conflict between the two slots).
__device__ __forceinline__ void store_pair_fp8(uint32_t slot_s, int m, int row, int q, uint4 v,
                                               float s) {
  uint4 lo, hi;
  dq16(v, s, lo, hi);
  const uint32_t slot = slot_s + (2 * m + (q >> 2)) * kSlotBytes;
  const int u = 2 * (q & 3);
  const bool swap = (q & 4) != 0;
  sts_v4(slot + sw128_off(row, u + (swap ? 1 : 0)), swap ? hi : lo);
  sts_v4(slot + sw128_off(row, u + (swap ? 0 : 1)), swap ? lo : hi);
}

template <int L>
__device__ void run_producer(const dsv4b_decode_params& p, const dsv4b_sched_meta& sm, int g,
                             uint32_t q_s, uint32_t slot_s, Misc& M, int* err, const CUtensorMap* q_map) {
  using LT = LayoutT<L>;
  constexpr int NCH = LT::kChunks;
  const int ptid = threadIdx.x;
  const int w = ptid >> 5, lane = ptid & 31;
  const int q = lane & 7;
  const int row0 = 16 * w + (lane >> 3);  // row of pass k: row0 + 4k

  TileCursor cur = cursor_begin(p, sm);
  if (!cur.valid) return;
  TileCursor nxt = cursor_next(p, sm, cur);

  // Test hook (read here, off the critical path: the load completes
  // while the first tile's rows are in flight).
  const bool withhold_first_q = ptid == 0 && g_decode_test_stall != 0;
  // The first row's Q^T is in flight together with the first tile's loads.
  if (ptid == 0 && !withhold_first_q) load_q_tma<NCH>(q_map, q_s, g, cur, M);

  ProdRegs<L> R;
  int idx[kRowsPerThread];
  if (ptid == 0) DSV4B_TR_ROLE(0, 42, cur.t);
#pragma unroll
  for (int k = 0; k < kRowsPerThread; ++k) idx[k] = producer_index(p, cur, row0 + 4 * k);
  rows_of<L>(p, cur, idx, R);
  if (ptid == 0) DSV4B_TR_ROLE(0, 43, idx[0] & 0xFFFF);
#pragma unroll
  for (int m = 0; m < 4; ++m) load_pair<L>(m, q, R);
  load_scales_all<L>(R);
  if constexpr (LT::kPInRopeSlot) load_rope_v32<L>(q, R);
#pragma unroll
  for (int k = 0; k < kRowsPerThread; ++k) idx[k] = nxt.valid ? producer_index(p, nxt, row0 + 4 * k) : -1;

  int tile_count = 0, seg_count = 0;
  volatile int* abort_flag = &M.abort;
  while (cur.valid) {
    if (cur.t == cur.t_lo) {
      // New query row: (re)load Q^T once the previous row's last QK^T is done.
      if (seg_count > 0 && ptid == 0) {
        if (!mbar_wait(&M.q_empty, (seg_count - 1) & 1, abort_flag, err)) return;
        load_q_tma<NCH>(q_map, q_s, g, cur, M);
      }
      if (ptid == 0) DSV4B_TR_ROLE(0, 5, seg_count);
      ++seg_count;
    }
    if (ptid == 0) DSV4B_TR_ROLE(0, 1, tile_count);
    const uint32_t wait_par = (tile_count - 1) & 1;
    const bool more = nxt.valid;
    // This tile's loads are all issued: the row addresses of the next tile
    // (its indices were loaded during the previous tile) take their place.
    if (more) rows_of<L>(p, nxt, idx, R);
    if (more && q == 0) {
      // The next tile's rows into L2 now (one bulk prefetch per row by the
      // TMA unit, no load-path slot): its pair loads, issued one by one as
      // this tile's pairs are stored, then hit L2 (config 1 45.1 -> 43.0 us,
      // config 4 376 -> 362 us).
      uint32_t bytes;
      if constexpr (L == DSV4B_LAYOUT_V32) bytes = LayoutT<L>::kRecordBytes; else bytes = LayoutT<L>::kRowBytes;
#pragma unroll
      for (int k = 0; k < kRowsPerThread; ++k)
        if (R.rs[k].valid) prefetch_l2_bulk(R.rs[k].rec, bytes);
    }

#pragma unroll
    for (int m = 0; m < 4; ++m) {
      DSV4B_TR_WARP(55, m);
      if (tile_count > 0 && !mbar_wait(&M.empty[m], wait_par, abort_flag, err)) return;
      DSV4B_TR_WARP(51, m);
#pragma unroll
      for (int k = 0; k < kRowsPerThread; ++k) {
        const int row = row0 + 4 * k;
        if (L == DSV4B_LAYOUT_MODEL1 && m == 3 && q >= 4) {
          const uint32_t slot = slot_s + 7 * kSlotBytes;  // MODEL1 RoPE chunk
          sts_v4(slot + sw128_off(row, 2 * (q - 4)), R.f[3][k]);
          sts_v4(slot + sw128_off(row, 2 * (q - 4) + 1), R.rp[k]);
        } else {
          store_pair_fp8(slot_s, m, row, q, R.f[m][k], pair_scale<L>(R.sc[k], m, q));
        }
      }
      DSV4B_TR_WARP(56, m);
      fence_proxy_async_smem();
      mbar_arrive(&M.full[2 * m]);
      mbar_arrive(&M.full[2 * m + 1]);
      DSV4B_TR_WARP(52, m);
      if (ptid == 0) DSV4B_TR_ROLE(0, 2, 2 * m + 1);
      if (more) load_pair<L>(m, q, R);
    }
    if constexpr (LT::kPInRopeSlot) {
      // V32 RoPE chunk (slot NCH-1, shared with P^T): after the previous PV.
      DSV4B_TR_WARP(55, 4);
      if (tile_count > 0 && !mbar_wait(&M.empty[4], wait_par, abort_flag, err)) return;
      DSV4B_TR_WARP(51, 4);
      const uint32_t slot = slot_s + (NCH - 1) * kSlotBytes;
#pragma unroll
      for (int k = 0; k < kRowsPerThread; ++k) sts_v4(slot + sw128_off(row0 + 4 * k, q), R.rp[k]);
      DSV4B_TR_WARP(56, 4);
      fence_proxy_async_smem();
      mbar_arrive(&M.full[NCH - 1]);
      DSV4B_TR_WARP(52, 4);
      if (ptid == 0) DSV4B_TR_ROLE(0, 2, NCH - 1);
      if (more) load_rope_v32<L>(q, R);
    }
    const TileCursor nn = cursor_next(p, sm, nxt);
    if (more) {
      load_scales_all<L>(R);
#pragma unroll
      for (int k = 0; k < kRowsPerThread; ++k) idx[k] = nn.valid ? producer_index(p, nn, row0 + 4 * k) : -1;
    }
    if (ptid == 0) DSV4B_TR_ROLE(0, 6, tile_count);

    cur = nxt;
    nxt = nn;
    ++tile_count;
  }
}

// ------------------------------------------------------------- prefill producer
// Sparse prefill (bf16 KV rows): nothing to dequantise, the producers copy
// each row's 16-byte units into the swizzled chunk slots.  Same mapping as
// the decode gather (warp w: rows 16w + 4k + (lane >> 3); lane q = lane & 7
// takes columns 128m + 16q .. +15 of chunk pair m, i.e. 32 bytes), in two
// register halves per tile (pairs 0-1, then pairs 2-3 and the 576-column
// RoPE chunk): a thread's release arrive waits for its loads in flight, so
// each half is loaded, landed and stored before the next is issued.  The
// rows of the next tile are prefetched into L2 at the start of each tile.
// Invalid positions are copied as zeros; the softmax leaves them out.
template <int L>
__device__ void run_producer_bf16(const dsv4b_decode_params& p, const dsv4b_sched_meta& sm, int g,
                                  uint32_t q_s, uint32_t slot_s, Misc& M, int* err, const CUtensorMap* q_map) {
  using LT = LayoutT<L>;
  constexpr int NCH = LT::kChunks;
  const int ptid = threadIdx.x;
  const int w = ptid >> 5, lane = ptid & 31;
  const int q = lane & 7;
  const int row0 = 16 * w + (lane >> 3);
  volatile int* abort_flag = &M.abort;
  const bool withhold_first_q = ptid == 0 && g_decode_test_stall != 0;

  TileCursor cur = cursor_begin(p, sm);
  if (!cur.valid) return;

  // Address of tile row r, or nullptr for an invalid position.
  auto row_ptr = [&](const TileCursor& c, int r) -> const uint8_t* {
    if (!c.valid) return nullptr;
    const TileSpan ts = tile_span(p, c);
    const int lim = min(ts.npos, c.ri.len_valid - c.t * kTileTokens);
    const int ix = r < lim ? __ldg(ts.idx + r) : -1;
    return (ix >= 0 && ix < ts.num_tokens) ? ts.kv + (int64_t)ix * ts.stride_block : nullptr;
  };
  const uint4 z = make_uint4(0, 0, 0, 0);
  auto ld = [&](const uint8_t* s, int off) { return s ? ldg_nc_v4(s + off) : z; };
  // Stores lane q's 16 columns of pair m of one row (units lo, hi) where
  // the decode gather puts its dequantised pair (store_pair_fp8).
  auto st_pair = [&](int m, int row, uint4 lo, uint4 hi) {
    const uint32_t slot = slot_s + (2 * m + (q >> 2)) * kSlotBytes;
    const int u = 2 * (q & 3);
    const bool swap = (q & 4) != 0;
    sts_v4(slot + sw128_off(row, u + (swap ? 1 : 0)), swap ? hi : lo);
    sts_v4(slot + sw128_off(row, u + (swap ? 0 : 1)), swap ? lo : hi);
  };

  const uint8_t* src[kRowsPerThread];
#pragma unroll
  for (int k = 0; k < kRowsPerThread; ++k) src[k] = row_ptr(cur, row0 + 4 * k);
  if (ptid == 0 && !withhold_first_q) load_q_tma<NCH>(q_map, q_s, g, cur, M);
  int tile = 0, seg = 0;
  while (cur.valid) {
    if (cur.t == cur.t_lo) {
      // New query row: (re)load Q^T once the previous row's last QK^T is done.
      if (seg > 0 && ptid == 0) {
        if (!mbar_wait(&M.q_empty, (seg - 1) & 1, abort_flag, err)) break;
        load_q_tma<NCH>(q_map, q_s, g, cur, M);
      }
      ++seg;
    }
    const TileCursor nxt = cursor_next(p, sm, cur);
    if (ptid < kTileTokens) {  // the next tile's rows into L2
      const uint8_t* r = row_ptr(nxt, ptid);
      if (r) prefetch_l2_bulk(r, (uint32_t)LT::kDqk * 2u);
    }
    const uint32_t par = (tile - 1) & 1;
    bool ok = true;
#pragma unroll
    for (int h = 0; h < 2 && ok; ++h) {  // pairs 2h, 2h + 1
      uint4 v[2][kRowsPerThread][2];
#pragma unroll
      for (int mm = 0; mm < 2; ++mm)
#pragma unroll
        for (int k = 0; k < kRowsPerThread; ++k) {
          const int m = 2 * h + mm;
          v[mm][k][0] = ld(src[k], 256 * m + 32 * q);
          v[mm][k][1] = ld(src[k], 256 * m + 32 * q + 16);
        }
#pragma unroll
      for (int mm = 0; mm < 2; ++mm) {
        const int m = 2 * h + mm;
        if (tile > 0 && !mbar_wait(&M.empty[m], par, abort_flag, err)) {
          ok = false;
          break;
        }
#pragma unroll
        for (int k = 0; k < kRowsPerThread; ++k) st_pair(m, row0 + 4 * k, v[mm][k][0], v[mm][k][1]);
        fence_proxy_async_smem();
        mbar_arrive(&M.full[2 * m]);
        mbar_arrive(&M.full[2 * m + 1]);
      }
    }
    if (!ok) break;
    if constexpr (LT::kPInRopeSlot) {
      // RoPE chunk (columns 512..575; its slot holds P^T during PV)
      uint4 rp[kRowsPerThread];
#pragma unroll
      for (int k = 0; k < kRowsPerThread; ++k) rp[k] = ld(src[k], 1024 + 16 * q);
      if (tile > 0 && !mbar_wait(&M.empty[4], par, abort_flag, err)) break;
      const uint32_t slot = slot_s + (NCH - 1) * kSlotBytes;
#pragma unroll
      for (int k = 0; k < kRowsPerThread; ++k) sts_v4(slot + sw128_off(row0 + 4 * k, q), rp[k]);
      fence_proxy_async_smem();
      mbar_arrive(&M.full[NCH - 1]);
    }
#pragma unroll
    for (int k = 0; k < kRowsPerThread; ++k) src[k] = row_ptr(nxt, row0 + 4 * k);
    cur = nxt;
    ++tile;
  }
  cp_async_wait_all();  // no copy may land after the CTA exits
}

// ------------------------------------------------------------- MMA issuer
// One thread (lane 0 of the first softmax warp) issues every tcgen05.mma,
// between that warp's softmax passes: QK^T of tile t+1 follows PV of tile
// t, which follows the softmax of tile t, so no MMA is delayed by sharing
// the warp.
struct MmaState {
  int tile_count = 0, seg_count = 0;
};

// S^T[128 tok, 64 heads] = K_tile[128, d_qk] . Q^T (K-major A and B), chunk
// by chunk as the producers land them.
// One lane of the converged MMA warp (the lowest active one) issues each
// group of tcgen05.mma / tcgen05.commit; issuing from a converged warp
// measured slightly faster on B200 than a lane-0-only branch.
__device__ __forceinline__ bool elect_one() {
  uint32_t e;
  asm volatile("{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\tselp.u32 %0, 1, 0, e;\n\t}" : "=r"(e));
  return e != 0;
}
// mbarrier wait whose result is uniform across the (converged) MMA warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err) {
  const bool ok = mbar_wait(bar, parity, abort_flag, err);
  return __all_sync(0xffffffffu, ok);
}

template <int L>
__device__ bool mma_qk(const TileCursor& cur, const MmaState& st, uint32_t q_s, uint32_t slot_s,
                       uint32_t tmem, Misc& M, int* err) {
  constexpr int NCH = LayoutT<L>::kChunks;
  constexpr uint32_t idesc_qk = idesc_bf16_f32(128, 64, false, false);
  volatile int* abort_flag = &M.abort;
  if (cur.t == cur.t_lo && !warp_wait(&M.q_full, st.seg_count & 1, abort_flag, err)) return false;
  for (int c = 0; c < NCH; ++c) {
    if (!warp_wait(&M.full[c], st.tile_count & 1, abort_flag, err)) return false;
    if ((threadIdx.x & 31) == 0) DSV4B_TR_ROLE(1, 10, c);
    tc_fence_after();
    if (elect_one()) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t ad = sdesc_sw128(slot_s + c * kSlotBytes + kk * 32, 16, 1024);
        const uint64_t bd = sdesc_sw128(q_s + c * kQChunkBytes + kk * 32, 16, 1024);
        umma_bf16_ss(tmem + kColS, ad, bd, idesc_qk, (c | kk) != 0);
      }
    }
    __syncwarp();
  }
  if (elect_one()) {
    umma_commit(&M.s_full);
    if (cur.t + 1 == cur.t_hi) umma_commit(&M.q_empty);
  }
  __syncwarp();
  if ((threadIdx.x & 31) == 0) DSV4B_TR_ROLE(1, 11, st.tile_count);
  return true;
}

// O^T[512 dims, 64 heads] += V^T[dims, 128 tok] . P^T[128 tok, heads], then
// the row sums; releases the chunk slots M-block by M-block.
template <int L>
__device__ bool mma_pv(const TileCursor& cur, const MmaState& st, uint32_t slot_s, uint32_t p_s,
                       uint32_t tmem, Misc& M, int* err) {
  constexpr uint32_t idesc_pv = idesc_bf16_f32(128, 64, true, true);
  constexpr uint32_t idesc_sum = idesc_bf16_f32(64, 64, false, true);
  const uint32_t ones_s = smem_u32(&M.stage[0][0]);
  const bool seg_first = cur.t == cur.t_lo;
  if (!warp_wait(&M.p_full, st.tile_count & 1, &M.abort, err)) return false;
  if ((threadIdx.x & 31) == 0) DSV4B_TR_ROLE(1, 12, st.tile_count);
  tc_fence_after();
  if (elect_one()) {
#pragma unroll 1
  for (int m = 0; m < 4; ++m) {
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint64_t ad = sdesc_sw128(slot_s + (2 * m) * kSlotBytes + kk * 2048, kSlotBytes, 1024);
      const uint64_t bd = sdesc_sw128(p_s + kk * 2048, 8192, 1024);
      umma_bf16_ss(tmem + kColO + 64 * m, ad, bd, idesc_pv, !(seg_first && kk == 0));
    }
    umma_commit(&M.empty[m]);
  }
  // Row sums on the tensor core: L[64 x heads] += ones[64 x 128 tok] .
  // P^T, so every row of L (TMEM lane 0 included) holds sum_tok P for
  // each head, summed from the same bf16 P that enters O.
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    umma_bf16_ss(tmem + kColL, sdesc_sw128(ones_s, 16, 1024), sdesc_sw128(p_s + kk * 2048, 8192, 1024),
                 idesc_sum, !(seg_first && kk == 0));
  if (LayoutT<L>::kPInRopeSlot) umma_commit(&M.empty[4]);
  if (cur.t + 1 == cur.t_hi) umma_commit(&M.o_full);
  }
  __syncwarp();
  if ((threadIdx.x & 31) == 0) DSV4B_TR_ROLE(1, 13, st.tile_count);
  return true;
}

// ------------------------------------------------------------- softmax
__device__ __forceinline__ void apply_sink(float sink, int lse_includes_sink, float& lse,
                                           float& scale) {
  // tests/reference.py:124-129
  scale *= 1.0f / (1.0f + expf(sink - lse));
  if (lse_includes_sink) {
    const float m = fmaxf(lse, sink);
    lse = m + logf(expf(lse - m) + expf(sink - m));
  }
}

// Epilogue of one (query row, split): row sums, LSE (+ sink for a row
// finished in this CTA), then either the bf16 output (whole row here) or
// the fp32 split partial [split][h_q][512 dims].
__device__ __forceinline__ void epilogue(const dsv4b_decode_params& p, const dsv4b_sched_meta& sm,
                                         int g, const TileCursor& cur, float m_run,
                                         const int32_t* num_splits, float* lse_accum, float* o_accum,
                                         uint32_t tl, Misc& M) {
  const int st = threadIdx.x - kProducerThreads;
  const int q = st >> 5, lane = st & 31;
  // Row sums: the row-sum UMMA left sum_tok P of head j in column kColL + j
  // of every row; warp 0 reads TMEM lane 0.
  if (q == 0) {
    float lv[64];
    tmem_ld64(tl + kColL, lv);
    tc_wait_ld();
    if (lane == 0) {
#pragma unroll
      for (int j = 0; j < 64; ++j) M.red[0][j] = lv[j];
    }
  }
  named_bar_sync(1, kSoftmaxThreads);
  const bool final_out = (cur.t_lo == 0 && cur.t_hi == cur.ri.nt);
  const int split = (cur.req == sm.begin_req_idx) ? sm.begin_split_idx : __ldg(num_splits + cur.req);
  if (st < 64) {
    const float l = M.red[0][st];
    const int head = g * kHeadsPerCta + st;
    float lse = (m_run + log2f(l)) * kLn2;
    float scale = 1.0f / l;
    const bool empty = p.prefill && !(l > 0.0f);  // no valid position (prefill)
    if (empty) {  // FlashMLA sparse prefill: lse = +inf, max_logits = -inf, output 0
      lse = INFINITY;
      scale = 0.0f;
    }
    if (head < p.h_q) {
      if (final_out) {
        if (p.attn_sink && !empty) apply_sink(__ldg(p.attn_sink + head), p.lse_includes_sink, lse, scale);
        p.lse[((int64_t)cur.ri.b * p.h_q + head) * p.s_q + cur.ri.s] = lse;
        if (p.max_logits)
          p.max_logits[((int64_t)cur.ri.b * p.s_q + cur.ri.s) * p.h_q + head] = empty ? -INFINITY : m_run * kLn2;
      } else {
        lse_accum[(int64_t)split * p.h_q + head] = lse;
      }
    } else {
      scale = 0.0f;
    }
    M.scale_o[st] = scale;
  }
  named_bar_sync(1, kSoftmaxThreads);
  if (final_out) {
    // bf16 [heads, dims] through a 32-head x 128-dim staging tile so the
    // global stores are 16-byte and contiguous along dims.
    __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out) + (int64_t)cur.ri.b * p.stride_o_b +
                         (int64_t)cur.ri.s * p.stride_o_s;
    const int r = st >> 2, part = st & 3;
#pragma unroll 1
    for (int mh = 0; mh < 8; ++mh) {  // 4 M-blocks x 2 head halves
      const int m = mh >> 1, hf = mh & 1;
      float ov[32];
      tmem_ld32(tl + kColO + 64 * m + 32 * hf, ov);
      tc_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) M.stage[j][st] = __float2bfloat16_rn(ov[j] * M.scale_o[32 * hf + j]);
      named_bar_sync(1, kSoftmaxThreads);
      const int head = g * kHeadsPerCta + 32 * hf + r;
      if (head < p.h_q) {
        uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)head * p.stride_o_h + 128 * m + 32 * part);
        const uint4* src = reinterpret_cast<const uint4*>(&M.stage[r][32 * part]);
#pragma unroll
        for (int k = 0; k < 4; ++k) dst[k] = src[k];
      }
      named_bar_sync(1, kSoftmaxThreads);
    }
  } else {
    // fp32 partial [split][h_q][512]: thread st holds dim 128 m + st of each
    // M-block for all 64 heads, so one store per head is already coalesced
    // (a warp's 32 adjacent dims write 128 contiguous bytes); no staging.
    const int hmax = min(kHeadsPerCta, p.h_q - g * kHeadsPerCta);
    float* dst = o_accum + ((int64_t)split * p.h_q + g * kHeadsPerCta) * kDv;
#pragma unroll 1
    for (int m = 0; m < 4; ++m) {
      float ov[64];
      tmem_ld64(tl + kColO + 64 * m, ov);
      tc_wait_ld();
      const int d = 128 * m + st;
#pragma unroll
      for (int j = 0; j < 64; ++j)
        if (j < hmax) dst[(int64_t)j * kDv + d] = ov[j] * M.scale_o[j];
    }
  }
}

// Writes bf16 ones over the staging tile (the row-sum UMMA's A operand)
// and makes them visible to the tensor core.
__device__ __forceinline__ void fill_ones(Misc& M, int st) {
  uint4* dst = reinterpret_cast<uint4*>(&M.stage[0][0]);
  const uint4 one = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);
#pragma unroll
  for (int i = st; i < (int)(sizeof(M.stage) / 16); i += kSoftmaxThreads) dst[i] = one;
  fence_proxy_async_smem();
}

// Per-head stabiliser update: column max of the tile via redux.sync and a
// 4-warp exchange, m_use / alpha for every head, and, when some head's max
// rose by more than 2^8 after the row's first tile, the rescale of that
// head's O and row-sum columns in TMEM.
__device__ __forceinline__ void softmax_max_path(uint32_t tl, float row_scale, bool seg_first,
                                                 float& m_run, Misc& M, float thr) {
  const int st = threadIdx.x - kProducerThreads;
  const int q = st >> 5, lane = st & 31;
  {
    float sv[64];
    tmem_ld64(tl + kColS, sv);
    tc_wait_ld();
#pragma unroll
    for (int j = 0; j < 64; ++j) {
      const float mx = warp_max_f32(row_scale != 0.0f ? sv[j] * row_scale : -INFINITY);
      if (lane == 0) M.red[q][j] = mx;
    }
  }
  named_bar_sync(1, kSoftmaxThreads);
  bool resc = false;
  if (st < 64) {
    const float mt = fmaxf(fmaxf(M.red[0][st], M.red[1][st]), fmaxf(M.red[2][st], M.red[3][st]));
    const float m_old = m_run;
    float m_new = m_old, alpha = 1.0f;
    if (m_old == -INFINITY) {
      m_new = mt;
    } else if (mt > m_old + thr) {
      m_new = mt;
      alpha = fast_exp2(m_old - m_new);
      resc = true;
    }
    m_run = m_new;
    M.m_use[st] = (m_new == -INFINITY) ? 0.0f : m_new;
    M.alpha[st] = alpha;
  }
  const bool any_resc = named_bar_or(1, kSoftmaxThreads, resc);
  if (any_resc && !seg_first) {
    // 4 O M-blocks (64 head columns each) + the row sums.
#pragma unroll 1
    for (int cc = 0; cc < 5; ++cc) {
      const uint32_t col = cc < 4 ? kColO + 64 * cc : kColL;
      float ov[64];
      tmem_ld64(tl + col, ov);
      tc_wait_ld();
#pragma unroll
      for (int j = 0; j < 64; ++j) ov[j] *= M.alpha[j];
      tmem_st32(tl + col, *reinterpret_cast<float(*)[32]>(&ov[0]));
      tmem_st32(tl + col + 32, *reinterpret_cast<float(*)[32]>(&ov[32]));
    }
  }
}

// P = 2^(s * scale - m_use) rounded to bf16, stored as P^T row st in
// shared memory.  Returns whether any of this row's logits exceeds its
// head's stabiliser by more than 2^8 (the P just written is then redone).
__device__ __forceinline__ bool softmax_p_pass(uint32_t tl, float row_scale, uint32_t p_s,
                                               const Misc& M, float thr) {
  const int st = threadIdx.x - kProducerThreads;
  bool exceed = false;
  float sa[64];
  tmem_ld64(tl + kColS, sa);
  tc_wait_ld();
#pragma unroll
  for (int c16 = 0; c16 < 4; ++c16) {
    const float* sv = sa + 16 * c16;
    uint32_t pk[8];
#pragma unroll
    for (int j4 = 0; j4 < 4; ++j4) {
      const float4 mu = *reinterpret_cast<const float4*>(&M.m_use[16 * c16 + 4 * j4]);
      const float x0 = fmaf(sv[4 * j4 + 0], row_scale, -mu.x);
      const float x1 = fmaf(sv[4 * j4 + 1], row_scale, -mu.y);
      const float x2 = fmaf(sv[4 * j4 + 2], row_scale, -mu.z);
      const float x3 = fmaf(sv[4 * j4 + 3], row_scale, -mu.w);
      const bool live = row_scale != 0.0f;
      exceed |= live && (fmaxf(fmaxf(x0, x1), fmaxf(x2, x3)) > thr);
      pk[2 * j4] = pack_bf16(live ? fast_exp2(x0) : 0.0f, live ? fast_exp2(x1) : 0.0f);
      pk[2 * j4 + 1] = pack_bf16(live ? fast_exp2(x2) : 0.0f, live ? fast_exp2(x3) : 0.0f);
    }
    sts_v4(p_s + sw128_off(st, 2 * c16), make_uint4(pk[0], pk[1], pk[2], pk[3]));
    sts_v4(p_s + sw128_off(st, 2 * c16 + 1), make_uint4(pk[4], pk[5], pk[6], pk[7]));
  }
  return exceed && row_scale != 0.0f;
}

// (m, l) of head j for the cluster merge, adjacent so that a peer reads
// both with one distributed-shared-memory load (red[2..3]; the max-path
// exchange rows are free once the row's last tile is done).
__device__ __forceinline__ float2* merge_ml(Misc& M) { return reinterpret_cast<float2*>(&M.red[2][0]); }

// Cluster plan: instead of the epilogue, publish this CTA's per-head
// stabiliser and row sum (merge_ml) for the cluster merge.
__device__ __forceinline__ void publish_partial(uint32_t tl, float m_run, Misc& M) {
  const int st = threadIdx.x - kProducerThreads;
  if ((st >> 5) == 0) {
    float lv[64];
    tmem_ld64(tl + kColL, lv);
    tc_wait_ld();
    if (st == 0) {
#pragma unroll
      for (int j = 0; j < 64; ++j) merge_ml(M)[j].y = lv[j];
    }
  }
  if (st < 64) merge_ml(M)[st].x = m_run;
}

// The softmax threads leave on a wait failure only all together: each
// thread's own bounded wait can give up at a slightly different moment (its
// time limit, or the CTA abort flag raised by another role, possibly just
// as the barrier completes), and a thread that went on while another left
// would wait forever at the group's next named barrier.  group_ok() ORs
// the failures over named barrier 1 (one vote, every thread gets the same
// answer).  A failed MMA issuer stops issuing but stays in the group.
__device__ __forceinline__ bool group_ok(bool ok) {
  __syncwarp();  // bar.red is warp-aligned: the lanes left their polls at different times
  return !named_bar_or(1, kSoftmaxThreads, !ok);
}

template <int L>
__device__ void run_softmax(const dsv4b_decode_params& p, const dsv4b_sched_meta& sm, int g,
                            const int32_t* num_splits, float* lse_accum, float* o_accum,
                            uint32_t q_s, uint32_t slot_s, uint32_t p_s, uint32_t tmem, Misc& M, int* err,
                            int cluster_c) {
  const int st = threadIdx.x - kProducerThreads;  // 0..127 = token row = TMEM lane
  const int q = st >> 5;
  const bool mma_lane = q == 0;  // warp kMmaWarp issues the MMAs (one elected lane)
  MmaState ms;
  const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16);
  const float scale_log2 = p.sm_scale * kLog2e;
  // Prefill reports the exact max logit: any growth of a head's max then
  // takes the stabiliser path (threshold 0), so m_run is the running max.
  const float thr = p.prefill ? 0.0f : kRescaleThreshold;
  volatile int* abort_flag = &M.abort;

  TileCursor cur = cursor_begin(p, sm);
  int tile_count = 0, seg_count = 0;
  float m_run = -INFINITY;  // stabiliser of head `st` (threads 0..63), log2 units
  if (cluster_c > 1 && !cur.valid && st < 64) {  // a cluster rank with no tiles
    merge_ml(M)[st] = make_float2(-INFINITY, 0.0f);
  }
  // MMA issue of the first tile; later tiles' QK^T follows the previous PV.
  bool mma_ok = true;  // lane 0 of warp kMmaWarp: false once an MMA-side wait gave up
  if (mma_lane && cur.valid) mma_ok = mma_qk<L>(cur, ms, q_s, slot_s, tmem, M, err);
  __syncwarp();
  while (cur.valid) {
    const bool seg_first = cur.t == cur.t_lo;
    const bool seg_last = cur.t + 1 == cur.t_hi;
    if (seg_first) m_run = -INFINITY;
    // 0 marks a row left out of the softmax: padding past the row's length,
    // and in prefill mode every invalid position (index < 0, >= the number
    // of KV rows, or past topk_length), which FlashMLA masks out.
    float row_scale = st < tile_span(p, cur).npos ? scale_log2 : 0.0f;
    if (p.prefill) {
      const TileSpan ts = tile_span(p, cur);
      const int ix = st < ts.npos ? __ldg(ts.idx + st) : -1;  // prefill has no extra (SWA) tiles
      if (st >= cur.ri.len_valid - cur.t * kTileTokens || ix < 0 || ix >= ts.num_tokens) row_scale = 0.0f;
    }

    // On a failed wait the thread still runs this tile's softmax pass on
    // whatever TMEM holds (harmless) so that the group's vote below, which
    // the pass needs anyway, also carries the failure: no extra barrier per
    // tile.
    const bool s_ok = mbar_wait(&M.s_full, tile_count & 1, abort_flag, err);
    if (st == 0) DSV4B_TR_ROLE(2, 20, tile_count);
    tc_fence_after();

    // A row's first tile sets the stabilisers.  After that the kept
    // stabilisers are used directly; only when some logit exceeds its
    // head's by more than 2^8 (a block-wide vote) are they raised, O and
    // the row sums rescaled and P recomputed.
    // (tcgen05.ld / wait::ld are .sync.aligned: every lane executes them,
    // padding rows included.)
    if (seg_first) {
      if (!group_ok(s_ok)) return;
      softmax_max_path(tl, row_scale, true, m_run, M, thr);
      softmax_p_pass(tl, row_scale, p_s, M, thr);
    } else {
      const bool exceed = softmax_p_pass(tl, row_scale, p_s, M, thr);
      __syncwarp();
      if (named_bar_or(1, kSoftmaxThreads, exceed || !s_ok)) {
        if (!group_ok(s_ok)) return;
        softmax_max_path(tl, row_scale, false, m_run, M, thr);
        softmax_p_pass(tl, row_scale, p_s, M, thr);
      }
    }
    tc_wait_st();
    fence_proxy_async_smem();
    tc_fence_before();
    mbar_arrive(&M.p_full);
    if (st == 0) DSV4B_TR_ROLE(2, 23, tile_count);
    const TileCursor nxt = cursor_next(p, sm, cur);
    if (mma_lane && mma_ok) {  // the MMA issuer's turn: PV of this tile, QK^T of the next
      mma_ok = mma_pv<L>(cur, ms, slot_s, p_s, tmem, M, err);
      if (cur.t + 1 == cur.t_hi) ++ms.seg_count;
      ++ms.tile_count;
      if (mma_ok && nxt.valid) mma_ok = mma_qk<L>(nxt, ms, q_s, slot_s, tmem, M, err);
    }
    __syncwarp();

    if (seg_last) {
      if (!group_ok(mbar_wait(&M.o_full, seg_count & 1, abort_flag, err))) return;
      if (st == 0) DSV4B_TR_ROLE(2, 24, seg_count);
      tc_fence_after();
      if (cluster_c > 1) {
        publish_partial(tl, m_run, M);
        return;  // a cluster CTA owns one segment; the merge follows the role loops
      }
      epilogue(p, sm, g, cur, m_run, num_splits, lse_accum, o_accum, tl, M);
      named_bar_sync(1, kSoftmaxThreads);  // staging tile reads done
      fill_ones(M, st);
      tc_fence_before();
      if (st == 0) DSV4B_TR_ROLE(2, 25, seg_count);
      ++seg_count;
    }
    ++tile_count;
    cur = nxt;
  }
}

// Cluster merge of one query row over the C = cluster_c CTAs that split
// it (cluster ranks 0..C-1; rank i holds m_i, l_i per head in merge_ml
// and its unnormalised O_i^T in TMEM).  With M = max_i m_i and
// L = sum_i l_i 2^(m_i - M): out = sum_i (2^(m_i - M) / L) O_i, then the
// sink epilogue (tests/reference.py:124-129), lse = (M + log2 L) ln 2.
// Rank j owns dims [j*512/C, (j+1)*512/C): every other rank stores its
// weighted O for those dims into rank j's K-slot region (free once every
// rank's PV is done) through distributed shared memory, as bf16
// [sender][head octet][dim][8 heads] (the weighted partial rounded once to
// bf16; distributed shared memory runs at about 30 GB/s per SM, so the
// bytes sent set the merge's floor), so a warp's 32 consecutive dims write
// and read 512 contiguous bytes; rank j adds its own fp32 part from TMEM
// and writes bf16.
// Every thread of the CTA calls this; all waits before it are bounded, so
// every CTA of the cluster reaches both cluster barriers.
__device__ void cluster_epilogue(const dsv4b_decode_params& p, int g, int C, uint32_t tmem,
                                 uint32_t recv_s, uint8_t* qarea, Misc& M) {
  const bool softmax = threadIdx.x >= kProducerThreads && threadIdx.x < kProducerThreads + kSoftmaxThreads;
  // The merge's data movement is latency-bound with one warp per SM
  // sub-partition, so producer warps 0-3 (idle by now; they read the same
  // TMEM lane quarters) take half of it: M-blocks 2-3 of the send and heads
  // 32-63 of the output.
  const bool helper = threadIdx.x < kSoftmaxThreads;
  const bool worker = softmax || helper;
  const int st = threadIdx.x - kProducerThreads;
  const int lane_row = softmax ? st : (int)threadIdx.x;  // TMEM lane = dim within an M-block
  const int half = helper ? 1 : 0;
  const uint32_t self = cluster_ctarank();
  const int D = kDv / C;
  const uint32_t blk_bytes = (uint32_t)D * 128u;  // one sender block: D dims x 64 heads x bf16
  const uint32_t tl = tmem + ((uint32_t)((lane_row >> 5) * 32) << 16);
  const int row = blockIdx.x / C;
  const int rb = row / p.s_q, rs = row - rb * p.s_q;

  if (st == 0) DSV4B_TR_ROLE(2, 30, 0);
  cluster_sync_all();  // 1: every rank's (m, l) is published and its PV is done
  if (st == 0) DSV4B_TR_ROLE(2, 31, 0);
  if (softmax && st < 64) {
    float mi[8], li[8];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      mi[i] = -INFINITY;
      li[i] = 0.0f;
      if (i < C) {
        const float2 ml = dsmem_ld_f32x2(dsmem_addr(smem_u32(&merge_ml(M)[st]), i));
        mi[i] = ml.x;
        li[i] = ml.y;
      }
    }
    // all C remote loads are issued above before any is used
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (li[i] > 0.0f) mx = fmaxf(mx, mi[i]);
    float l = 0.0f;
    uint32_t live = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (li[i] > 0.0f) {
        l += li[i] * fast_exp2(mi[i] - mx);
        live |= 1u << i;
      }
    float w = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i == (int)self && li[i] > 0.0f) w = fast_exp2(mi[i] - mx) / l;
    const int head = g * kHeadsPerCta + st;
    float lse = (mx + log2f(l)) * kLn2;
    if (head < p.h_q) {
      if (p.attn_sink) apply_sink(__ldg(p.attn_sink + head), p.lse_includes_sink, lse, w);
      if (self == 0) p.lse[((int64_t)rb * p.h_q + head) * p.s_q + rs] = lse;
    } else {
      w = 0.0f;
    }
    M.scale_o[st] = w;
    if (st == 0) M.cl_live = live;
  }
  if (st == 0) DSV4B_TR_ROLE(2, 35, 0);
  if (worker) named_bar_sync(kMergeBar, 2 * kSoftmaxThreads);
  if (st == 0) DSV4B_TR_ROLE(2, 36, 0);
  if (worker && ((M.cl_live >> self) & 1u)) {
#pragma unroll 1
    for (int m = 2 * half; m < 2 * half + 2; ++m) {
      const int d = 128 * m + lane_row;
      const int owner = d / D, dl = d - owner * D;
      const uint32_t dst = dsmem_addr(recv_s + self * blk_bytes + (uint32_t)dl * 16u, owner);
      float ov[64];
      tmem_ld64(tl + kColO + 64 * m, ov);
      tc_wait_ld();
      if (owner != (int)self) {
        // weighted O of 8 heads per 16-byte store, rounded to bf16: half
        // the distributed-shared-memory bytes of fp32
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float4 wa = *reinterpret_cast<const float4*>(&M.scale_o[8 * u]);
          const float4 wb = *reinterpret_cast<const float4*>(&M.scale_o[8 * u + 4]);
          const float* o8 = ov + 8 * u;
          dsmem_st_v4(dst + (uint32_t)u * (uint32_t)D * 16u,
                      __uint_as_float(pack_bf16(o8[0] * wa.x, o8[1] * wa.y)),
                      __uint_as_float(pack_bf16(o8[2] * wa.z, o8[3] * wa.w)),
                      __uint_as_float(pack_bf16(o8[4] * wb.x, o8[5] * wb.y)),
                      __uint_as_float(pack_bf16(o8[6] * wb.z, o8[7] * wb.w)));
        }
      }
    }
  }
  if (st == 0) DSV4B_TR_ROLE(2, 32, 0);
  cluster_sync_all();  // 2: every rank's contribution has landed at its owner
  if (st == 0) DSV4B_TR_ROLE(2, 33, 0);
  if (!worker) return;
  const uint32_t live = M.cl_live;
  __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out) + (int64_t)rb * p.stride_o_b +
                       (int64_t)rs * p.stride_o_s;
  const int lo = (int)self * D, hi = lo + D;
  const bool own = (live >> self) & 1u;
  // Dim d = 128 m + lane_row of each M-block in [lo, hi), heads 32*half ..
  // +31: the own weighted part from TMEM, plus every other live rank's bf16
  // part from the receive area (all loads issued before any is summed),
  // then through this half's [32 heads][128 dims] bf16 staging tile (in the
  // Q^T region, free after the last QK^T) so that the global stores are 16
  // bytes and contiguous along dims.
  __nv_bfloat16(*stage)[128] = reinterpret_cast<__nv_bfloat16(*)[128]>(qarea + half * 32 * 128 * 2);
  const int r = lane_row >> 2, part = lane_row & 3;
  // Every thread of the half runs every iteration and both barriers: with
  // C = 8 (D = 64) only half of an M-block's dims belong to this rank.
#pragma unroll 1
  for (int m = lo / 128; m * 128 < hi; ++m) {
    const int d = 128 * m + lane_row;
    const bool mine = d >= lo && d < hi;  // uniform per warp (D >= 64)
    const int dl = d - lo;
    if (mine) {
      float acc[32];
      tmem_ld32(tl + kColO + 64 * m + 32 * half, acc);
      tc_wait_ld();
      if (st == 0) DSV4B_TR_ROLE(2, 38, m);
#pragma unroll
      for (int j = 0; j < 32; ++j) acc[j] = own ? acc[j] * M.scale_o[32 * half + j] : 0.0f;
#pragma unroll 1
      for (int i = 0; i < C; ++i) {
        if (i == (int)self || !((live >> i) & 1u)) continue;
        uint32_t v[4][4];
#pragma unroll
        for (int u = 0; u < 4; ++u)  // 8 heads per 16-byte unit
          asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(v[u][0]), "=r"(v[u][1]), "=r"(v[u][2]), "=r"(v[u][3])
                       : "r"(recv_s + (uint32_t)i * blk_bytes +
                             ((uint32_t)(4 * half + u) * (uint32_t)D + (uint32_t)dl) * 16u));
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            acc[8 * u + 2 * e] += __uint_as_float(v[u][e] << 16);
            acc[8 * u + 2 * e + 1] += __uint_as_float(v[u][e] & 0xFFFF0000u);
          }
      }
      if (st == 0) DSV4B_TR_ROLE(2, 39, m);
#pragma unroll
      for (int j = 0; j < 32; ++j) stage[j][lane_row] = __float2bfloat16_rn(acc[j]);
    }
    named_bar_sync(kMergeBar + 1 + half, kSoftmaxThreads);
    const int head = g * kHeadsPerCta + 32 * half + r;
    const int dq = 128 * m + 32 * part;
    if (head < p.h_q && dq >= lo && dq < hi) {
      uint4* dst = reinterpret_cast<uint4*>(out + (int64_t)head * p.stride_o_h + dq);
      const uint4* src = reinterpret_cast<const uint4*>(&stage[r][32 * part]);
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) dst[q4] = src[q4];
    }
    named_bar_sync(kMergeBar + 1 + half, kSoftmaxThreads);
  }
  if (st == 0) DSV4B_TR_ROLE(2, 34, 0);
}

template <int L>
__global__ void __launch_bounds__(kThreads, 1)
    sparse_decode_kernel(const dsv4b_decode_params p, const dsv4b_sched_meta* __restrict__ sched,
                         const int32_t* __restrict__ num_splits, float* __restrict__ lse_accum,
                         float* __restrict__ o_accum, int* __restrict__ err, int cluster_c,
                         const __grid_constant__ CUtensorMap q_map) {
  using SP = SmemPlan<L>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base_addr = (raw_addr + 1023u) & ~1023u;
  uint8_t* base = smem_raw + (base_addr - raw_addr);
  Misc& M = *reinterpret_cast<Misc*>(base + SP::kMiscOff);
  const uint32_t q_s = base_addr + SP::kQOff;
  const uint32_t slot_s = base_addr + SP::kSlotOff;
  const uint32_t p_s = base_addr + SP::kPOff;

  const int warp = threadIdx.x >> 5;
  // A dependent combine launch may be scheduled now; it waits in-kernel
  // for this grid's completion (griddepcontrol.wait).
  asm volatile("griddepcontrol.launch_dependents;");
  // Head group and scheduler part.  Decode: grid (parts, groups).  Prefill:
  // one column of tokens x groups CTAs with a token's head groups adjacent,
  // so that they run together and the second reader of each gathered row
  // finds it in L2 (7.22 -> 7.06 ms on the prefill bench; the same order
  // measured 1 % slower for decode at config 4).
  const int ngroups = (p.h_q + kHeadsPerCta - 1) / kHeadsPerCta;
  const int g = p.prefill ? (int)blockIdx.x % ngroups : (int)blockIdx.y;
  const int part = p.prefill ? (int)blockIdx.x / ngroups : (int)blockIdx.x;

  if (threadIdx.x == 0) {
    for (int c = 0; c < 9; ++c) mbar_init(&M.full[c], kProducerThreads);
    for (int e = 0; e < 5; ++e) mbar_init(&M.empty[e], 1);
    mbar_init(&M.s_full, 1);
    mbar_init(&M.p_full, kSoftmaxThreads);
    mbar_init(&M.q_full, 1);  // one arrive (+ the Q^T bytes) per load
    M.q_loads = 0;
    mbar_init(&M.q_empty, 1);
    mbar_init(&M.o_full, 1);
    mbar_init(&M.drain, 1);
    M.abort = 0;
#ifdef DSV4B_TRACE
    s_trace_n[0] = s_trace_n[1] = s_trace_n[2] = 0;
    for (int i = 0; i < 8; ++i) s_trace_wn[i] = 0;
    s_trace_base = (blockIdx.x < kTraceCtas && blockIdx.y == 0) ? g_trace + blockIdx.x * 3 * 128 : nullptr;
    if (s_trace_base) {
      for (int i = 0; i < 3 * 128; ++i) s_trace_base[i] = 0;
      s_trace_base[0] = (unsigned long long)clock64() << 24;  // role 0 slot 0: kernel start
      s_trace_n[0] = 1;
      unsigned long long gt;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(gt));
      s_trace_base[127] = gt;  // role 0 last slot: globaltimer at start
      s_trace_base[126] = (unsigned long long)clock64();
      DSV4B_TR_ROLE(0, 44, 0);
    }
#endif
    fence_mbarrier_init();
  }
  if (warp >= kProducerWarps) fill_ones(M, threadIdx.x - kProducerThreads);
  if (warp == kMmaWarp) {
    tmem_alloc(&M.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = M.tmem_base;
  // This grid may be a programmatic dependent of the scheduler (or of the
  // previous decode): everything above touched only on-chip state; from
  // here on the prerequisite grid has completed and its writes are visible.
  if (threadIdx.x == 0) DSV4B_TR_ROLE(0, 40, 0);
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const dsv4b_sched_meta sm = sched[part];
  if (threadIdx.x == 0) DSV4B_TR_ROLE(0, 41, sm.begin_req_idx);

  if (warp < kProducerWarps) {
    if constexpr (is_bf16_layout(L)) {
      run_producer_bf16<L>(p, sm, g, q_s, slot_s, M, err, &q_map);
    } else {
      run_producer<L>(p, sm, g, q_s, slot_s, M, err, &q_map);
    }
    cp_async_wait_all();
    if (threadIdx.x == 0 && M.abort && M.q_loads > 0) {
      // aborted: the last Q^T load lands before the CTA's shared memory goes
      // away (its barrier completes on its bytes alone; bounded wait)
      const long long t0 = clock64();
      while (!mbar_try_wait(smem_u32(&M.q_full), (M.q_loads - 1) & 1) && clock64() - t0 < 2000000) {
      }
    }
  } else {
    run_softmax<L>(p, sm, g, num_splits, lse_accum, o_accum, q_s, slot_s, p_s, tmem, M, err, cluster_c);
    if (warp == kMmaWarp) {
      // Every tcgen05.mma the issuer started must be complete before shared
      // memory is reused by the cluster merge and TMEM is freed.  On the
      // normal path the last o_full commit already covered them; after an
      // abort this commit + wait does (a bounded wait that ignores the
      // abort flag: MMAs always complete, their operands are resident).
      if (threadIdx.x == kProducerThreads) umma_commit(&M.drain);
      __syncwarp();
      const long long t0 = clock64();
      while (!mbar_try_wait(smem_u32(&M.drain), 0) && clock64() - t0 < kWaitLimitCycles) {
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (cluster_c > 1) {
    tc_fence_after();
    cluster_epilogue(p, g, cluster_c, tmem, slot_s, base + SP::kQOff, M);
    tc_fence_before();
    __syncthreads();
  }
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
#ifdef DSV4B_TRACE
  if (threadIdx.x == 0 && s_trace_base) {
    unsigned long long gt;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(gt));
    s_trace_base[255] = gt;  // role 1 last slot: globaltimer at end
    s_trace_base[254] = (unsigned long long)clock64();
  }
#endif
}

template <int L>
cudaError_t set_smem_attr() {
  static bool attr_done[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_done[dev]) {
    e = cudaFuncSetAttribute(sparse_decode_kernel<L>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SmemPlan<L>::kBytes);
    if (e != cudaSuccess) return e;
    attr_done[dev] = true;
  }
  return cudaSuccess;
}

// How many clusters of c decode CTAs can be resident at once on this device
// (one CTA per SM, clusters confined to a GPC).  Cached per device.
template <int L>
int clusters_resident(int c) {
  static int cache[64][4] = {};  // 0 unknown, else count + 1; index log2(c) - 1
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  const int k = c == 2 ? 0 : c == 4 ? 1 : 2;
  if (cache[dev][k] == 0) {
    int n = 0;
    if (set_smem_attr<L>() == cudaSuccess) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(c, 1, 1);
      cfg.blockDim = dim3(kThreads, 1, 1);
      cfg.dynamicSmemBytes = SmemPlan<L>::kBytes;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = c;
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&n, sparse_decode_kernel<L>, &cfg) != cudaSuccess) n = 0;
      cudaGetLastError();  // a refused query leaves no sticky error
    }
    cache[dev][k] = n + 1;
  }
  return cache[dev][k] - 1;
}

// Whether the decode launch is a programmatic dependent: always on stream
// launches, and inside CUDA-graph capture too unless DSV4B_PDL_IN_GRAPH=0
// (with the scheduler captured before it, a graphed b 1-32 step measured
// ~2 us faster with the programmatic edge; without it, the same).
bool pdl_allowed(cudaStream_t stream) {
  static const bool in_graph = [] {
    const char* e = getenv("DSV4B_PDL_IN_GRAPH");
    return !(e && e[0] == '0');
  }();
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) return false;
  return cap == cudaStreamCaptureStatusNone || in_graph;
}

// 4-D TMA map of q, dims (innermost first) {d_qk, h_q, s_q, b}, box
// {64, 64, 1, 1} with SWIZZLE_128B: one box = one Q^T chunk slot.  A size-1
// dimension gets a nominal stride (its coordinate is always 0).
template <int L>
cudaError_t make_q_map(const dsv4b_decode_params& p, CUtensorMap* map) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t sh = (cuuint64_t)p.stride_q_h * 2;
  const cuuint64_t ss = p.s_q > 1 ? (cuuint64_t)p.stride_q_s * 2 : sh * (cuuint64_t)p.h_q;
  const cuuint64_t sb = p.b > 1 ? (cuuint64_t)p.stride_q_b * 2 : ss * (cuuint64_t)p.s_q;
  const cuuint64_t dims[4] = {(cuuint64_t)LayoutT<L>::kDqk, (cuuint64_t)p.h_q, (cuuint64_t)p.s_q, (cuuint64_t)p.b};
  const cuuint64_t strides[3] = {sh, ss, sb};
  const cuuint32_t box[4] = {64u, (cuuint32_t)kHeadsPerCta, 1u, 1u};
  const cuuint32_t es[4] = {1u, 1u, 1u, 1u};
  if (enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(p.q), dims, strides, box, es,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  return cudaSuccess;
}

template <int L>
cudaError_t launch_decode_impl(const dsv4b_decode_params& p, const dsv4b_sched_meta* sched,
                               const int32_t* num_splits, int num_sm_parts, float* lse_accum,
                               float* o_accum, int* err, cudaStream_t stream) {
  cudaError_t e = set_smem_attr<L>();
  if (e != cudaSuccess) return e;
  CUtensorMap q_map;
  if ((e = make_q_map<L>(p, &q_map)) != cudaSuccess) return e;
  const int c = plan_cluster_size(p, num_sm_parts);
  const int groups = (p.h_q + kHeadsPerCta - 1) / kHeadsPerCta;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(c > 1 ? p.b * p.s_q * c : num_sm_parts, groups, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = SmemPlan<L>::kBytes;
  cfg.stream = stream;
  // Programmatic dependent launch: the CTAs set up while the previous grid
  // (typically the scheduler of get_mla_metadata) drains, and wait for it
  // in-kernel (griddepcontrol.wait) before reading anything it wrote.
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (pdl_allowed(stream)) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (c > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = c;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, sparse_decode_kernel<L>, p, sched, num_splits, lse_accum, o_accum, err,
                            c > 1 ? c : 1, q_map);
}

// Sparse prefill: one CTA per (query token, 64-head group), no split, no
// cluster (every row ends in the CTA's own epilogue).
template <int L>
cudaError_t launch_prefill_impl(const dsv4b_decode_params& p, const dsv4b_sched_meta* sched,
                                const int32_t* num_splits, int* err, cudaStream_t stream) {
  cudaError_t e = set_smem_attr<L>();
  if (e != cudaSuccess) return e;
  CUtensorMap q_map;
  if ((e = make_q_map<L>(p, &q_map)) != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.b * p.s_q * ((p.h_q + kHeadsPerCta - 1) / kHeadsPerCta), 1, 1);  // a token's groups adjacent
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = SmemPlan<L>::kBytes;
  cfg.stream = stream;
  return cudaLaunchKernelEx(&cfg, sparse_decode_kernel<L>, p, sched, num_splits, (float*)nullptr,
                            (float*)nullptr, err, 1, q_map);
}

}  // namespace

// Cluster size of the plan for this batch; 1 = no cluster (split partials
// are merged by the combine kernel).  Candidates are C in {8, 4, 2} with
// b*s_q*C <= num_sm_parts, C <= the most tiles a row can have, and every
// cluster of the launch resident at once (one wave).  The largest such C
// gives k_c = ceil(tiles / C) tiles per CTA; it is used unless the
// row-aligned plan would give its parts fewer tiles (k_r), since a tile
// (~7 us) costs more than the combine step that plan adds.
int plan_cluster_size(const dsv4b_decode_params& p, int num_sm_parts) {
  static const bool clusters_off = [] {
    const char* e = getenv("DSV4B_CLUSTER");  // "0": never use the cluster plan
    return e && e[0] == '0';
  }();
  if (clusters_off) return 1;
  const int64_t rows = (int64_t)p.b * p.s_q;
  const int groups = (p.h_q + kHeadsPerCta - 1) / kHeadsPerCta;
  const int tiles_max = (p.topk + kTileTokens - 1) / kTileTokens +
                        (p.extra_kv ? (p.extra_topk + kTileTokens - 1) / kTileTokens : 0);
  if (rows > num_sm_parts) return 1;
  int kr = 1;  // row-aligned cap: smallest t with rows * ceil(tiles / t) <= parts
  while (rows * ((tiles_max + kr - 1) / kr) > num_sm_parts) ++kr;
  for (int c = 8; c >= 2; c >>= 1) {
    if (rows * c > num_sm_parts || c > tiles_max) continue;
    const int resident = p.layout == DSV4B_LAYOUT_V32 ? clusters_resident<DSV4B_LAYOUT_V32>(c)
                                                      : clusters_resident<DSV4B_LAYOUT_MODEL1>(c);
    if (resident < rows * groups) continue;
    const int kc = (tiles_max + c - 1) / c;
    return kc <= kr ? c : 1;
  }
  return 1;
}

cudaError_t launch_sparse_decode(const dsv4b_decode_params& p, const dsv4b_sched_meta* sched,
                                 const int32_t* num_splits, int num_sm_parts, float* lse_accum,
                                 float* o_accum, int* err, cudaStream_t stream) {
  if (p.layout == DSV4B_LAYOUT_V32)
    return launch_decode_impl<DSV4B_LAYOUT_V32>(p, sched, num_splits, num_sm_parts, lse_accum, o_accum,
                                                err, stream);
  return launch_decode_impl<DSV4B_LAYOUT_MODEL1>(p, sched, num_splits, num_sm_parts, lse_accum, o_accum,
                                                 err, stream);
}

cudaError_t launch_sparse_prefill(const dsv4b_decode_params& p, const dsv4b_sched_meta* sched,
                                  const int32_t* num_splits, int* err, cudaStream_t stream) {
  if (p.layout == DSV4B_LAYOUT_BF16_576)
    return launch_prefill_impl<DSV4B_LAYOUT_BF16_576>(p, sched, num_splits, err, stream);
  return launch_prefill_impl<DSV4B_LAYOUT_BF16_512>(p, sched, num_splits, err, stream);
}

#ifdef DSV4B_TRACE
extern "C" DSV4B_API int dsv4b_debug_trace_read_warps(unsigned long long* dst, int max_words) {
  const int n = kTraceCtas * 8 * 64 < max_words ? kTraceCtas * 8 * 64 : max_words;
  cudaMemcpyFromSymbol(dst, g_trace_w, n * sizeof(unsigned long long));
  return n;
}

extern "C" DSV4B_API int dsv4b_debug_trace_read(unsigned long long* dst, int max_words) {
  const int n = kTraceCtas * 3 * 128 < max_words ? kTraceCtas * 3 * 128 : max_words;
  cudaMemcpyFromSymbol(dst, g_trace, n * sizeof(unsigned long long));
  return n;
}
#endif

int decode_smem_bytes(int layout) {
  return layout == DSV4B_LAYOUT_V32 ? SmemPlan<DSV4B_LAYOUT_V32>::kBytes
                                    : SmemPlan<DSV4B_LAYOUT_MODEL1>::kBytes;
}

cudaError_t set_decode_test_stall(int stall) {
  return cudaMemcpyToSymbol(g_decode_test_stall, &stall, sizeof(stall));
}

}  // namespace dsv4b
