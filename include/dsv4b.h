/*
 * dsv4b.h - C ABI of the B200 (sm_100a) sparse FP8 MLA decode path.
 *
 * Plain C: pointers, sizes, int status codes.  No torch or C++ types.
 * Every entry point runs asynchronously on the given CUDA stream (passed as
 * void*, a cudaStream_t) and never synchronises the device.  All return
 * DSV4B_OK (0) or a negative dsv4b_status; dsv4b_status_string() names it.
 *
 * Each declaration cites the reference interface it replaces
 * (0xSero/deepseek-v4-flash-sm120, paths relative to that project).
 */
#ifndef DSV4B_H_
#define DSV4B_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DSV4B_API __attribute__((visibility("default")))
#else
#define DSV4B_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The reference aborts the process on CUDA errors
 * (csrc/common/defines.h:11-21) and raises TORCH_CHECK on bad arguments
 * (csrc/api/sparse_decode.cpp:43-75); here both become return codes. */
typedef enum dsv4b_status {
  DSV4B_OK = 0,
  DSV4B_ERR_INVALID_ARGUMENT = -1, /* shape / stride / pointer check failed */
  DSV4B_ERR_UNSUPPORTED = -2,      /* valid request this build does not run */
  DSV4B_ERR_CUDA = -3,             /* a CUDA runtime call failed */
  DSV4B_ERR_WORKSPACE = -4,        /* workspace too small */
  DSV4B_ERR_ARCH = -5,             /* device is not sm_100 */
  DSV4B_ERR_KERNEL_TIMEOUT = -6,   /* a kernel wait hit its time limit */
  DSV4B_ERR_SCRATCH_LIMIT = -7     /* request needs more than the fixed
                                      scratch of dsv4b_sparse_decode_noalloc */
} dsv4b_status;

/* KV-cache byte layouts (csrc/common/params.h:12-15, ModelType). */
typedef enum dsv4b_layout {
  /* DeepSeek-V3.2: d_qk 576, d_v 512, 656 B/token, token-contiguous
   * [512 x e4m3 | 4 x fp32 scale per 128 | 64 x bf16 RoPE]. */
  DSV4B_LAYOUT_V32 = 0,
  /* DeepSeek-V4-Flash: d_qk = d_v = 512; per page P x 576 B
   * [448 x e4m3 | 64 x bf16 RoPE] rows, then P x 8 B UE8M0 scales
   * (tests/reference.py:7-19). */
  DSV4B_LAYOUT_MODEL1 = 1,
  /* Sparse prefill only (dsv4b_sparse_prefill): a bf16 [s_kv, d_qk] KV
   * tensor, row stride stride_kv_block bytes, d_qk = 576 (V3.2 latent +
   * RoPE; V = the first 512 columns) or 512 (V4; V = the whole row). */
  DSV4B_LAYOUT_BF16_576 = 2,
  DSV4B_LAYOUT_BF16_512 = 3
} dsv4b_layout;

/* One record per SM part, 32 bytes, field order of the reference's
 * DecodingSchedMeta (csrc/common/params.h:17-32).  Tiles are 128 top-k
 * positions.  A part covers (begin_req_idx, begin_block_idx) up to
 * (end_req_idx, end_block_idx) with the end tile exclusive; an empty part
 * has end_req_idx < begin_req_idx.  "req" is a query row b * s_q + s. */
typedef struct dsv4b_sched_meta {
  int32_t begin_req_idx;
  int32_t end_req_idx;
  int32_t begin_block_idx;
  int32_t end_block_idx;
  int32_t begin_split_idx;
  int32_t is_first_req_splitted;
  int32_t is_last_req_splitted;
  int32_t num_tiles;
} dsv4b_sched_meta;

/* Arguments of one decode call; mirrors SparseAttnDecodeParams
 * (csrc/common/params.h:34-97) with 64-bit strides.  Element strides for
 * q / out, byte strides for caches, element strides for indices. */
typedef struct dsv4b_decode_params {
  int32_t layout;            /* dsv4b_layout */
  int32_t b, s_q, h_q, d_qk, d_v, topk;
  float sm_scale;
  int32_t lse_includes_sink; /* 1: lse = logaddexp(lse, sink) (reference
                                tests/reference.py:124-129); 0: FlashMLA doc */

  const void* q;             /* bf16 [b, s_q, h_q, d_qk], last dim contiguous */
  int64_t stride_q_b, stride_q_s, stride_q_h;

  const void* kv;            /* uint8/fp8 cache */
  int32_t num_blocks, page_block_size;
  int64_t stride_kv_block;   /* bytes between pages */
  int64_t stride_kv_row;     /* bytes between tokens in a page (V32) */

  const int32_t* indices;    /* [b, s_q, topk] flat page*P+offset, -1 = pad */
  int64_t stride_idx_b, stride_idx_s;
  const int32_t* topk_length;/* [b] or NULL */
  const float* attn_sink;    /* [h_q] or NULL */

  const void* extra_kv;      /* optional SWA sidecar cache, same layout */
  int32_t extra_num_blocks, extra_page_block_size, extra_topk;
  int64_t stride_extra_kv_block, stride_extra_kv_row;
  const int32_t* extra_indices;     /* [b, s_q, extra_topk] */
  int64_t stride_extra_idx_b, stride_extra_idx_s;
  const int32_t* extra_topk_length; /* [b] or NULL */

  void* out;                 /* bf16 [b, s_q, h_q, d_v] */
  int64_t stride_o_b, stride_o_s, stride_o_h;
  float* lse;                /* fp32 [b, h_q, s_q], contiguous */

  /* Sparse prefill (dsv4b_sparse_prefill) only; 0 / NULL for decode. */
  int32_t prefill;           /* 1: FlashMLA sparse-prefill semantics (see there) */
  float* max_logits;         /* fp32 [b, h_q] (s_q = 1) or NULL */
} dsv4b_decode_params;

/* Library version (major*10000 + minor*100 + patch). */
DSV4B_API int dsv4b_version(void);

/* Human-readable name of a dsv4b_status. */
DSV4B_API const char* dsv4b_status_string(int status);

/* DSV4B_OK if `device` is an sm_100 part this build can run on.
 * Replaces the Arch probe + SM_120 gate (csrc/common/params.h:100-116,
 * csrc/api/sparse_decode.cpp:160-168). */
DSV4B_API int dsv4b_check_device(int device);

/* Number of SM parts (scheduler records) to use for h_q heads on `device`
 * (148 SMs on B200; heads are processed in groups of 64).  Replaces the
 * fixed num_sm_parts = 1 (csrc/api/sparse_decode.cpp:147-158). */
DSV4B_API int dsv4b_num_sm_parts(int device, int h_q, int32_t* num_sm_parts);

/* Bytes of device workspace a decode call needs (split-KV partials and
 * the kernel status word); depends on shapes only. */
DSV4B_API size_t dsv4b_workspace_bytes(int b, int s_q, int h_q, int num_sm_parts);

/* get_mla_metadata: plan the split-KV tile schedule on the device from
 * topk / topk_length / extra_topk_length (no host synchronisation, CUDA
 * graph capturable).  Writes num_sm_parts records and num_splits
 * [b*s_q + 1] (prefix offsets of each query row's splits).  Replaces the
 * placeholder scheduler tensors of csrc/api/sparse_decode.cpp:147-158 and
 * the FlashMLA get_mla_metadata protocol (flash_mla_interface.py:38-51). */
DSV4B_API int dsv4b_get_mla_metadata(const dsv4b_decode_params* p, int num_sm_parts,
                           dsv4b_sched_meta* sched_meta, int32_t* num_splits,
                           void* stream);

/* Cluster size of the tile plan dsv4b_get_mla_metadata makes for these
 * shapes and num_sm_parts (a pure function of b*s_q, topk, extra_topk,
 * the layout and the device).  C >= 2: each query row is split over the C
 * CTAs of one thread-block cluster, which merge the row in distributed
 * shared memory, so the combine kernel has nothing to do and
 * num_splits = [0, 1, ..., b*s_q]; 1: split rows are merged by
 * dsv4b_combine().  Part of the get_mla_metadata protocol it extends
 * (flash_mla_interface.py:38-51); the reference has no split plan. */
DSV4B_API int dsv4b_plan_cluster_size(const dsv4b_decode_params* p, int num_sm_parts,
                                      int32_t* cluster_size);

/* Sparse decode forward: decode kernel (K1) plus split combine (K3).
 * Replaces dsv4_kernel::sparse_decode_fwd (csrc/api/sparse_decode.cpp:29-172)
 * and sm120::launch_dsv4_sparse_decode_v32
 * (csrc/sm120/decode/sparse_decode_instantiation.cu:10-23).  Writes
 * p->out and p->lse ([b, h_q, s_q], so no transpose copy is needed). */
DSV4B_API int dsv4b_sparse_decode(const dsv4b_decode_params* p,
                        const dsv4b_sched_meta* sched_meta,
                        const int32_t* num_splits, int num_sm_parts,
                        void* workspace, size_t workspace_bytes, void* stream);

/* The split-KV combine kernel alone (K3), for callers that run the decode
 * kernel through dsv4b_sparse_decode_partial().  New: the reference has no
 * combine (csrc/common/params.h:83-96 holds unused fields). */
DSV4B_API int dsv4b_combine(const dsv4b_decode_params* p, const int32_t* num_splits,
                  int num_sm_parts, void* workspace, size_t workspace_bytes,
                  void* stream);

/* The decode kernel alone (K1): rows whose work spans several parts leave
 * fp32 partials in the workspace for dsv4b_combine().  Same inputs as
 * dsv4b_sparse_decode. */
DSV4B_API int dsv4b_sparse_decode_partial(const dsv4b_decode_params* p,
                                const dsv4b_sched_meta* sched_meta,
                                const int32_t* num_splits, int num_sm_parts,
                                void* workspace, size_t workspace_bytes,
                                void* stream);

/* Debug: gather + dequantise n rows (flat indices) of a cache into bf16
 * [n, d_qk] with the decode kernel's own row decoder; -1 / out-of-range
 * rows come out as zeros.  Mirrors load_kv_chunk
 * (csrc/sm120/decode/sparse_decode_kernel.cuh:116-197) and the oracle
 * unpack (tests/reference.py:45-79) for bit-exact checks. */
DSV4B_API int dsv4b_gather_dequant(int layout, const void* kv, int num_blocks,
                         int page_block_size, int64_t stride_kv_block,
                         int64_t stride_kv_row, const int32_t* indices, int n,
                         void* out_bf16, void* stream);

/* Measurement: time the decode kernel's tcgen05.mma shapes with resident
 * shared-memory operands, one chain per CTA on `ctas` CTAs.  out (device,
 * 16-byte aligned, 2 * ctas int64): per CTA the best of six repetitions in
 * SM cycles (-1 if its bounded wait gave up) and the number of MMAs in the
 * chain.  shape 0: QK^T (M 128, N 64, A and B K-major, 36 MMAs); 1: PV
 * (M 128, N 64, A and B MN-major, 32 MMAs); 2: the QK^T A operand with
 * N 128 (16 MMAs); 3: with N 256 (8 MMAs); 4, 5: shapes 0, 1 issued from
 * precomputed descriptors.  No reference counterpart: it
 * backs the tensor-core figures of the decode roofline. */
DSV4B_API int dsv4b_mma_rate_probe(int shape, int ctas, long long* out, void* stream);

/* Measurement: gather the n rows listed in `rows` (row_bytes each, a
 * multiple of 16 up to 1536, at kv + row * row_stride) into 148 CTAs with
 * one mechanism and nothing else running: 0 = 16-byte register loads by
 * 256 threads per CTA, 1 = one cp.async.bulk per row into a shared-memory
 * ring (8 issuing lanes per CTA).  scratch (device, >= (148 * 256 + 4) * 4
 * bytes): a sink for the loaded words, then an int status word (set to a
 * nonzero value if a bounded wait gave up; the caller zeroes it).  Time it
 * with events on `stream`.  No reference counterpart: it backs the
 * gather-ceiling figures of the decode roofline. */
DSV4B_API int dsv4b_gather_rate_probe(int mechanism, const void* kv, int64_t row_stride, int row_bytes,
                                      const int32_t* rows, int n, void* scratch, size_t scratch_bytes,
                                      void* stream);

/* KV-cache writer: quantise n bf16 tokens into the cache's FP8 format and
 * scatter them to their slots (flat page * page_block_size + offset).
 *   layout V32:    nope = latent [n, 512], rope = [n, 64]; 656-B records
 *                  [512 e4m3 | 4 fp32 scales | 64 bf16 RoPE] at
 *                  page * stride_kv_block + offset * stride_kv_row;
 *                  scale = max(amax / 448, FLT_MIN) per 128 columns
 *                  (vLLM's fp8_ds_mla rule; an all-zero tile gets FLT_MIN).
 *   layout MODEL1: nope = [n, 448], rope = [n, 64] (for a [n, 512] k, pass
 *                  k and k + 448 with the same stride); per page P x 576-B
 *                  rows [448 e4m3 | 64 bf16 RoPE] then P x 8 UE8M0 bytes,
 *                  scale = 2^ceil(log2(max(amax, 1e-4) / 448)) per 64
 *                  columns (stride_kv_row is ignored).
 * e4m3 values are x / scale clamped to +-448, rounded to nearest even.
 * Element row strides (multiples of 8), 16-byte aligned rows.  slot_bytes
 * is 8 (int64 slots, vLLM's slot_mapping) or 4 (int32).  Tokens whose slot
 * is negative or >= num_blocks * page_block_size are skipped.
 * The producer of the bytes the decode path reads: SGLang's
 * quant_k_cache_v4 (tests/reference.py:45-58 unpacks its output); same
 * bytes as vLLM's quantize_and_insert_k_cache (MODEL1) and
 * concat_and_cache_mla with kv_cache_dtype "fp8_ds_mla" (V32). */
DSV4B_API int dsv4b_kv_cache_write(int layout, const void* nope, int64_t stride_nope,
                                   const void* rope, int64_t stride_rope,
                                   const void* slot_mapping, int slot_bytes, int64_t n,
                                   void* kv, int num_blocks, int page_block_size,
                                   int64_t stride_kv_block, int64_t stride_kv_row,
                                   void* stream);

/* Reads (and clears) this device's status word of dsv4b_kv_cache_write
 * into *flags (0 = no error; 1 = a kernel wait hit its time limit and the
 * write is incomplete).  Synchronises `stream`.  New: the reference has
 * no writer. */
DSV4B_API int dsv4b_kv_cache_write_status(int* flags, void* stream);

/* Self-test of the V32 writer's quotient x / scale (an FMA refinement of
 * one reciprocal per scale tile instead of a division per element): every
 * finite bf16 x against each of the n_scales device floats in `scales`
 * with |x| <= 448 * scale (the writer's domain).  Adds to mismatches[0]
 * (device uint64[2]) the e4m3 bytes that differ from those of the
 * hardware division, to mismatches[1] the differing fp32 quotients of
 * normal magnitude.  For tests. */
DSV4B_API int dsv4b_kv_write_selftest(const float* scales, int n_scales,
                                      unsigned long long* mismatches, void* stream);

/* ---------------------------------------------------------------------
 * Indexer logits (the step that produces `indices`): fp8_paged_mqa_logits.
 *
 * For every query row (b, i), i < next_n, and every cache position t:
 *   logits[b*next_n + i][t] = k_scale[t] *
 *       sum_h weights[b*next_n + i][h] * relu(sum_d q[b][i][h][d] * k[t][d])
 * for t < context_lens[b] and t <= context_lens[b] - next_n + i; positions
 * inside the row's last 128-token tile that fail the test get -inf; with
 * clean_logits, every later position up to max_model_len gets -inf too.
 * q and k are e4m3, products are accumulated in fp32 on the tensor cores.
 * The cache holds, per page, P x d e4m3 values followed by P x fp32 scales
 * (vLLM's indexer K cache: indexer_k_quant_and_cache).  Same contract as
 * DeepGEMM's fp8_paged_mqa_logits (vLLM utils/deep_gemm.py:407-460, torch
 * statement at v1/attention/ops/rocm_aiter_mla_sparse.py:256-300), the
 * kernel SGLang's DeepSeek-V4 indexer calls on sm_100; the reference only
 * wraps SGLang's fallbacks (deepseek_v4_kernel/_patch.py:199-236). */
typedef struct dsv4b_mqa_logits_params {
  int32_t b, next_n, h, d;        /* d = 128; h in {32, 64, 128}; next_n * h in {32, 64, 128, 256} */
  const void* q;                  /* e4m3 [b, next_n, h, d], contiguous */
  const void* kv;                 /* uint8 pages, see above */
  int32_t num_blocks, page_block_size;  /* P in {32, 64, 128} */
  int64_t stride_kv_block;        /* bytes between pages (>= P * (d + 4), % 16 == 0) */
  const float* weights;           /* [b * next_n, h] fp32, contiguous */
  const int32_t* context_lens;    /* [b] */
  const int32_t* block_table;     /* [b, >= ceil(context_len / P)] physical page ids */
  int64_t stride_block_table;     /* elements between rows */
  float* logits;                  /* [b * next_n, >= max_model_len] fp32 */
  int64_t stride_logits;          /* elements between rows */
  int32_t max_model_len;
  int32_t clean_logits;
} dsv4b_mqa_logits_params;

/* Schedule for dsv4b_fp8_paged_mqa_logits on num_sms CTAs: writes
 * sched[num_sms + 1][2] int32 (request, 128-token tile) start positions,
 * splitting all requests' tiles evenly (on the device, graph capturable).
 * Mirrors DeepGEMM's get_paged_mqa_logits_metadata (vLLM
 * utils/deep_gemm.py:386-405).  b <= 16384. */
DSV4B_API int dsv4b_mqa_logits_metadata(const int32_t* context_lens, int b, int num_sms,
                                        int32_t* sched, void* stream);

/* The logits kernel (one persistent CTA per schedule entry). */
DSV4B_API int dsv4b_fp8_paged_mqa_logits(const dsv4b_mqa_logits_params* p, const int32_t* sched,
                                         int num_sms, void* stream);

/* Reads (and clears) this device's status word of the logits kernel
 * (0 = no error; 1 = a kernel wait hit its time limit).  Synchronises. */
DSV4B_API int dsv4b_mqa_logits_status(int* flags, void* stream);

/* Reads (and clears) the kernel status word kept in the workspace into
 * *flags (0 = no error; bit 0 = a bounded wait ran out of time, the call's
 * outputs are then invalid).  Synchronises `stream`.  workspace = NULL
 * with workspace_bytes = 0 reads (and clears) the status word of
 * dsv4b_sparse_decode_noalloc's built-in scratch on the current device. */
DSV4B_API int dsv4b_read_kernel_status(void* workspace, size_t workspace_bytes,
                             int* flags, void* stream);

/* Test hook for the kernels' failure path, on the current device.  Every
 * mbarrier wait inside the library's kernels gives up after a time limit
 * (4e9 SM cycles, about 2 s); the CTA then raises an abort flag, every
 * role leaves (waiting, bounded, for its own copies and tensor-core work
 * in flight), TMEM is freed and the kernel's status word gets bit 0.  The
 * kernel returns normally: no fault, no hang, the context stays usable,
 * and the call's outputs are invalid.  For each kernel whose bit is set in
 * `kernels`, one thread per CTA withholds one arrival on a barrier nothing
 * else completes, so that a wait can only run out:
 *   DSV4B_STALL_DECODE      decode: the first Q^T arrival (status:
 *                           dsv4b_read_kernel_status);
 *   DSV4B_STALL_KV_WRITE    KV-cache writer: the first chunk's copies
 *                           (status: dsv4b_kv_cache_write_status);
 *   DSV4B_STALL_MQA_LOGITS  indexer logits: the first page-id batch
 *                           (status: dsv4b_mqa_logits_status).
 * A test sets a bit, runs the call (about 2-4 s), checks the status, then
 * clears the hook (kernels = 0).  Replaces nothing in the reference, whose
 * kernels have no bounded waits (csrc/common/defines.h:11-21 aborts the
 * process on CUDA errors instead). */
#define DSV4B_STALL_DECODE 1
#define DSV4B_STALL_KV_WRITE 2
#define DSV4B_STALL_MQA_LOGITS 4
DSV4B_API int dsv4b_set_test_stall(int kernels);

/* Size of the library's built-in device scratch used by
 * dsv4b_sparse_decode_noalloc (32 MiB on each GPU where the library's
 * device code has been loaded). */
#define DSV4B_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)

/* Sparse decode forward that allocates nothing.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory at
 * call time -- e.g. a serving engine that has already handed all free HBM
 * to its KV-cache pool, or a C / FFI caller that has no access to a caching
 * allocator and must not call cudaMalloc in the middle of a decode step
 * (cudaMalloc can synchronise the device).  Same inputs, outputs and
 * results as dsv4b_sparse_decode, but the split-KV partials and the kernel
 * status word live in a fixed DSV4B_NOALLOC_SCRATCH_BYTES array inside the
 * library instead of a caller workspace; requests whose workspace
 * (dsv4b_workspace_bytes) would exceed it return DSV4B_ERR_SCRATCH_LIMIT
 * before launching anything.  The scratch is device memory of the library's
 * module: CUDA allocates it when it loads the module on a device, which
 * with lazy module loading (the CUDA default) happens at the first call of
 * the library that touches that device, not when the library is opened.  So
 * make one call of this function on each device BEFORE sizing a KV-cache
 * pool from the free memory, and before any stream capture; from then on a
 * call allocates nothing (cudaMemGetInfo does not change across calls).
 * Read a call's status word with dsv4b_read_kernel_status(NULL, 0, ...).
 * All calls
 * on a device share the one scratch array and it keeps the last call's
 * contents (the status word is cleared at the start of every call): calls
 * that overlap on the GPU -- different streams without ordering between
 * them -- race on it and must not be issued. */
DSV4B_API int dsv4b_sparse_decode_noalloc(const dsv4b_decode_params* p,
                                          const dsv4b_sched_meta* sched_meta,
                                          const int32_t* num_splits, int num_sm_parts,
                                          void* stream);

/* Bytes of device workspace dsv4b_sparse_prefill needs for `rows` query
 * tokens (its tile schedule and the kernel status word). */
DSV4B_API size_t dsv4b_prefill_workspace_bytes(int rows);

/* Sparse attention prefill, FlashMLA's flash_mla_sparse_fwd
 * (vLLM flash_mla_interface.py:180-217; the reference has no prefill: its
 * kernel flattens s_q into the batch, csrc/sm120/decode/
 * sparse_decode_kernel.cuh:38-40).  Each of the b query tokens (s_q = 1)
 * attends, with all h_q heads, to the top-k rows of one bf16 KV tensor:
 *   layout   DSV4B_LAYOUT_BF16_576 or DSV4B_LAYOUT_BF16_512 (d_qk 576/512);
 *   kv       bf16 [num_blocks = s_kv rows, d_qk], page_block_size = 1,
 *            stride_kv_block = row stride in bytes (multiple of 16);
 *   indices  [b, topk] row numbers (stride_idx_b); -1 or >= s_kv: none;
 *   topk_length [b] or NULL: only the first topk_length[i] indices count;
 *   attn_sink [h_q] or NULL: the output (not lse / max_logits) is scaled by
 *            exp(lse) / (exp(lse) + exp(sink)); lse_includes_sink must be 0;
 *   prefill = 1; max_logits fp32 [b, h_q] or NULL; lse fp32 [b, h_q].
 * Invalid positions are left out of the softmax (not zero rows, unlike
 * decode).  lse is the natural-log log-sum-exp of sm_scale * q.k over the
 * valid positions, max_logits their maximum; a token with no valid
 * position gets lse = +inf, max_logits = -inf and a zero output (FlashMLA's
 * conventions, checked against vLLM 0.22's kernel on B200).  Every token is
 * one CTA per 64 heads (no split-KV); extra_kv is not supported.  Status
 * word: dsv4b_read_kernel_status on the same workspace. */
DSV4B_API int dsv4b_sparse_prefill(const dsv4b_decode_params* p, void* workspace,
                                   size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DSV4B_H_ */
