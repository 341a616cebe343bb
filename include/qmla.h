/*
 * qmla — B200 (sm_100a) paged latent-KV MLA / GLA decode attention.
 *
 * C ABI of libqmla.so.  Plain pointers and sizes only; every device pointer is
 * a CUDA device address, `stream` is a cudaStream_t passed as void*.  No entry
 * point allocates device memory or synchronises the device (the qmla_dcp_buffer_*
 * set-up calls and the status readers excepted).  qmla_mla_decode, the DCP and
 * cache-writer kernels and the context gather may be recorded into a CUDA graph.
 * Entry points that take a `device` make it current for the call and restore the
 * caller's current device before they return.
 * Host-side the library keeps only per-device attributes and a small cache of
 * TMA descriptors.  Entry points return 0 on success or a negative QMLA_E_*
 * code.
 *
 * Reference interfaces replaced (paths inside sootaugur/qwen-mla-vllm):
 *   qmla_mla_decode   <- qwen_mla/ops/mla_decode_attention.py:1264-1359
 *                        decode_attention_fwd(q, k_buffer, v_buffer, o, lse,
 *                        req_to_token, b_seq_len, attn_logits, num_kv_splits,
 *                        sm_scale, page_size, logit_cap, k_scale, v_scale,
 *                        is_mla, rms_offset, rms_bf16, rms_log8, qrows), and
 *                        the FlashInfer fork's run() called from
 *                        qwen_mla/fi_decode.py:381-384 (BatchMLAPagedAttention
 *                        launcher, qwen_mla/kernels/qwen_mla.cuh:1386-1480).
 *   qmla_plan         <- qwen_mla/fi_decode.py:235-270 (_RankPlan.plan_cpu) and
 *                        the MLAPlan work partition it feeds
 *                        (qwen_mla/kernels/qwen_scheduler.cuh:1599-1871).
 *   qmla_dcp_correct  <- qwen_mla/dcp_fix.py:31-130 (_mla_correct_attn_out).
 *   qmla_dcp_merge    <- the all-gather + correct + reduce-scatter sequence of
 *                        vLLM's cp_lse_ag_out_rs that dcp_fix.py:133-142 patches,
 *                        fused into one merge of N (out, lse) partials.
 *   qmla_fp8_cache_write <- qwen_mla/mla_impl.py:309-342
 *                        (QwenMLATritonImpl.do_kv_cache_update, FP8 row writer).
 *   qmla_gather_cache <- qwen_mla/ops/mla_gather.py:28-76 (gather_cache_torch, the
 *                        chunked-prefill context gather with FP8 dequantisation).
 *   qmla_dcp_p2p_merge <- the same cp_lse_ag_out_rs sequence (dcp_fix.py:133-142)
 *                        done by one kernel over NVLink peer memory instead of
 *                        NCCL; no counterpart in the reference, which refuses
 *                        DCP (qwen_mla/mla_impl.py:552).
 */
#ifndef QMLA_H_
#define QMLA_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* error codes */
#define QMLA_OK 0
#define QMLA_E_INVALID (-1)        /* bad argument (null pointer, negative size, ...) */
#define QMLA_E_UNSUPPORTED (-2)    /* shape / dtype combination this build has no kernel for */
#define QMLA_E_ALIGNMENT (-3)      /* a cache pointer or stride is not 16-byte aligned */
#define QMLA_E_WORKSPACE (-4)      /* workspace smaller than qmla_decode_workspace_bytes() */
#define QMLA_E_CUDA (-5)           /* a CUDA runtime / driver call failed */
#define QMLA_E_DEVICE_TIMEOUT (-6) /* a kernel gave up waiting (see qmla_read_status) */

/* element types */
#define QMLA_DT_BF16 0
#define QMLA_DT_F16 1
#define QMLA_DT_F32 2
#define QMLA_DT_FP8E4M3 3

/* how the per-(token, head) score divisor is stored in the cache row
 * (qwen_mla/ops/mla_decode_attention.py:466-505) */
#define QMLA_RMS_NONE 0   /* rms_offset < 0: no divide                                  */
#define QMLA_RMS_NATIVE 1 /* one element per head in the cache dtype (bf16; e4m3 x k_scale) */
#define QMLA_RMS_BF16 2   /* FP8 row, raw bf16, two bytes per head                       */
#define QMLA_RMS_LOG8 3   /* FP8 row, uint8 code of log2(rms) over [-3, 3]               */

typedef struct qmla_decode_params {
  /* Query rows.  Element (row, head, d):
   *   d <  rank        : q   [row*q_stride_row   + head*q_stride_head   + d]
   *   rank <= d < qk_dim: q_pe[row*qpe_stride_row + head*qpe_stride_head + d - rank]
   * Pass q_pe = q + rank (same strides) for a single [rows, heads, Lq] tensor. */
  const void* q;
  int64_t q_stride_row, q_stride_head;
  const void* q_pe;
  int64_t qpe_stride_row, qpe_stride_head;
  int32_t q_dtype; /* QMLA_DT_BF16 or QMLA_DT_F16 */

  /* Paged latent cache: token t of page p starts at
   * kv_cache + (p*kv_stride_page + t*kv_stride_token) elements.  One row is
   * [latent (rank) | rope (qk_dim - rank) | rms tail | pad]. */
  const void* kv_cache;
  int64_t kv_stride_page, kv_stride_token;
  int64_t kv_num_pages;
  int32_t kv_row_width; /* elements per row that may be read (>= qk_dim and rms tail) */
  int32_t kv_dtype;     /* QMLA_DT_BF16 or QMLA_DT_FP8E4M3 (f16 caches: unsupported) */
  int32_t page_size;    /* tokens per page (> 0); multiples of 16 use TMA boxes */

  /* block_table[row*block_table_stride + i] is the i-th page of a row;
   * seq_lens[row] its length in tokens (values < 0 are treated as 0). */
  const int32_t* block_table;
  int64_t block_table_stride;
  const int32_t* seq_lens;

  int32_t num_rows;   /* decode rows (already flattened for MTP verify)      */
  int32_t num_heads;  /* query heads per row (<= 48)                          */
  int32_t rank;       /* latent width = value width: 256, 384, 512, 768 or 1792 */
  int32_t qk_dim;     /* attention width: latent + rope (reference Lk), <= 2048 */
  int32_t rms_offset; /* element (byte for FP8 rows) offset of the rms tail  */
  int32_t rms_mode;   /* QMLA_RMS_*                                           */
  float sm_scale;
  float logit_cap;      /* <= 0: off                                          */
  const float* k_scale; /* device fp32 scalar, FP8 dequant scale; NULL = 1.0  */
  int32_t qrows;        /* MTP verify tokens per request (rows already flattened:
                         * the qrows consecutive rows of a request share its block-table
                         * row; row j's length is that draft's causal length).  When
                         * qrows > 1 divides num_rows, up to 48 / num_heads of a request's
                         * rows are decoded together, so its cache is read once per such
                         * group instead of once per row; results are the same.           */

  /* Outputs: o[row*o_stride_row + head*o_stride_head + d], d < rank;
   * lse[row*lse_stride_row + head] natural-log LSE of the scaled scores
   * (may be NULL). */
  void* o;
  int64_t o_stride_row, o_stride_head;
  int32_t o_dtype; /* QMLA_DT_BF16, QMLA_DT_F16 or QMLA_DT_F32 */
  void* lse;
  int64_t lse_stride_row;
  int32_t lse_dtype; /* QMLA_DT_F32, QMLA_DT_BF16 or QMLA_DT_F16 */

  /* Caller-owned device scratch of at least qmla_decode_workspace_bytes(). */
  void* workspace;
  int64_t workspace_bytes;

  /* Optional precomputed plan from qmla_plan (device copy of tile_prefix,
   * num_rows + 1 entries).  NULL: the plan is built on the device.  Ignored when
   * MTP rows are decoded together (qrows > 1), whose plan is per group. */
  const int32_t* plan_tile_prefix;

  int32_t num_ctas; /* persistent CTAs; 0 = one per SM */
  int32_t device;   /* CUDA device ordinal the pointers live on */
} qmla_decode_params;

/* Bytes of workspace qmla_mla_decode needs for these parameters. */
int qmla_decode_workspace_bytes(const qmla_decode_params* p, int64_t* bytes);

/* Paged MLA decode: o, lse <- softmax((q . k) / rms * sm_scale) . v per row
 * and head, reading each row's cache once.  Launches a plan kernel (a bounds
 * kernel when plan_tile_prefix is given), the persistent decode kernel and a
 * merge kernel for rows cut at CTA boundaries on `stream`. */
int qmla_mla_decode(const qmla_decode_params* p, void* stream);

/* qmla_mla_decode for callers that cannot allocate device memory.  No counterpart in the
 * reference: its decode always receives scratch that vLLM's workspace manager owns.  Here the
 * callers are hosts that reach this library through a foreign-function layer that hands over
 * only the input and output buffers (no device allocator, nowhere to keep a workspace between
 * calls), and serving processes whose device memory pool is sized and locked at start-up, where
 * a later cudaMalloc would fail.  The call ignores p->workspace and uses a 32 MiB device array
 * inside the library instead; it calls no cudaMalloc, cudaFree or other allocating routine.
 *  - Limit: shapes whose qmla_decode_workspace_bytes() exceeds 32 MiB return QMLA_E_WORKSPACE
 *    before anything is launched (about 513,000 rows at 160 CTAs x 32 heads x rank 768).
 *  - Every GPU that loads the library holds one such array until the process exits.  The first
 *    call on a device looks up the array's device address (cudaGetSymbolAddress) with that
 *    device current; make that first call before any stream capture.
 *  - Every call on a device shares its array, which keeps the last call's contents (the status
 *    word is cleared by each call).  Two calls whose executions overlap on the GPU (for example calls
 *    on different streams) race on it: order them on one stream or with events.
 *  - qmla_static_read_status reads the status word of the last static call on a device. */
int qmla_mla_decode_static(const qmla_decode_params* p, void* stream);

/* Status word of the last qmla_mla_decode_static call on `device` (same bits as
 * qmla_read_status).  Copies 4 bytes device->host on `stream` and synchronises that stream. */
int qmla_static_read_status(int32_t device, void* stream, int32_t* status);

/* Device status word of the last call that used `workspace`: 0, or bit 0 set
 * when a kernel wait timed out.  Copies 4 bytes device->host on `stream` and
 * synchronises that stream (host-side diagnostic, not for graph capture). */
int qmla_read_status(const void* workspace, void* stream, int32_t* status);

/* Host planner (no CUDA calls).  From host sequence lengths it writes, into
 * caller-owned host arrays:
 *   tile_prefix[num_rows+1]  exclusive prefix of ceil(len/128) (the decode
 *                            kernel's work partition; copy it to the device
 *                            and pass as plan_tile_prefix),
 *   kv_indptr[num_rows+1]    page-count prefix  (fi_decode.py:235-270),
 *   kv_len[num_rows]         clamped lengths,
 * and *total_tiles / *total_pages.  kv_indptr / kv_len may be NULL. */
int qmla_plan(const int32_t* seq_lens_host, int32_t num_rows, int32_t page_size,
              int32_t* tile_prefix, int32_t* kv_indptr, int32_t* kv_len,
              int64_t* total_tiles, int64_t* total_pages);

/* DCP output correction for one rank (dcp_fix.py:31-130):
 *   lse_g[b,h] = logsumexp_n lses[n,b,h]  (NaN / +inf treated as -inf)
 *   out[b,h,:] *= exp(lses[cp_rank,b,h] - lse_g[b,h])  (0 where the factor is 0)
 * out: [B,H,D] (dtype out_dtype, strides in elements), lses: [N,B,H] fp32,
 * lse_out: [B,H] fp32 (may be NULL). */
int qmla_dcp_correct(void* out, int32_t out_dtype, int64_t out_stride_b, int64_t out_stride_h,
                     const float* lses, int64_t lses_stride_n, int64_t lses_stride_b,
                     float* lse_out, int32_t n_ranks, int32_t cp_rank, int32_t B, int32_t H,
                     int32_t D, int32_t is_base_e, void* stream);

/* Fused DCP merge of N partial results (what correct + reduce-scatter compute
 * together): o = sum_n exp(lse_n - lse_g) * o_n, lse = lse_g.
 * parts: [N,B,H,D] dtype parts_dtype, contiguous; part_lse: [N,B,H] fp32
 * (natural log); o: [B,H,D] o_dtype contiguous; lse: [B,H] fp32 (may be NULL). */
int qmla_dcp_merge(const void* parts, int32_t parts_dtype, const float* part_lse, void* o,
                   int32_t o_dtype, float* lse, int32_t n_parts, int32_t B, int32_t H, int32_t D,
                   void* stream);

/* FP8 cache writer (mla_impl.py:309-342): for each token i with slot
 * s = max(slot_mapping[i], 0), writes row s of the byte cache as
 *   [e4m3(latent/k_scale) | e4m3(rope/k_scale) | rms tail | untouched pad]
 * with values clamped to +-448 and rounded to nearest-even; the rms tail is
 * one log8 code per head (rms_mode QMLA_RMS_LOG8) or two bf16 bytes per head
 * (QMLA_RMS_BF16).  latent: [n, rank] bf16, k_pe: [n, >= rope + heads] bf16
 * ([rope | rms | ...]), row strides in elements; cache rows are
 * cache_row_stride bytes apart (slot = page*page_size + token). */
int qmla_fp8_cache_write(const void* latent, int64_t latent_stride, const void* k_pe,
                         int64_t k_pe_stride, const int64_t* slot_mapping, int32_t n_tokens,
                         int32_t rank, int32_t rope, int32_t heads, int32_t rms_mode,
                         const float* k_scale, void* cache, int64_t cache_row_stride,
                         void* stream);

/* ---- prefill context gather ----------------------------------------------
 * (qwen_mla/ops/mla_gather.py:28-76)  Destination row j (0 <= j < num_tokens)
 * belongs to sequence s = token_to_seq[j] and holds that sequence's token
 *   tok = j - cu_seq_lens[s] + (seq_starts ? seq_starts[s] : 0),
 * read from page block_table[s * block_table_stride + tok / page_size] at offset
 * tok % page_size.
 *   2-byte cache (QMLA_DT_BF16 / F16): the first row_elems elements of the row are
 *     copied, converted to dst_dtype.
 *   FP8 cache: columns [0, rms_offset) become e4m3 * (*scale); the rms_heads columns
 *     from rms_offset are decoded per rms_mode: QMLA_RMS_LOG8 (one code byte per
 *     head, 2^(-3 + code * 6/255)), QMLA_RMS_BF16 (two raw bf16 bytes per head) or
 *     QMLA_RMS_NATIVE (e4m3 * scale, like the latent).  Later columns are untouched.
 * Rows whose sequence, token or page index falls outside the tables are skipped and
 * OR QMLA_STATUS_BAD_INDEX into *status (when status is not NULL); a wait of the
 * staged variant that gives up ORs QMLA_STATUS_TIMEOUT.  Neither happens on valid
 * tables. */
#define QMLA_STATUS_TIMEOUT 1   /* a device wait gave up (every kernel with waits) */
#define QMLA_STATUS_BAD_INDEX 2 /* context gather: a row's index fell outside the tables */
typedef struct qmla_gather_params {
  const void* src_cache;                    /* element (p, t, c) at p*stride_page + t*stride_token + c */
  int64_t src_stride_page, src_stride_token; /* elements of src_dtype */
  int32_t page_size, num_pages;
  int32_t src_dtype;                        /* QMLA_DT_BF16, QMLA_DT_F16 or QMLA_DT_FP8E4M3 */
  int32_t row_elems;                        /* 2-byte cache: elements copied per row */
  int32_t rms_offset, rms_heads, rms_mode;  /* FP8 cache only */
  const float* scale;                       /* FP8 cache: per-layer scale (device scalar) */
  const int32_t* block_table;               /* [num_seqs][block_table_cols] page ids */
  int64_t block_table_stride;
  int32_t block_table_cols;
  const int32_t* cu_seq_lens;               /* [num_seqs + 1] first destination row of each sequence */
  const int32_t* token_to_seq;              /* [num_tokens] */
  const int32_t* seq_starts;                /* [num_seqs] first token of the chunk, or NULL */
  int32_t num_seqs, num_tokens;
  void* dst;                                /* [num_tokens][dst_stride_row] */
  int64_t dst_stride_row;                   /* elements of dst_dtype */
  int32_t dst_dtype;                        /* QMLA_DT_BF16, QMLA_DT_F16 or QMLA_DT_F32 */
  int32_t* status;                          /* optional device word (QMLA_STATUS_* bits) */
  int32_t device;
} qmla_gather_params;

int qmla_gather_cache(const qmla_gather_params* p, void* stream);

/* ---- DCP over NVLink peer memory ------------------------------------------
 * Each rank of a DCP group (one process per GPU) owns one exchange buffer:
 *   [header 256 B: flags[8] u32 (epoch published by each rank), status u32 at byte 32,
 *    last merged epoch u32 at byte 36 and a block counter u32 at byte 40 (device-epoch mode),
 *    merge stats u64[4] at byte 64 (merges, ns spent waiting for the peers' flags, ns from
 *    entry to exit, ns to publish; block 0 of each qmla_dcp_p2p_merge adds to them; the host
 *    may zero them)]
 *   [o partial, 2 slots of B*H*D f32, each 256-B aligned]
 *   [lse partial, 2 slots of B*H f32 (natural log), each 256-B aligned]
 * qmla_dcp_buffer_layout returns the byte offsets.  A decode step e writes the
 * rank's partial into slot e&1 of its own buffer (qmla_mla_decode with o / lse
 * pointing there, f32 o); qmla_dcp_p2p_merge(epoch = e) then merges all ranks'
 * slot-e&1 partials, reading the peers' buffers through their IPC mappings.
 * Epochs start at 1 and grow by one per step on every rank.  With epoch = 0 the kernel
 * takes the epoch from the device instead (one past the last epoch this rank merged, kept in
 * its header and advanced by the merge itself), so a captured CUDA graph can be replayed; a
 * captured sequence then needs an even number of merges per replay so each replay starts on
 * the same slot.  A group uses one mode for its whole life. */
#define QMLA_DCP_MAX_WORLD 8
#define QMLA_DCP_ALL_HEADS 0     /* every rank gets o[B, H, D] */
#define QMLA_DCP_HEAD_SCATTER 1  /* rank r gets heads [r*H/world, (r+1)*H/world): o[B, H/world, D] */

int qmla_dcp_buffer_layout(int32_t B, int32_t H, int32_t D, int64_t* total_bytes,
                           int64_t* o_offset, int64_t* o_slot_bytes, int64_t* lse_offset,
                           int64_t* lse_slot_bytes);
/* cudaMalloc + zero-fill of an exchange buffer on `device`; writes its 64-byte
 * CUDA IPC handle to ipc_handle.  Free with qmla_dcp_buffer_free. */
int qmla_dcp_buffer_alloc(int32_t device, int64_t bytes, void** ptr, void* ipc_handle);
/* Map a peer's exchange buffer (its IPC handle) on `device`; undo with
 * qmla_dcp_buffer_close. */
int qmla_dcp_buffer_open(int32_t device, const void* ipc_handle, void** ptr);
int qmla_dcp_buffer_close(void* ptr);
int qmla_dcp_buffer_free(void* ptr);

typedef struct qmla_dcp_p2p_params {
  void* bufs[QMLA_DCP_MAX_WORLD]; /* every rank's exchange buffer as mapped on this device */
  int32_t world, rank;            /* 1 <= world <= 8 */
  int32_t num_rows, num_heads, head_dim; /* head_dim % 4 == 0; H % world == 0 for scatter */
  int32_t mode;                   /* QMLA_DCP_ALL_HEADS or QMLA_DCP_HEAD_SCATTER */
  uint32_t epoch;                 /* this step's epoch (>= 1, equal on every rank); 0 = device epoch */
  void* out;                      /* [B, heads of this rank, D] */
  int64_t out_stride_row, out_stride_head; /* elements */
  int32_t out_dtype;              /* QMLA_DT_BF16 / F16 / F32 */
  float* lse_out;                 /* [B, heads of this rank] natural log, contiguous; may be NULL */
  int64_t timeout_ns;             /* bound on the wait for the peers' flags (<= 0: 2 s) */
  int32_t device;
} qmla_dcp_p2p_params;

/* Publish this rank's epoch to every peer, wait (bounded) for theirs, merge:
 *   o = sum_n exp(lse_n - lse_g) o_n,  lse_g = logsumexp_n lse_n
 * (NaN / +inf partial LSEs count as -inf).  A wait that runs out sets the
 * status word of this rank's buffer (qmla_dcp_read_status) and leaves `out`
 * unwritten; the launch itself still succeeds. */
int qmla_dcp_p2p_merge(const qmla_dcp_p2p_params* p, void* stream);
/* Status word of an exchange buffer (0 = ok, 1 = a merge wait timed out);
 * synchronises `stream`. */
int qmla_dcp_read_status(const void* buffer, void* stream, int32_t* status);

/* Human-readable text for a QMLA_E_* code. */
const char* qmla_error_string(int code);

/* ABI version (major*100 + minor). */
int qmla_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* QMLA_H_ */
