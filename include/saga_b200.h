/*
 * saga_b200 -- C ABI of the SAGA decode-attention path on NVIDIA B200 (sm_100a).
 *
 * Every entry point takes plain pointers, element strides and sizes, and a
 * CUDA stream passed as `void*` (a cudaStream_t; NULL = legacy default
 * stream). Nothing here allocates device memory: the caller passes outputs
 * and a workspace of `saga_workspace_bytes()` bytes. All work is enqueued
 * on the given stream with no host synchronisation, so calls can be captured
 * in a CUDA graph.
 *
 * Return value: SAGA_OK (0) or a negative saga_status. On error,
 * `saga_last_error()` returns a message for the calling thread.
 *
 * Shapes follow the reference (noamelata/SAGA, attention/attention.py):
 *   query  q [B, Hq, 1, D]   key cache k [B, Hk, L, D]   value cache v [B, Hv, L, D]
 *   Hq % Hk == 0, Hq % Hv == 0. Query head h uses key head h / (Hq/Hk) and
 *   value head h / (Hq/Hv). Row r = b*Hq + h indexes per-(batch, query head)
 *   quantities. The innermost (D) stride of every tensor must be 1.
 */
#ifndef SAGA_B200_H
#define SAGA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SAGA_API __attribute__((visibility("default")))
#else
#define SAGA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  SAGA_BF16 = 0,
  SAGA_FP16 = 1,
  SAGA_FP32 = 2,
  SAGA_BOOL = 3, /* masks only: True adds 1.0, False adds 0.0 (attention.py:124-126) */
  SAGA_INT64 = 4 /* index outputs */
} saga_dtype;

typedef enum {
  SAGA_OK = 0,
  SAGA_ERR_INVALID = -1,     /* bad shape, stride, dtype or null pointer */
  SAGA_ERR_UNSUPPORTED = -2, /* valid request outside what the kernels cover */
  SAGA_ERR_WORKSPACE = -3,   /* workspace missing or too small */
  SAGA_ERR_CUDA = -4         /* CUDA runtime error (launch, attribute, ...) */
} saga_status;

/* Device status word bits, written with atomicOr by the kernels (never a trap).
 * The caller reads the int32 word outside timed regions. */
#define SAGA_STATUS_WAIT_TIMEOUT 0x1   /* a bounded inter-CTA wait gave up */
#define SAGA_STATUS_NONFINITE_THR 0x2  /* some row's logit threshold was NaN/inf */
#define SAGA_STATUS_OVERFLOW 0x4       /* some row had more than K passing positions */
#define SAGA_STATUS_EMPTY_ROW 0x8      /* some row selected nothing (output is NaN) */
#define SAGA_STATUS_APPEND_RANGE 0x10  /* append_pos_dev held a position outside [0, L): no append */
#define SAGA_STATUS_PAGE_RANGE 0x20    /* a page table entry outside [0, num_pages): page 0 was read */

/* Descriptor shared by the attention entry points. Unused fields are ignored.
 * Strides are in elements. */
typedef struct SagaAttnArgs {
  int32_t dtype; /* saga_dtype of q, k, v, out (and of k_new/v_new) */
  int32_t B, Hq, Hk, Hv, D;
  int32_t L; /* key/value positions seen by the kernel (key.shape[2]) */

  const void* q;  int64_t q_sb, q_sh;          /* [B, Hq, 1, D] */
  const void* k;  int64_t k_sb, k_sh, k_sl;    /* [B, Hk, L, D] */
  const void* v;  int64_t v_sb, v_sh, v_sl;    /* [B, Hv, L, D] */

  /* Additive mask [B, 1|Hq, 1, >=L] sliced to L (attention.py:124-126), or NULL.
   * mask_dtype is SAGA_BOOL or equal to dtype. Strides may be 0 (broadcast). */
  const void* mask; int32_t mask_dtype; int64_t m_sb, m_sh, m_sl;

  float scaling;       /* logits scale; the reference default is 1/sqrt(D) */
  int32_t top_n;       /* N of Atop-N */
  const float* thr_in; /* amortized: softmax-space threshold per row [B*Hq] */
  float* thr_out;      /* calibration: N-th largest probability per row [B*Hq] */

  void* out; int64_t o_sb, o_sh; /* [B, Hq, 1, D], dtype */

  /* Optional fused append of the decode token at position append_pos
   * (transformers StaticLayer.update's index_copy_): k[b, kh, pos] = k_new[b, kh],
   * v[b, vh, pos] = v_new[b, vh] before the step reads the cache. NULL = no append. */
  const void* k_new; int64_t kn_sb, kn_sh; /* [B, Hk, 1, D] */
  const void* v_new; int64_t vn_sb, vn_sh; /* [B, Hv, 1, D] */
  int32_t append_pos;

  /* Optional per-row outputs (NULL = not written). */
  float* logit_thr_out;  /* amortized: logit-space threshold t [R] */
  int32_t* count_out;    /* amortized: positions with logit > t [R] (before the cap);
                            calibration: positions with probability > threshold [R] */
  int32_t* sel_idx_out;  /* kept positions, ascending, [R, sel_ld]; unused slots untouched */
  int32_t sel_ld;
  void* logits_out; int64_t lo_ld; /* logits [R, lo_ld >= L] in dtype (saga_attn_logits) */

  void* workspace; size_t workspace_bytes; /* see saga_workspace_bytes */
  int32_t* status; /* device status word (SAGA_STATUS_*), or NULL */

  /* Optional phase trace (NULL = off), int64 [1024][128]. CTA c < 1024 writes
   * stamps of its first work item into row c: column k < 16 = SM clock
   * (clock64) at phase point k (0 start, 1 logits done, 7 item done, the rest
   * after the exchanges and gather steps), column 64 + k = global timer (ns)
   * at the same point; 16 + t / 32 + t / 48 + t = SM clock when key tile t
   * (< 16) was issued by TMA / multiplied / stored; 127 = value rows
   * gathered. Diagnostics only: written only by a library built with
   * SAGA_PHASE_TRACE=1 in the environment (python -m saga_b200.build --force),
   * ignored otherwise. */
  int64_t* trace;

  /* Sequence sharding (config 4 of the reference's benchmarks): the positions
   * of every group are split over `shards` devices, one call per device, all
   * in flight together. This call owns positions [0, nsel) of its caches, which
   * are global positions pos_offset + [0, nsel); when nsel < L, positions
   * [nsel, L) are a replica of the sequence's last kTail (256) rows, used
   * only for the tail max (attention.py:142-143). The exchanges of the fused
   * kernel (exp-sums, counts, partial outputs, completion) run between the
   * devices through their workspaces: shard_workspaces[s] is shard s's
   * workspace mapped into this device (peer memory over NVLink), and
   * shard_workspaces[shard] == workspace. All shards must use the same
   * shapes and nsel. Every shard writes the full output (and, for the
   * calibration, its own copy of every row's threshold). Supported for
   * saga_atopn_decode, saga_atopn_calibrate and saga_dense_decode.
   * shards = 0 or 1: not sharded. */
  int32_t nsel;        /* 0 = L */
  int32_t pos_offset;  /* added to the positions written to sel_idx_out */
  int32_t shards;
  int32_t shard;
  void* shard_workspaces[8];

  /* Optional: device address of the append position (int64, first element),
   * read by the kernel instead of append_pos, so that a CUDA graph can replay
   * the append at a position that advances (an HF static cache's length).
   * Not with shards > 1. */
  const int64_t* append_pos_dev;

  /* Optional paged caches (no counterpart in the reference, whose caches are
   * contiguous [B, H, L, D] tensors; it copies a prefilled cache per batch
   * row, speedup.py:155-160). With page_table non-NULL, k and v point at page
   * pools [num_pages][H][page_len][D]: k_sb / v_sb are the page strides, and
   * k_sh, k_sl / v_sh, v_sl the head and row strides inside a page (elements).
   * Logical position pos of sequence b lives in page
   * page_table[b * pt_sb + pos / page_len]; rows of several sequences may
   * share a page, but an appended row must go to a page of its own sequence.
   * page_len is a power of two and a multiple of 128; L is the logical
   * context length (<= pt_sb * page_len). A page number outside
   * [0, num_pages) sets SAGA_STATUS_PAGE_RANGE and page 0 is read instead.
   * saga_atopn_decode, saga_atopn_calibrate, saga_dense_decode and
   * saga_attn_logits only; not with shards > 1. */
  const int32_t* page_table;
  int64_t pt_sb;
  int32_t page_len;
  int32_t num_pages;
} SagaAttnArgs;

/* Ops understood by saga_workspace_bytes. */
typedef enum {
  SAGA_OP_ATOPN_DECODE = 0,
  SAGA_OP_ATOPN_CALIBRATE = 1,
  SAGA_OP_DENSE_DECODE = 2,
  SAGA_OP_LOGITS = 3
} saga_op;

/* Bytes of workspace the op needs for these shapes (0 plus an error message if
 * the shapes are invalid). A workspace belongs to one op and one set of shapes
 * (dtype, B, Hq, Hk, Hv, D, L): its layout depends on them. It must be
 * zero-filled when allocated; each successful call leaves its counters zeroed
 * again, so later calls with the same shapes can reuse it. Zero it again before
 * using it for other shapes, and after a call that reported
 * SAGA_STATUS_WAIT_TIMEOUT. Calls that share a workspace must not overlap on
 * the GPU (one stream at a time). */
SAGA_API size_t saga_workspace_bytes(const SagaAttnArgs* args, int32_t op);

/* Steady-state Atop-N decode step. Replaces approx_top_n_attention_amortized
 * (attention.py:192-209): logits (113-128), the softmax->logit threshold
 * transform (136-149), threshold selection with K = min(2N, L)
 * (triton_atopn.py:59-113, kernel 6-53) and the softmax-weighted V gather
 * (attention.py:152-170), fused in one persistent kernel. When more than K
 * positions pass, the K lowest positions are kept. */
SAGA_API int saga_atopn_decode(const SagaAttnArgs* args, void* stream);

/* saga_atopn_decode without a caller workspace. It has no counterpart in the
 * reference: it serves hosts that cannot allocate device memory at call time.
 * The scratch is a fixed array of saga_noalloc_scratch_bytes() (8 MiB) in the
 * library's own device memory, one per device; shapes that need more are
 * refused with SAGA_ERR_WORKSPACE (args->workspace is ignored). The array is
 * part of the library's device image, so every CUDA context that loads the
 * library holds those 8 MiB until exit, whether or not this entry point is
 * called. Sequence sharding (shards > 1) is refused with SAGA_ERR_UNSUPPORTED.
 * A call is fully validated before it touches the scratch; then it zero-fills
 * the bytes it uses with one cudaMemsetAsync on `stream`. Calls on one device
 * must not overlap on the GPU: they share the scratch. Make the first call on
 * a device outside stream capture (it may load the library's device code
 * there). Nothing is allocated. */
SAGA_API int saga_atopn_decode_noalloc(const SagaAttnArgs* args, void* stream);

/* Capacity in bytes of the static scratch of saga_atopn_decode_noalloc. */
SAGA_API size_t saga_noalloc_scratch_bytes(void);

/* Calibration step. Replaces approx_top_n_attention_amortized_cal
 * (attention.py:173-189): full softmax, exact top-min(N, L) probabilities,
 * thr_out[r] = the N-th largest probability (184-187), output from the
 * renormalised top-N probabilities. Ties at the N-th value are kept in
 * ascending position order. */
SAGA_API int saga_atopn_calibrate(const SagaAttnArgs* args, void* stream);

/* Dense GQA decode. Replaces full_einsum_forward (attention.py:64-85). */
SAGA_API int saga_dense_decode(const SagaAttnArgs* args, void* stream);

/* Logits only: writes logits_out [R, L]. Replaces _compute_attn_weights
 * (attention.py:113-128). */
SAGA_API int saga_attn_logits(const SagaAttnArgs* args, void* stream);

/* Softmax-space -> logit-space threshold. Replaces _transform_softmax_threshold
 * (attention.py:136-149): t[r] = m + log(max(thr[r], 1e-30) * s), with m the max
 * of the last min(tail, L) logits and s = sum(exp(logits - m)) rounded as the
 * reference does in the logits dtype. m_out / s_out may be NULL. */
SAGA_API int saga_transform_threshold(int32_t dtype, const void* logits, int64_t ld, int32_t rows,
                             int32_t L, const float* thr, int32_t tail, float* t_out,
                             float* m_out, float* s_out, void* stream);

/* Threshold selection. Replaces threshold_topk_fast (triton_atopn.py:59-113)
 * and its kernel (6-53). For row r, every x[r, i] > thr[r % thr_count] is
 * written in ascending i to vals[r, :] / idx[r, :] (at most k per row).
 * Unused slots get vals = -inf and idx = 0 (triton_atopn.py:82-84).
 * counts[r] = number passing before the cap (may be NULL). */
SAGA_API int saga_threshold_select(int32_t dtype, const void* x, int64_t ldx, int32_t rows, int32_t L,
                          int32_t k, const float* thr, int32_t thr_count, void* vals,
                          int64_t* idx, int32_t* counts, void* stream);

/* Sparse V gather + output. Replaces _atopn_gather_and_output
 * (attention.py:152-170) for a [R, K] buffer of weights (logits when
 * input_is_logits != 0, else probabilities) and int64 positions. */
SAGA_API int saga_gather_output(int32_t dtype, const void* w, const int64_t* idx, int32_t K,
                       int32_t input_is_logits, const void* v, int64_t v_sb, int64_t v_sh,
                       int64_t v_sl, int32_t B, int32_t Hq, int32_t Hv, int32_t D, int32_t L,
                       void* out, int64_t o_sb, int64_t o_sh, void* stream);

/* KV append of one decode token at position pos: the index_copy_ of
 * transformers' StaticLayer.update on the asymmetric cache of
 * speedup.py:119-139 (Hk key heads, Hv value heads). */
SAGA_API int saga_kv_append(int32_t dtype, int32_t B, int32_t Hk, int32_t Hv, int32_t D, int32_t L,
                   int32_t pos, void* k, int64_t k_sb, int64_t k_sh, int64_t k_sl, void* v,
                   int64_t v_sb, int64_t v_sh, int64_t v_sl, const void* k_new, int64_t kn_sb,
                   int64_t kn_sh, const void* v_new, int64_t vn_sb, int64_t vn_sh,
                   void* stream);

/* Set-up helpers of sequence sharding (no counterpart in the reference).
 * saga_ipc_handle writes the 64-byte cudaIpcMemHandle of the device
 * allocation that contains `ptr` and the byte offset of `ptr` in it (the
 * allocation must come from cudaMalloc, as torch's caching allocator does by
 * default). saga_ipc_open maps another process's allocation into the CURRENT
 * device with peer access enabled, so that kernels on this device read and
 * write it over NVLink; *ptr receives the allocation's base (add the offset).
 * saga_ipc_close unmaps it. */
SAGA_API int saga_ipc_handle(const void* ptr, void* handle64, size_t* offset);
SAGA_API int saga_ipc_open(const void* handle64, void** ptr);
SAGA_API int saga_ipc_close(void* ptr);

/* Message of the last error on the calling thread ("" if none). */
SAGA_API const char* saga_last_error(void);

/* Library version string. */
SAGA_API const char* saga_version(void);

/* Names of the kernels the last call on this thread launched, separated by
 * ',' (diagnostics; also used to count launches). */
SAGA_API const char* saga_last_launches(void);

#ifdef __cplusplus
}
#endif

#endif /* SAGA_B200_H */
