/*
 * C ABI of the Blackwell (sm_100a) FlashAttention-2 forward.
 *
 * This is the drop-in boundary for the reference's hot path. In the reference
 * (roy6n23/triton-fa2-forward) the Python wrapper `attention()` validates its inputs
 * (fa2/kernel.py:218-244) and launches the Triton kernel `_attn_fwd[grid](...)` with
 * q/k/v/out pointers, their 16 strides, (H_q, N_q, N_kv, qk_scale) and the constexprs
 * GQA_GROUP / PACK / HEAD_DIM / CAUSAL (fa2/kernel.py:246-259). `fa2_fwd_sm100` takes
 * the same information as plain pointers, sizes and strides and launches the CUDA kernel
 * asynchronously on the caller's stream. No torch types cross this boundary.
 *
 * Layout: q and o are [B, H_q, N_q, D], k and v are [B, H_kv, N_kv, D], each with
 * arbitrary element strides given in the order (b, h, n, d). The d stride must be 1,
 * every other stride must be a multiple of 8 elements (16 bytes) and the base pointers
 * must be 16-byte aligned (TMA rules); otherwise FA2_ERR_LAYOUT is returned and the
 * caller should pass contiguous copies.
 *
 * Variable-length batches (cu_seqlens_q != NULL): the sequences are packed along one token
 * axis, q and o [total_q, H_q, D], k and v [total_kv, H_kv, D] (the layout of
 * flash_attn_varlen_func). Sequence b owns q rows [cu_seqlens_q[b], cu_seqlens_q[b + 1]) and
 * k/v rows [cu_seqlens_kv[b], cu_seqlens_kv[b + 1]); seqlen_q / seqlen_kv are the largest
 * lengths, and the (b, h, n, d) strides give the token axis as n (the b stride is unused).
 *
 * Paged K/V (block_table != NULL): k and v are caches of pages [num_pages, page_size, H_kv, D]
 * (the layout of flash_attn_with_kvcache); sequence b's keys j live in page
 * block_table[b * block_table_stride + j / page_size], row j % page_size, and seqlens_kv[b]
 * says how many there are (at most seqlen_kv). The k/v strides are given as (page, h, row, d).
 * q and o keep the fixed-length layout [B, H_q, N_q, D].
 */
#ifndef FA2_SM100_H_
#define FA2_SM100_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FA2_SM100_ABI_VERSION 5

#if defined(__GNUC__)
#define FA2_API __attribute__((visibility("default")))
#else
#define FA2_API
#endif

enum Fa2DType { FA2_DTYPE_FP16 = 0, FA2_DTYPE_BF16 = 1 };

/* Alignment of the causal mask (Fa2FwdParams::causal_align). Top-left is the reference's
 * (fa2/kernel.py:225-228): query i sees keys j <= i and N_q must equal N_kv. Bottom-right
 * lines the last query up with the last key, query i sees keys j <= i + (N_kv - N_q), for
 * chunked prefill and decode against a longer K/V; it needs N_q <= N_kv (the reference has
 * no such mode, its README lists it out of scope). With N_q == N_kv the two are the same. */
enum Fa2CausalAlign { FA2_CAUSAL_TOP_LEFT = 0, FA2_CAUSAL_BOTTOM_RIGHT = 1 };

enum Fa2Status {
  FA2_OK = 0,
  FA2_ERR_NULL = 1,          /* a required pointer is NULL */
  FA2_ERR_SHAPE = 2,         /* non-positive size, N_q != N_kv under top-left causal, N_q > N_kv
                                under bottom-right causal, unknown causal_align, num_splits > 256 */
  FA2_ERR_DTYPE = 3,         /* dtype is neither fp16 nor bf16 */
  FA2_ERR_HEAD_DIM = 4,      /* head_dim not supported by the compiled kernels */
  FA2_ERR_GQA = 5,           /* H_q % H_kv != 0 */
  FA2_ERR_PACK = 6,          /* pack_gqa requested but the group does not divide BLOCK_M (128) */
  FA2_ERR_SCALE = 7,         /* qk_scale not finite or not > 0 */
  FA2_ERR_LAYOUT = 8,        /* strides / alignment not usable by TMA */
  FA2_ERR_TMA_ENCODE = 9,    /* cuTensorMapEncodeTiled rejected a descriptor */
  FA2_ERR_LAUNCH = 10,       /* the CUDA launch failed (cudaGetLastError) */
  FA2_ERR_DEVICE = 11,       /* current device is not sm_100 / driver entry point missing */
  FA2_ERR_TIMEOUT = 12,      /* value written to err_flag by a kernel whose bounded wait expired */
  FA2_ERR_WORKSPACE = 13,    /* num_splits > 1 without a large enough, 16-byte aligned workspace */
  FA2_ERR_SCRATCH_LIMIT = 14 /* fa2_fwd_sm100_noalloc: the split-KV scratch this call needs is
                                larger than FA2_NOALLOC_SCRATCH_BYTES */
};
/* Device-side reports in err_flag: the kernel writes FA2_ERR_TIMEOUT (a bounded wait expired)
 * or FA2_ERR_SHAPE (a variable-length or paged sequence longer than seqlen_q / seqlen_kv, or
 * negative) into a zero word; the first report wins. */

/* Size of the library-owned device scratch behind fa2_fwd_sm100_noalloc (32 MiB). */
#define FA2_NOALLOC_SCRATCH_BYTES (32ll << 20)

typedef struct Fa2FwdParams {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  int64_t q_stride[4]; /* element strides, order (b, h, n, d) */
  int64_t k_stride[4];
  int64_t v_stride[4];
  int64_t o_stride[4];
  int32_t batch;
  int32_t heads_q;
  int32_t heads_kv;
  int32_t seqlen_q;
  int32_t seqlen_kv;
  int32_t head_dim;  /* 16, 32, 64 or 128 (16 and 32 run on the 64 build, read and written in place) */
  int32_t dtype;     /* Fa2DType */
  int32_t causal;    /* causal mask, aligned as causal_align says (per sequence when variable-length) */
  int32_t pack_gqa;  /* 1: a GQA group's query heads share one 128-row tile */
  float qk_scale;    /* sm_scale * log2(e), > 0 (fa2/kernel.py:240-244) */
  int32_t* err_flag; /* optional device int32 for device-side reports (see above). NULL: none. */
  int64_t timeout_cycles; /* per-wait limit in SM clocks; <= 0 selects the default (~1 s) */
  const int32_t* gate;     /* optional device int32 start gate: the kernel issues its first
                              load only once *gate != 0 (set by an upstream kernel or a copy
                              on another stream). The wait is bounded by timeout_cycles; when
                              it expires the kernel writes FA2_ERR_TIMEOUT to err_flag and
                              returns without touching o. NULL: start at once. */
  int32_t num_splits;      /* split-KV: >1 splits every CTA's K/V range into num_splits parts that
                              run as separate CTAs and are merged by a second kernel (short
                              queries against long K/V). <= 1: no split, no workspace. */
  int32_t causal_align;    /* Fa2CausalAlign; 0 (top-left) is the reference's behaviour */
  void* workspace;         /* device scratch for num_splits > 1 (fp32 partial O + row
                              log-sum-exp), at least fa2_fwd_sm100_workspace_bytes() bytes */
  int64_t workspace_bytes;
  const int32_t* cu_seqlens_q;  /* variable-length batch: device int32 [batch + 1], the prefix sums
                                   of the query lengths (cu_seqlens_q[0] == 0). NULL: every
                                   sequence has seqlen_q queries and seqlen_kv keys. */
  const int32_t* cu_seqlens_kv; /* the same for the keys; set together with cu_seqlens_q */
  int32_t total_q;              /* variable-length batch: rows of q and o on the token axis */
  int32_t total_kv;             /* variable-length batch: rows of k and v on the token axis */
  const int32_t* block_table;   /* paged K/V: device int32 [batch][block_table_stride] page indices.
                                   NULL: k and v are contiguous [B, H_kv, N_kv, D] (or varlen). */
  const int32_t* seqlens_kv;    /* paged K/V: device int32 [batch], keys of each sequence */
  int32_t block_table_stride;   /* paged K/V: entries per sequence in block_table */
  int32_t page_size;            /* paged K/V: keys per page, 16, 32, 64 or a multiple of 128 */
  int32_t num_pages;            /* paged K/V: pages in k and v */
  int32_t reserved1;
} Fa2FwdParams;

/* Host-only validation of `p` (no CUDA calls). Replaces the asserts and ValueErrors of
 * fa2/kernel.py:218-244 at the C level. Returns FA2_OK or the first failing Fa2Status. */
FA2_API int fa2_fwd_sm100_check(const Fa2FwdParams* p);

/* out = softmax(q k^T * sm_scale [+ causal mask]) v, launched on `stream` (a
 * cudaStream_t / CUstream; NULL = legacy default stream). Asynchronous: returns after
 * the launch, without synchronising. Replaces `_attn_fwd[grid](...)`
 * (fa2/kernel.py:246-259). */
FA2_API int fa2_fwd_sm100(const Fa2FwdParams* p, void* stream);

/* Bytes of device workspace fa2_fwd_sm100 needs for `p` (0 when p->num_splits <= 1).
 * Host only; the reference has no split-KV (its README lists it out of scope). */
FA2_API int64_t fa2_fwd_sm100_workspace_bytes(const Fa2FwdParams* p);

/* Split-KV forward that allocates nothing. No counterpart in the reference.
 *
 * For callers that cannot allocate device memory at call time: code running inside a
 * CUDA graph being captured or a custom allocator callback, inference runtimes that own
 * every device allocation and forbid cudaMalloc on the hot path, or plugins that receive
 * only input and output pointers. Same contract as fa2_fwd_sm100, but the split-KV partials
 * (fp32 partial O and row log-sum-exp, see fa2_fwd_sm100_workspace_bytes) go to a static
 * device array of FA2_NOALLOC_SCRATCH_BYTES that belongs to this library; p->workspace and
 * p->workspace_bytes are ignored. The caller still passes q, k, v and o.
 *
 * Limits and behaviour:
 *  - returns FA2_ERR_SCRATCH_LIMIT (and launches nothing) when the call needs more scratch
 *    than FA2_NOALLOC_SCRATCH_BYTES; use fewer splits or fa2_fwd_sm100 with a workspace;
 *  - the array is created when the library's GPU code is loaded and every GPU that loads the
 *    library holds it until the process exits;
 *  - the first call on each device, whatever its num_splits, looks up the array's device
 *    address (cudaGetSymbolAddress, once per device, with that device current); make that
 *    first call before any stream capture. Like fa2_fwd_sm100, the first launch of each
 *    kernel variant on a device also sets its shared-memory attribute
 *    (cudaFuncSetAttribute); no call allocates;
 *  - all calls share the one array and it keeps the previous call's contents (nothing in it
 *    needs to start at zero: every slot a call reads is written earlier in the same call), so
 *    calls that overlap on the GPU (other streams, other host threads) race on it: serialise
 *    them, e.g. issue them on one stream;
 *  - calls no cudaMalloc/cudaFree or allocating library routine.
 * With num_splits <= 1 no scratch is used and this behaves as fa2_fwd_sm100. */
FA2_API int fa2_fwd_sm100_noalloc(const Fa2FwdParams* p, void* stream);

/* Static description of the compiled kernel family (fa2/kernel.py:186-195 analogue):
 * fills BLOCK_M, BLOCK_N, threads per CTA, K/V pipeline stages and dynamic shared memory
 * bytes for `head_dim` (16 and 32 report the 64 build that serves them). Returns FA2_OK or
 * FA2_ERR_HEAD_DIM. Host only. */
FA2_API int fa2_fwd_sm100_config(int32_t head_dim, int32_t* block_m, int32_t* block_n,
                         int32_t* threads, int32_t* stages, int32_t* smem_bytes);

/* Human-readable text for a Fa2Status. Never NULL. */
FA2_API const char* fa2_sm100_strerror(int status);

/* FA2_SM100_ABI_VERSION of the loaded library. */
FA2_API int fa2_sm100_abi_version(void);

/* sizeof(Fa2FwdParams) as compiled into the library, so a binding (ctypes, cgo, ...) can
 * verify its mirror of the struct before the first call. */
FA2_API int64_t fa2_sm100_params_size(void);

#ifdef __cplusplus
}
#endif

#endif /* FA2_SM100_H_ */
