/*
 * b200_attn.h — C ABI of the sm_100a fused attention forward.
 *
 * This is the drop-in boundary for the reference's attention operator.  Every
 * entry point takes plain pointers, sizes and strides (no framework types) so a
 * Python ctypes stub, a C++ host or any other FFI can bind it.
 *
 * Semantics follow the reference operator
 *   triton_fused_attention(q, k, v, valid_token_mask, causal, scale, output_bshd)
 *   (model/triton_fused_attention.py:1877-1891), whose value definition is
 *   _reference_attention (model/triton_fused_attention.py:1256-1285):
 *     scores = (q @ k^T) * scale
 *     scores[i, j] = -inf  where causal and j > i            (triu(1) mask, :1273-1279)
 *     scores[:, j] = -inf  where valid_token_mask[b, j] == 0  (key padding, :1280-1283)
 *     out = softmax_fp32(scores).to(dtype) @ v               (:1284-1285)
 *   A row whose keys are all masked yields NaN, as torch.softmax does.
 *
 * Tensors are [B, H, S, D] views whose last dimension is contiguous; the three
 * outer strides are given in ELEMENTS and may describe transposed projection
 * views ([B, S, H*D] seen as [B, H, S, D]) or a contiguous [B, S, H, D] output
 * (the reference's output_bshd=True layout, :1950-1957).
 */
#ifndef B200_ATTN_H_
#define B200_ATTN_H_

#include <stdint.h>

#if defined(__GNUC__)
#define B200_ATTN_API __attribute__((visibility("default")))
#else
#define B200_ATTN_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define B200_ATTN_ABI_VERSION 2

/* Element types of q, k, v and the output.  fp32 inputs are multiplied on the
 * tensor cores as TF32 (10-bit mantissa products, fp32 accumulation), the
 * reference's fp32 tiled kernel's precision (model/triton_fused_attention.py:
 * 235-356); the softmax and the output stay fp32. */
enum {
  B200_ATTN_DTYPE_BF16 = 0,
  B200_ATTN_DTYPE_FP16 = 1,
  B200_ATTN_DTYPE_FP32 = 2
};

/* Return codes.  Entry points never abort the process. */
enum {
  B200_ATTN_OK = 0,
  B200_ATTN_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad size, non-positive scale   */
  B200_ATTN_ERR_UNSUPPORTED = 2,      /* dtype / head_dim outside the kernel envelope */
  B200_ATTN_ERR_ALIGNMENT = 3,        /* base or stride not 16-byte aligned            */
  B200_ATTN_ERR_DEVICE = 4,           /* no sm_100 device, or pointer not on a device  */
  B200_ATTN_ERR_LAUNCH = 5,           /* CUDA launch / tensor-map encoding failed      */
  B200_ATTN_ERR_TIMEOUT = 6,          /* an earlier launch reported a pipeline wait
                                         timeout in the (host) error word; nothing
                                         was launched                                */
  B200_ATTN_ERR_DEVICE_BOUNDS = 7     /* an earlier launch reported a failed bounds
                                         check (checked build) in the (host) error
                                         word; nothing was launched                  */
};

/* Bits the kernel ORs into *error_word (when error_word != NULL). */
enum {
  B200_ATTN_DEVERR_WAIT_TIMEOUT = 1,
  /* checked build only: a TMA coordinate, shared-memory tile address or
   * tensor-memory column range failed its check; the access was skipped */
  B200_ATTN_DEVERR_BOUNDS = 2
};

typedef struct b200_attn_fwd_params {
  const void* q;           /* [B,H,S,D] */
  const void* k;           /* [B,H,S,D] */
  const void* v;           /* [B,H,S,D] */
  void* o;                 /* [B,H,S,D] view of the output */
  int64_t batch;
  int64_t heads;
  int64_t seq_len;
  int64_t head_dim;
  /* strides in elements: {batch, head, seq}; the D stride must be 1 */
  int64_t q_stride[3];
  int64_t k_stride[3];
  int64_t v_stride[3];
  int64_t o_stride[3];
  /* optional bool [B,S] key-validity mask (1 = valid key), NULL = no mask */
  const uint8_t* key_mask;
  int64_t mask_stride[2];  /* {batch, seq} in bytes */
  float scale;             /* softmax scale, > 0 (reference default D**-0.5) */
  int32_t dtype;           /* B200_ATTN_DTYPE_* */
  int32_t causal;          /* 1: key j visible to query i iff j <= i (top-left aligned) */
  int32_t zero_masked_queries; /* 1: rows whose own mask bit is 0 are written as 0 */
  int32_t* error_word;     /* optional int32 the kernel reports B200_ATTN_DEVERR_* bits in
                              (see "Error word" below) */
} b200_attn_fwd_params;

/* Error word.  `error_word` (here and in the linear and softmax params) is
 * NULL, a device int32, or a pinned host int32 the device addresses directly
 * (cudaHostAlloc, or any pinned allocation under unified addressing).
 *   - device word: kernels OR their B200_ATTN_DEVERR_* bits in atomically; the
 *     caller reads it after synchronising.
 *   - host word: the caller can read it at any time without synchronising.
 *     Every entry point reads it before launching and, while it is non-zero,
 *     launches nothing and returns B200_ATTN_ERR_TIMEOUT (timeout bit set) or
 *     B200_ATTN_ERR_DEVICE_BOUNDS; the caller clears it (writes 0) once it has
 *     handled the report.  Kernels write a host word with plain stores, so two
 *     CTAs reporting at once may keep only one CTA's bits; a report never
 *     leaves the word zero.
 * A launch whose kernel reported an error has undefined output. */

/* ABI version (B200_ATTN_ABI_VERSION). */
B200_ATTN_API int32_t b200_attn_abi_version(void);

/* Host-only envelope query: 1 when the kernel computes (dtype, head_dim) for
 * the given causal/mask flags (bf16/fp16: head_dim any multiple of 8 up to 128;
 * fp32: any multiple of 8 up to 64), else 0.
 * Makes no CUDA call.  Head dims below 64 (above 64) run the 64-wide (128-wide)
 * kernel instance with the missing columns read as zeros by TMA; the result is
 * that of the true head dim.
 * Replaces the support test of triton_fused_attention
 * (model/triton_fused_attention.py:1906-1921) and the planner's envelope
 * (model/attention_dispatch.py:399-459). */
B200_ATTN_API int32_t b200_attn_query(int32_t dtype, int64_t head_dim, int32_t causal, int32_t has_mask);

/* Host-only argument validation (shape, dtype, alignment, strides).  Returns a
 * B200_ATTN_* code and makes no CUDA call.  Replaces _validate_inputs
 * (model/triton_fused_attention.py:1217-1253) for the device path. */
B200_ATTN_API int32_t b200_attn_check(const b200_attn_fwd_params* p);

/* Launch the forward on `stream` (a cudaStream_t of the tensors' device; NULL =
 * legacy default stream).  The device is taken from the q pointer; the caller's
 * current device is left as it was.  Asynchronous: no device synchronisation,
 * no allocation.  The kernel is launched with programmatic stream
 * serialization: its set-up may overlap the previous kernel's tail, and it
 * touches global memory only after that kernel has completed, so stream order
 * holds as for a plain launch.  Replaces the kernel
 * launch of triton_fused_attention (model/triton_fused_attention.py:1968-2001). */
B200_ATTN_API int32_t b200_attn_fwd(const b200_attn_fwd_params* p, void* stream);

/* Static text for a return code. */
B200_ATTN_API const char* b200_attn_error_string(int32_t code);

/* Number of kernel launches b200_attn_fwd issues per call for these params
 * (host-only; used by benchmarks to count launches). */
B200_ATTN_API int32_t b200_attn_launches_per_call(const b200_attn_fwd_params* p);

/* Text of the last host-side failure on the calling thread (CUDA error string,
 * tensor-map encoding failure); empty when none. */
B200_ATTN_API const char* b200_attn_last_error_detail(void);

/* Kernel launches issued so far by every entry point of this library in this
 * process (attention, linear, LayerNorm, softmax), counted on the host after
 * each successful launch (no reference counterpart; benchmarks count their
 * launches with it).  Launches replayed from a CUDA graph are counted once, at
 * capture. */
B200_ATTN_API int64_t b200_attn_launch_count(void);

/* Launch shape of the kernel instance b200_attn_fwd runs for (dtype,
 * head_dim), host-only: query rows per tensor-memory tile, query rows per CTA,
 * keys per K/V tile, warps per CTA and K/V ring slots (one K or one V tile per
 * slot).  Returns 1 and fills the outputs when the pair is supported, else 0.
 * Replaces the launch metadata the reference planner attaches to its plans
 * (model/attention_dispatch.py:303-354). */
B200_ATTN_API int32_t b200_attn_launch_shape(int32_t dtype, int64_t head_dim, int32_t* block_m,
                                             int32_t* rows_per_cta, int32_t* block_n,
                                             int32_t* num_warps, int32_t* ring_slots);

/* One step of context-parallel attention (no reference counterpart: the
 * reference runs every sequence on one device).  A sequence too long for one
 * GPU is split into chunks of equal length; the query chunk attends to one key
 * chunk per call, and the calls for all key chunks the query chunk sees are
 * merged in the output, exactly as attention over the whole key sequence:
 *   lse[b, h, i] = log(sum_j exp(scores[i, j]))      (this chunk's visible keys)
 *   accumulate = 0:  O = softmax over this chunk (as b200_attn_fwd),  lse written
 *   accumulate = 1:  O, lse = the merge of the (O, lse) in memory with this chunk's:
 *                    lse' = log(exp(lse) + exp(lse_chunk)),
 *                    O'   = O * exp(lse - lse') + O_chunk * exp(lse_chunk - lse')
 * `base.causal` is the diagonal chunk's mask (key j visible to query i iff
 * j <= i inside the chunk pair); a key chunk wholly before the query chunk is
 * passed with causal = 0 and one wholly after it is not passed.  A row that saw
 * no visible key in any chunk is NaN with lse -inf.  Key masks and
 * zero_masked_queries are not taken (B200_ATTN_ERR_UNSUPPORTED).  O is read
 * and written in the element type, so each accumulating call rounds it once. */
typedef struct b200_attn_partial_params {
  b200_attn_fwd_params base;
  float* lse;              /* [B, H, S] fp32 log-sum-exp (natural log), read when accumulating */
  int64_t lse_stride[3];   /* {batch, head, seq} in elements */
  int32_t accumulate;      /* 0: first chunk; 1: merge into (base.o, lse) */
  int32_t reserved;        /* 0 */
} b200_attn_partial_params;

B200_ATTN_API int32_t b200_attn_fwd_partial(const b200_attn_partial_params* p, void* stream);

/* Largest batch * heads * seq_len b200_attn_fwd_partial_static takes: its
 * log-sum-exp array holds this many fp32 values (4 MiB) on every device. */
#define B200_ATTN_STATIC_LSE_MAX_ROWS (1 << 20)

/* Allocation-free form of b200_attn_fwd_partial (no counterpart in the
 * reference, which allocates every buffer through torch).  It is for callers
 * that cannot call cudaMalloc: a host whose memory pool already owns the
 * device's memory, a loop that cannot take the device-wide synchronisation of
 * cudaMalloc/cudaFree, or a foreign-language binding with no device allocator.
 * Such a caller passes q, k, v and o as for b200_attn_fwd_partial (base.key_mask
 * NULL, base.zero_masked_queries 0); the per-row log-sum-exp that carries one
 * query chunk's merge from call to call lives in a fixed array inside this
 * library instead of a caller buffer, so nothing is allocated.
 *   - Limit: batch * heads * seq_len <= B200_ATTN_STATIC_LSE_MAX_ROWS, else
 *     B200_ATTN_ERR_INVALID_ARGUMENT and nothing is launched.
 *   - accumulate = 0 writes every row's log-sum-exp (nothing needs clearing);
 *     accumulate = 1 merges into what the last call on this device left, and
 *     is refused (B200_ATTN_ERR_INVALID_ARGUMENT) unless the last launched
 *     first-chunk call on this device had the same batch, heads and seq_len.
 *   - The array is shared by every call on a device and keeps the last call's
 *     contents: calls that overlap on the GPU (two streams, or another query
 *     chunk's first call between a chunk's calls) race and give undefined
 *     output.  Issue one query chunk's calls in order on one stream.
 *   - The first call on each device looks up the array's device address
 *     (once, with that device current); make that first call before any
 *     stream capture.  The array itself occupies its 4 MiB on every device
 *     that loads the library, until the process exits.
 * Return codes and the error word are those of b200_attn_fwd_partial. */
B200_ATTN_API int32_t b200_attn_fwd_partial_static(const b200_attn_fwd_params* p,
                                                   int32_t accumulate, void* stream);

/* Self-test of failure detection (no reference counterpart).  Launches the
 * forward exactly like b200_attn_fwd, except that in every CTA the K/V load
 * number `skipped_load` (0 = first K tile, 1 = first V tile, ...) is announced
 * to its barrier but never issued.  The pipeline wait on it runs out after its
 * one-second bound: the kernel ORs B200_ATTN_DEVERR_WAIT_TIMEOUT into
 * *error_word, lets every role fall through, waits (bounded) for its own copies
 * and MMAs, frees TMEM and returns, leaving the CUDA context usable.  Supported
 * for bf16, head_dim 128, causal, no mask, with a non-null error_word
 * (B200_ATTN_ERR_UNSUPPORTED otherwise).  A CTA that reaches the skipped load
 * takes about two seconds; the output is undefined. */
B200_ATTN_API int32_t b200_attn_selftest_stall(const b200_attn_fwd_params* p, int32_t skipped_load,
                                               void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200_ATTN_H_ */
