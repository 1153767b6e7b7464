/*
 * b200_softmax.h — C ABI of the row softmax over materialised attention
 * scores (the reference's unfused attention seam).
 *
 * Semantics of the reference's triton_attention_softmax
 * (model/triton_softmax.py:99-161, kernel :19-96), the softmax stage of the
 * organiser's BaselineSelfAttention (torch_transformer_benchmark.py:98-112):
 *   x = round_to_dtype(scores * scale)                 (the scale multiply in dtype)
 *   x[i, j] = -inf  where causal and j > i              (i = the row's query index)
 *   x[:, j] = -inf  where key_mask[b, j] == 0
 *   probs = exp(x - max(x)) / sum(exp(x - max(x)))      (fp32, IEEE division)
 *   rounded once to the dtype.  A row whose keys are all masked is NaN, as
 *   torch.softmax of an all -inf row is.
 *
 * scores and probs are contiguous [B, H, S, S] tensors of one element type
 * (B200_ATTN_DTYPE_* from b200_attn.h: bf16, fp16 or fp32); probs may be
 * scores itself (in place) but must not overlap it otherwise.  Return codes are
 * the B200_ATTN_* codes.
 */
#ifndef B200_SOFTMAX_H_
#define B200_SOFTMAX_H_

#include "b200_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Longest row the kernels take (the reference's row-kernel limit,
 * model/triton_softmax.py:138-140). */
#define B200_SOFTMAX_MAX_SEQ 65536

typedef struct b200_softmax_params {
  const void* scores;      /* [B, H, S, S] contiguous, unscaled q k^T */
  void* probs;             /* [B, H, S, S] contiguous output (may be scores) */
  int64_t batch;
  int64_t heads;
  int64_t seq_len;         /* S, 1..B200_SOFTMAX_MAX_SEQ */
  const uint8_t* key_mask; /* optional bool [B, S] (1 = valid key); NULL = no mask */
  int64_t mask_stride[2];  /* {batch, seq} in bytes */
  float scale;             /* > 0 */
  int32_t dtype;           /* B200_ATTN_DTYPE_* */
  int32_t causal;          /* 1: key j visible to query i iff j <= i */
  int32_t reserved;        /* 0 */
} b200_softmax_params;

/* Host-only validation (sizes, dtype, scale, 16-byte base alignment, and
 * aliasing: probs is scores or disjoint from it).  Makes no CUDA call.
 * Replaces the checks of triton_attention_softmax (model/triton_softmax.py:
 * 106-140) for the device path. */
B200_ATTN_API int32_t b200_softmax_check(const b200_softmax_params* p);

/* Launch the softmax on `stream` (NULL = legacy default stream): one kernel,
 * no allocation, no synchronisation; the caller's current device is left as it
 * was.  Replaces the Triton launch of triton_attention_softmax
 * (model/triton_softmax.py:142-161). */
B200_ATTN_API int32_t b200_softmax_fwd(const b200_softmax_params* p, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200_SOFTMAX_H_ */
