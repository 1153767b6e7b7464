/*
 * b200_layernorm.h — C ABI of the LayerNorm that runs between the block's
 * linear layers.
 *
 * Semantics of nn.LayerNorm over the last dimension (the block's norm1 and
 * norm2, torch_transformer_benchmark.py:129-131, 141-142, and the model's
 * final_norm, :161, :170):
 *   y = (x - mean(x)) / sqrt(var(x) + eps) * weight + bias
 * with the biased variance; mean, variance and the affine step in fp32, the
 * result rounded once to the element type.
 *
 * x and y are row-major [rows, cols] with a contiguous last dimension (row
 * strides in ELEMENTS); weight and bias are [cols] or NULL (1 and 0).  Element
 * types are B200_ATTN_DTYPE_* (b200_attn.h); return codes are B200_ATTN_*.
 *
 * With an addend the call first forms the block's residual sum
 *   s = x + addend            (an fp32 add rounded once, like a 16-bit tensor add)
 * writes it to `sum` (when not NULL) and normalises s instead of x: the
 * residual add that ends one reference block (torch_transformer_benchmark.py:142)
 * fused with the LayerNorm that starts the next (:141) or the final norm (:170).
 */
#ifndef B200_LAYERNORM_H_
#define B200_LAYERNORM_H_

#include "b200_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct b200_layernorm_params {
  const void* x;          /* [rows, cols] */
  const void* weight;     /* [cols] or NULL */
  const void* bias;       /* [cols] or NULL */
  void* y;                /* [rows, cols]; may be x (or the addend) itself */
  int64_t rows;
  int64_t cols;           /* multiple of 8, at most 4096 */
  int64_t x_row_stride;   /* elements */
  int64_t y_row_stride;
  float eps;              /* > 0 */
  int32_t dtype;          /* B200_ATTN_DTYPE_* */
  const void* addend;     /* [rows, cols] or NULL: normalise x + addend */
  void* sum;              /* [rows, cols] or NULL: receives x + addend (may be x or the
                             addend itself, never y) */
  int64_t addend_row_stride;
  int64_t sum_row_stride;
} b200_layernorm_params;

/* Host-only validation (sizes, dtype, eps, 16-byte alignment of bases and row
 * strides, and aliasing: an output may be exactly an input -- the same base
 * and row stride -- but any other overlap of an output with an input, or of y
 * with sum, returns B200_ATTN_ERR_INVALID_ARGUMENT).  Makes no CUDA call.  Replaces the shape checks of
 * torch.nn.functional.layer_norm for these calls. */
B200_ATTN_API int32_t b200_layernorm_check(const b200_layernorm_params* p);

/* Launch the LayerNorm on `stream` (NULL = legacy default stream): one kernel,
 * no allocation, no synchronisation; the caller's current device is left as it
 * was.  Replaces nn.LayerNorm's forward in the reference block
 * (torch_transformer_benchmark.py:141-142, 170). */
B200_ATTN_API int32_t b200_layernorm_fwd(const b200_layernorm_params* p, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200_LAYERNORM_H_ */
