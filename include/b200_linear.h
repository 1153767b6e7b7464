/*
 * b200_linear.h — C ABI of the sm_100a linear layer with fused epilogues.
 *
 * The layers on either side of the attention operator in the reference's
 * transformer block, with the elementwise passes that follow them folded into
 * the GEMM's epilogue:
 *
 *   y = x W^T + bias                         nn.Linear (q/k/v_proj, out_proj, ffn_in, ffn_out)
 *   y = gelu(x W^T + bias)                   ffn_in followed by the exact GELU
 *                                            (torch_transformer_benchmark.py:142)
 *   y = residual + (x W^T + bias)            the block's residual adds
 *                                            (torch_transformer_benchmark.py:141-142)
 *   rows whose row_mask byte is 0 become 0, or copy the residual unchanged:
 *                                            padded-query zeroing after out_proj
 *                                            (model/triton_fused_attention.py:2456-2461;
 *                                             torch_transformer_benchmark.py:119-122, :144-145)
 *
 * Rounding follows the unfused sequence of 16-bit tensors: the fp32 product
 * plus bias is rounded to the element type; GELU is evaluated in fp32 on that
 * rounded value as x * 0.5 * (1 + erf(x / sqrt(2))) and rounded again; the
 * residual add is an fp32 add of the two 16-bit values, rounded once.
 *
 * Matrices are row-major with a contiguous last dimension; row strides are in
 * ELEMENTS.  x is [M, K], W is [N, K] (the nn.Linear weight layout), bias is
 * [N], residual and y are [M, N], row_mask is [M] bytes.  The element type of
 * every operand is the one `dtype` names (B200_ATTN_DTYPE_* from b200_attn.h);
 * return codes are the B200_ATTN_* codes.
 */
#ifndef B200_LINEAR_H_
#define B200_LINEAR_H_

#include "b200_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

enum {
  B200_LINEAR_ACT_NONE = 0,
  B200_LINEAR_ACT_GELU = 1 /* exact (erf) GELU, torch's approximate="none" */
};

/* What a row whose row_mask byte is 0 receives. */
enum {
  B200_LINEAR_MASKED_ZERO = 0,         /* zeros */
  B200_LINEAR_MASKED_KEEP_RESIDUAL = 1 /* the residual row, unchanged (needs residual) */
};

typedef struct b200_linear_params {
  const void* x;            /* [M, K] */
  const void* w;            /* [N, K] */
  const void* bias;         /* [N] or NULL */
  const void* residual;     /* [M, N] or NULL */
  const uint8_t* row_mask;  /* [M] bytes, 1 = valid row; NULL = every row valid */
  void* y;                  /* [M, N] output; its bytes must not overlap any input's
                               (b200_linear_check returns B200_ATTN_ERR_INVALID_ARGUMENT) */
  int64_t m;
  int64_t n;
  int64_t k;
  int64_t x_row_stride;     /* elements */
  int64_t w_row_stride;
  int64_t residual_row_stride;
  int64_t y_row_stride;
  int32_t dtype;            /* B200_ATTN_DTYPE_* */
  int32_t activation;       /* B200_LINEAR_ACT_* */
  int32_t masked_rows;      /* B200_LINEAR_MASKED_*; used only with row_mask */
  int32_t reserved;         /* 0 */
  int32_t* error_word;      /* optional int32 the kernel reports B200_ATTN_DEVERR_* bits in:
                               a device word or a pinned host word (see "Error word" in
                               b200_attn.h; a host word that holds a report makes
                               b200_linear_fwd return B200_ATTN_ERR_TIMEOUT / _DEVICE_BOUNDS
                               without launching) */
} b200_linear_params;

/* Host-only validation (sizes, dtype, flags, 16-byte alignment of every base
 * and row stride, N and K multiples of 8, y disjoint from every input).  Makes
 * no CUDA call.  Replaces the
 * shape checks torch's nn.Linear applies to these calls. */
B200_ATTN_API int32_t b200_linear_check(const b200_linear_params* p);

/* Launch y = epilogue(x W^T + bias) on `stream` (a cudaStream_t of the
 * tensors' device; NULL = legacy default stream).  One kernel launch, no
 * allocation, no synchronisation; the caller's current device is left as it
 * was.  Replaces the cuBLAS GEMM of nn.Linear plus the elementwise GELU,
 * residual-add and masked_fill passes of the reference block
 * (torch_transformer_benchmark.py:141-145; model/triton_fused_attention.py:2456-2461). */
B200_ATTN_API int32_t b200_linear_fwd(const b200_linear_params* p, void* stream);

/* Output-tile width (128 or 256 columns) b200_linear_fwd picks for these
 * params on a device with `num_sms` SMs (148 on a B200), 0 when the params are
 * invalid.  Host-only, no CUDA call; for benchmarks and tests. */
B200_ATTN_API int32_t b200_linear_tile_n(const b200_linear_params* p, int32_t num_sms);

#ifdef __cplusplus
}
#endif

#endif /* B200_LINEAR_H_ */
