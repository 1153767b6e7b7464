// torch_op.cpp — the attention operator as a torch custom op over the C ABI.
//
// torch.ops.b200.fused_attention keeps the argument meaning, checks and
// exception types of the reference operator triton_fused_attention
// (model/triton_fused_attention.py:1877-1891; _validate_inputs :1217-1253):
// contract violations raise ValueError / TypeError (TORCH_CHECK_VALUE /
// TORCH_CHECK_TYPE), inputs outside the kernel envelope raise ValueError
// (there is no fallback), a launch refused because the error word holds an
// earlier launch's report raises RuntimeError with the "b200 device error"
// prefix.  It validates, allocates the output and launches b200_attn_fwd on the
// current stream in one C++ call, so a call costs no Python-side argument
// packing; the kernel, its tensor maps and its checks are the C library's.
#include <ATen/ATen.h>
#include <c10/core/GradMode.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <cmath>
#include <optional>

#include "b200_attn.h"

namespace {

const char* dtype_name(at::ScalarType t) {
  switch (t) {
    case at::kBFloat16: return "bfloat16";
    case at::kHalf: return "float16";
    case at::kFloat: return "float32";
    default: return c10::toString(t);
  }
}

int32_t dtype_code(at::ScalarType t) {
  switch (t) {
    case at::kBFloat16: return B200_ATTN_DTYPE_BF16;
    case at::kHalf: return B200_ATTN_DTYPE_FP16;
    case at::kFloat: return B200_ATTN_DTYPE_FP32;
    default: return -1;
  }
}

void fill_strides(int64_t dst[3], const at::Tensor& t) {
  dst[0] = t.stride(0);
  dst[1] = t.stride(1);
  dst[2] = t.stride(2);
}

at::Tensor fused_attention(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                           const std::optional<at::Tensor>& valid_token_mask, bool causal,
                           std::optional<double> scale, bool output_bshd,
                           bool zero_masked_queries, const std::optional<at::Tensor>& out,
                           int64_t error_word) {
  // the reference's _validate_inputs (model/triton_fused_attention.py:1217-1253)
  TORCH_CHECK_VALUE(q.dim() == 4, "q must have shape [B, H, S, D], got ", q.sizes());
  TORCH_CHECK_VALUE(k.sizes() == q.sizes() && v.sizes() == q.sizes(),
                    "q, k, and v must have the same [B, H, S, D] shape; got q=", q.sizes(),
                    ", k=", k.sizes(), ", v=", v.sizes());
  TORCH_CHECK_VALUE(q.device() == k.device() && q.device() == v.device(),
                    "q, k, and v must be on the same device");
  TORCH_CHECK_TYPE(q.scalar_type() == k.scalar_type() && q.scalar_type() == v.scalar_type(),
                   "q, k, and v must have the same dtype");
  TORCH_CHECK_TYPE(at::isFloatingType(q.scalar_type()),
                   "q/k/v must use a floating-point dtype, got ", q.scalar_type());
  const int64_t B = q.size(0), H = q.size(1), S = q.size(2), D = q.size(3);
  TORCH_CHECK_VALUE(S > 0 && D > 0, "sequence length and head dimension must be positive");
  const at::Tensor* mask = valid_token_mask.has_value() ? &valid_token_mask.value() : nullptr;
  if (mask) {
    TORCH_CHECK_VALUE(mask->dim() == 2 && mask->size(0) == B && mask->size(1) == S,
                      "valid_token_mask must have shape (", B, ", ", S, "), got ", mask->sizes());
    TORCH_CHECK_TYPE(mask->scalar_type() == at::kBool, "valid_token_mask must have dtype torch.bool");
    TORCH_CHECK_VALUE(mask->device() == q.device(),
                      "valid_token_mask and q must be on the same device");
  }
  const double sc = scale.has_value() ? scale.value() : std::pow(static_cast<double>(D), -0.5);
  TORCH_CHECK_VALUE(sc > 0.0, "scale must be positive");
  // the kernel envelope: no fallback, unsupported inputs raise
  TORCH_CHECK_VALUE(q.is_cuda(), "unsupported sm_100a attention invocation: inputs must be CUDA tensors");
  const int32_t dt = dtype_code(q.scalar_type());
  TORCH_CHECK_VALUE(dt >= 0, "unsupported sm_100a attention invocation: dtype ",
                    dtype_name(q.scalar_type()),
                    " is outside the kernel envelope (bfloat16, float16, float32)");
  TORCH_CHECK_VALUE(b200_attn_query(dt, D, causal ? 1 : 0, mask ? 1 : 0) == 1,
                    "unsupported sm_100a attention invocation: head_dim ", D,
                    " is outside the kernel envelope for ", dtype_name(q.scalar_type()),
                    " (multiples of 8 up to ", dt == B200_ATTN_DTYPE_FP32 ? 64 : 128, ")");
  TORCH_CHECK_VALUE(q.stride(3) == 1 && k.stride(3) == 1 && v.stride(3) == 1,
                    "unsupported sm_100a attention invocation: q/k/v must have a contiguous last "
                    "dimension");
  TORCH_CHECK_VALUE(!(c10::GradMode::is_enabled() &&
                      (q.requires_grad() || k.requires_grad() || v.requires_grad())),
                    "unsupported sm_100a attention invocation: the kernel is inference-only "
                    "(autograd requested)");
  TORCH_CHECK_VALUE(!zero_masked_queries || mask, "zero_masked_queries requires valid_token_mask");

  const std::vector<int64_t> shape = output_bshd ? std::vector<int64_t>{B, S, H, D}
                                                 : std::vector<int64_t>{B, H, S, D};
  at::Tensor result;
  if (out.has_value()) {
    result = out.value();
    TORCH_CHECK_VALUE(result.sizes() == at::IntArrayRef(shape), "out must have shape ", shape);
  } else {
    result = at::empty(shape, q.options());
  }
  const at::Tensor o = output_bshd ? result.transpose(1, 2) : result;
  TORCH_CHECK_VALUE(result.scalar_type() == q.scalar_type() && result.device() == q.device() &&
                        o.stride(3) == 1,
                    "out must match q's dtype and device with a contiguous last dim");

  b200_attn_fwd_params p{};
  p.q = q.data_ptr();
  p.k = k.data_ptr();
  p.v = v.data_ptr();
  p.o = o.data_ptr();
  p.batch = B;
  p.heads = H;
  p.seq_len = S;
  p.head_dim = D;
  fill_strides(p.q_stride, q);
  fill_strides(p.k_stride, k);
  fill_strides(p.v_stride, v);
  fill_strides(p.o_stride, o);
  if (mask) {
    p.key_mask = static_cast<const uint8_t*>(mask->data_ptr());
    p.mask_stride[0] = mask->stride(0);
    p.mask_stride[1] = mask->stride(1);
  }
  p.scale = static_cast<float>(sc);
  p.dtype = dt;
  p.causal = causal ? 1 : 0;
  p.zero_masked_queries = zero_masked_queries ? 1 : 0;
  p.error_word = reinterpret_cast<int32_t*>(static_cast<intptr_t>(error_word));

  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(q.device().index()).stream();
  const int32_t rc = b200_attn_fwd(&p, stream);
  if (rc == B200_ATTN_OK) return result;
  const char* text = b200_attn_error_string(rc);
  TORCH_CHECK_VALUE(rc != B200_ATTN_ERR_INVALID_ARGUMENT && rc != B200_ATTN_ERR_ALIGNMENT,
                    "b200_attn_fwd: ", text);
  TORCH_CHECK_VALUE(rc != B200_ATTN_ERR_UNSUPPORTED, "unsupported sm_100a attention invocation: ",
                    text);
  TORCH_CHECK(rc != B200_ATTN_ERR_TIMEOUT && rc != B200_ATTN_ERR_DEVICE_BOUNDS,
              "b200 device error: b200_attn_fwd refused to launch: ", text);
  TORCH_CHECK(false, "b200_attn_fwd: ", text, " (", b200_attn_last_error_detail(), ")");
}

}  // namespace

TORCH_LIBRARY(b200, m) {
  m.def(
      "fused_attention(Tensor q, Tensor k, Tensor v, Tensor? valid_token_mask, bool causal, "
      "float? scale, bool output_bshd, bool zero_masked_queries, Tensor? out, int error_word) "
      "-> Tensor",
      &fused_attention);
}
