// layernorm.cu — LayerNorm over the last dimension of the block's 16-bit
// activations (the reference block's norm1 / norm2 and the final norm,
// torch_transformer_benchmark.py:141-142, 170):
//   y = (x - mean) * rsqrt(var + eps) * weight + bias
// mean and biased variance in fp32 (two passes over the row held in
// registers, widened once), the affine step ((x - mean) * rstd * weight + bias)
// in fp32, one rounding to the element type.
//
// HBM-bound: one warp per row, 16-byte loads and stores (a warp reads and
// writes whole contiguous 512-byte segments), the row kept in registers
// between the mean and variance reductions, so every byte of x is read once
// and every byte of y written once.  Eight rows per 256-thread block.
// With an addend, the residual add that precedes the norm in the reference
// block is done in the same pass (x + addend rounded once, optionally stored).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <mutex>

#include "b200_layernorm.h"
#include "byte_range.h"
#include "error_word.cuh"

namespace b200ln {

using b200attn::ByteRange;
using b200attn::count_launch;
using b200attn::rows_range;
using b200attn::set_error;

constexpr int kRowsPerBlock = 8;
constexpr int kThreads = 32 * kRowsPerBlock;
constexpr int kMaxCols = 4096;  // the row stays in registers (16 vectors per lane)

struct LnArgs {
  const uint16_t* x;
  const uint16_t* w;
  const uint16_t* b;
  uint16_t* y;
  const uint16_t* add;  // addend or null
  uint16_t* sum;        // x + addend out, or null
  int64_t rows, ldx, ldy, lda, lds;
  int32_t cols;
  float eps;
};

template <bool BF16>
__device__ __forceinline__ float2 unpack2(uint32_t v) {
  if constexpr (BF16) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
  } else {
    __half2 h = *reinterpret_cast<__half2*>(&v);
    return __half22float2(h);
  }
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (BF16) {
    __nv_bfloat162 r = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&r);
  } else {
    __half2 r = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&r);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Packed fp32 pairs (sm_100 .f32x2): each lane rounds like the scalar op.
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// 16 bytes of a row: through the non-coherent (read-only) path when no
// output of the launch aliases the row's tensor, else a plain global load.
template <bool NC>
__device__ __forceinline__ uint4 load16(const uint16_t* p) {
  if constexpr (NC) {
    return __ldg(reinterpret_cast<const uint4*>(p));
  } else {
    return *reinterpret_cast<const uint4*>(p);
  }
}

// VPL: 16-byte vectors per lane (8 elements each), cols <= 256 * VPL.  The
// row is widened to fp32 once and kept in registers (4 * VPL pairs per lane).
// ADD: normalise x + addend (rounded once to the element type), optionally
// writing that sum; each lane reads its columns in full before it writes
// them, so y or the sum may overwrite x in place.  NC: x and the addend stay
// read-only for the whole launch (no output aliases them), so they may be
// read through the non-coherent path.
template <int VPL, bool BF16, bool ADD, bool NC>
__global__ void __launch_bounds__(kThreads) layernorm_kernel(const LnArgs a) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kRowsPerBlock + warp;
  if (row >= a.rows) return;
  const uint16_t* xr = a.x + row * a.ldx;
  float2 f[VPL][4];
  float2 s2 = make_float2(0.f, 0.f);
  uint4 v[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int col = (i * 32 + lane) * 8;
    v[i] = col < a.cols ? load16<NC>(xr + col) : make_uint4(0u, 0u, 0u, 0u);
  }
  if constexpr (ADD) {
    const uint16_t* ar = a.add + row * a.lda;
    uint16_t* sr = a.sum ? a.sum + row * a.lds : nullptr;
    uint4 tv[VPL];  // every load of the row is in flight before the first add
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int col = (i * 32 + lane) * 8;
      tv[i] = col < a.cols ? load16<NC>(ar + col) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      const int col = (i * 32 + lane) * 8;
      if (col >= a.cols) continue;
      uint32_t* w = reinterpret_cast<uint32_t*>(&v[i]);
      const uint32_t* tw = reinterpret_cast<const uint32_t*>(&tv[i]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 sum = add2(unpack2<BF16>(w[j]), unpack2<BF16>(tw[j]));
        w[j] = pack2<BF16>(sum.x, sum.y);  // the 16-bit residual sum
      }
      if (sr) *reinterpret_cast<uint4*>(sr + col) = v[i];
    }
  }
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&v[i]);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      f[i][j] = unpack2<BF16>(w[j]);
      s2 = add2(s2, f[i][j]);
    }
  }
  const float inv_n = 1.f / static_cast<float>(a.cols);
  const float mean = warp_sum(s2.x + s2.y) * inv_n;
  const float2 neg_mean = make_float2(-mean, -mean);
  float2 q2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int col = (i * 32 + lane) * 8;
    if (col >= a.cols) continue;  // padding lanes hold zeros, not x - mean
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 d = add2(f[i][j], neg_mean);
      q2 = fma2(d, d, q2);
    }
  }
  const float rstd = rsqrtf(warp_sum(q2.x + q2.y) * inv_n + a.eps);
  const float2 r2 = make_float2(rstd, rstd);
  uint16_t* yr = a.y + row * a.ldy;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int col = (i * 32 + lane) * 8;
    if (col >= a.cols) continue;
    const uint4 g4 = a.w ? __ldg(reinterpret_cast<const uint4*>(a.w + col)) : make_uint4(0u, 0u, 0u, 0u);
    const uint4 b4 = a.b ? __ldg(reinterpret_cast<const uint4*>(a.b + col)) : make_uint4(0u, 0u, 0u, 0u);
    const uint32_t* gw = reinterpret_cast<const uint32_t*>(&g4);
    const uint32_t* bw = reinterpret_cast<const uint32_t*>(&b4);
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 n = mul2(add2(f[i][j], neg_mean), r2);  // (x - mean) * rstd
      const float2 g = a.w ? unpack2<BF16>(gw[j]) : make_float2(1.f, 1.f);
      const float2 bb = a.b ? unpack2<BF16>(bw[j]) : make_float2(0.f, 0.f);
      const float2 y = fma2(n, g, bb);
      o[j] = pack2<BF16>(y.x, y.y);
    }
    *reinterpret_cast<uint4*>(yr + col) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <bool BF, bool ADD, bool NC>
void launch_vpl(const LnArgs& a, unsigned grid, cudaStream_t s) {
  const int vpl = (a.cols + 255) / 256;
  if (vpl <= 1) layernorm_kernel<1, BF, ADD, NC><<<grid, kThreads, 0, s>>>(a);
  else if (vpl <= 2) layernorm_kernel<2, BF, ADD, NC><<<grid, kThreads, 0, s>>>(a);
  else if (vpl <= 4) layernorm_kernel<4, BF, ADD, NC><<<grid, kThreads, 0, s>>>(a);
  else if (vpl <= 8) layernorm_kernel<8, BF, ADD, NC><<<grid, kThreads, 0, s>>>(a);
  else layernorm_kernel<16, BF, ADD, NC><<<grid, kThreads, 0, s>>>(a);
}

template <bool BF>
int launch(const LnArgs& a, bool in_place, cudaStream_t s) {
  const unsigned grid = static_cast<unsigned>((a.rows + kRowsPerBlock - 1) / kRowsPerBlock);
  if (a.add) {
    if (in_place) launch_vpl<BF, true, false>(a, grid, s);
    else launch_vpl<BF, true, true>(a, grid, s);
  } else {
    if (in_place) launch_vpl<BF, false, false>(a, grid, s);
    else launch_vpl<BF, false, true>(a, grid, s);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(cudaGetErrorString(e));
    return B200_ATTN_ERR_LAUNCH;
  }
  count_launch();
  return B200_ATTN_OK;
}

ByteRange x_range(const b200_layernorm_params* p) {
  return rows_range(p->x, p->rows, p->cols, p->x_row_stride);
}
ByteRange y_range(const b200_layernorm_params* p) {
  return rows_range(p->y, p->rows, p->cols, p->y_row_stride);
}
ByteRange add_range(const b200_layernorm_params* p) {
  return rows_range(p->addend, p->rows, p->cols, p->addend_row_stride);
}
ByteRange sum_range(const b200_layernorm_params* p) {
  return rows_range(p->sum, p->rows, p->cols, p->sum_row_stride);
}

// An output may be an input itself (same base and row stride: each lane reads
// its columns before it writes them); any other overlap between an output and
// an input, or between the two outputs, lets warps write rows another warp
// still reads or writes.
bool same_rows(const void* a, int64_t lda, const void* b, int64_t ldb, int64_t rows) {
  return a == b && (rows == 1 || lda == ldb);
}

// Whether an output aliases an input (the launch then reads x and the addend
// with coherent loads).  Call only after b200_layernorm_check passed.
bool aliases(const b200_layernorm_params* p) {
  const ByteRange y = y_range(p);
  if (y.overlaps(x_range(p))) return true;
  if (p->addend && y.overlaps(add_range(p))) return true;
  if (p->sum) {
    const ByteRange s = sum_range(p);
    if (s.overlaps(x_range(p)) || s.overlaps(add_range(p))) return true;
  }
  return false;
}

struct DeviceGuard {
  int prev = -1;
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

}  // namespace b200ln

using namespace b200ln;

extern "C" int32_t b200_layernorm_check(const b200_layernorm_params* p) {
  if (!p || !p->x || !p->y) return B200_ATTN_ERR_INVALID_ARGUMENT;
  // one block per kRowsPerBlock rows, at most 2^31 - 1 blocks
  if (p->rows < 1 || p->cols < 1 || p->rows > static_cast<int64_t>(kRowsPerBlock) * 0x7fffffffll)
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (!(p->eps > 0.f) || !std::isfinite(p->eps)) return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->dtype != B200_ATTN_DTYPE_BF16 && p->dtype != B200_ATTN_DTYPE_FP16)
    return B200_ATTN_ERR_UNSUPPORTED;
  if (p->cols > kMaxCols) return B200_ATTN_ERR_UNSUPPORTED;
  if (p->rows > 1 && (p->x_row_stride < p->cols || p->y_row_stride < p->cols))
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->cols % 8 != 0) return B200_ATTN_ERR_ALIGNMENT;
  if (!aligned16(p->x) || !aligned16(p->y)) return B200_ATTN_ERR_ALIGNMENT;
  if ((p->weight && !aligned16(p->weight)) || (p->bias && !aligned16(p->bias)))
    return B200_ATTN_ERR_ALIGNMENT;
  if (p->rows > 1 && (p->x_row_stride % 8 != 0 || p->y_row_stride % 8 != 0))
    return B200_ATTN_ERR_ALIGNMENT;
  if (!p->addend && p->sum) return B200_ATTN_ERR_INVALID_ARGUMENT;  // a sum needs an addend
  if (p->addend) {
    if (p->rows > 1 && p->addend_row_stride < p->cols) return B200_ATTN_ERR_INVALID_ARGUMENT;
    if (p->sum && p->rows > 1 && p->sum_row_stride < p->cols) return B200_ATTN_ERR_INVALID_ARGUMENT;
    if (p->sum && p->sum == p->y) return B200_ATTN_ERR_INVALID_ARGUMENT;
    if (!aligned16(p->addend) || (p->sum && !aligned16(p->sum))) return B200_ATTN_ERR_ALIGNMENT;
    if (p->rows > 1 &&
        (p->addend_row_stride % 8 != 0 || (p->sum && p->sum_row_stride % 8 != 0)))
      return B200_ATTN_ERR_ALIGNMENT;
  }
  // outputs: each either disjoint from an input or exactly that input
  const ByteRange y = y_range(p);
  if (y.overlaps(x_range(p)) && !same_rows(p->y, p->y_row_stride, p->x, p->x_row_stride, p->rows))
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->addend && y.overlaps(add_range(p)) &&
      !same_rows(p->y, p->y_row_stride, p->addend, p->addend_row_stride, p->rows))
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->sum) {
    const ByteRange s = sum_range(p);
    if (s.overlaps(y)) return B200_ATTN_ERR_INVALID_ARGUMENT;
    if (s.overlaps(x_range(p)) &&
        !same_rows(p->sum, p->sum_row_stride, p->x, p->x_row_stride, p->rows))
      return B200_ATTN_ERR_INVALID_ARGUMENT;
    if (s.overlaps(add_range(p)) &&
        !same_rows(p->sum, p->sum_row_stride, p->addend, p->addend_row_stride, p->rows))
      return B200_ATTN_ERR_INVALID_ARGUMENT;
  }
  return B200_ATTN_OK;
}

extern "C" int32_t b200_layernorm_fwd(const b200_layernorm_params* p, void* stream) {
  const int32_t rc = b200_layernorm_check(p);
  if (rc != B200_ATTN_OK) return rc;
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, p->x) != cudaSuccess || attr.device < 0 ||
      (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)) {
    cudaGetLastError();
    set_error("x is not a device pointer");
    return B200_ATTN_ERR_DEVICE;
  }
  DeviceGuard guard;
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != attr.device) {
    if (cudaSetDevice(attr.device) != cudaSuccess) {
      cudaGetLastError();
      set_error("cudaSetDevice failed");
      return B200_ATTN_ERR_DEVICE;
    }
    guard.prev = cur;
  }
  LnArgs a;
  a.x = static_cast<const uint16_t*>(p->x);
  a.w = static_cast<const uint16_t*>(p->weight);
  a.b = static_cast<const uint16_t*>(p->bias);
  a.y = static_cast<uint16_t*>(p->y);
  a.rows = p->rows;
  a.cols = static_cast<int32_t>(p->cols);
  a.ldx = p->x_row_stride;
  a.ldy = p->y_row_stride;
  a.eps = p->eps;
  a.add = static_cast<const uint16_t*>(p->addend);
  a.sum = static_cast<uint16_t*>(p->sum);
  a.lda = p->addend ? p->addend_row_stride : 0;
  a.lds = p->sum ? p->sum_row_stride : 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool in_place = aliases(p);
  return p->dtype == B200_ATTN_DTYPE_BF16 ? launch<true>(a, in_place, s)
                                          : launch<false>(a, in_place, s);
}
