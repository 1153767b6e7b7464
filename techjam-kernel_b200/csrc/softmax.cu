// softmax.cu — row softmax over materialised attention scores for B200: the
// reference's unfused attention seam (model/triton_softmax.py:19-161), whose
// value is the softmax stage of the organiser's BaselineSelfAttention
// (torch_transformer_benchmark.py:98-112):
//   x = round_to_dtype(score * scale); causal / key-mask positions -> -inf;
//   p = exp(x - max) / sum(exp(x - max)) in fp32 (IEEE division), rounded once.
//
// HBM-bound: one read of the scores and one write of the probabilities.  A row
// is owned by a group of G threads (a warp for rows up to 2048 keys, up to a
// 512-thread CTA for 32768 keys) that holds it in registers, EPT elements per
// thread, loaded with 16-byte vectors when rows are 16-byte aligned; the max
// and the sum are reduced with warp shuffles (and shared memory across the
// warps of a group), so every element is read once, exponentiated once and
// written once.  Rows longer than 32768 keys (up to 65536) run a three-pass
// form whose re-reads of the row come from L2.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <mutex>

#include "b200_softmax.h"
#include "byte_range.h"
#include "error_word.cuh"

namespace b200sm {

using b200attn::count_launch;
using b200attn::rows_range;
using b200attn::set_error;

constexpr int kMaxRegisterRow = 32768;  // longest row held in registers
constexpr int kLongThreads = 1024;

struct SmArgs {
  const void* x;
  void* y;
  int64_t rows;  // B * H * S
  int32_t seq;   // S (row length; the query index is row % S)
  int32_t heads;
  const uint8_t* mask;
  int64_t mask_sb, mask_ss;  // bytes
  float scale;
  int32_t causal;
};

// Element type traits: widen to fp32, round an fp32 value to the type.
template <int DT>
struct Elem;
// narrow2 / widen2: a pair in one 32-bit word (low half first), rounded
// like two narrow calls.
template <>
struct Elem<B200_ATTN_DTYPE_BF16> {
  using Raw = uint16_t;
  __device__ static float widen(Raw v) { return __uint_as_float(static_cast<uint32_t>(v) << 16); }
  __device__ static Raw narrow(float x) { return __bfloat16_as_ushort(__float2bfloat16_rn(x)); }
  __device__ static uint32_t narrow2(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
  __device__ static float2 widen2(uint32_t w) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  }
};
template <>
struct Elem<B200_ATTN_DTYPE_FP16> {
  using Raw = uint16_t;
  __device__ static float widen(Raw v) { return __half2float(__ushort_as_half(v)); }
  __device__ static Raw narrow(float x) { return __half_as_ushort(__float2half_rn(x)); }
  __device__ static uint32_t narrow2(float lo, float hi) {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
  __device__ static float2 widen2(uint32_t w) {
    return __half22float2(*reinterpret_cast<const __half2*>(&w));
  }
};
template <>
struct Elem<B200_ATTN_DTYPE_FP32> {
  using Raw = float;
  __device__ static float widen(Raw v) { return v; }
  __device__ static Raw narrow(float x) { return x; }
};

// The score after the scale multiply rounded to the dtype, or -inf when the
// key is not visible to the row's query.
template <int DT>
__device__ __forceinline__ float visible_score(const SmArgs& a, float raw, int64_t col, int64_t q,
                                               const uint8_t* mrow) {
  using E = Elem<DT>;
  bool vis = col < a.seq;
  if (a.causal) vis = vis && col <= q;
  if (mrow) vis = vis && col < a.seq && mrow[col * a.mask_ss] != 0;
  return vis ? E::widen(E::narrow(raw * a.scale)) : -INFINITY;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Packed fp32 pairs (sm_100 .f32x2): each lane rounds like the scalar op.
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
// 2^x on the MUFU; subnormal results are kept (bf16 probabilities share
// fp32's exponent range)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// A pair of scores after the scale multiply, rounded to the dtype.
template <int DT>
__device__ __forceinline__ float2 scaled_pair(float2 x, float scale) {
  using E = Elem<DT>;
  const float2 s = mul2(x, make_float2(scale, scale));
  if constexpr (DT == B200_ATTN_DTYPE_FP32) return s;
  else return E::widen2(E::narrow2(s.x, s.y));
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
// Three-input maximum (sm_100 max.f32 with three sources).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// G threads per row (32 to 512), EPT elements per thread.  VEC:
// rows start on 16-byte boundaries, each thread loads EPT / V vectors of V
// elements at vector index n * G + t.  Without VEC it loads single elements at
// n * G + t.  Both are coalesced across the group.
//
// 16-bit outputs take exp(x - m) as ex2(x * log2e - m * log2e) (one FMA and
// one MUFU operation; the argument's fp32 rounding changes the result by a
// few fp32 units, far below the 16-bit rounding) and multiply by the row sum's
// reciprocal; fp32 outputs keep expf and an IEEE division per element.
template <int G, int EPT, int DT, bool VEC>
__global__ void __launch_bounds__(G < 256 ? 256 : G) softmax_rows_kernel(const SmArgs a) {
  using E = Elem<DT>;
  using Raw = typename E::Raw;
  constexpr bool kExact = DT == B200_ATTN_DTYPE_FP32;
  constexpr float kLog2e = 1.4426950408889634f;
  constexpr int kThreads = G < 256 ? 256 : G;
  constexpr int kRows = kThreads / G;       // rows per CTA
  constexpr int kWarps = G / 32;            // warps per row
  constexpr int V = VEC ? 16 / static_cast<int>(sizeof(Raw)) : 1;
  constexpr int NV = EPT / V;
  static_assert(EPT % V == 0 && EPT % 2 == 0, "whole vectors and pairs per thread");
  __shared__ float red[kRows][kWarps > 1 ? kWarps : 1][2];

  const int t = threadIdx.x % G;
  const int r = threadIdx.x / G;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kRows + r;
  const bool active = row < a.rows;  // inactive threads still join the barriers
  const int64_t S = a.seq;
  const int64_t q = active ? row % S : 0;
  const int64_t b = active ? row / (static_cast<int64_t>(a.heads) * S) : 0;
  const Raw* xr = static_cast<const Raw*>(a.x) + (active ? row : 0) * S;
  Raw* yr = static_cast<Raw*>(a.y) + (active ? row : 0) * S;
  const uint8_t* mrow = a.mask ? a.mask + b * a.mask_sb : nullptr;
  // V mask bytes in one load: a byte-contiguous, V-aligned mask row
  const bool mask_vec = VEC && mrow && a.mask_ss == 1 &&
                        (reinterpret_cast<uintptr_t>(mrow) & (V - 1)) == 0;

  auto col_of = [&](int n, int v) -> int64_t {
    return VEC ? static_cast<int64_t>(n * G + t) * V + v : static_cast<int64_t>(n * G + t);
  };

  float x[EPT];
#pragma unroll
  for (int n = 0; n < NV; ++n) {
    const int64_t c0 = col_of(n, 0);
    if constexpr (VEC) {
      Raw raw[V];
      if (active && c0 < S) {
        *reinterpret_cast<uint4*>(raw) = *reinterpret_cast<const uint4*>(xr + c0);
      } else {
#pragma unroll
        for (int v = 0; v < V; ++v) raw[v] = Raw(0);
      }
#pragma unroll
      for (int v = 0; v < V; ++v) x[n * V + v] = E::widen(raw[v]);
    } else {
      x[n] = (active && c0 < S) ? E::widen(xr[c0]) : 0.f;
    }
  }

  float m = -INFINITY;
  if constexpr (VEC) {
#pragma unroll
    for (int n = 0; n < NV; ++n) {
      const int64_t c0 = col_of(n, 0);
      float* xv = x + n * V;
#pragma unroll
      for (int v = 0; v < V; v += 2) {
        const float2 sp = scaled_pair<DT>(make_float2(xv[v], xv[v + 1]), a.scale);
        xv[v] = sp.x;
        xv[v + 1] = sp.y;
      }
      // the whole vector is in the row (S is a multiple of V); causality and
      // the mask are tested only where they can hide a key
      if (!active || c0 >= S) {
#pragma unroll
        for (int v = 0; v < V; ++v) xv[v] = -INFINITY;
      } else {
        if (a.causal && c0 + V - 1 > q) {
#pragma unroll
          for (int v = 0; v < V; ++v)
            if (c0 + v > q) xv[v] = -INFINITY;
        }
        if (mrow) {
          uint8_t mb[V];
          if (mask_vec) {
            if constexpr (V == 8) *reinterpret_cast<uint2*>(mb) = *reinterpret_cast<const uint2*>(mrow + c0);
            else *reinterpret_cast<uint32_t*>(mb) = *reinterpret_cast<const uint32_t*>(mrow + c0);
          } else {
#pragma unroll
            for (int v = 0; v < V; ++v) mb[v] = mrow[(c0 + v) * a.mask_ss];
          }
#pragma unroll
          for (int v = 0; v < V; ++v)
            if (!mb[v]) xv[v] = -INFINITY;
        }
      }
#pragma unroll
      for (int v = 0; v < V; ++v) m = fmaxf(m, xv[v]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      x[i] = active ? visible_score<DT>(a, x[i], col_of(i, 0), q, mrow) : -INFINITY;
      m = fmaxf(m, x[i]);
    }
  }
  m = warp_max(m);
  if constexpr (kWarps > 1) {
    if ((t & 31) == 0) red[r][t >> 5][0] = m;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < kWarps; ++w) m = fmaxf(m, red[r][w][0]);
  }

  // a row with no visible key keeps m = -inf: x - m is NaN and so is the
  // row, as torch.softmax of an all -inf row
  float sum = 0.f;
  if constexpr (kExact) {
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      x[i] = expf(x[i] - m);
      sum += x[i];
    }
  } else {
    const float2 l2 = make_float2(kLog2e, kLog2e);
    const float2 nm = make_float2(-m * kLog2e, -m * kLog2e);
    float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int i = 0; i < EPT; i += 2) {
      const float2 arg = fma2(make_float2(x[i], x[i + 1]), l2, nm);
      x[i] = ex2_approx(arg.x);
      x[i + 1] = ex2_approx(arg.y);
      s2.x += x[i];
      s2.y += x[i + 1];
    }
    sum = s2.x + s2.y;
  }
  sum = warp_sum(sum);
  if constexpr (kWarps > 1) {
    if ((t & 31) == 0) red[r][t >> 5][1] = sum;
    __syncthreads();
    sum = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) sum += red[r][w][1];
  }

  if (!active) return;
  const float inv = kExact ? 0.f : __frcp_rn(sum);
#pragma unroll
  for (int n = 0; n < NV; ++n) {
    const int64_t c0 = col_of(n, 0);
    if (c0 >= S) continue;
    if constexpr (VEC) {
      Raw out[V];
#pragma unroll
      for (int v = 0; v < V; v += 2) {
        if constexpr (kExact) {
          out[v] = E::narrow(__fdiv_rn(x[n * V + v], sum));
          out[v + 1] = E::narrow(__fdiv_rn(x[n * V + v + 1], sum));
        } else {
          const float2 pv = mul2(make_float2(x[n * V + v], x[n * V + v + 1]), make_float2(inv, inv));
          out[v] = E::narrow(pv.x);
          out[v + 1] = E::narrow(pv.y);
        }
      }
      *reinterpret_cast<uint4*>(yr + c0) = *reinterpret_cast<const uint4*>(out);
    } else {
      yr[c0] = E::narrow(kExact ? __fdiv_rn(x[n], sum) : x[n] * inv);
    }
  }
}

// Warp per row, persistent: each warp walks rows warp, warp + stride, ...
// and loads the next row's vectors before it reduces and stores the current
// one, so a warp keeps two rows of loads in flight.  Rows start on 16-byte
// boundaries (the vector path); EPT elements per lane.  Two CTAs per SM (the
// register cap of __launch_bounds__): 16 warps, each with its row in
// registers and the next row's loads in flight.
template <int EPT, int DT>
__global__ void __launch_bounds__(256, 2) softmax_warp_rows_kernel(const SmArgs a) {
  using E = Elem<DT>;
  using Raw = typename E::Raw;
  constexpr bool kExact = DT == B200_ATTN_DTYPE_FP32;
  constexpr float kLog2e = 1.4426950408889634f;
  constexpr int V = 16 / static_cast<int>(sizeof(Raw));
  constexpr int NV = EPT / V;
  static_assert(EPT % V == 0 && EPT % 2 == 0, "whole vectors and pairs per lane");
  const int lane = threadIdx.x & 31;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  const int64_t S = a.seq;
  int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);

  auto load_row = [&](int64_t r, uint4 (&raw)[NV]) {
    const Raw* xr = static_cast<const Raw*>(a.x) + r * S;
#pragma unroll
    for (int n = 0; n < NV; ++n) {
      const int64_t c0 = static_cast<int64_t>(n * 32 + lane) * V;
      raw[n] = c0 < S ? *reinterpret_cast<const uint4*>(xr + c0) : make_uint4(0u, 0u, 0u, 0u);
    }
  };

  uint4 cur[NV];
  if (row < a.rows) load_row(row, cur);
  for (; row < a.rows; row += stride) {
    // widen this row first, then put the next row's loads in flight: live
    // are the fp32 row and the next row's raw vectors, not three buffers
    float x[EPT];
#pragma unroll
    for (int n = 0; n < NV; ++n) {
      const Raw* raw = reinterpret_cast<const Raw*>(&cur[n]);
#pragma unroll
      for (int v = 0; v < V; ++v) x[n * V + v] = E::widen(raw[v]);
    }
    const int64_t next = row + stride;
    if (next < a.rows) load_row(next, cur);

    // 32-bit column arithmetic (S <= B200_SOFTMAX_MAX_SEQ).  A chunk n covers
    // the warp's columns [n * 32 * V, (n + 1) * 32 * V); with causality every
    // chunk that starts past this row's query index holds only -inf scores,
    // whose probabilities are exact zeros: the warp skips their arithmetic
    // (a warp-uniform test) and stores zeros.
    const int Si = static_cast<int>(S);
    const int q = static_cast<int>(row % S);
    const int64_t b = row / (static_cast<int64_t>(a.heads) * S);
    const uint8_t* mrow = a.mask ? a.mask + b * a.mask_sb : nullptr;
    const bool mask_vec = mrow && a.mask_ss == 1 && (reinterpret_cast<uintptr_t>(mrow) & (V - 1)) == 0;
    auto chunk_live = [&](int n) { return n * 32 * V < Si && !(a.causal && n * 32 * V > q); };
    float m = -INFINITY;
#pragma unroll
    for (int n = 0; n < NV; ++n) {
      if (!chunk_live(n)) continue;
      const int c0 = (n * 32 + lane) * V;
      float* xv = x + n * V;
#pragma unroll
      for (int v = 0; v < V; v += 2) {
        const float2 sp = scaled_pair<DT>(make_float2(xv[v], xv[v + 1]), a.scale);
        xv[v] = sp.x;
        xv[v + 1] = sp.y;
      }
      if (c0 >= Si) {
#pragma unroll
        for (int v = 0; v < V; ++v) xv[v] = -INFINITY;
      } else {
        if (a.causal && c0 + V - 1 > q) {
#pragma unroll
          for (int v = 0; v < V; ++v)
            if (c0 + v > q) xv[v] = -INFINITY;
        }
        if (mrow) {
          uint8_t mb[V];
          if (mask_vec) {
            if constexpr (V == 8) *reinterpret_cast<uint2*>(mb) = *reinterpret_cast<const uint2*>(mrow + c0);
            else *reinterpret_cast<uint32_t*>(mb) = *reinterpret_cast<const uint32_t*>(mrow + c0);
          } else {
#pragma unroll
            for (int v = 0; v < V; ++v) mb[v] = mrow[static_cast<int64_t>(c0 + v) * a.mask_ss];
          }
#pragma unroll
          for (int v = 0; v < V; ++v)
            if (!mb[v]) xv[v] = -INFINITY;
        }
      }
#pragma unroll
      for (int v = 0; v < V; v += 2) m = fmax3(m, xv[v], xv[v + 1]);
    }
    m = warp_max(m);

    float sum = 0.f;
    if constexpr (kExact) {
#pragma unroll
      for (int n = 0; n < NV; ++n) {
        if (!chunk_live(n)) continue;
#pragma unroll
        for (int v = 0; v < V; ++v) {
          const int i = n * V + v;
          x[i] = expf(x[i] - m);
          sum += x[i];
        }
      }
    } else {
      const float2 l2 = make_float2(kLog2e, kLog2e);
      const float2 nm = make_float2(-m * kLog2e, -m * kLog2e);
      float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int n = 0; n < NV; ++n) {
        if (!chunk_live(n)) continue;
#pragma unroll
        for (int v = 0; v < V; v += 2) {
          const int i = n * V + v;
          const float2 arg = fma2(make_float2(x[i], x[i + 1]), l2, nm);
          x[i] = ex2_approx(arg.x);
          x[i + 1] = ex2_approx(arg.y);
          s2 = add2(s2, make_float2(x[i], x[i + 1]));
        }
      }
      sum = s2.x + s2.y;
    }
    sum = warp_sum(sum);

    const float inv = kExact ? 0.f : __frcp_rn(sum);
    Raw* yr = static_cast<Raw*>(a.y) + row * S;
#pragma unroll
    for (int n = 0; n < NV; ++n) {
      const int c0 = (n * 32 + lane) * V;
      if (c0 >= Si) continue;
      Raw out[V];
      if (!chunk_live(n)) {
        // a row with no visible key is NaN throughout, as torch.softmax of
        // an all -inf row
        const float z = m == -INFINITY ? __int_as_float(0x7fc00000) : 0.f;
#pragma unroll
        for (int v = 0; v < V; ++v) out[v] = E::narrow(z);
      } else {
#pragma unroll
        for (int v = 0; v < V; v += 2) {
          if constexpr (kExact) {
            out[v] = E::narrow(__fdiv_rn(x[n * V + v], sum));
            out[v + 1] = E::narrow(__fdiv_rn(x[n * V + v + 1], sum));
          } else {
            const float2 pv = mul2(make_float2(x[n * V + v], x[n * V + v + 1]), make_float2(inv, inv));
            *reinterpret_cast<uint32_t*>(&out[v]) = E::narrow2(pv.x, pv.y);
          }
        }
      }
      *reinterpret_cast<uint4*>(yr + c0) = *reinterpret_cast<const uint4*>(out);
    }
  }
}

// Rows longer than the register form holds: one 1024-thread CTA per row,
// three passes (max, sum, write) whose second and third reads of the row come
// from L2 (a row is at most 256 KB and one CTA per SM is resident).
template <int DT>
__global__ void __launch_bounds__(kLongThreads) softmax_long_kernel(const SmArgs a) {
  using E = Elem<DT>;
  using Raw = typename E::Raw;
  constexpr int kWarps = kLongThreads / 32;
  __shared__ float red[kWarps][2];
  const int64_t row = blockIdx.x;
  const int t = threadIdx.x;
  const int64_t S = a.seq;
  const int64_t q = row % S;
  const int64_t b = row / (static_cast<int64_t>(a.heads) * S);
  const Raw* xr = static_cast<const Raw*>(a.x) + row * S;
  Raw* yr = static_cast<Raw*>(a.y) + row * S;
  const uint8_t* mrow = a.mask ? a.mask + b * a.mask_sb : nullptr;

  float m = -INFINITY;
  for (int64_t c = t; c < S; c += kLongThreads)
    m = fmaxf(m, visible_score<DT>(a, E::widen(xr[c]), c, q, mrow));
  m = warp_max(m);
  if ((t & 31) == 0) red[t >> 5][0] = m;
  __syncthreads();
  for (int w = 0; w < kWarps; ++w) m = fmaxf(m, red[w][0]);

  float sum = 0.f;
  for (int64_t c = t; c < S; c += kLongThreads)
    sum += expf(visible_score<DT>(a, E::widen(xr[c]), c, q, mrow) - m);
  sum = warp_sum(sum);
  if ((t & 31) == 0) red[t >> 5][1] = sum;
  __syncthreads();
  sum = 0.f;
  for (int w = 0; w < kWarps; ++w) sum += red[w][1];

  // each thread rewrites only the elements it read, so probs may be scores
  for (int64_t c = t; c < S; c += kLongThreads) {
    const float e = expf(visible_score<DT>(a, E::widen(xr[c]), c, q, mrow) - m);
    yr[c] = E::narrow(__fdiv_rn(e, sum));
  }
}

int64_t elem_bytes(int32_t dtype) { return dtype == B200_ATTN_DTYPE_FP32 ? 4 : 2; }

// The persistent warp-per-row kernel: enough CTAs to fill every SM several
// times over, each warp walking the rows with a grid stride.
template <int EPT, int DT>
void launch_warp_rows(const SmArgs& a, int num_sms, cudaStream_t s) {
  const int64_t need = (a.rows + 7) / 8;
  const int64_t cap = static_cast<int64_t>(num_sms) * 8;
  const unsigned grid = static_cast<unsigned>(need < cap ? need : cap);
  softmax_warp_rows_kernel<EPT, DT><<<grid, 256, 0, s>>>(a);
}

template <int G, int EPT, int DT>
void launch_rows(const SmArgs& a, bool vec, cudaStream_t s) {
  constexpr int kRows = (G < 256 ? 256 : G) / G;
  const unsigned grid = static_cast<unsigned>((a.rows + kRows - 1) / kRows);
  constexpr int kThreads = G < 256 ? 256 : G;
  if (vec) softmax_rows_kernel<G, EPT, DT, true><<<grid, kThreads, 0, s>>>(a);
  else softmax_rows_kernel<G, EPT, DT, false><<<grid, kThreads, 0, s>>>(a);
}

// Row groups by row length: the smallest group that covers the row with up
// to 64 elements per thread.  A warp per row up to 2048 keys needs no
// barrier, and more rows per SM keep more of the row loads in flight.
template <int DT>
void launch(const SmArgs& a, bool vec, int num_sms, cudaStream_t s) {
  const int S = a.seq;
  // 64 fp32 values per lane fit the two-CTA register budget for 16-bit rows
  // (raw next-row vectors of 32 registers); fp32 rows take at most 32
  constexpr int kWarpMax = (DT == B200_ATTN_DTYPE_FP32 ? 32 : 64) * 32;
  if (vec && S <= kWarpMax) {
    if (S <= 8 * 32) launch_warp_rows<8, DT>(a, num_sms, s);
    else if (S <= 32 * 32 || DT == B200_ATTN_DTYPE_FP32) launch_warp_rows<32, DT>(a, num_sms, s);
    else launch_warp_rows<64, DT>(a, num_sms, s);
    return;
  }
  if (S <= 256) launch_rows<32, 8, DT>(a, vec, s);
  else if (S <= 1024) launch_rows<32, 32, DT>(a, vec, s);
  else if (S <= 2048) launch_rows<32, 64, DT>(a, vec, s);
  else if (S <= 4096) launch_rows<64, 64, DT>(a, vec, s);
  else if (S <= 8192) launch_rows<128, 64, DT>(a, vec, s);
  else if (S <= 16384) launch_rows<256, 64, DT>(a, vec, s);
  else if (S <= kMaxRegisterRow) launch_rows<512, 64, DT>(a, vec, s);
  else softmax_long_kernel<DT><<<static_cast<unsigned>(a.rows), kLongThreads, 0, s>>>(a);
}

struct DeviceGuard {
  int prev = -1;
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// SMs of a device, queried once per device (the persistent kernel's grid).
int sm_count(int device) {
  constexpr int kMaxDevices = 64;
  static std::once_flag once[kMaxDevices];
  static int sms[kMaxDevices];
  if (device < 0 || device >= kMaxDevices) return 148;
  std::call_once(once[device], [device] {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n < 1) {
      cudaGetLastError();
      n = 148;
    }
    sms[device] = n;
  });
  return sms[device];
}

}  // namespace b200sm

using namespace b200sm;

extern "C" int32_t b200_softmax_check(const b200_softmax_params* p) {
  if (!p || !p->scores || !p->probs) return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->batch < 1 || p->heads < 1 || p->seq_len < 1 || p->seq_len > B200_SOFTMAX_MAX_SEQ)
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  // one CTA per row (or per group of rows): rows within the grid limit
  if (p->batch * p->heads > (1ll << 31) || p->batch * p->heads * p->seq_len > 0x7fffffffll)
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (!(p->scale > 0.f) || !std::isfinite(p->scale) || p->reserved != 0)
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->dtype != B200_ATTN_DTYPE_BF16 && p->dtype != B200_ATTN_DTYPE_FP16 &&
      p->dtype != B200_ATTN_DTYPE_FP32)
    return B200_ATTN_ERR_UNSUPPORTED;
  const int64_t eb = elem_bytes(p->dtype);
  if ((reinterpret_cast<uintptr_t>(p->scores) | reinterpret_cast<uintptr_t>(p->probs)) %
          static_cast<uintptr_t>(eb) != 0)
    return B200_ATTN_ERR_ALIGNMENT;
  // probs is scores itself (each group reads its row before writing it) or
  // disjoint from it
  const int64_t rows = p->batch * p->heads * p->seq_len;
  if (p->probs != p->scores &&
      rows_range(p->probs, rows, p->seq_len, p->seq_len, eb)
          .overlaps(rows_range(p->scores, rows, p->seq_len, p->seq_len, eb)))
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  return B200_ATTN_OK;
}

extern "C" int32_t b200_softmax_fwd(const b200_softmax_params* p, void* stream) {
  const int32_t rc = b200_softmax_check(p);
  if (rc != B200_ATTN_OK) return rc;
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, p->scores) != cudaSuccess || attr.device < 0 ||
      (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)) {
    cudaGetLastError();
    set_error("scores is not a device pointer");
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
  SmArgs a;
  a.x = p->scores;
  a.y = p->probs;
  a.rows = p->batch * p->heads * p->seq_len;
  a.seq = static_cast<int32_t>(p->seq_len);
  a.heads = static_cast<int32_t>(p->heads);
  a.mask = p->key_mask;
  a.mask_sb = p->key_mask ? p->mask_stride[0] : 0;
  a.mask_ss = p->key_mask ? p->mask_stride[1] : 0;
  a.scale = p->scale;
  a.causal = p->causal ? 1 : 0;
  const int64_t eb = elem_bytes(p->dtype);
  const bool vec = (p->seq_len * eb) % 16 == 0 &&
                   ((reinterpret_cast<uintptr_t>(p->scores) |
                     reinterpret_cast<uintptr_t>(p->probs)) & 15u) == 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int num_sms = sm_count(attr.device);
  switch (p->dtype) {
    case B200_ATTN_DTYPE_BF16: launch<B200_ATTN_DTYPE_BF16>(a, vec, num_sms, s); break;
    case B200_ATTN_DTYPE_FP16: launch<B200_ATTN_DTYPE_FP16>(a, vec, num_sms, s); break;
    default: launch<B200_ATTN_DTYPE_FP32>(a, vec, num_sms, s); break;
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(cudaGetErrorString(e));
    return B200_ATTN_ERR_LAUNCH;
  }
  count_launch();
  return B200_ATTN_OK;
}
