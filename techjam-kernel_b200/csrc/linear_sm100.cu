// linear_sm100.cu — linear layer with fused epilogues for B200 (sm_100a).
//
//   y = epilogue(x W^T + bias)      x [M,K], W [N,K] (nn.Linear layout), y [M,N]
//
// The epilogue folds in the elementwise passes that follow the reference
// block's GEMMs (torch_transformer_benchmark.py:141-145 and the padded-query
// zeroing after out_proj, model/triton_fused_attention.py:2456-2461):
//   t = round(acc + bias)                       16-bit rounding of the GEMM output
//   t = round(t * 0.5 * (1 + erf(t / sqrt 2)))  exact GELU (optional)
//   y = round(residual + t)                     residual add (optional)
//   masked rows (row_mask byte 0): y = 0, or y = residual unchanged
// which is the rounding sequence of the unfused 16-bit tensor ops.
//
// Two persistent, warp-specialised kernels walk the output tiles
// t = cta (or CTA pair), + number of CTAs (pairs), ..., row-block major so the
// tiles in flight share x rows in L2:
//
// * linear_sm100_pair_kernel (N > 128 and M > 128): clusters of two CTAs on
//   two SMs compute 256 x 256 tiles with cta_group::2 products.  Each CTA
//   loads 128 rows of x and 128 rows of W per 64-wide K step, so every SM
//   streams half the W bytes a one-CTA 128 x 256 tile needs; the leader CTA
//   issues M=256 x N=256 x K=16 products that read both CTAs' shared memory
//   and write 128 accumulator rows into each CTA's tensor memory.
// * linear_sm100_kernel: one CTA per SM, 128 x BN tiles (BN = 128 or 256).
//
// Warp roles (both kernels):
//   warp  0     TMA producer: 64-column slices of x and W into a ring of
//               shared-memory stages, 128-byte swizzle
//   warp  1     TMEM owner; tcgen05 issuer (one thread; the leader CTA's only
//               in the pair kernel)
//   warps 2-9   epilogue: one output row per thread (TMEM lane); warp w reads
//               lanes 32*(w%4)..+31, warps 2-5 the first half of the columns
//               and warps 6-9 the rest; bias, GELU, residual, row mask, then
//               16-byte stores straight to global memory
// Two accumulators (2 x BN <= 512 TMEM columns) let the epilogue of one tile
// overlap the tensor-core work of the next.
//
// In the pair kernel both CTAs' loads complete on the leader CTA's stage
// barriers (the leader's producer announces the bytes of both), the leader's
// issuer commits each stage release and each finished accumulator to the
// barriers at the same offset in both CTAs, and the other CTA's epilogue
// warps arrive remotely on the leader's accumulator-release barrier.
//
// Every mbarrier wait is bounded (wall clock, ~1 s).  On expiry the thread
// sets a CTA abort flag and B200_ATTN_DEVERR_WAIT_TIMEOUT in the caller's
// error word, every role leaves its loop (in the pair kernel the other CTA's
// waits then run out as well), the producer and the issuer wait (bounded) for
// their copies and MMAs in flight, TMEM is freed and the kernel returns.
// There is no trap and no unbounded spin.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "b200_linear.h"
#include "byte_range.h"
#include "error_word.cuh"
#include "sm100_ptx.cuh"

namespace b200lin {

namespace ptx = b200attn::ptx;
using b200attn::ByteRange;
using b200attn::count_launch;
using b200attn::rows_range;
using b200attn::report_error;
using b200attn::resolve_error_word;
using b200attn::set_error;

constexpr int kBM = 128;  // output rows per tile = TMEM lanes
constexpr int kBK = 64;   // K elements per stage = one 128-byte swizzle row
constexpr int kProducerWarp = 0;
constexpr int kMmaWarp = 1;
constexpr int kEpiWarp0 = 2;
constexpr int kEpiWarps = 8;
constexpr int kThreads = 32 * (kEpiWarp0 + kEpiWarps);
constexpr uint64_t kWaitTimeoutNs = 1000000000ull;
constexpr int kIssuerSpin = 4096;
#ifndef B200_LINEAR_TILE_N
#define B200_LINEAR_TILE_N 0
#endif
// 0: the host picks the tile width per shape; 128 or 256 forces it.
constexpr int kForceTileN = B200_LINEAR_TILE_N;
#ifndef B200_LINEAR_CLUSTER_ACQUIRE
#define B200_LINEAR_CLUSTER_ACQUIRE 0
#endif
// Pair kernel: waits on barriers the other CTA (or its loads) completes use
// cluster-scope acquire (1) or the default CTA scope (0).
constexpr bool kClusterAcquire = B200_LINEAR_CLUSTER_ACQUIRE != 0;
#ifndef B200_LINEAR_GROUP_M
#define B200_LINEAR_GROUP_M 8
#endif
// Tile raster: groups of this many row blocks are walked column by column, so
// the tiles in flight share both x rows and W rows in L2 (0: row by row).
constexpr int kGroupM = B200_LINEAR_GROUP_M;

struct LinArgs {
  int32_t m, n, k;
  int32_t num_m_tiles;
  int32_t num_n_tiles;
  int32_t num_tiles;
  int32_t k_blocks;
  const uint16_t* bias;      // [N] or null
  const uint16_t* residual;  // [M, N] or null
  int64_t ld_res;            // elements
  const uint8_t* row_mask;   // [M] or null
  int32_t masked_keep_residual;
  uint16_t* y;
  int64_t ld_y;
  int32_t* err;
};

// Row block and column block of tile t (num_m row blocks, num_n column blocks).
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& tm, int& tn) {
  if (kGroupM > 0) {
    const int per_group = kGroupM * num_n;
    const int g = t / per_group;
    const int rows = min(kGroupM, num_m - g * kGroupM);  // the last group may be shorter
    const int r = t - g * per_group;
    tm = g * kGroupM + r % rows;
    tn = r / rows;
  } else {
    tm = t / num_n;
    tn = t % num_n;
  }
}

template <int BN_>
struct LinCfg {
  static constexpr int BN = BN_;
  static_assert(BN == 128 || BN == 256, "tile width 128 or 256");
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = BN == 256 ? 4 : 6;
  static constexpr int kOffBar = kStages * kStageBytes;
  static constexpr int kBarFull = 0;
  static constexpr int kBarEmpty = kStages;
  static constexpr int kBarAccFull = 2 * kStages;       // [2]
  static constexpr int kBarAccEmpty = 2 * kStages + 2;  // [2]
  static constexpr int kBarDrain = 2 * kStages + 4;
  static constexpr int kNumBars = kBarDrain + 1;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 16 + 1024;  // + alignment slack
  static_assert(kSmemBytes <= 232448, "exceeds the 227 KB per-block shared memory limit");
  static constexpr uint32_t kTmemCols = 2 * BN;
  static constexpr int kHalfCols = BN / 2;    // columns per epilogue warpgroup
  static constexpr int kChunks = kHalfCols / 32;
};

// CTA-pair tiles: 256 x 256 per pair; per CTA and stage 128 rows of x and
// 128 rows (N) of W, and 128 x 256 fp32 per accumulator.
struct PairCfg {
  static constexpr int BN = 256;
  static constexpr int kHalfN = 128;  // W rows per CTA
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = kHalfN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = 5;
  // Output staging: per epilogue half two buffers of 128 rows x 64 columns
  // (16-bit, 128-byte swizzle), written by the threads and stored by TMA; with
  // a residual, TMA first loads the residual block into the same buffer.
  static constexpr int kOutBlockCols = 64;
  static constexpr int kOutBufBytes = kBM * kOutBlockCols * 2;
  static constexpr int kOffOut = kStages * kStageBytes;
  static constexpr int kOffBar = kOffOut + 4 * kOutBufBytes;
  static constexpr int kBarFull = 0;
  static constexpr int kBarEmpty = kStages;
  static constexpr int kBarAccFull = 2 * kStages;       // [2]
  static constexpr int kBarAccEmpty = 2 * kStages + 2;  // [2]
  static constexpr int kBarDrain = 2 * kStages + 4;
  static constexpr int kBarRes = 2 * kStages + 5;       // [half][buffer]
  static constexpr int kNumBars = kBarRes + 4;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 16 + 1024;
  static_assert(kSmemBytes <= 232448, "exceeds the 227 KB per-block shared memory limit");
  static constexpr uint32_t kTmemCols = 2 * BN;
  static constexpr int kHalfCols = BN / 2;
  static constexpr int kBlocksPerHalf = kHalfCols / kOutBlockCols;
};

// ---------------------------------------------------------------- helpers
template <bool kCluster>
__device__ __forceinline__ bool try_wait(uint32_t bar, uint32_t parity) {
  if constexpr (kCluster) {
    return ptx::mbar_try_wait_cluster(bar, parity);
  } else {
    return ptx::mbar_try_wait(bar, parity);
  }
}

template <bool kCluster>
__device__ __noinline__ bool wait_bar_slow(uint32_t bar, uint32_t parity,
                                           volatile uint32_t* abort_flag, int32_t* err) {
  const uint64_t t0 = ptx::globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int k = 0; k < 32; ++k)
      if (try_wait<kCluster>(bar, parity)) return true;
    if (*abort_flag) return false;
    if (ptx::globaltimer_ns() - t0 > kWaitTimeoutNs) {
      *abort_flag = 1u;
      report_error(err, B200_ATTN_DEVERR_WAIT_TIMEOUT);
      return false;
    }
  }
}

// Bounded wait on an mbarrier phase.  Returns false when the CTA was aborted
// (by this thread's timeout or another's).  kCluster: acquire at cluster
// scope, for barriers another CTA arrives on.
template <bool kCluster = false>
__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity,
                                         volatile uint32_t* abort_flag, int32_t* err) {
  if (try_wait<kCluster>(bar, parity)) return true;
  return wait_bar_slow<kCluster>(bar, parity, abort_flag, err);
}

// Issuer-side wait: poll without suspending first, then the bounded wait.
template <bool kCluster = false>
__device__ __forceinline__ bool issuer_wait(uint32_t bar, uint32_t parity,
                                            volatile uint32_t* abort_flag, int32_t* err) {
#pragma unroll 1
  for (int k = 0; k < kIssuerSpin; ++k) {
    const bool done = kCluster ? ptx::mbar_test_wait_cluster(bar, parity)
                               : ptx::mbar_test_wait(bar, parity);
    if (done) return true;
  }
  return wait_bar<kCluster>(bar, parity, abort_flag, err);
}

// Wait by every lane of a warp, made warp-uniform for the warp-collective
// tcgen05 loads that follow.
template <bool kCluster = false>
__device__ __forceinline__ bool warp_wait_bar(uint32_t bar, uint32_t parity,
                                              volatile uint32_t* abort_flag, int32_t* err) {
  const bool ok = wait_bar<kCluster>(bar, parity, abort_flag, err);
  const bool all = __all_sync(0xffffffffu, ok);
  if (!all) *abort_flag = 1u;
  return all;
}

// The two 16-bit values of a packed pair, widened to fp32.
template <bool BF16>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  if constexpr (BF16) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  } else {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    return __half22float2(h);
  }
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}

// x rounded to the element type and widened back.
template <bool BF16>
__device__ __forceinline__ float round16(float x) {
  if constexpr (BF16) {
    return __bfloat162float(__float2bfloat16_rn(x));
  } else {
    return __half2float(__float2half_rn(x));
  }
}

#ifndef B200_LINEAR_GELU_AS
#define B200_LINEAR_GELU_AS 1
#endif
// 1: GELU from the Abramowitz-Stegun erfc formula below, in packed pairs;
// 0: x * 0.5 * (1 + erff(x / sqrt 2)) with CUDA's erff.
constexpr bool kGeluAS = B200_LINEAR_GELU_AS != 0;

// Exact GELU in fp32 in the evaluation order x * 0.5 * (1 + erf(x / sqrt 2)).
__device__ __forceinline__ float gelu_erf(float x) {
  return x * 0.5f * (1.0f + erff(x * 0.70710678118654752440f));
}

// Packed fp32 pairs (sm_100 .f32x2): each lane rounds like the scalar op.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// GELU of a pair, x * Phi(x) with the normal CDF Phi from the complementary
// error function: for z = |x| / sqrt 2, Abramowitz & Stegun (Handbook of
// Mathematical Functions, 7.1.26, after Hastings) give
//   erfc(z) = (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-z^2),  t = 1 / (1 + p z)
// with absolute error <= 1.5e-7.  q = erfc(z) / 2 = Phi(-|x|), so Phi(x) = q for
// x < 0 and 1 - q otherwise; taking erfc directly avoids the cancellation of
// 1 + erf(x / sqrt 2) at negative x.  The coefficients below carry the 1/2.
__device__ __forceinline__ float2 gelu2_as(float2 x) {
  constexpr float kInvSqrt2 = 0.70710678118654752f;
  constexpr float kP = 0.3275911f;
  const float2 z = make_float2(fabsf(x.x) * kInvSqrt2, fabsf(x.y) * kInvSqrt2);
  const float2 den = fma2(make_float2(kP, kP), z, make_float2(1.f, 1.f));
  const float2 t = make_float2(rcp_approx(den.x), rcp_approx(den.y));
  float2 poly = fma2(make_float2(0.5307027145f, 0.5307027145f), t,
                     make_float2(-0.7265760135f, -0.7265760135f));
  poly = fma2(poly, t, make_float2(0.7107068705f, 0.7107068705f));
  poly = fma2(poly, t, make_float2(-0.142248368f, -0.142248368f));
  poly = fma2(poly, t, make_float2(0.127414796f, 0.127414796f));
  poly = mul2(poly, t);
  const float2 arg = mul2(mul2(z, z), make_float2(-1.4426950408889634f, -1.4426950408889634f));
  const float2 e = make_float2(ptx::ex2_approx(arg.x), ptx::ex2_approx(arg.y));
  const float2 q = mul2(poly, e);
  const float2 phi = make_float2(x.x < 0.f ? q.x : 1.f - q.x, x.y < 0.f ? q.y : 1.f - q.y);
  return mul2(x, phi);
}

__device__ __forceinline__ uint4 ld_nc_v4(const uint16_t* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// Residual of one row over 32 columns from col0 (zeros past the row's end and
// for rows outside the matrix).
__device__ __forceinline__ void load_res32(const LinArgs& args, int row, int col0,
                                           uint4 (&r)[4]) {
  const bool row_in = row < args.m;
  const uint16_t* rrow = args.residual + static_cast<int64_t>(row_in ? row : 0) * args.ld_res;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int col = col0 + 8 * g;
    r[g] = (row_in && col < args.n) ? ld_nc_v4(rrow + col) : make_uint4(0u, 0u, 0u, 0u);
  }
}

// Epilogue of 8 consecutive columns of one row: accumulators a[0..7], bias
// and residual as packed 16-bit words; returns the 8 packed outputs.
template <bool kBF16, bool kGelu, bool kRes>
__device__ __forceinline__ uint4 epi8(const uint32_t* a, uint4 bias, uint4 res, bool keep,
                                      int32_t keep_residual) {
  const uint32_t* bw = reinterpret_cast<const uint32_t*>(&bias);
  const uint32_t* rw = reinterpret_cast<const uint32_t*>(&res);
  uint32_t out[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 acc = make_float2(__uint_as_float(a[2 * j]), __uint_as_float(a[2 * j + 1]));
    const float2 sum = add2(acc, unpack2<kBF16>(bw[j]));
    float2 t = make_float2(round16<kBF16>(sum.x), round16<kBF16>(sum.y));
    if constexpr (kGelu) {
      if constexpr (kGeluAS) {
        const float2 g = gelu2_as(t);
        t = make_float2(round16<kBF16>(g.x), round16<kBF16>(g.y));
      } else {
        t = make_float2(round16<kBF16>(gelu_erf(t.x)), round16<kBF16>(gelu_erf(t.y)));
      }
    }
    if constexpr (kRes) {
      const float2 y = add2(unpack2<kBF16>(rw[j]), t);
      out[j] = keep ? pack2<kBF16>(y.x, y.y) : (keep_residual ? rw[j] : 0u);
    } else {
      out[j] = keep ? pack2<kBF16>(t.x, t.y) : 0u;
    }
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

// Epilogue of this thread's output row over kChunks x 32 accumulator columns:
// `tacc` is the TMEM address of the row's first column, the output columns are
// [cbase, cbase + 32 * kChunks), `rnext` holds the first chunk's residual.
// `release()` runs on every lane once the warp's last tcgen05.ld of the tile
// has completed, after which the accumulator may be overwritten.
template <int kChunks, bool kBF16, bool kGelu, bool kRes, class Release>
__device__ __forceinline__ void epilogue_row(const LinArgs& args, uint32_t tacc, int row,
                                             int cbase, uint4 (&rnext)[4], Release&& release) {
  const int N = args.n;
  const bool row_in = row < args.m;
  bool keep = true;
  if (args.row_mask && row_in) keep = args.row_mask[row] != 0;
  uint16_t* yrow = args.y + static_cast<int64_t>(row_in ? row : 0) * args.ld_y;
#pragma unroll 1
  for (int c = 0; c < kChunks; ++c) {
    const int col0 = cbase + 32 * c;
    uint32_t a[32];
    ptx::tmem_ld_32x32b_x32(tacc + 32 * c, a);
    uint4 rcur[4];
    if constexpr (kRes) {
#pragma unroll
      for (int g = 0; g < 4; ++g) rcur[g] = rnext[g];
      if (c + 1 < kChunks) load_res32(args, row, col0 + 32, rnext);
    }
    ptx::tmem_wait_ld();
    if (c == kChunks - 1) release();
    uint4 outv[4];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int col = col0 + 8 * g;
      const uint4 bias = (args.bias && col < N) ? ld_nc_v4(args.bias + col) : make_uint4(0u, 0u, 0u, 0u);
      outv[g] = epi8<kBF16, kGelu, kRes>(a + 8 * g, bias, kRes ? rcur[g] : make_uint4(0u, 0u, 0u, 0u),
                                         keep, args.masked_keep_residual);
    }
    const uint32_t* out = reinterpret_cast<const uint32_t*>(outv);
    if (row_in) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        const int col = col0 + 8 * g;
        if (col < N)
          *reinterpret_cast<uint4*>(yrow + col) =
              make_uint4(out[4 * g], out[4 * g + 1], out[4 * g + 2], out[4 * g + 3]);
      }
    }
  }
}

// ----------------------------------------------------------------- kernel
template <class C, bool kBF16, bool kGelu, bool kRes>
__global__ void __launch_bounds__(kThreads, 1)
    linear_sm100_kernel(const __grid_constant__ CUtensorMap tm_x,
                        const __grid_constant__ CUtensorMap tm_w, const LinArgs args) {
  constexpr int BN = C::BN;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(smem + C::kOffMisc);
  // misc[0] TMEM base, misc[1] abort flag
  volatile uint32_t* abort_flag = misc + 1;
  const uint32_t bar0 = sbase + C::kOffBar;
  auto bar = [&](int idx) { return bar0 + 8u * static_cast<uint32_t>(idx); };

  if (threadIdx.x == 0) {
    misc[1] = 0u;
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(bar(C::kBarFull + s), 1);
      ptx::mbar_init(bar(C::kBarEmpty + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(bar(C::kBarAccFull + b), 1);
      ptx::mbar_init(bar(C::kBarAccEmpty + b), kEpiWarps);  // one arrival per epilogue warp
    }
    ptx::mbar_init(bar(C::kBarDrain), 1);
    ptx::fence_mbar_init();
    ptx::fence_proxy_async_smem();
    ptx::tma_prefetch_desc(&tm_x);
    ptx::tma_prefetch_desc(&tm_w);
  }
  if (warp == kMmaWarp) {
    ptx::tmem_alloc(sbase + C::kOffMisc, C::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = misc[0];
  const int k_blocks = args.k_blocks;

  if (warp == kProducerWarp) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      uint32_t L = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < args.num_tiles; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, args.num_m_tiles, args.num_n_tiles, tm, tn);
        const int m0 = tm * kBM;
        const int n0 = tn * BN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          const uint32_t s = L % S, r = L / S;
          if (!issuer_wait(bar(C::kBarEmpty + s), (r & 1u) ^ 1u, abort_flag, args.err)) {
            ok = false;
            break;
          }
          const uint32_t a_dst = sbase + s * C::kStageBytes;
          ptx::mbar_arrive_expect_tx(bar(C::kBarFull + s), C::kStageBytes);
          ptx::tma_load_2d(a_dst, &tm_x, bar(C::kBarFull + s), kb * kBK, m0);
          ptx::tma_load_2d(a_dst + C::kABytes, &tm_w, bar(C::kBarFull + s), kb * kBK, n0);
          ++L;
        }
      }
      if (!ok) {
        // Let copies already issued land before the CTA's shared memory goes away.
        const uint32_t first = L > static_cast<uint32_t>(S) ? L - S : 0u;
        for (uint32_t x = first; x < L; ++x) {
          const uint64_t t0 = ptx::globaltimer_ns();
          while (!ptx::mbar_try_wait(bar(C::kBarFull + x % S), (x / S) & 1u) &&
                 ptx::globaltimer_ns() - t0 < kWaitTimeoutNs) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------ tcgen05 issuer
    // acc(buf) = x_tile W_tile^T: A = x (K-major), B = W (K-major, BN rows).
    if (lane == 0) {
      constexpr uint32_t idesc = ptx::idesc_f16(kBF16, kBM, BN, false);
      uint32_t L = 0;
      int tc = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < args.num_tiles; t += gridDim.x, ++tc) {
        const int buf = tc & 1;
        const uint32_t use = static_cast<uint32_t>(tc >> 1);
        // the epilogue has read this accumulator's previous tile
        if (!issuer_wait(bar(C::kBarAccEmpty + buf), (use & 1u) ^ 1u, abort_flag, args.err)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t acc = tmem + static_cast<uint32_t>(buf * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          const uint32_t s = L % S, r = L / S;
          if (!issuer_wait(bar(C::kBarFull + s), r & 1u, abort_flag, args.err)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t a_addr = sbase + s * C::kStageBytes;
          const uint32_t b_addr = a_addr + C::kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            ptx::tc_mma_ss(acc, ptx::smem_desc_sw128(a_addr + kk * 32, 16, 1024),
                           ptx::smem_desc_sw128(b_addr + kk * 32, 16, 1024), idesc,
                           (kb > 0 || kk > 0) ? 1u : 0u);
          ptx::tc_commit(bar(C::kBarEmpty + s));  // stage free once these MMAs completed
          ++L;
        }
        if (ok) ptx::tc_commit(bar(C::kBarAccFull + buf));
      }
      // Drain: every MMA this thread issued completes before TMEM is freed.
      ptx::tc_commit(bar(C::kBarDrain));
      const uint64_t t0 = ptx::globaltimer_ns();
      while (!ptx::mbar_try_wait(bar(C::kBarDrain), 0) &&
             ptx::globaltimer_ns() - t0 < kWaitTimeoutNs) {
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - kEpiWarp0;
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int half = e >> 2;    // column half of the tile
    const int rl = quad * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    int tc = 0;
    for (int t = blockIdx.x; t < args.num_tiles; t += gridDim.x, ++tc) {
      const int buf = tc & 1;
      const uint32_t use = static_cast<uint32_t>(tc >> 1);
      int tm, tn;
      tile_coords(t, args.num_m_tiles, args.num_n_tiles, tm, tn);
      const int row = tm * kBM + rl;
      const int cbase = tn * BN + half * C::kHalfCols;
      uint4 rnext[4];  // residual of the first chunk, before the accumulator is ready
      if constexpr (kRes) load_res32(args, row, cbase, rnext);
      if (!warp_wait_bar(bar(C::kBarAccFull + buf), use & 1u, abort_flag, args.err)) break;
      ptx::tc_fence_after();
      const uint32_t tacc = tmem + lane_off + static_cast<uint32_t>(buf * BN + half * C::kHalfCols);
      epilogue_row<C::kChunks, kBF16, kGelu, kRes>(args, tacc, row, cbase, rnext, [&] {
        // this warp's last read of the accumulator: hand it back to the issuer
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(bar(C::kBarAccEmpty + buf));
      });
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------ pair kernel
template <bool kBF16, bool kGelu, bool kRes>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    linear_sm100_pair_kernel(const __grid_constant__ CUtensorMap tm_x,
                             const __grid_constant__ CUtensorMap tm_w,
                             const __grid_constant__ CUtensorMap tm_y,
                             const __grid_constant__ CUtensorMap tm_r, const LinArgs args) {
  using C = PairCfg;
  constexpr int BN = C::BN;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = ptx::cluster_ctarank();  // 0: leader (issues the products)
  const bool leader = rank == 0;
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int num_pairs = static_cast<int>(gridDim.x >> 1);
  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(smem + C::kOffMisc);
  // misc[0] TMEM base, misc[1] abort flag
  volatile uint32_t* abort_flag = misc + 1;
  const uint32_t bar0 = sbase + C::kOffBar;
  auto bar = [&](int idx) { return bar0 + 8u * static_cast<uint32_t>(idx); };

  if (threadIdx.x == 0) {
    misc[1] = 0u;
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(bar(C::kBarFull + s), 1);   // leader: its producer's expect_tx
      ptx::mbar_init(bar(C::kBarEmpty + s), 1);  // the leader's commit, in both CTAs
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(bar(C::kBarAccFull + b), 1);  // the leader's commit, in both CTAs
      ptx::mbar_init(bar(C::kBarAccEmpty + b), 2 * kEpiWarps);  // leader: both CTAs' warps
    }
    ptx::mbar_init(bar(C::kBarDrain), 1);
    for (int b = 0; b < 4; ++b) ptx::mbar_init(bar(C::kBarRes + b), 1);
    ptx::fence_mbar_init();
    ptx::fence_proxy_async_smem();
    ptx::tma_prefetch_desc(&tm_x);
    ptx::tma_prefetch_desc(&tm_w);
    ptx::tma_prefetch_desc(&tm_y);
    if (kRes) ptx::tma_prefetch_desc(&tm_r);
  }
  if (warp == kMmaWarp) {
    ptx::tmem_alloc_pair(sbase + C::kOffMisc, C::kTmemCols);
    ptx::tmem_relinquish_pair();
  }
  ptx::tc_fence_before();
  ptx::cluster_sync();  // barriers initialised and TMEM allocated in both CTAs
  ptx::tc_fence_after();
  const uint32_t tmem = misc[0];
  const int k_blocks = args.k_blocks;

  if (warp == kProducerWarp) {
    // ---------------------------------------------------------- producer
    if (lane == 0) {
      const uint32_t full_leader = ptx::mapa_shared(bar(C::kBarFull), 0);
      uint32_t L = 0;
      bool ok = true;
      for (int t = pair; ok && t < args.num_tiles; t += num_pairs) {
        int tm, tn;
        tile_coords(t, args.num_m_tiles, args.num_n_tiles, tm, tn);
        const int m0 = tm * (2 * kBM) + static_cast<int>(rank) * kBM;
        const int n0 = tn * BN + static_cast<int>(rank) * C::kHalfN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          const uint32_t s = L % S, r = L / S;
          if (!issuer_wait<kClusterAcquire>(bar(C::kBarEmpty + s), (r & 1u) ^ 1u, abort_flag, args.err)) {
            ok = false;
            break;
          }
          if (leader) ptx::mbar_arrive_expect_tx(bar(C::kBarFull + s), 2u * C::kStageBytes);
          const uint32_t a_dst = sbase + s * C::kStageBytes;
          ptx::tma_load_2d_pair(a_dst, &tm_x, full_leader + 8u * s, kb * kBK, m0);
          ptx::tma_load_2d_pair(a_dst + C::kABytes, &tm_w, full_leader + 8u * s, kb * kBK, n0);
          ++L;
        }
      }
      if (!ok && leader) {
        // Let copies already issued land before shared memory goes away.
        const uint32_t first = L > static_cast<uint32_t>(S) ? L - S : 0u;
        for (uint32_t x = first; x < L; ++x) {
          const uint64_t t0 = ptx::globaltimer_ns();
          while (!try_wait<kClusterAcquire>(bar(C::kBarFull + x % S), (x / S) & 1u) &&
                 ptx::globaltimer_ns() - t0 < kWaitTimeoutNs) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------- tcgen05 issuer (leader)
    // acc(buf) rows of both CTAs = x_tile W_tile^T, one M=256 x N=256 x K=16
    // product per 16 columns of K.
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = ptx::idesc_f16(kBF16, 2 * kBM, BN, false);
      uint32_t L = 0;
      int tc = 0;
      bool ok = true;
      for (int t = pair; ok && t < args.num_tiles; t += num_pairs, ++tc) {
        const int buf = tc & 1;
        const uint32_t use = static_cast<uint32_t>(tc >> 1);
        // both CTAs' epilogues have read this accumulator's previous tile
        if (!issuer_wait<kClusterAcquire>(bar(C::kBarAccEmpty + buf), (use & 1u) ^ 1u, abort_flag, args.err)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t acc = tmem + static_cast<uint32_t>(buf * BN);
        for (int kb = 0; kb < k_blocks; ++kb) {
          const uint32_t s = L % S, r = L / S;
          if (!issuer_wait<kClusterAcquire>(bar(C::kBarFull + s), r & 1u, abort_flag, args.err)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t a_addr = sbase + s * C::kStageBytes;
          const uint32_t b_addr = a_addr + C::kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            ptx::tc_mma_ss_pair(acc, ptx::smem_desc_sw128(a_addr + kk * 32, 16, 1024),
                                ptx::smem_desc_sw128(b_addr + kk * 32, 16, 1024), idesc,
                                (kb > 0 || kk > 0) ? 1u : 0u);
          // stage s of both CTAs is free once these products completed
          ptx::tc_commit_pair_both(bar(C::kBarEmpty + s));
          ++L;
        }
        if (ok) ptx::tc_commit_pair_both(bar(C::kBarAccFull + buf));
      }
      // Drain: every product this thread issued completes before TMEM is freed.
      ptx::tc_commit_pair(bar(C::kBarDrain));
      const uint64_t t0 = ptx::globaltimer_ns();
      while (!ptx::mbar_try_wait(bar(C::kBarDrain), 0) &&
             ptx::globaltimer_ns() - t0 < kWaitTimeoutNs) {
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // Each half (4 warps, 128 threads = 128 rows) writes its 128 columns as two
    // 64-column blocks, block b through staging buffer b of the half; one
    // elected thread per half loads the tile's residual blocks (before the
    // accumulator is ready) and issues the output stores.
    const int e = warp - kEpiWarp0;
    const int quad = warp & 3;
    const int half = e >> 2;
    const int rl = quad * 32 + lane;
    const bool elected = (e & 3) == 0 && lane == 0;
    const uint32_t named = 1u + static_cast<uint32_t>(half);  // named barrier of the half
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t acc_empty_leader = ptx::mapa_shared(bar(C::kBarAccEmpty), 0);
    const uint32_t out0 = sbase + C::kOffOut + static_cast<uint32_t>(half * 2 * C::kOutBufBytes);
    static_assert(C::kBlocksPerHalf == 2, "one staging buffer per block of the tile");
    int tc = 0;
    int armed_tc = -1;  // elected thread: last tile whose residual loads it issued
    for (int t = pair; t < args.num_tiles; t += num_pairs, ++tc) {
      const int buf = tc & 1;
      const uint32_t use = static_cast<uint32_t>(tc >> 1);
      int tm, tn;
      tile_coords(t, args.num_m_tiles, args.num_n_tiles, tm, tn);
      const int row0 = tm * (2 * kBM) + static_cast<int>(rank) * kBM;
      const int row = row0 + rl;
      const int cbase = tn * BN + half * C::kHalfCols;
      if (elected) {
        // the previous tile's stores have read both buffers: refill them
        ptx::bulk_wait_group_read_all();
        if constexpr (kRes) {
#pragma unroll
          for (int b = 0; b < C::kBlocksPerHalf; ++b) {
            const uint32_t rb = bar(C::kBarRes + half * 2 + b);
            ptx::mbar_arrive_expect_tx(rb, C::kOutBufBytes);
            ptx::tma_load_2d(out0 + b * C::kOutBufBytes, &tm_r, rb, cbase + b * C::kOutBlockCols,
                             row0);
          }
          armed_tc = tc;
        }
      }
      bool keep = true;
      if (args.row_mask && row < args.m) keep = args.row_mask[row] != 0;
      // the four warps of the half agree before any of them passes a named
      // barrier (this one also orders the buffer refill above before any write)
      const bool acc_ok =
          warp_wait_bar<kClusterAcquire>(bar(C::kBarAccFull + buf), use & 1u, abort_flag, args.err);
      if (!ptx::named_barrier_and(named, 128, acc_ok)) break;
      ptx::tc_fence_after();
      const uint32_t tacc = tmem + lane_off + static_cast<uint32_t>(buf * BN + half * C::kHalfCols);
      bool ok = true;
#pragma unroll 1
      for (int b = 0; b < C::kBlocksPerHalf; ++b) {
        const uint32_t stage = out0 + b * C::kOutBufBytes;
        const int col0 = cbase + b * C::kOutBlockCols;
        uint32_t a0[32], a1[32];
        ptx::tmem_ld_32x32b_x32(tacc + b * C::kOutBlockCols, a0);
        ptx::tmem_ld_32x32b_x32(tacc + b * C::kOutBlockCols + 32, a1);
        ptx::tmem_wait_ld();
        if (b == C::kBlocksPerHalf - 1) {
          // this warp's last read of the accumulator: hand it back to the issuer
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive_cluster(acc_empty_leader + 8u * buf);
        }
        bool res_ok = true;
        if constexpr (kRes)
          res_ok = warp_wait_bar(bar(C::kBarRes + half * 2 + b), static_cast<uint32_t>(tc) & 1u,
                                 abort_flag, args.err);
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          const int col = col0 + 8 * g;
          const uint32_t addr = stage + static_cast<uint32_t>(rl * 128) +
                                ((static_cast<uint32_t>(g) ^ static_cast<uint32_t>(rl & 7)) << 4);
          uint4 res = make_uint4(0u, 0u, 0u, 0u);
          if constexpr (kRes) {
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(res.x), "=r"(res.y), "=r"(res.z), "=r"(res.w)
                         : "r"(addr));
          }
          const uint4 bias =
              (args.bias && col < args.n) ? ld_nc_v4(args.bias + col) : make_uint4(0u, 0u, 0u, 0u);
          const uint32_t* src = g < 4 ? a0 + 8 * g : a1 + 8 * (g - 4);
          const uint4 o = epi8<kBF16, kGelu, kRes>(src, bias, res, keep, args.masked_keep_residual);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(o.x), "r"(o.y),
                       "r"(o.z), "r"(o.w)
                       : "memory");
        }
        ptx::fence_proxy_async_smem();
        // the block is in shared memory (unless a residual load never arrived)
        ok = ptx::named_barrier_and(named, 128, res_ok);
        if (!ok) break;
        if (elected) {
          ptx::tma_store_2d(&tm_y, stage, col0, row0);
          ptx::bulk_commit_group();
        }
      }
      if (!ok) break;
    }
    if constexpr (kRes) {
      // After an abort, residual loads of the last tile may still be writing
      // shared memory: let them land (bounded) before the CTA can exit.  On
      // the normal path every armed barrier has completed and this returns at
      // once.
      if (elected && armed_tc >= 0) {
#pragma unroll
        for (int b = 0; b < C::kBlocksPerHalf; ++b) {
          const uint32_t rb = bar(C::kBarRes + half * 2 + b);
          const uint64_t t0 = ptx::globaltimer_ns();
          while (!ptx::mbar_try_wait(rb, static_cast<uint32_t>(armed_tc) & 1u) &&
                 ptx::globaltimer_ns() - t0 < kWaitTimeoutNs) {
          }
        }
      }
    }
    if (elected) ptx::bulk_wait_group_all();  // stores complete before the CTA ends
  }

  ptx::tc_fence_before();
  ptx::cluster_sync();  // no CTA frees TMEM or leaves while the pair still uses it
  if (warp == kMmaWarp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem, C::kTmemCols);
  }
}

// ------------------------------------------------------------------- host
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D row-major [rows, cols] map with a {64, box_rows} box, 128-byte swizzle;
// reads past either edge fill zeros.
int encode_rows(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int64_t ld,
                uint32_t box_rows, bool bf16) {
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled entry point unavailable");
    return B200_ATTN_ERR_LAUNCH;
  }
  const int64_t stride = rows > 1 ? ld * 2 : ((cols * 2 + 15) / 16) * 16;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kBK), box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed");
    return B200_ATTN_ERR_LAUNCH;
  }
  return B200_ATTN_OK;
}

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  std::once_flag probed;
  bool sm100 = false;
  int num_sms = 0;
};
DeviceInfo g_dev[kMaxDevices];

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Tile width for a shape.
int pick_tile_n(int64_t m, int64_t n, int num_sms) {
  if (kForceTileN == 128 || kForceTileN == 256) return kForceTileN;
  (void)m;
  (void)num_sms;
  // Measured on the decoder's shapes (M = 16384; N, K in {1024, 3072, 4096}):
  // the 256-wide tile is faster everywhere, by 1.3-1.6x, also where the
  // narrow one would fill the last wave better.
  return n <= 128 ? 128 : 256;
}

// The CTA-pair kernel for every shape with more than one 128-row block and
// more than 128 output columns (unless a tile width is forced at build time).
bool use_pair(int64_t m, int64_t n) { return kForceTileN == 0 && m > kBM && n > 128; }

struct DeviceGuard {
  int prev = -1;
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

template <int BN, bool BF, bool G, bool R>
int launch(const CUtensorMap& mx, const CUtensorMap& mw, const LinArgs& a, int dev, int grid,
           cudaStream_t stream) {
  using C = LinCfg<BN>;
  auto kernel = linear_sm100_kernel<C, BF, G, R>;
  static std::once_flag attr_once[kMaxDevices];
  static cudaError_t attr_err[kMaxDevices];
  std::call_once(attr_once[dev], [&] {
    attr_err[dev] =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  });
  if (attr_err[dev] != cudaSuccess) {
    set_error(cudaGetErrorString(attr_err[dev]));
    return B200_ATTN_ERR_LAUNCH;
  }
  kernel<<<grid, kThreads, C::kSmemBytes, stream>>>(mx, mw, a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(cudaGetErrorString(e));
    return B200_ATTN_ERR_LAUNCH;
  }
  count_launch();
  return B200_ATTN_OK;
}

template <bool BF, bool G, bool R>
int launch_pair(const CUtensorMap& mx, const CUtensorMap& mw, const CUtensorMap& my,
                const CUtensorMap& mr, const LinArgs& a, int dev, int num_sms,
                cudaStream_t stream) {
  auto kernel = linear_sm100_pair_kernel<BF, G, R>;
  static std::once_flag once[kMaxDevices];
  static cudaError_t attr_err[kMaxDevices];
  static int max_pairs[kMaxDevices];
  std::call_once(once[dev], [&] {
    attr_err[dev] = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         PairCfg::kSmemBytes);
    if (attr_err[dev] != cudaSuccess) return;
    // pairs that can be resident at once (SMs that cannot be paired stay idle)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(num_sms - num_sms % 2), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = PairCfg::kSmemBytes;
    int n = 0;
    attr_err[dev] = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
    max_pairs[dev] = n;
  });
  if (attr_err[dev] != cudaSuccess || max_pairs[dev] < 1) {
    set_error(attr_err[dev] != cudaSuccess ? cudaGetErrorString(attr_err[dev])
                                           : "no CTA pair fits on the device");
    return B200_ATTN_ERR_LAUNCH;
  }
  const int pairs = a.num_tiles < max_pairs[dev] ? a.num_tiles : max_pairs[dev];
  kernel<<<2 * pairs, kThreads, PairCfg::kSmemBytes, stream>>>(mx, mw, my, mr, a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(cudaGetErrorString(e));
    return B200_ATTN_ERR_LAUNCH;
  }
  count_launch();
  return B200_ATTN_OK;
}

int dispatch_pair(const CUtensorMap* maps, const LinArgs& a, const b200_linear_params* p, int dev,
                  int num_sms, cudaStream_t s) {
  const bool bf = p->dtype == B200_ATTN_DTYPE_BF16;
  const bool g = p->activation == B200_LINEAR_ACT_GELU;
  const bool r = p->residual != nullptr;
  const CUtensorMap &mx = maps[0], &mw = maps[1], &my = maps[2], &mr = maps[3];
  if (bf) {
    if (g) return r ? launch_pair<true, true, true>(mx, mw, my, mr, a, dev, num_sms, s)
                    : launch_pair<true, true, false>(mx, mw, my, mr, a, dev, num_sms, s);
    return r ? launch_pair<true, false, true>(mx, mw, my, mr, a, dev, num_sms, s)
             : launch_pair<true, false, false>(mx, mw, my, mr, a, dev, num_sms, s);
  }
  if (g) return r ? launch_pair<false, true, true>(mx, mw, my, mr, a, dev, num_sms, s)
                  : launch_pair<false, true, false>(mx, mw, my, mr, a, dev, num_sms, s);
  return r ? launch_pair<false, false, true>(mx, mw, my, mr, a, dev, num_sms, s)
           : launch_pair<false, false, false>(mx, mw, my, mr, a, dev, num_sms, s);
}

template <int BN>
int dispatch(const CUtensorMap& mx, const CUtensorMap& mw, const LinArgs& a,
             const b200_linear_params* p, int dev, int grid, cudaStream_t s) {
  const bool bf = p->dtype == B200_ATTN_DTYPE_BF16;
  const bool g = p->activation == B200_LINEAR_ACT_GELU;
  const bool r = p->residual != nullptr;
  if (bf) {
    if (g) return r ? launch<BN, true, true, true>(mx, mw, a, dev, grid, s)
                    : launch<BN, true, true, false>(mx, mw, a, dev, grid, s);
    return r ? launch<BN, true, false, true>(mx, mw, a, dev, grid, s)
             : launch<BN, true, false, false>(mx, mw, a, dev, grid, s);
  }
  if (g) return r ? launch<BN, false, true, true>(mx, mw, a, dev, grid, s)
                  : launch<BN, false, true, false>(mx, mw, a, dev, grid, s);
  return r ? launch<BN, false, false, true>(mx, mw, a, dev, grid, s)
           : launch<BN, false, false, false>(mx, mw, a, dev, grid, s);
}

}  // namespace
}  // namespace b200lin

// ------------------------------------------------------------------ C ABI
using namespace b200lin;

extern "C" int32_t b200_linear_check(const b200_linear_params* p) {
  if (!p || !p->x || !p->w || !p->y) return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->m < 1 || p->n < 1 || p->k < 1) return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->m > 0x7fffffffll || p->n > 0x7fffffffll || p->k > 0x7fffffffll)
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (ceil_div(p->m, kBM) * ceil_div(p->n, 128) > 0x7fffffffll) return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->dtype != B200_ATTN_DTYPE_BF16 && p->dtype != B200_ATTN_DTYPE_FP16)
    return B200_ATTN_ERR_UNSUPPORTED;
  if (p->activation != B200_LINEAR_ACT_NONE && p->activation != B200_LINEAR_ACT_GELU)
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->masked_rows != B200_LINEAR_MASKED_ZERO && p->masked_rows != B200_LINEAR_MASKED_KEEP_RESIDUAL)
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->reserved != 0) return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->row_mask && p->masked_rows == B200_LINEAR_MASKED_KEEP_RESIDUAL && !p->residual)
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->m > 1 && p->x_row_stride < p->k) return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->n > 1 && p->w_row_stride < p->k) return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->m > 1 && p->y_row_stride < p->n) return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->residual && p->m > 1 && p->residual_row_stride < p->n) return B200_ATTN_ERR_INVALID_ARGUMENT;
  // 16-byte rows and bases: TMA strides for x and W, vector accesses for the rest
  if (p->n % 8 != 0 || p->k % 8 != 0) return B200_ATTN_ERR_ALIGNMENT;
  if (!aligned16(p->x) || !aligned16(p->w) || !aligned16(p->y)) return B200_ATTN_ERR_ALIGNMENT;
  if (p->bias && !aligned16(p->bias)) return B200_ATTN_ERR_ALIGNMENT;
  if (p->residual && !aligned16(p->residual)) return B200_ATTN_ERR_ALIGNMENT;
  if (p->m > 1 && (p->x_row_stride % 8 != 0 || p->y_row_stride % 8 != 0))
    return B200_ATTN_ERR_ALIGNMENT;
  if (p->n > 1 && p->w_row_stride % 8 != 0) return B200_ATTN_ERR_ALIGNMENT;
  if (p->residual && p->m > 1 && p->residual_row_stride % 8 != 0) return B200_ATTN_ERR_ALIGNMENT;
  // y must not overlap any input: its stores would race the TMA loads of x,
  // W and the residual prefetch
  const ByteRange yr = rows_range(p->y, p->m, p->n, p->y_row_stride);
  if (yr.overlaps(rows_range(p->x, p->m, p->k, p->x_row_stride)) ||
      yr.overlaps(rows_range(p->w, p->n, p->k, p->w_row_stride)) ||
      (p->bias && yr.overlaps(rows_range(p->bias, 1, p->n, p->n))) ||
      (p->residual && yr.overlaps(rows_range(p->residual, p->m, p->n, p->residual_row_stride))) ||
      (p->row_mask && yr.overlaps(ByteRange{reinterpret_cast<uintptr_t>(p->row_mask),
                                            reinterpret_cast<uintptr_t>(p->row_mask) +
                                                static_cast<uintptr_t>(p->m)})))
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  return B200_ATTN_OK;
}

extern "C" int32_t b200_linear_tile_n(const b200_linear_params* p, int32_t num_sms) {
  if (b200_linear_check(p) != B200_ATTN_OK) return 0;
  return pick_tile_n(p->m, p->n, num_sms);
}

extern "C" int32_t b200_linear_fwd(const b200_linear_params* p, void* stream) {
  int32_t rc = b200_linear_check(p);
  if (rc != B200_ATTN_OK) return rc;

  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, p->x) != cudaSuccess || attr.device < 0 ||
      attr.device >= kMaxDevices ||
      (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)) {
    cudaGetLastError();
    set_error("x is not a device pointer");
    return B200_ATTN_ERR_DEVICE;
  }
  const int dev = attr.device;
  DeviceGuard guard;
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess || cur != dev) {
    if (cudaSetDevice(dev) != cudaSuccess) {
      cudaGetLastError();
      set_error("cudaSetDevice failed");
      return B200_ATTN_ERR_DEVICE;
    }
    guard.prev = cur;
  }
  std::call_once(g_dev[dev].probed, [dev] {
    int major = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) == cudaSuccess)
      g_dev[dev].sm100 = (major == 10);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess)
      g_dev[dev].num_sms = sms;
  });
  if (!g_dev[dev].sm100 || g_dev[dev].num_sms < 1) {
    set_error("device is not compute capability 10.x");
    return B200_ATTN_ERR_DEVICE;
  }

  const bool bf = p->dtype == B200_ATTN_DTYPE_BF16;
  const int bn = pick_tile_n(p->m, p->n, g_dev[dev].num_sms);
  const bool pair = use_pair(p->m, p->n);
  // each CTA of a pair loads 128 rows of W; a single CTA loads all bn rows
  const uint32_t w_rows = pair ? static_cast<uint32_t>(PairCfg::kHalfN) : static_cast<uint32_t>(bn);
  CUtensorMap mx, mw;
  if ((rc = encode_rows(&mx, p->x, p->m, p->k, p->x_row_stride, kBM, bf)) != B200_ATTN_OK ||
      (rc = encode_rows(&mw, p->w, p->n, p->k, p->w_row_stride, w_rows, bf)) != B200_ATTN_OK)
    return rc;

  LinArgs a;
  a.m = static_cast<int32_t>(p->m);
  a.n = static_cast<int32_t>(p->n);
  a.k = static_cast<int32_t>(p->k);
  a.num_n_tiles = static_cast<int32_t>(ceil_div(p->n, bn));
  a.num_m_tiles = static_cast<int32_t>(ceil_div(p->m, pair ? 2 * kBM : kBM));
  a.num_tiles = a.num_m_tiles * a.num_n_tiles;
  a.k_blocks = static_cast<int32_t>(ceil_div(p->k, kBK));
  a.bias = static_cast<const uint16_t*>(p->bias);
  a.residual = static_cast<const uint16_t*>(p->residual);
  a.ld_res = p->residual ? p->residual_row_stride : 0;
  a.row_mask = p->row_mask;
  a.masked_keep_residual = p->masked_rows == B200_LINEAR_MASKED_KEEP_RESIDUAL ? 1 : 0;
  a.y = static_cast<uint16_t*>(p->y);
  a.ld_y = p->y_row_stride;
  if ((rc = resolve_error_word(p->error_word, &a.err)) != B200_ATTN_OK) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (pair) {
    // the output (and the residual) leave and enter through 64 x 128 TMA boxes
    CUtensorMap maps[4] = {mx, mw, {}, {}};
    if ((rc = encode_rows(&maps[2], p->y, p->m, p->n, p->y_row_stride, kBM, bf)) != B200_ATTN_OK)
      return rc;
    if (p->residual) {
      if ((rc = encode_rows(&maps[3], p->residual, p->m, p->n, p->residual_row_stride, kBM, bf)) !=
          B200_ATTN_OK)
        return rc;
    } else {
      maps[3] = maps[2];
    }
    return dispatch_pair(maps, a, p, dev, g_dev[dev].num_sms, s);
  }
  const int grid = static_cast<int>(
      a.num_tiles < g_dev[dev].num_sms ? a.num_tiles : g_dev[dev].num_sms);
  return bn == 256 ? dispatch<256>(mx, mw, a, p, dev, grid, s)
                   : dispatch<128>(mx, mw, a, p, dev, grid, s);
}
