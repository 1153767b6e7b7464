// attn_fwd_sm100.cu — fused attention forward for B200 (sm_100a).
//
// Value definition: the reference's _reference_attention
// (model/triton_fused_attention.py:1256-1285): scores = q k^T * scale, causal
// triu(1) and key-padding positions set to -inf, fp32 softmax, probabilities in
// the input dtype, times v.  Fully masked rows give NaN like torch.softmax.
//
// Work decomposition.  One CTA owns 256 query rows of one (batch, head) as two
// 128-row tiles Q0, Q1 and streams 128-key K/V tiles through a shared-memory
// ring.  Eleven warps, one job each:
//   warps 0-3  softmax for Q0 (one thread per query row = one TMEM lane)
//   warps 4-7  softmax for Q1
//   warp  8    TMA producer (Q once, then K_j, V_j into the ring)
//   warp  9    tcgen05 issuer of the QK products (one thread) and TMEM owner
//   warp 10    tcgen05 issuer of the PV products (one thread)
// Tensor memory (512 columns x 128 lanes of 32 bit) holds the scores
// S = Q_i K_j^T (128 fp32 columns, one buffer shared by Q0 and Q1), one
// buffer of P_i per query tile (64 columns of packed 16-bit pairs) and the
// fp32 accumulators O_i (D columns):
//   D = 128: S (128) | P0 P1 (2x64) | O0 O1 (2x128) = 512 columns
//   D =  64: S (128) | P0 P1 (2x64) | O0 O1 (2x64)  = 384 columns
// P never aliases S, so a QK product only waits until the previous scores in
// the S buffer were copied to registers by their softmax warpgroup, never for
// a PV product; PV_i(j) is issued once P_i(j) is written.  The shared S buffer
// makes the two softmax warpgroups alternate (S0(j), S1(j), S0(j+1), ...), so
// the warps that share an SM sub-partition do not run their exponentials at
// the same time, while the tensor core computes the next scores and the
// previous PV products.
// The running max is updated lazily: O and the row sum are rescaled only when
// the max grows by more than 2^8, which keeps the unnormalised P in range and
// makes rescaling rare; the final O / l is exact either way.
//
// Every mbarrier wait is bounded (wall clock, ~1 s).  On expiry the kernel
// sets a CTA abort flag and an error bit in the caller's error word, lets all
// roles fall through, waits (bounded) for its own copies and MMAs in flight,
// frees TMEM and returns.  There is no trap and no unbounded spin.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <atomic>
#include <cstring>
#include <mutex>

#include "b200_attn.h"
#include "error_word.cuh"
#include "sm100_ptx.cuh"

namespace b200attn {

constexpr int kBlockM = 128;  // query rows per tile = TMEM lanes
constexpr int kRowsPerCta = 2 * kBlockM;
constexpr int kSoftmaxWarps = 8;
constexpr int kLoadWarp = 8;
constexpr int kQkWarp = 9;   // issues QK products, owns TMEM
constexpr int kPvWarp = 10;  // issues PV products
constexpr int kThreads = 352;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.0f;  // rescale O when the max grows by > 2^8
constexpr uint64_t kWaitTimeoutNs = 1000000000ull;
constexpr float kLog2e = 1.4426950408889634f;
#ifndef B200_ATTN_POLY_PER8
#define B200_ATTN_POLY_PER8 0
#endif
// Of every 8 probabilities, this many are computed with the FMA-pipe exp2.
constexpr int kPolyPer8 = B200_ATTN_POLY_PER8;
#ifndef B200_ATTN_F32X2
#define B200_ATTN_F32X2 1
#endif
#ifndef B200_ATTN_SPLIT_LD
#define B200_ATTN_SPLIT_LD 1
#endif
#ifndef B200_ATTN_ISSUER_SPIN
#define B200_ATTN_ISSUER_SPIN 1
#endif
// MMA issuers poll their barriers without suspending before the bounded
// wait: a suspended issuer was measured to resume hundreds of cycles after
// the softmax signalled, which sits directly on the scores -> softmax chain.
// (Softmax warps keep suspending waits: their polling would take issue slots
// from the other softmax warpgroup on the same SM sub-partition.)
constexpr int kIssuerSpin = B200_ATTN_ISSUER_SPIN ? 4096 : 0;
#ifndef B200_ATTN_CHECKED
#define B200_ATTN_CHECKED 0
#endif
// Checked build (libb200_attention_checked.so): every TMA coordinate, shared-
// memory tile address and tensor-memory column range is verified before use.
// A failed check ORs B200_ATTN_DEVERR_BOUNDS into the error word, sets the CTA
// abort flag and skips the access; the kernel then winds down through its
// bounded waits.  No trap, no device assert.
constexpr bool kChecked = B200_ATTN_CHECKED != 0;
#ifndef B200_ATTN_GROUP_MB
#define B200_ATTN_GROUP_MB 48
#endif
// Packed fp32x2 FMA/ADD in the softmax (same rounding, half the instructions).
constexpr bool kF32x2 = B200_ATTN_F32X2 != 0;
// Row max of the first 64 score columns overlaps the TMEM load of the rest.
constexpr bool kSplitLoad = B200_ATTN_SPLIT_LD != 0;
// CTAs of heads whose K and V fit in this many MB of L2 run together.
constexpr int64_t kGroupBytes = static_cast<int64_t>(B200_ATTN_GROUP_MB) << 20;

struct KernelArgs {
  int32_t seq_len;
  int32_t heads;
  int32_t batch;
  int32_t num_q_blocks;  // ceil(S / 256)
  int32_t head_dim;      // the tensors' head dim (<= the instance's D)
  int32_t group_heads;   // (batch, head) pairs per L2 group of CTAs
  float scale;           // softmax scale
  float scale_log2;      // scale * log2(e)
  int32_t zero_masked_queries;
  const uint8_t* mask;   // [B,S] bool or null
  int64_t mask_sb;       // bytes
  int64_t mask_ss;
  void* o;               // output base (for zero rows of skipped blocks)
  int64_t o_sb, o_sh, o_ss;  // elements
  int32_t* err;          // error word as resolve_error_word returns it (bit 0: host word)
  int32_t skip_load;     // stall self-test only: K/V load left out (see b200_attn_selftest_stall)
};

// Arguments of the partial instances (b200_attn_fwd_partial): the per-row
// log-sum-exp of this key chunk, merged into the existing (O, lse) when
// accumulate is set.  A separate type, so the other instances' arguments
// (and their code) are unchanged.
struct PartialKernelArgs : KernelArgs {
  float* lse;
  int64_t lse_sb, lse_sh, lse_ss;  // elements
  int32_t accumulate;
};

template <bool kPartial>
struct ArgsOf {
  using type = KernelArgs;
};
template <>
struct ArgsOf<true> {
  using type = PartialKernelArgs;
};

// Compile-time shape of one kernel instance.  ELEM is the element size: 2
// for bf16/fp16 (kind::f16 products), 4 for fp32 (kind::tf32 products).
template <int D_, int BN_, int PB_, int NSLOT_, bool SHARED_S_, int ELEM_ = 2>
struct Cfg {
  static constexpr int D = D_;          // head dim
  static constexpr int BN = BN_;        // keys per K/V tile
  static constexpr int PB = PB_;        // P buffers per query tile
  static constexpr int NSLOT = NSLOT_;  // K/V ring slots (one K or V tile each)
  static constexpr bool kSharedS = SHARED_S_;  // one S buffer for both query tiles
  static constexpr int ELEM = ELEM_;
  static constexpr int kSBufs = kSharedS ? 1 : 2;
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static_assert(BN == 64 || BN == 128, "BN 64 or 128");
  static_assert(ELEM == 2 || ELEM == 4, "16- or 32-bit elements");
  static constexpr int kChunkCols = 128 / ELEM;       // elements per 128-byte swizzle row
  static constexpr int kChunks = D / kChunkCols;      // 128-byte swizzle chunks per row
  static constexpr int kKStep = 32 / ELEM;            // K elements per tcgen05.mma
  static constexpr int kPCols = BN * ELEM / 4;        // TMEM columns of one P buffer
  static constexpr int kQChunkBytes = kBlockM * 128;  // one chunk of a 128-row tile
  static constexpr int kKVChunkBytes = BN * 128;      // one chunk of a BN-row tile
  static constexpr int kQTileBytes = kBlockM * D * ELEM;
  static constexpr int kKVTileBytes = BN * D * ELEM;
  static constexpr int kOffQ = 0;
  static constexpr int kOffRing = 2 * kQTileBytes;
  static constexpr int kOffBar = kOffRing + NSLOT * kKVTileBytes;
  // barrier indices
  static constexpr int kBarQ = 0;  // [2], one per query tile
  static constexpr int kBarSlotFull = 2;
  static constexpr int kBarSlotEmpty = kBarSlotFull + NSLOT;
  static constexpr int kBarSFull = kBarSlotEmpty + NSLOT;  // [2]
  static constexpr int kBarSFree = kBarSFull + 2;          // [2]
  static constexpr int kBarPFull = kBarSFree + 2;          // [2][PB]
  static constexpr int kBarPVDone = kBarPFull + 2 * PB;    // [2][PB]
  static constexpr int kBarOFull = kBarPVDone + 2 * PB;    // [2]
  static constexpr int kBarDrain = kBarOFull + 2;
  static constexpr int kNumBars = kBarDrain + 1;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 16 + 1024;  // + alignment slack
  static_assert(kSmemBytes <= 232448, "exceeds the 227 KB per-block shared memory limit");
  // TMEM columns
  __host__ __device__ static constexpr uint32_t col_s(int i) { return kSharedS ? 0u : BN * i; }
  __host__ __device__ static constexpr uint32_t col_p(int i, int b) {
    return kSBufs * BN + (i * PB + b) * kPCols;
  }
  __host__ __device__ static constexpr uint32_t col_o(int i) {
    return kSBufs * BN + 2 * PB * kPCols + D * i;
  }
  static_assert(kSBufs * BN + 2 * PB * kPCols + 2 * D <= 512, "TMEM budget");
  // Query tiles whose visible keys all lie in the first kExactKeys keys take
  // the exact-rounding path (keys held in registers across <= 2 tiles).
  static constexpr int kExactKeys = 128;
  static constexpr int kExactTiles = kExactKeys / BN;
};

// ---------------------------------------------------------------- helpers
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

// x rounded to the input dtype and widened back to fp32 (fp32: x itself).
template <int DT>
__device__ __forceinline__ float round_to_input(float x) {
  if constexpr (DT == B200_ATTN_DTYPE_BF16) {
    return __bfloat162float(__float2bfloat16_rn(x));
  } else if constexpr (DT == B200_ATTN_DTYPE_FP16) {
    return __half2float(__float2half_rn(x));
  } else {
    return x;
  }
}

// Packed fp32x2 a*b+c and a+b (sm_100 fma/add .f32x2): two lanes per
// instruction, each rounded exactly like the scalar operation.
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0,
                                      float b1, float c0, float c1) {
  asm("{\n\t.reg .b64 a, b, c, d;\n\t"
      "mov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\tmov.b64 c, {%6, %7};\n\t"
      "fma.rn.f32x2 d, a, b, c;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void fadd2(float& d0, float& d1, float a0, float a1, float b0,
                                      float b1) {
  asm("{\n\t.reg .b64 a, b, d;\n\t"
      "mov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
      "add.rn.f32x2 d, a, b;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}

// Three-input maximum (sm_100 max.f32 with three sources).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x on the FMA pipe, for -126 <= x <= 64.  x = n + f with n = rint(x)
// obtained by adding 1.5*2^23 (the sum's low mantissa bits hold n, f in
// [-0.5, 0.5]); 2^f from a degree-3 polynomial fitted here by a Remez
// iteration for minimax relative error on [-0.5, 0.5] (max 7.5e-5, below the
// 2^-9 rounding of the 16-bit probabilities); 2^n is added to the exponent
// field as (bits(x + 1.5*2^23) << 23), whose high bits shift out.
__device__ __forceinline__ float ex2_poly(float x) {
  constexpr float kRound = 12582912.0f;  // 1.5 * 2^23
  const float t = x + kRound;
  const float f = x - (t - kRound);
  const float p = fmaf(fmaf(fmaf(0.05517167f, f, 0.24261113f), f, 0.69326097f), f, 0.99992806f);
  return __uint_as_float(__float_as_uint(p) + (__float_as_uint(t) << 23));
}

// Max of s[OFF, OFF + CNT) (CNT a multiple of 32) as a 3-input tree.
template <int OFF, int CNT, int N>
__device__ __forceinline__ float range_max(const uint32_t (&s)[N]) {
  static_assert(CNT % 32 == 0 && OFF % 32 == 0 && OFF + CNT <= N, "chunks of 32");
  float cm[CNT / 32];
#pragma unroll
  for (int cc = 0; cc < CNT / 32; ++cc) {
    const int c = OFF / 32 + cc;
    float v[11];
#pragma unroll
    for (int t = 0; t < 10; ++t)
      v[t] = fmax3(__uint_as_float(s[32 * c + 3 * t]), __uint_as_float(s[32 * c + 3 * t + 1]),
                   __uint_as_float(s[32 * c + 3 * t + 2]));
    v[10] = fmaxf(__uint_as_float(s[32 * c + 30]), __uint_as_float(s[32 * c + 31]));
    cm[cc] = fmax3(fmax3(v[0], v[1], v[2]), fmax3(v[3], v[4], v[5]),
                   fmax3(v[6], v[7], fmax3(v[8], v[9], v[10])));
  }
  float m = cm[0];
#pragma unroll
  for (int c = 1; c < CNT / 32; ++c) m = fmaxf(m, cm[c]);
  return m;
}

template <int N>
__device__ __forceinline__ float row_max(const uint32_t (&s)[N]) {
  return range_max<0, N, N>(s);
}

__device__ __forceinline__ int warp_max_i(int v) {
#pragma unroll
  for (int off = 16; off; off >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// Bounded wait on an mbarrier phase.  Returns false when the CTA was aborted
// (by this thread's timeout or another's).
__device__ __noinline__ bool wait_bar_slow(uint32_t bar, uint32_t parity,
                                           volatile uint32_t* abort_flag, int32_t* err) {
  const uint64_t t0 = ptx::globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int k = 0; k < 32; ++k)
      if (ptx::mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (ptx::globaltimer_ns() - t0 > kWaitTimeoutNs) {
      *abort_flag = 1u;
      report_error(err, B200_ATTN_DEVERR_WAIT_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity,
                                         volatile uint32_t* abort_flag, int32_t* err) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  return wait_bar_slow(bar, parity, abort_flag, err);
}

// Issuer-side wait: poll without suspending first (a suspended thread resumes
// late), then the bounded wait.
__device__ __forceinline__ bool issuer_wait(uint32_t bar, uint32_t parity,
                                            volatile uint32_t* abort_flag, int32_t* err) {
#pragma unroll 1
  for (int k = 0; k < kIssuerSpin; ++k)
    if (ptx::mbar_test_wait(bar, parity)) return true;
  return wait_bar(bar, parity, abort_flag, err);
}

// Wait by every lane of a warp; the result is made warp-uniform so the
// warp-collective tcgen05 instructions that follow stay converged.
__device__ __forceinline__ bool warp_wait_bar(uint32_t bar, uint32_t parity,
                                              volatile uint32_t* abort_flag, int32_t* err) {
  const bool ok = wait_bar(bar, parity, abort_flag, err);
  const bool all = __all_sync(0xffffffffu, ok);
  if (!all) *abort_flag = 1u;
  return all;
}

// One arrival per warp after all lanes finished their tcgen05 accesses.
__device__ __forceinline__ void warp_arrive(uint32_t bar, int lane) {
  ptx::tc_fence_before();
  __syncwarp();
  if (lane == 0) ptx::mbar_arrive(bar);
}

// Last valid key + 1 of one mask row (0 when none).  One warp, scanning
// backwards in 512-byte windows when the row is byte-contiguous and aligned.
__device__ int mask_extent(const uint8_t* mrow, int64_t ss, int S, int lane) {
  int last = -1;
  const bool vec = (ss == 1) && ((reinterpret_cast<uintptr_t>(mrow) & 15u) == 0);
  if (vec) {
    const int nvec = S / 16;
    for (int k = nvec * 16 + lane; k < S; k += 32)
      if (mrow[k]) last = k;
    last = warp_max_i(last);
    for (int base = nvec - 32; last < 0 && base > -32; base -= 32) {
      const int c = base + lane;
      int found = -1;
      if (c >= 0) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(mrow) + c);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (ws[q]) found = 16 * c + 4 * q + ((31 - __clz(ws[q])) >> 3);
      }
      last = warp_max_i(found);
    }
  } else {
    for (int k = lane; k < S; k += 32)
      if (mrow[static_cast<int64_t>(k) * ss]) last = k;
    last = warp_max_i(last);
  }
  return last + 1;
}

// Load N fp32 score columns of this thread's row from TMEM.
template <int N>
__device__ __forceinline__ void load_row(uint32_t taddr, uint32_t (&s)[N]) {
#pragma unroll
  for (int c = 0; c < N / 32; ++c)
    ptx::tmem_ld_32x32b_x32(taddr + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&s[32 * c]));
  ptx::tmem_wait_ld();
}

// Set scores of invisible keys to -inf: key k of the tile is visible iff
// k <= lim and its mask bit is set.
template <int N>
__device__ __forceinline__ void mask_row(uint32_t (&s)[N], int lim, const uint32_t* mw) {
#pragma unroll
  for (int k = 0; k < N; ++k) {
    const bool vis = (k <= lim) && (((mw[k >> 5] >> (k & 31)) & 1u) != 0u);
    if (!vis) s[k] = __float_as_uint(-INFINITY);
  }
}

// ----------------------------------------------------------------- kernel
// kStallProbe (self-test instance only): K/V load number args.skip_load of
// every CTA is announced to its barrier but never issued, so the pipeline
// waits on it run out and exercise the abort path.
// kPartial (b200_attn_fwd_partial): the CTA also writes each row's
// log-sum-exp over this key chunk and, with args.accumulate, merges its
// normalised output into the O and lse already in memory (the context-parallel
// step over one chunk of a longer key sequence).
template <class C, bool kCausal, bool kMask, int kDtype, bool kStallProbe = false,
          bool kPartial = false>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                          const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v,
                          const __grid_constant__ CUtensorMap tm_o,
                          const typename ArgsOf<kPartial>::type args) {
  constexpr int D = C::D, BN = C::BN, PB = C::PB, NSLOT = C::NSLOT;
  constexpr int kMaskWords = BN / 32;
  constexpr bool kBF16 = kDtype == B200_ATTN_DTYPE_BF16;
  constexpr bool kTF32 = kDtype == B200_ATTN_DTYPE_FP32;  // fp32 inputs, TF32 products
  static_assert(kTF32 == (C::ELEM == 4), "fp32 runs the 32-bit instance");
  static_assert(!(kPartial && kMask), "partial instances take no key mask");
  constexpr int kCC = C::kChunkCols;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = args.seq_len;

  // CTAs run in groups of group_heads (batch, head) pairs whose K and V fit
  // in L2, so the query blocks of a head re-read K/V from L2 rather than HBM;
  // inside a group the heaviest query blocks (causal) are launched first.
  const int bh_count = args.batch * args.heads;
  const int per_group = args.group_heads * args.num_q_blocks;
  const int grp = static_cast<int>(blockIdx.x) / per_group;
  const int rem = static_cast<int>(blockIdx.x) - grp * per_group;
  const int gsize = min(args.group_heads, bh_count - grp * args.group_heads);
  const int qb = args.num_q_blocks - 1 - rem / gsize;
  const int bh = grp * args.group_heads + rem % gsize;
  const int b = bh / args.heads;
  const int h = bh % args.heads;
  const int q0 = qb * kRowsPerCta;

  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(smem + C::kOffMisc);
  // misc[0] TMEM base, misc[1] abort flag, misc[2] key extent
  volatile uint32_t* abort_flag = misc + 1;
  const uint32_t bar0 = sbase + C::kOffBar;
  auto bar = [&](int idx) { return bar0 + 8u * static_cast<uint32_t>(idx); };
  // checked builds: true when the access may proceed
  auto chk = [&](bool cond) {
    if constexpr (kChecked) {
      if (!cond) {
        report_error(args.err, B200_ATTN_DEVERR_BOUNDS);
        *abort_flag = 1u;
      }
      return cond;
    } else {
      return true;
    }
  };
  // a whole tile of `bytes` at smem address `a`, 1024-byte aligned (128-byte
  // swizzle atoms), inside [lo, hi)
  auto tile_ok = [&](uint32_t a, uint32_t bytes, uint32_t lo, uint32_t hi) {
    return a >= lo && a + bytes <= hi && ((a - sbase) & 1023u) == 0u;
  };
  auto coord_ok = [&](int x, int row, int hh, int bb, int row_hi) {
    return x >= 0 && x + kCC <= D && (x % kCC) == 0 && row >= 0 && row < row_hi && hh >= 0 &&
           hh < args.heads && bb >= 0 && bb < args.batch;
  };

  const uint8_t* mrow = nullptr;
  if constexpr (kMask) mrow = args.mask + static_cast<int64_t>(b) * args.mask_sb;

  // TMA loads (one thread of the load warp): query tile i, and key (kv = 0)
  // or value (kv = 1) tile j into ring slot s
  auto load_q = [&](int i) {
    ptx::mbar_arrive_expect_tx(bar(C::kBarQ + i), C::kQTileBytes);
#pragma unroll
    for (int c = 0; c < C::kChunks; ++c) {
      const uint32_t dst = sbase + C::kOffQ + i * C::kQTileBytes + c * C::kQChunkBytes;
      if (chk(tile_ok(dst, C::kQChunkBytes, sbase + C::kOffQ, sbase + C::kOffRing) &&
              coord_ok(kCC * c, q0 + kBlockM * i, h, b, args.num_q_blocks * kRowsPerCta)))
        ptx::tma_load_4d(dst, &tm_q, bar(C::kBarQ + i), kCC * c, q0 + kBlockM * i, h, b);
    }
  };
  auto load_kv = [&](int j, int kv, uint32_t s) {
    const CUtensorMap* tm = kv ? &tm_v : &tm_k;
#pragma unroll
    for (int c = 0; c < C::kChunks; ++c) {
      const uint32_t dst = sbase + C::kOffRing + s * C::kKVTileBytes + c * C::kKVChunkBytes;
      if (chk(tile_ok(dst, C::kKVChunkBytes, sbase + C::kOffRing, sbase + C::kOffBar) &&
              coord_ok(kCC * c, BN * j, h, b, S)))
        ptx::tma_load_4d(dst, tm, bar(C::kBarSlotFull + s), kCC * c, BN * j, h, b);
    }
  };
  // The first key tile goes out with the query tiles, before the set-up
  // barriers (not in the stall self-test when it is the load left out).
  const bool early_k0 = !(kStallProbe && args.skip_load == 0);

  // ---------------------------------------------------------- prologue
  // Launched with programmatic stream serialization: the next kernel in the
  // stream may start its set-up now, and this CTA's set-up (barriers, TMEM,
  // tensor-map prefetch) overlaps the previous kernel's tail.  No thread
  // touches global memory before grid_dependency_wait.
  if (threadIdx.x == 0) ptx::launch_dependents();
  if (warp == kLoadWarp) {
    if (lane == 0) {
      misc[1] = 0u;
      ptx::mbar_init(bar(C::kBarQ), 1);
      ptx::mbar_init(bar(C::kBarQ + 1), 1);
      for (int s = 0; s < NSLOT; ++s) {
        ptx::mbar_init(bar(C::kBarSlotFull + s), 1);
        ptx::mbar_init(bar(C::kBarSlotEmpty + s), 1);
      }
      for (int i = 0; i < 2; ++i) {
        ptx::mbar_init(bar(C::kBarSFull + i), 1);
        ptx::mbar_init(bar(C::kBarSFree + i), 4);  // one arrival per softmax warp
        for (int pb = 0; pb < PB; ++pb) {
          // per P buffer, so neither barrier can complete twice unobserved:
          // buffer b is rewritten only after PV on b completed
          ptx::mbar_init(bar(C::kBarPFull + i * PB + pb), 4);
          ptx::mbar_init(bar(C::kBarPVDone + i * PB + pb), 1);
        }
        ptx::mbar_init(bar(C::kBarOFull + i), 1);
      }
      ptx::mbar_init(bar(C::kBarDrain), 2);  // one commit per issuing thread
      ptx::fence_mbar_init();
      ptx::fence_proxy_async_smem();
      ptx::tma_prefetch_desc(&tm_q);
      ptx::tma_prefetch_desc(&tm_k);
      ptx::tma_prefetch_desc(&tm_v);
      ptx::tma_prefetch_desc(&tm_o);
    }
    ptx::grid_dependency_wait();
    int extent = S;
    if constexpr (kMask) extent = mask_extent(mrow, args.mask_ss, S, lane);
    if (lane == 0) {
      misc[2] = static_cast<uint32_t>(extent);
      // Q0, K(0), Q1 overlap the set-up below; the first product needs only
      // Q0 and K(0).  A block that returns at once (all its query rows
      // masked) loads nothing.
      if (!(kMask && args.zero_masked_queries && q0 >= extent)) {
        load_q(0);
        if (early_k0) {
          ptx::mbar_arrive_expect_tx(bar(C::kBarSlotFull), C::kKVTileBytes);
          load_kv(0, 0, 0u);
        }
        load_q(1);
      }
    }
  }
  __syncthreads();
  if (warp != kLoadWarp) ptx::grid_dependency_wait();
  const int extent = static_cast<int>(misc[2]);

  // A block whose rows all lie at or past the last valid key has only masked
  // query rows: with zero_masked_queries its output is all zeros.
  if (kMask && args.zero_masked_queries && q0 >= extent) {
    if (warp < kSoftmaxWarps) {
      const int row = q0 + threadIdx.x;
      if (row < S) {
        uint4* dst = reinterpret_cast<uint4*>(
            reinterpret_cast<uint8_t*>(args.o) +
            C::ELEM * (static_cast<int64_t>(b) * args.o_sb + static_cast<int64_t>(h) * args.o_sh +
                       static_cast<int64_t>(row) * args.o_ss));
#pragma unroll
        for (int c = 0; c < args.head_dim * C::ELEM / 16; ++c) dst[c] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    return;
  }

  if (warp == kQkWarp) {
    ptx::tmem_alloc(sbase + C::kOffMisc, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = misc[0];

  // Key tiles each query tile visits.
  const int kv_keys = kMask ? max(1, extent) : S;
  const int n_kv = (kv_keys + BN - 1) / BN;
  int n_tiles[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int q_end = q0 + kBlockM * (i + 1);  // one past the tile's last row
    n_tiles[i] = kCausal ? min((q_end + BN - 1) / BN, n_kv) : n_kv;
  }
  const int n_max = n_tiles[1];  // Q1 never needs fewer tiles than Q0

  if (warp == kLoadWarp) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      // ring load L = 2 j + kv; load 0 (K(0)) went out in the prologue
      uint32_t L = 0;
      bool ok = true;
      for (int j = 0; ok && j < n_max; ++j) {
        for (int kv = 0; kv < 2; ++kv) {
          if (L == 0 && early_k0) {
            ++L;
            continue;
          }
          const uint32_t s = L % NSLOT, r = L / NSLOT;
          if (!wait_bar(bar(C::kBarSlotEmpty + s), (r & 1u) ^ 1u, abort_flag, args.err)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_expect_tx(bar(C::kBarSlotFull + s), C::kKVTileBytes);
          if (kStallProbe && static_cast<int32_t>(L) == args.skip_load) {
            ++L;  // the announced bytes never arrive
            continue;
          }
          load_kv(j, kv, s);
          ++L;
        }
      }
      if (!ok) {
        // Let copies already issued land before the CTA's shared memory goes away.
        const uint32_t first = L > NSLOT ? L - NSLOT : 0u;
        for (uint32_t x = first; x < L; ++x) {
          const uint64_t t0 = ptx::globaltimer_ns();
          while (!ptx::mbar_try_wait(bar(C::kBarSlotFull + x % NSLOT), (x / NSLOT) & 1u) &&
                 ptx::globaltimer_ns() - t0 < kWaitTimeoutNs) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == kQkWarp) {
    // -------------------------------------------- tcgen05 issuer: scores
    // S_i(j) = Q_i K(j)^T: A = Q (K-major), B = K (K-major, BN rows).  A QK
    // product may overwrite its S buffer once the previous scores in that
    // buffer were copied to registers by their softmax warpgroup.  With one
    // shared S buffer the occupancy order is S0(0), S1(0), S0(1), S1(1), ...
    if (lane == 0) {
      constexpr uint32_t id_qk =
          kTF32 ? ptx::idesc_tf32(kBlockM, BN, false) : ptx::idesc_f16(kBF16, kBlockM, BN, false);
      bool ok = true;
      int prev_i[2] = {-1, -1}, prev_j[2] = {-1, -1};  // last occupant per S buffer
      for (int j = 0; ok && j < n_max; ++j) {
        const uint32_t kL = 2u * j, ks = kL % NSLOT;
        ok = wait_bar(bar(C::kBarSlotFull + ks), (kL / NSLOT) & 1u, abort_flag, args.err);
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          if (!ok || j >= n_tiles[i]) continue;
          if (j == 0 && !wait_bar(bar(C::kBarQ + i), 0, abort_flag, args.err)) {
            ok = false;
            break;
          }
          const int sb = C::kSharedS ? 0 : i;
          if (prev_i[sb] >= 0 &&
              !issuer_wait(bar(C::kBarSFree + prev_i[sb]), prev_j[sb] & 1, abort_flag, args.err)) {
            ok = false;
            break;
          }
          prev_i[sb] = i;
          prev_j[sb] = j;
          ptx::tc_fence_after();
          const uint32_t qaddr = sbase + C::kOffQ + i * C::kQTileBytes;
          const uint32_t kaddr = sbase + C::kOffRing + ks * C::kKVTileBytes;
          if (!chk(tile_ok(qaddr, C::kQTileBytes, sbase + C::kOffQ, sbase + C::kOffRing) &&
                   tile_ok(kaddr, C::kKVTileBytes, sbase + C::kOffRing, sbase + C::kOffBar) &&
                   C::col_s(i) + BN <= kTmemCols)) {
            ok = false;
            break;
          }
          // 32 bytes of K per product: four products per 128-byte swizzle row
#pragma unroll
          for (int kk = 0; kk < D / C::kKStep; ++kk) {
            const uint32_t qo = (kk >> 2) * C::kQChunkBytes + (kk & 3) * 32;
            const uint32_t ko = (kk >> 2) * C::kKVChunkBytes + (kk & 3) * 32;
            const uint64_t qd = ptx::smem_desc_sw128(qaddr + qo, 16, 1024);
            const uint64_t kd = ptx::smem_desc_sw128(kaddr + ko, 16, 1024);
            if constexpr (kTF32)
              ptx::tc_mma_ss_tf32(tmem + C::col_s(i), qd, kd, id_qk, kk > 0 ? 1u : 0u);
            else
              ptx::tc_mma_ss(tmem + C::col_s(i), qd, kd, id_qk, kk > 0 ? 1u : 0u);
          }
          ptx::tc_commit(bar(C::kBarSFull + i));
        }
        // Q1 is K(j)'s last reader (Q0 never needs more key tiles than Q1)
        if (ok) ptx::tc_commit(bar(C::kBarSlotEmpty + ks));
      }
      // Drain: every MMA this thread issued completes before TMEM is freed.
      ptx::tc_commit(bar(C::kBarDrain));
      const uint64_t t0 = ptx::globaltimer_ns();
      while (!ptx::mbar_try_wait(bar(C::kBarDrain), 0) &&
             ptx::globaltimer_ns() - t0 < kWaitTimeoutNs) {
      }
    }
    __syncwarp();
  } else if (warp == kPvWarp) {
    // --------------------------------------- tcgen05 issuer: PV products
    // O_i += P_i(j) V(j): A = P from TMEM, B = V (MN-major, D contiguous),
    // issued as soon as the softmax warpgroup has written P_i(j).
    if (lane == 0) {
      constexpr uint32_t id_pv =
          kTF32 ? ptx::idesc_tf32(kBlockM, D, true) : ptx::idesc_f16(kBF16, kBlockM, D, true);
      bool ok = true;
      for (int j = 0; ok && j < n_max; ++j) {
        const uint32_t vL = 2u * j + 1u, vs = vL % NSLOT;
        ok = wait_bar(bar(C::kBarSlotFull + vs), (vL / NSLOT) & 1u, abort_flag, args.err);
        const uint32_t vaddr = sbase + C::kOffRing + vs * C::kKVTileBytes;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          if (!ok || j >= n_tiles[i]) continue;
          if (!issuer_wait(bar(C::kBarPFull + i * PB + (j % PB)), (j / PB) & 1, abort_flag,
                           args.err)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          if (!chk(tile_ok(vaddr, C::kKVTileBytes, sbase + C::kOffRing, sbase + C::kOffBar) &&
                   C::col_p(i, j % PB) + C::kPCols <= kTmemCols && C::col_o(i) + D <= kTmemCols)) {
            ok = false;
            break;
          }
          const uint32_t pcol = tmem + C::col_p(i, j % PB);
          // kKStep keys per product: kKStep rows of V (128 bytes each) and
          // 8 TMEM columns of P (16-bit pairs, or single fp32 values)
#pragma unroll
          for (int kk = 0; kk < BN / C::kKStep; ++kk) {
            const uint64_t bdesc =
                ptx::smem_desc_sw128(vaddr + kk * (C::kKStep * 128), C::kKVChunkBytes, 1024);
            if constexpr (kTF32) {
              // fp32 V is MN-major in the 32-byte-atom swizzle: 4-row K groups
              const uint64_t vdesc = ptx::smem_desc_sw128_base32(vaddr + kk * (C::kKStep * 128),
                                                                 C::kKVChunkBytes, 512);
              ptx::tc_mma_ts_tf32(tmem + C::col_o(i), pcol + kk * 8, vdesc, id_pv,
                                  (j > 0 || kk > 0) ? 1u : 0u);
            } else {
              ptx::tc_mma_ts(tmem + C::col_o(i), pcol + kk * 8, bdesc, id_pv,
                             (j > 0 || kk > 0) ? 1u : 0u);
            }
          }
          ptx::tc_commit(bar(C::kBarPVDone + i * PB + (j % PB)));
          if (j == n_tiles[i] - 1) ptx::tc_commit(bar(C::kBarOFull + i));
        }
        if (ok) ptx::tc_commit(bar(C::kBarSlotEmpty + vs));  // Q1 is V(j)'s last reader
      }
      ptx::tc_commit(bar(C::kBarDrain));
      const uint64_t t0 = ptx::globaltimer_ns();
      while (!ptx::mbar_try_wait(bar(C::kBarDrain), 0) &&
             ptx::globaltimer_ns() - t0 < kWaitTimeoutNs) {
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    const int i = warp >> 2;              // query tile
    const int quad = warp & 3;            // TMEM lane quadrant of this warp
    const int rl = quad * 32 + lane;      // row within the tile = TMEM lane
    const int qstart = q0 + kBlockM * i;  // first row of the tile
    const int row = qstart + rl;          // global query row
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + lane_off + C::col_s(i);
    const uint32_t tO = tmem + lane_off + C::col_o(i);
    const float scale_log2 = args.scale_log2;
    const int n = n_tiles[i];
    const uint32_t bar_s_full = bar(C::kBarSFull + i), bar_s_free = bar(C::kBarSFree + i);
    auto bar_p_full = [&](int j) { return bar(C::kBarPFull + i * PB + (j % PB)); };

    // mask bits of key tile j for the warp (all ones without a mask)
    auto mask_words = [&](int j, uint32_t (&mw)[kMaskWords]) {
#pragma unroll
      for (int q = 0; q < kMaskWords; ++q) {
        if constexpr (kMask) {
          const int key = j * BN + 32 * q + lane;
          const bool v = key < S && mrow[static_cast<int64_t>(key) * args.mask_ss] != 0;
          mw[q] = __ballot_sync(0xffffffffu, v);
        } else {
          mw[q] = ~0u;
        }
      }
    };
    // largest visible in-tile key index given bounds and causality
    auto visible_limit = [&](int j) {
      const int key0 = j * BN;
      int lim = S - 1 - key0;
      if (kCausal) lim = min(lim, row - key0);
      return lim;
    };
    auto partial_tile = [&](int j, const uint32_t (&mw)[kMaskWords]) {
      const int key0 = j * BN;
      bool p = key0 + BN > S || (kCausal && key0 + BN - 1 > qstart);
      if constexpr (kMask) {
        uint32_t all = ~0u;
#pragma unroll
        for (int q = 0; q < kMaskWords; ++q) all &= mw[q];
        p = p || all != ~0u;
      }
      return p;
    };

    float m_run = -INFINITY;
    float l_run = 0.f;
    float lse_row = -INFINITY;  // partial instances: natural-log log-sum-exp of the row
    bool ok = true;

    if (n <= C::kExactTiles) {
      // Every visible key of this query tile lies in the first 128 keys, so
      // the whole row fits in registers: reproduce the reference's rounding
      // points exactly (model/triton_fused_attention.py:1272-1284): scores
      // rounded to the input dtype, the scale multiply rounded again, fp32
      // softmax normalised before P is rounded.  These rows have few keys and
      // large outputs, where a different rounding order would show as whole
      // output ulps.
      constexpr int NE = C::kExactKeys;
      uint32_t sr[NE];
#pragma unroll
      for (int k = 0; k < NE; ++k) sr[k] = __float_as_uint(-INFINITY);
#pragma unroll
      for (int j = 0; j < C::kExactTiles; ++j) {
        if (j < n && ok) {
          uint32_t mw[kMaskWords];
          mask_words(j, mw);
          if (!warp_wait_bar(bar_s_full, j & 1, abort_flag, args.err)) {
            ok = false;
          } else {
            ptx::tc_fence_after();
            uint32_t part[BN];
            load_row<BN>(tS, part);
            warp_arrive(bar_s_free, lane);
            mask_row<BN>(part, visible_limit(j), mw);
#pragma unroll
            for (int k = 0; k < BN; ++k) sr[j * BN + k] = part[k];
          }
        }
      }
      if (ok) {
        const float scale = args.scale;
        float mx = -INFINITY;
#pragma unroll
        for (int k = 0; k < NE; ++k) {
          const float v =
              round_to_input<kDtype>(round_to_input<kDtype>(__uint_as_float(sr[k])) * scale);
          sr[k] = __float_as_uint(v);
          mx = fmaxf(mx, v);
        }
        const float sub = (mx == -INFINITY) ? 0.f : mx;
        float tot = 0.f;
#pragma unroll
        for (int k = 0; k < NE; ++k) {
          const float pe = expf(__uint_as_float(sr[k]) - sub);
          sr[k] = __float_as_uint(pe);
          tot += pe;
        }
        const float inv = 1.f / tot;
#pragma unroll
        for (int j = 0; j < C::kExactTiles; ++j) {
          if (j < n) {
            const uint32_t tP = tmem + lane_off + C::col_p(i, j % PB);
            if constexpr (kTF32) {
              // fp32 P, one column per key (the product reads it as TF32)
#pragma unroll
              for (int k = 0; k < BN; ++k)
                sr[j * BN + k] = __float_as_uint(__uint_as_float(sr[j * BN + k]) * inv);
#pragma unroll
              for (int c = 0; c < BN / 32; ++c)
                ptx::tmem_st_32x32b_x32(tP + 32 * c,
                                        *reinterpret_cast<uint32_t(*)[32]>(&sr[j * BN + 32 * c]));
            } else {
              uint32_t pk[BN / 2];
#pragma unroll
              for (int e = 0; e < BN / 2; ++e)
                pk[e] = pack2<kBF16>(__uint_as_float(sr[j * BN + 2 * e]) * inv,
                                     __uint_as_float(sr[j * BN + 2 * e + 1]) * inv);
#pragma unroll
              for (int c = 0; c < BN / 64; ++c)
                ptx::tmem_st_32x32b_x32(tP + 32 * c,
                                        *reinterpret_cast<uint32_t(*)[32]>(&pk[32 * c]));
            }
            ptx::tmem_wait_st();
            warp_arrive(bar_p_full(j), lane);
          }
        }
        m_run = mx;   // -inf only when the row has no visible key (NaN output)
        l_run = 1.f;  // P is already normalised
        if constexpr (kPartial) lse_row = (mx == -INFINITY) ? -INFINITY : sub + logf(tot);
      }
    } else {
      for (int j = 0; j < n; ++j) {
        uint32_t mw[kMaskWords];
        mask_words(j, mw);
        if (!warp_wait_bar(bar_s_full, j & 1, abort_flag, args.err)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
        uint32_t sr[BN];
        float mx;
        if (partial_tile(j, mw)) {
          load_row<BN>(tS, sr);
          warp_arrive(bar_s_free, lane);  // the MMA warp may now overwrite S_i
          mask_row<BN>(sr, visible_limit(j), mw);
          mx = row_max<BN>(sr);
        } else if constexpr (kSplitLoad && BN == 128) {
          // max of columns [0,64) while columns [64,128) are still in flight
          if constexpr (D == 64) {
            // one 64-column load per half: measured +4 % for head dim 64 (and
            // slower for 128, where the two 32-column loads stay)
            ptx::tmem_ld_32x32b_x64(tS, *reinterpret_cast<uint32_t(*)[64]>(&sr[0]));
            ptx::tmem_wait_ld();
            ptx::tmem_ld_32x32b_x64(tS + 64, *reinterpret_cast<uint32_t(*)[64]>(&sr[64]));
          } else {
            ptx::tmem_ld_32x32b_x32(tS, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
            ptx::tmem_ld_32x32b_x32(tS + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
            ptx::tmem_wait_ld();
            ptx::tmem_ld_32x32b_x32(tS + 64, *reinterpret_cast<uint32_t(*)[32]>(&sr[64]));
            ptx::tmem_ld_32x32b_x32(tS + 96, *reinterpret_cast<uint32_t(*)[32]>(&sr[96]));
          }
          const float m_lo = range_max<0, 64, BN>(sr);
          ptx::tmem_wait_ld();
          warp_arrive(bar_s_free, lane);
          mx = fmaxf(m_lo, range_max<64, 64, BN>(sr));
        } else {
          load_row<BN>(tS, sr);
          warp_arrive(bar_s_free, lane);
          mx = row_max<BN>(sr);
        }

        const float m_cand = mx * scale_log2;
        const bool resc = m_cand > m_run + kRescaleLog2;
        const float m_new = resc ? m_cand : m_run;
        const float alpha = resc ? ptx::ex2_approx(m_run - m_new) : 1.f;
        l_run *= alpha;
        m_run = m_new;
        const float neg_m = (m_run == -INFINITY) ? 0.f : -m_run;

        // p = 2^(s*scale*log2e - m); kPolyPer8 of every 8 on the FMA pipe
        // (ex2_poly), the rest on the MUFU; four independent partial sums.
        float sum[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t pk[kTF32 ? 1 : BN / 2];  // packed 16-bit P (fp32 P overwrites sr in place)
#pragma unroll
        for (int e = 0; e < BN / 2; ++e) {
          float x[2], p2[2];
          if constexpr (kF32x2) {
            ffma2(x[0], x[1], __uint_as_float(sr[2 * e]), __uint_as_float(sr[2 * e + 1]),
                  scale_log2, scale_log2, neg_m, neg_m);
          } else {
            x[0] = fmaf(__uint_as_float(sr[2 * e]), scale_log2, neg_m);
            x[1] = fmaf(__uint_as_float(sr[2 * e + 1]), scale_log2, neg_m);
          }
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int k = 2 * e + hh;
            p2[hh] = ((k & 7) < kPolyPer8) ? ex2_poly(fmaxf(x[hh], -126.f))
                                           : ptx::ex2_approx(x[hh]);
          }
          if constexpr (kF32x2) {
            const int a = 2 * (e & 1);
            fadd2(sum[a], sum[a + 1], sum[a], sum[a + 1], p2[0], p2[1]);
          } else {
            sum[e & 3] += p2[0] + p2[1];
          }
          if constexpr (kTF32) {
            sr[2 * e] = __float_as_uint(p2[0]);
            sr[2 * e + 1] = __float_as_uint(p2[1]);
          } else {
            pk[e] = pack2<kBF16>(p2[0], p2[1]);
          }
        }
        l_run += (sum[0] + sum[1]) + (sum[2] + sum[3]);

        // P buffer j % PB was last read by PV_i(j - PB).
        if (j >= PB) {
          const int pb = j % PB;
          if (!warp_wait_bar(bar(C::kBarPVDone + i * PB + pb), ((j / PB) + 1) & 1, abort_flag,
                             args.err)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
        }
        if (j > 0 && __any_sync(0xffffffffu, resc)) {
          // O_i must hold the sum over tiles < j: wait for PV_i(j-1).
          const int pb = (j - 1) % PB;
          if (!warp_wait_bar(bar(C::kBarPVDone + i * PB + pb), ((j - 1) / PB) & 1, abort_flag,
                             args.err)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            ptx::tmem_ld_32x32b_x32(tO + 32 * c, o);
            ptx::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            ptx::tmem_st_32x32b_x32(tO + 32 * c, o);
          }
        }
        const uint32_t tP = tmem + lane_off + C::col_p(i, j % PB);
        if constexpr (kTF32) {
#pragma unroll
          for (int c = 0; c < BN / 32; ++c)
            ptx::tmem_st_32x32b_x32(tP + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&sr[32 * c]));
        } else {
#pragma unroll
          for (int c = 0; c < BN / 64; ++c)
            ptx::tmem_st_32x32b_x32(tP + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&pk[32 * c]));
        }
        ptx::tmem_wait_st();
        warp_arrive(bar_p_full(j), lane);
      }
      if constexpr (kPartial)
        lse_row = (m_run == -INFINITY) ? -INFINITY
                                       : (m_run + log2f(l_run)) * 0.6931471805599453f;
    }

    // ------------------------------------------------------------ epilogue
    if (ok) ok = warp_wait_bar(bar(C::kBarOFull + i), 0, abort_flag, args.err);
    uint32_t all_ok;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.and.pred q, %2, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(all_ok)
        : "r"(ok ? 1u : 0u), "r"(1 + i)
        : "memory");
    if (all_ok) {
      ptx::tc_fence_after();
      bool zero_row = false;
      if constexpr (kMask) {
        if (args.zero_masked_queries && row < S)
          zero_row = mrow[static_cast<int64_t>(row) * args.mask_ss] == 0;
      }
      // a row that saw no visible key is NaN, as torch.softmax of all -inf
      const float inv_l =
          zero_row ? 0.f : (m_run == -INFINITY ? __int_as_float(0x7fc00000) : 1.f / l_run);
      const uint32_t stage = sbase + C::kOffQ + i * C::kQTileBytes;  // Q_i is no longer read
      // Partial instances: out = w_new * (this chunk's output) + w_old * (the
      // output in memory), the weights from the two log-sum-exps.  A side with
      // no visible key (lse -inf) has weight 0 and is not read into the sum;
      // when neither side saw a key the row keeps what it holds (NaN).
      float w_new = 1.f, w_old = 0.f;
      const uint8_t* orow = nullptr;
      if constexpr (kPartial) {
        if (row < S) {
          float* lp = args.lse + static_cast<int64_t>(b) * args.lse_sb +
                      static_cast<int64_t>(h) * args.lse_sh + static_cast<int64_t>(row) * args.lse_ss;
          float lse_out = lse_row;
          if (args.accumulate) {
            const float lo = *lp;
            const float mx2 = fmaxf(lo, lse_row);
            if (mx2 == -INFINITY) {
              w_new = 0.f;
              w_old = 1.f;
            } else {
              w_old = lo == -INFINITY ? 0.f : expf(lo - mx2);
              w_new = lse_row == -INFINITY ? 0.f : expf(lse_row - mx2);
              const float tot = w_old + w_new;
              lse_out = mx2 + logf(tot);
              w_old /= tot;
              w_new /= tot;
            }
            orow = reinterpret_cast<const uint8_t*>(args.o) +
                   C::ELEM * (static_cast<int64_t>(b) * args.o_sb + static_cast<int64_t>(h) * args.o_sh +
                              static_cast<int64_t>(row) * args.o_ss);
          }
          *lp = lse_out;
        }
      }
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        ptx::tmem_ld_32x32b_x32(tO + 32 * c, o);
        ptx::tmem_wait_ld();
        // 16-byte pieces of the row: 8 packed 16-bit or 4 fp32 elements each
        constexpr int kPer16 = 16 / C::ELEM;
#pragma unroll
        for (int u = 0; u < 32 / kPer16; ++u) {
          uint32_t w[4];
          if constexpr (kPartial) {
            // merge with the 16 bytes of this piece already in the output
            // (read before the tile's store is issued)
            uint4 old4 = make_uint4(0u, 0u, 0u, 0u);
            const int col = 32 * c + kPer16 * u;
            if (orow && col < args.head_dim)
              old4 = *reinterpret_cast<const uint4*>(orow + C::ELEM * col);
            const uint32_t ow[4] = {old4.x, old4.y, old4.z, old4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if constexpr (kTF32) {
                const float a = __uint_as_float(o[4 * u + e]) * inv_l;
                float r = w_new > 0.f ? w_new * a : 0.f;
                if (w_old > 0.f) r += w_old * __uint_as_float(ow[e]);
                if (w_new == 0.f && w_old == 1.f) r = __uint_as_float(ow[e]);
                w[e] = __float_as_uint(r);
              } else {
                const float a = __uint_as_float(o[8 * u + 2 * e]) * inv_l;
                const float bb = __uint_as_float(o[8 * u + 2 * e + 1]) * inv_l;
                const float oa = kBF16 ? __uint_as_float(ow[e] << 16)
                                       : __half2float(__ushort_as_half(static_cast<uint16_t>(ow[e])));
                const float ob = kBF16 ? __uint_as_float(ow[e] & 0xffff0000u)
                                       : __half2float(__ushort_as_half(static_cast<uint16_t>(ow[e] >> 16)));
                float ra = w_new > 0.f ? w_new * a : 0.f;
                float rb = w_new > 0.f ? w_new * bb : 0.f;
                if (w_old > 0.f) {
                  ra += w_old * oa;
                  rb += w_old * ob;
                }
                w[e] = (w_new == 0.f && w_old == 1.f) ? ow[e] : pack2<kBF16>(ra, rb);
              }
            }
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              if constexpr (kTF32) {
                const float a = __uint_as_float(o[4 * u + e]) * inv_l;
                w[e] = __float_as_uint(zero_row ? 0.f : a);
              } else {
                float a = __uint_as_float(o[8 * u + 2 * e]) * inv_l;
                float bb = __uint_as_float(o[8 * u + 2 * e + 1]) * inv_l;
                if (zero_row) a = bb = 0.f;
                w[e] = pack2<kBF16>(a, bb);
              }
            }
          }
          const int col = 32 * c + kPer16 * u;  // first element of this 16-byte piece
          const int cb = col / kCC;             // 128-byte swizzle block of the row
          const int lc = (col % kCC) / kPer16;  // logical 16-byte piece within the block
          const uint32_t addr = stage + cb * C::kQChunkBytes + rl * 128 + ((lc ^ (rl & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w[0]),
                       "r"(w[1]), "r"(w[2]), "r"(w[3])
                       : "memory");
        }
      }
      ptx::fence_proxy_async_smem();
      ptx::named_barrier_sync(1 + i, kBlockM);
      if (rl == 0 && qstart < S) {
#pragma unroll
        for (int cb = 0; cb < C::kChunks; ++cb) {
          const uint32_t src = stage + cb * C::kQChunkBytes;
          if (chk(tile_ok(src, C::kQChunkBytes, sbase + C::kOffQ, sbase + C::kOffRing) &&
                  coord_ok(kCC * cb, qstart, h, b, S)))
            ptx::tma_store_4d(&tm_o, src, kCC * cb, qstart, h, b);
        }
        ptx::bulk_commit_group();
        ptx::bulk_wait_group_read_all();  // shared memory may go once the store has read it
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kQkWarp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

// Instances: 128-key tiles, one P buffer per query tile and one S buffer
// shared by the two query tiles.  For D = 128 that fills the 512 TMEM
// columns.  D = 64 would have room for an S buffer per query tile, but the
// shared buffer was measured faster there too (+7 %): it makes the two softmax
// warpgroups alternate, so the warps that share an SM sub-partition do not
// run their exponentials at the same time and drift apart.
using Cfg128 = Cfg<128, 128, 1, 5, true>;
using Cfg64 = Cfg<64, 128, 1, 10, true>;
// fp32 inputs (TF32 products), head dims up to 64: Q0/Q1 64 KB plus five
// 32 KB K/V slots, and S | P0 P1 (128 fp32 columns each) | O0 O1 = 512 TMEM
// columns, the same budgets as Cfg128.
using CfgF32 = Cfg<64, 128, 1, 5, true, 4>;

// ------------------------------------------------------------------- host
// Text of the calling thread's last host-side failure, shared by every entry
// point of the library (b200_attn_last_error_detail).
thread_local char g_last_error[256] = {0};

void set_error(const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
}

std::atomic<int64_t> g_launch_count{0};

void count_launch() { g_launch_count.fetch_add(1, std::memory_order_relaxed); }

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

// 16-bit inputs: any multiple of 8 up to 128.  The instance with D = 64 serves
// head dims up to 64, D = 128 the rest: the tensor maps give the true head dim
// as the inner extent, so the TMA boxes read zeros past it (Q K^T and P V are
// unchanged by zero columns) and the output store clips the columns past it.
// fp32 inputs: any multiple of 8 up to 64, on the fp32 instance.
bool supported_dtype(int32_t dtype) {
  return dtype == B200_ATTN_DTYPE_BF16 || dtype == B200_ATTN_DTYPE_FP16 ||
         dtype == B200_ATTN_DTYPE_FP32;
}
bool supported_head_dim(int32_t dtype, int64_t d) {
  const int64_t hi = dtype == B200_ATTN_DTYPE_FP32 ? 64 : 128;
  return d >= 8 && d <= hi && d % 8 == 0;
}
bool wide_head(int64_t d) { return d > 64; }
int64_t elem_bytes(int32_t dtype) { return dtype == B200_ATTN_DTYPE_FP32 ? 4 : 2; }

// Alignment rules of the 4-D TMA view {D, S, H, B}: 16-byte base, 16-byte
// multiples for every stride whose dimension has extent > 1.
bool tensor_aligned(const void* ptr, const int64_t st[3], const b200_attn_fwd_params* p) {
  if (reinterpret_cast<uintptr_t>(ptr) & 15u) return false;
  const int64_t ext[3] = {p->batch, p->heads, p->seq_len};
  for (int a = 0; a < 3; ++a) {
    if (ext[a] <= 1) continue;
    if (st[a] <= 0) return false;
    if ((st[a] * elem_bytes(p->dtype)) % 16 != 0) return false;
  }
  return true;
}

// 4-D tensor map {D, S, H, B} with a {128 bytes, box_rows, 1, 1} box (64
// 16-bit or 32 fp32 elements), 128-byte swizzle.  `mn_major_tf32`: the box
// lands in the 128-byte swizzle with 32-byte atoms, the only shared-memory
// layout of an MN-major TF32 operand (fp32 V).
int encode_map(CUtensorMap* m, const void* ptr, const int64_t st[3],
               const b200_attn_fwd_params* p, uint32_t box_rows, bool mn_major_tf32 = false) {
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled entry point unavailable");
    return B200_ATTN_ERR_LAUNCH;
  }
  const int64_t D = p->head_dim, S = p->seq_len, H = p->heads, B = p->batch;
  const int64_t eb = elem_bytes(p->dtype);
  // Size-1 dimensions never move the address; give them a legal stride.
  const int64_t fill = D * eb * 16;
  const int64_t s_seq = S > 1 ? st[2] * eb : fill;
  const int64_t s_head = H > 1 ? st[1] * eb : fill;
  const int64_t s_batch = B > 1 ? st[0] * eb : fill;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S),
                        static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(s_seq), static_cast<cuuint64_t>(s_head),
                           static_cast<cuuint64_t>(s_batch)};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(128 / eb), box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt = p->dtype == B200_ATTN_DTYPE_BF16   ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : p->dtype == B200_ATTN_DTYPE_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                    : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const CUtensorMapSwizzle swz =
      mn_major_tf32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = fn(m, dt, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed");
    return B200_ATTN_ERR_LAUNCH;
  }
  return B200_ATTN_OK;
}

constexpr int kMaxDevices = 64;

struct DeviceState {
  std::once_flag probed;
  bool sm100 = false;
};
DeviceState g_dev[kMaxDevices];

template <class Cf, bool Ca, bool M, int DT, bool SP = false, bool PT = false>
int launch_one(const CUtensorMap maps[4], const typename ArgsOf<PT>::type& args, int device,
               cudaStream_t stream) {
  auto kernel = attn_fwd_sm100_kernel<Cf, Ca, M, DT, SP, PT>;
  static std::once_flag attr_once[kMaxDevices];
  static cudaError_t attr_err[kMaxDevices];
  std::call_once(attr_once[device], [&] {
    attr_err[device] = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            Cf::kSmemBytes);
  });
  if (attr_err[device] != cudaSuccess) {
    set_error(cudaGetErrorString(attr_err[device]));
    return B200_ATTN_ERR_LAUNCH;
  }
  const unsigned grid = static_cast<unsigned>(args.num_q_blocks) * args.batch * args.heads;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cf::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, maps[0], maps[1], maps[2], maps[3], args);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(cudaGetErrorString(e));
    return B200_ATTN_ERR_LAUNCH;
  }
  count_launch();
  return B200_ATTN_OK;
}

template <class Cf, int DT>
int dispatch_flags(const CUtensorMap maps[4], const KernelArgs& a, const b200_attn_fwd_params* p,
                   int dev, cudaStream_t s) {
  const bool c = p->causal != 0, m = p->key_mask != nullptr;
  if (c) {
    return m ? launch_one<Cf, true, true, DT>(maps, a, dev, s)
             : launch_one<Cf, true, false, DT>(maps, a, dev, s);
  }
  return m ? launch_one<Cf, false, true, DT>(maps, a, dev, s)
           : launch_one<Cf, false, false, DT>(maps, a, dev, s);
}

template <class Cf, int DT>
int dispatch_partial(const CUtensorMap maps[4], const PartialKernelArgs& a, bool causal, int dev,
                     cudaStream_t s) {
  return causal ? launch_one<Cf, true, false, DT, false, true>(maps, a, dev, s)
                : launch_one<Cf, false, false, DT, false, true>(maps, a, dev, s);
}

// Kernel instance for (dtype, head_dim): its keys per K/V tile and ring slots.
void instance_shape(int32_t dtype, int64_t head_dim, int* block_n, int* slots) {
  if (dtype == B200_ATTN_DTYPE_FP32) {
    *block_n = CfgF32::BN;
    *slots = CfgF32::NSLOT;
  } else if (wide_head(head_dim)) {
    *block_n = Cfg128::BN;
    *slots = Cfg128::NSLOT;
  } else {
    *block_n = Cfg64::BN;
    *slots = Cfg64::NSLOT;
  }
}

}  // namespace
}  // namespace b200attn

// ------------------------------------------------------------------ C ABI
using namespace b200attn;

extern "C" int32_t b200_attn_abi_version(void) { return B200_ATTN_ABI_VERSION; }

extern "C" int32_t b200_attn_query(int32_t dtype, int64_t head_dim, int32_t causal,
                                   int32_t has_mask) {
  (void)causal;
  (void)has_mask;
  if (!supported_dtype(dtype)) return 0;
  return supported_head_dim(dtype, head_dim) ? 1 : 0;
}

extern "C" const char* b200_attn_error_string(int32_t code) {
  switch (code) {
    case B200_ATTN_OK: return "ok";
    case B200_ATTN_ERR_INVALID_ARGUMENT: return "invalid argument";
    case B200_ATTN_ERR_UNSUPPORTED: return "unsupported dtype or head_dim";
    case B200_ATTN_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
    case B200_ATTN_ERR_DEVICE: return "no sm_100 device for the given pointers";
    case B200_ATTN_ERR_LAUNCH: return "kernel launch failed";
    case B200_ATTN_ERR_TIMEOUT: return "an earlier launch reported a device pipeline wait timeout";
    case B200_ATTN_ERR_DEVICE_BOUNDS:
      return "an earlier launch reported a failed device bounds check";
    default: return "unknown error";
  }
}

extern "C" const char* b200_attn_last_error_detail(void) { return g_last_error; }

extern "C" int64_t b200_attn_launch_count(void) {
  return g_launch_count.load(std::memory_order_relaxed);
}

extern "C" int32_t b200_attn_launch_shape(int32_t dtype, int64_t head_dim, int32_t* block_m,
                                          int32_t* rows_per_cta, int32_t* block_n,
                                          int32_t* num_warps, int32_t* ring_slots) {
  if (!b200_attn_query(dtype, head_dim, 0, 0)) return 0;
  int bn = 0, slots = 0;
  instance_shape(dtype, head_dim, &bn, &slots);
  if (block_m) *block_m = kBlockM;
  if (rows_per_cta) *rows_per_cta = kRowsPerCta;
  if (block_n) *block_n = bn;
  if (num_warps) *num_warps = kThreads / 32;
  if (ring_slots) *ring_slots = slots;
  return 1;
}

extern "C" int32_t b200_attn_check(const b200_attn_fwd_params* p) {
  if (!p || !p->q || !p->k || !p->v || !p->o) return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->batch < 1 || p->heads < 1 || p->seq_len < 1 || p->head_dim < 1)
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->batch * p->heads > (1ll << 24) || p->seq_len > (1ll << 30))
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (!(p->scale > 0.f) || !std::isfinite(p->scale)) return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (!supported_dtype(p->dtype)) return B200_ATTN_ERR_UNSUPPORTED;
  if (!supported_head_dim(p->dtype, p->head_dim)) return B200_ATTN_ERR_UNSUPPORTED;
  if (p->zero_masked_queries && !p->key_mask) return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (!tensor_aligned(p->q, p->q_stride, p) || !tensor_aligned(p->k, p->k_stride, p) ||
      !tensor_aligned(p->v, p->v_stride, p) || !tensor_aligned(p->o, p->o_stride, p))
    return B200_ATTN_ERR_ALIGNMENT;
  return B200_ATTN_OK;
}

extern "C" int32_t b200_attn_launches_per_call(const b200_attn_fwd_params* p) {
  return b200_attn_check(p) == B200_ATTN_OK ? 1 : 0;
}

namespace b200attn {
namespace {

// Restores the caller's current device when a call had to switch to the
// tensors' device.
struct DeviceGuard {
  int prev = -1;
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// Validates p, selects its device (restored by `guard` when the call ends) and
// fills the tensor maps and kernel arguments; returns a B200_ATTN_* code.
int32_t prepare(const b200_attn_fwd_params* p, CUtensorMap maps[4], KernelArgs& a, int& dev_out,
                DeviceGuard& guard) {
  int32_t rc = b200_attn_check(p);
  if (rc != B200_ATTN_OK) return rc;

  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, p->q) != cudaSuccess || attr.device < 0 ||
      attr.device >= kMaxDevices ||
      (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)) {
    cudaGetLastError();
    set_error("q is not a device pointer");
    return B200_ATTN_ERR_DEVICE;
  }
  const int dev = attr.device;
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
    int major = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) == cudaSuccess)
      g_dev[dev].sm100 = (major == 10);
  });
  if (!g_dev[dev].sm100) {
    set_error("device is not compute capability 10.x");
    return B200_ATTN_ERR_DEVICE;
  }

  int bn = 0, slots = 0;
  instance_shape(p->dtype, p->head_dim, &bn, &slots);
  const uint32_t kv_rows = static_cast<uint32_t>(bn);
  if ((rc = encode_map(&maps[0], p->q, p->q_stride, p, kBlockM)) != B200_ATTN_OK ||
      (rc = encode_map(&maps[1], p->k, p->k_stride, p, kv_rows)) != B200_ATTN_OK ||
      (rc = encode_map(&maps[2], p->v, p->v_stride, p, kv_rows,
                       p->dtype == B200_ATTN_DTYPE_FP32)) != B200_ATTN_OK ||
      (rc = encode_map(&maps[3], p->o, p->o_stride, p, kBlockM)) != B200_ATTN_OK)
    return rc;

  a.seq_len = static_cast<int32_t>(p->seq_len);
  a.head_dim = static_cast<int32_t>(p->head_dim);
  a.heads = static_cast<int32_t>(p->heads);
  a.batch = static_cast<int32_t>(p->batch);
  a.num_q_blocks = static_cast<int32_t>((p->seq_len + kRowsPerCta - 1) / kRowsPerCta);
  {
    const int64_t bh = p->batch * p->heads;
    const int64_t kv_bytes = 2 * elem_bytes(p->dtype) * p->seq_len * p->head_dim;  // K and V of one head
    // As few groups as the L2 budget allows, all of (nearly) equal size: a
    // small last group would start its heaviest query blocks late and
    // lengthen the tail (measured: -11 % for 4 heads of S = 32768).  When the
    // last group would still be less than half full (16 heads of S = 32768:
    // 3, 3, 3, 3, 3, 1), smaller groups that divide the pairs more evenly are
    // taken instead (8 groups of 2: measured +5.7 %).
    const int64_t n_groups = kGroupBytes > 0 ? (bh * kv_bytes + kGroupBytes - 1) / kGroupBytes : 1;
    int64_t g = (bh + n_groups - 1) / (n_groups < 1 ? 1 : n_groups);
    g = g < 1 ? 1 : (g > bh ? bh : g);
    if (2 * (bh % g) != 0 && 2 * (bh % g) < g) {
      int64_t h = g - 1;
      while (h > 1 && bh % h != 0 && 2 * (bh % h) < h) --h;
      g = h;
    }
    a.group_heads = static_cast<int32_t>(g);
  }
  a.scale = p->scale;
  a.scale_log2 = p->scale * kLog2e;
  a.zero_masked_queries = p->zero_masked_queries;
  a.mask = p->key_mask;
  a.mask_sb = p->key_mask ? p->mask_stride[0] : 0;
  a.mask_ss = p->key_mask ? p->mask_stride[1] : 0;
  a.o = p->o;
  a.o_sb = p->o_stride[0];
  a.o_sh = p->o_stride[1];
  a.o_ss = p->o_stride[2];
  if ((rc = resolve_error_word(p->error_word, &a.err)) != B200_ATTN_OK) return rc;
  a.skip_load = -1;
  if (static_cast<int64_t>(a.num_q_blocks) * p->batch * p->heads > 0x7fffffffll)
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  dev_out = dev;
  return B200_ATTN_OK;
}

}  // namespace
}  // namespace b200attn

extern "C" int32_t b200_attn_fwd(const b200_attn_fwd_params* p, void* stream) {
  CUtensorMap maps[4];
  KernelArgs a;
  int dev = 0;
  DeviceGuard guard;
  const int32_t rc = prepare(p, maps, a, dev, guard);
  if (rc != B200_ATTN_OK) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (p->dtype) {
    case B200_ATTN_DTYPE_FP32:
      return dispatch_flags<CfgF32, B200_ATTN_DTYPE_FP32>(maps, a, p, dev, s);
    case B200_ATTN_DTYPE_FP16:
      return wide_head(p->head_dim) ? dispatch_flags<Cfg128, B200_ATTN_DTYPE_FP16>(maps, a, p, dev, s)
                                    : dispatch_flags<Cfg64, B200_ATTN_DTYPE_FP16>(maps, a, p, dev, s);
    default:
      return wide_head(p->head_dim) ? dispatch_flags<Cfg128, B200_ATTN_DTYPE_BF16>(maps, a, p, dev, s)
                                    : dispatch_flags<Cfg64, B200_ATTN_DTYPE_BF16>(maps, a, p, dev, s);
  }
}

extern "C" int32_t b200_attn_fwd_partial(const b200_attn_partial_params* pp, void* stream) {
  if (!pp) return B200_ATTN_ERR_INVALID_ARGUMENT;
  const b200_attn_fwd_params* p = &pp->base;
  if (p->key_mask || p->zero_masked_queries) return B200_ATTN_ERR_UNSUPPORTED;
  if (!pp->lse || (reinterpret_cast<uintptr_t>(pp->lse) & 3u) || pp->reserved != 0 ||
      (pp->accumulate != 0 && pp->accumulate != 1))
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  for (int d = 0; d < 3; ++d)
    if (pp->lse_stride[d] < 0) return B200_ATTN_ERR_INVALID_ARGUMENT;
  CUtensorMap maps[4];
  PartialKernelArgs a;
  int dev = 0;
  DeviceGuard guard;
  const int32_t rc = prepare(p, maps, a, dev, guard);
  if (rc != B200_ATTN_OK) return rc;
  a.lse = pp->lse;
  a.lse_sb = pp->lse_stride[0];
  a.lse_sh = pp->lse_stride[1];
  a.lse_ss = pp->lse_stride[2];
  a.accumulate = pp->accumulate;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool c = p->causal != 0;
  switch (p->dtype) {
    case B200_ATTN_DTYPE_FP32:
      return dispatch_partial<CfgF32, B200_ATTN_DTYPE_FP32>(maps, a, c, dev, s);
    case B200_ATTN_DTYPE_FP16:
      return wide_head(p->head_dim) ? dispatch_partial<Cfg128, B200_ATTN_DTYPE_FP16>(maps, a, c, dev, s)
                                    : dispatch_partial<Cfg64, B200_ATTN_DTYPE_FP16>(maps, a, c, dev, s);
    default:
      return wide_head(p->head_dim) ? dispatch_partial<Cfg128, B200_ATTN_DTYPE_BF16>(maps, a, c, dev, s)
                                    : dispatch_partial<Cfg64, B200_ATTN_DTYPE_BF16>(maps, a, c, dev, s);
  }
}

extern "C" int32_t b200_attn_selftest_stall(const b200_attn_fwd_params* p, int32_t skipped_load,
                                             void* stream) {
  if (!p || p->head_dim != 128 || p->dtype != B200_ATTN_DTYPE_BF16 || !p->causal || p->key_mask ||
      !p->error_word || skipped_load < 0)
    return B200_ATTN_ERR_UNSUPPORTED;
  CUtensorMap maps[4];
  KernelArgs a;
  int dev = 0;
  DeviceGuard guard;
  const int32_t rc = prepare(p, maps, a, dev, guard);
  if (rc != B200_ATTN_OK) return rc;
  a.skip_load = skipped_load;
  return launch_one<Cfg128, true, false, B200_ATTN_DTYPE_BF16, true>(
      maps, a, dev, reinterpret_cast<cudaStream_t>(stream));
}

// ------------------------------------------- allocation-free partial step
// Log-sum-exp scratch of b200_attn_fwd_partial_static: one fp32 per (batch,
// head, query row), [B, H, S] contiguous.  It is a module variable, so every
// device that loads this library holds its 4 MiB until the process exits, and
// every call on a device shares it.  Host code must not pass its name to a
// kernel (on the host the name is only a stand-in); the entry point looks up
// its device address once per device instead.
static __device__ __align__(256) float b200_static_lse[B200_ATTN_STATIC_LSE_MAX_ROWS];

namespace b200attn {
namespace {

struct StaticLseState {
  std::once_flag resolved;
  cudaError_t err = cudaSuccess;
  float* ptr = nullptr;  // device address of b200_static_lse on this device
  std::mutex mu;
  // Shape of the last first-chunk call that launched on this device; an
  // accumulating call must match it (its rows merge into what that call left).
  int64_t shape[3] = {0, 0, 0};
};
StaticLseState g_static_lse[kMaxDevices];

}  // namespace
}  // namespace b200attn

extern "C" int32_t b200_attn_fwd_partial_static(const b200_attn_fwd_params* p, int32_t accumulate,
                                                void* stream) {
  if (!p) return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->key_mask || p->zero_masked_queries) return B200_ATTN_ERR_UNSUPPORTED;
  if (accumulate != 0 && accumulate != 1) return B200_ATTN_ERR_INVALID_ARGUMENT;
  int32_t rc = b200_attn_check(p);
  if (rc != B200_ATTN_OK) return rc;
  // batch * heads <= 2^24 and seq_len <= 2^30 (b200_attn_check): no overflow
  const int64_t rows = p->batch * p->heads * p->seq_len;
  if (rows > B200_ATTN_STATIC_LSE_MAX_ROWS) {
    set_error("batch * heads * seq_len exceeds B200_ATTN_STATIC_LSE_MAX_ROWS");
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  }
  CUtensorMap maps[4];
  PartialKernelArgs a;
  int dev = 0;
  DeviceGuard guard;
  rc = prepare(p, maps, a, dev, guard);  // leaves `dev` current until return
  if (rc != B200_ATTN_OK) return rc;
  StaticLseState& st = g_static_lse[dev];
  std::call_once(st.resolved, [&st] {
    st.err = cudaGetSymbolAddress(reinterpret_cast<void**>(&st.ptr), b200_static_lse);
    if (st.err != cudaSuccess) {
      cudaGetLastError();
      st.ptr = nullptr;
    }
  });
  if (st.err != cudaSuccess || !st.ptr) {
    set_error(st.err != cudaSuccess ? cudaGetErrorString(st.err)
                                    : "no device address for the static log-sum-exp array");
    return B200_ATTN_ERR_DEVICE;
  }
  if (accumulate) {
    std::lock_guard<std::mutex> lk(st.mu);
    if (st.shape[0] != p->batch || st.shape[1] != p->heads || st.shape[2] != p->seq_len) {
      set_error("accumulating call without a first-chunk call of the same shape on this device");
      return B200_ATTN_ERR_INVALID_ARGUMENT;
    }
  }
  a.lse = st.ptr;
  a.lse_sb = p->heads * p->seq_len;
  a.lse_sh = p->seq_len;
  a.lse_ss = 1;
  a.accumulate = accumulate;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool c = p->causal != 0;
  switch (p->dtype) {
    case B200_ATTN_DTYPE_FP32:
      rc = dispatch_partial<CfgF32, B200_ATTN_DTYPE_FP32>(maps, a, c, dev, s);
      break;
    case B200_ATTN_DTYPE_FP16:
      rc = wide_head(p->head_dim) ? dispatch_partial<Cfg128, B200_ATTN_DTYPE_FP16>(maps, a, c, dev, s)
                                  : dispatch_partial<Cfg64, B200_ATTN_DTYPE_FP16>(maps, a, c, dev, s);
      break;
    default:
      rc = wide_head(p->head_dim) ? dispatch_partial<Cfg128, B200_ATTN_DTYPE_BF16>(maps, a, c, dev, s)
                                  : dispatch_partial<Cfg64, B200_ATTN_DTYPE_BF16>(maps, a, c, dev, s);
      break;
  }
  if (rc == B200_ATTN_OK && !accumulate) {
    std::lock_guard<std::mutex> lk(st.mu);
    st.shape[0] = p->batch;
    st.shape[1] = p->heads;
    st.shape[2] = p->seq_len;
  }
  return rc;
}
