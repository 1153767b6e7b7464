// attn_fwd_sm100.cu — fused attention forward for B200 (sm_100a).
//
// Value definition: the reference's _reference_attention
// (model/triton_fused_attention.py:1256-1285): scores = q k^T * scale, causal
// triu(1) and key-padding positions set to -inf, fp32 softmax, probabilities in
// the input dtype, times v.  Fully masked rows give NaN like torch.softmax.
//
// Work decomposition.  One CTA owns 256 query rows of one (batch, head) as two
// 128-row tiles Q0, Q1 and streams 128-key K/V tiles through a shared-memory
// ring.  Ten warps, each with one job:
//   warps 0-3  softmax for Q0 (one thread per query row = one TMEM lane)
//   warps 4-7  softmax for Q1
//   warp  8    TMA producer (Q once, then K_j, V_j into the ring)
//   warp  9    tcgen05 issuer (one elected thread) and TMEM owner
// Tensor memory (512 columns x 128 lanes, fp32 cells):
//   [0,128)   S0 = Q0 K_j^T      (P0 as packed 16-bit pairs in [64,128))
//   [128,256) S1 = Q1 K_j^T      (P1 in [192,256))
//   [256,256+D) O0, [256+D,256+2D) O1  (fp32 accumulators)
// MMA issue order per key tile j: PV0(j-1), QK0(j), PV1(j-1), QK1(j), so the
// tensor core works on one query tile while the other tile's softmax runs.
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
#include <cstring>
#include <mutex>

#include "b200_attn.h"
#include "sm100_ptx.cuh"

namespace b200attn {

constexpr int kBlockM = 128;         // query rows per tile = TMEM lanes
constexpr int kBlockN = 128;         // keys per K/V tile
constexpr int kRowsPerCta = 2 * kBlockM;
constexpr int kSoftmaxWarps = 8;
constexpr int kLoadWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 320;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleLog2 = 8.0f;  // rescale O when the max grows by > 2^8
constexpr uint64_t kWaitTimeoutNs = 1000000000ull;
constexpr float kLog2e = 1.4426950408889634f;
#ifndef B200_ATTN_POLY_PER8
#define B200_ATTN_POLY_PER8 0
#endif
// Of every 8 probabilities, this many are computed with the FMA-pipe exp2.
constexpr int kPolyPer8 = B200_ATTN_POLY_PER8;

struct KernelArgs {
  int32_t seq_len;
  int32_t heads;
  int32_t batch;
  int32_t num_q_blocks;  // ceil(S / 256)
  float scale;           // softmax scale
  float scale_log2;      // scale * log2(e)
  int32_t zero_masked_queries;
  const uint8_t* mask;   // [B,S] bool or null
  int64_t mask_sb;       // bytes
  int64_t mask_ss;
  void* o;               // output base (for zero rows of skipped blocks)
  int64_t o_sb, o_sh, o_ss;  // elements
  int32_t* err;
};

template <int D, int NSLOT>
struct Cfg {
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static constexpr int kChunks = D / 64;               // 128-byte swizzle chunks per row
  static constexpr int kChunkBytes = kBlockM * 128;    // one chunk of a 128-row tile
  static constexpr int kTileBytes = kBlockM * D * 2;   // Q, K or V tile
  static constexpr int kOffQ = 0;
  static constexpr int kOffRing = 2 * kTileBytes;
  static constexpr int kOffBar = kOffRing + NSLOT * kTileBytes;
  // q_full, slot_full[NSLOT], slot_empty[NSLOT], s_full[2], p_full[2], o_full[2], drain
  static constexpr int kNumBars = 1 + 2 * NSLOT + 7;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kSmemBytes = kOffMisc + 16 + 1024;  // + alignment slack
  // TMEM column of S_i (P_i lives in its upper 64 columns) and of O_i
  __host__ __device__ static constexpr uint32_t col_s(int i) { return 128u * i; }
  __host__ __device__ static constexpr uint32_t col_o(int i) { return 256u + D * i; }
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

__device__ __forceinline__ int warp_max_i(int v) {
#pragma unroll
  for (int off = 16; off; off >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

// x rounded to the input dtype and widened back to fp32.
template <bool BF16>
__device__ __forceinline__ float round_to_input(float x) {
  if constexpr (BF16) {
    return __bfloat162float(__float2bfloat16_rn(x));
  } else {
    return __half2float(__float2half_rn(x));
  }
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

// Bounded wait on an mbarrier phase.  Returns false when the CTA was aborted
// (by this thread's timeout or another's).
__device__ __noinline__ bool wait_bar_slow(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag,
                                      int32_t* err) {
  const uint64_t t0 = ptx::globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int k = 0; k < 32; ++k)
      if (ptx::mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (ptx::globaltimer_ns() - t0 > kWaitTimeoutNs) {
      *abort_flag = 1u;
      if (err) atomicOr(err, B200_ATTN_DEVERR_WAIT_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity,
                                         volatile uint32_t* abort_flag, int32_t* err) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  return wait_bar_slow(bar, parity, abort_flag, err);
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

// ----------------------------------------------------------------- kernel
template <int D, int NSLOT, bool kCausal, bool kMask, bool kBF16>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                          const __grid_constant__ CUtensorMap tm_k,
                          const __grid_constant__ CUtensorMap tm_v,
                          const __grid_constant__ CUtensorMap tm_o, const KernelArgs args) {
  using C = Cfg<D, NSLOT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = ptx::smem_u32(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int S = args.seq_len;

  // Heaviest query blocks (causal) are launched first across all heads.
  const int bh_count = args.batch * args.heads;
  const int qb = args.num_q_blocks - 1 - static_cast<int>(blockIdx.x) / bh_count;
  const int bh = static_cast<int>(blockIdx.x) % bh_count;
  const int b = bh / args.heads;
  const int h = bh % args.heads;
  const int q0 = qb * kRowsPerCta;

  volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(smem + C::kOffMisc);
  // misc[0] TMEM base, misc[1] abort flag, misc[2] key extent
  volatile uint32_t* abort_flag = misc + 1;
  const uint32_t bar_base = sbase + C::kOffBar;
  const uint32_t bar_q = bar_base;
  auto slot_full = [&](uint32_t s) { return bar_base + 8u * (1u + s); };
  auto slot_empty = [&](uint32_t s) { return bar_base + 8u * (1u + NSLOT + s); };
  auto s_full = [&](int i) { return bar_base + 8u * (1u + 2u * NSLOT + i); };
  auto p_full = [&](int i) { return bar_base + 8u * (3u + 2u * NSLOT + i); };
  auto o_full = [&](int i) { return bar_base + 8u * (5u + 2u * NSLOT + i); };
  const uint32_t bar_drain = bar_base + 8u * (7u + 2u * NSLOT);

  const uint8_t* mrow = nullptr;
  if constexpr (kMask) mrow = args.mask + static_cast<int64_t>(b) * args.mask_sb;

  // ---------------------------------------------------------- prologue
  if (warp == kLoadWarp) {
    int extent = S;
    if constexpr (kMask) extent = mask_extent(mrow, args.mask_ss, S, lane);
    if (lane == 0) {
      misc[1] = 0u;
      misc[2] = static_cast<uint32_t>(extent);
      ptx::mbar_init(bar_q, 1);
      for (int s = 0; s < NSLOT; ++s) {
        ptx::mbar_init(slot_full(s), 1);
        ptx::mbar_init(slot_empty(s), 1);
      }
      for (int i = 0; i < 2; ++i) {
        ptx::mbar_init(s_full(i), 1);
        ptx::mbar_init(p_full(i), kBlockM);
        ptx::mbar_init(o_full(i), 1);
      }
      ptx::mbar_init(bar_drain, 1);
      ptx::fence_mbar_init();
      ptx::fence_proxy_async_smem();
      ptx::tma_prefetch_desc(&tm_q);
      ptx::tma_prefetch_desc(&tm_k);
      ptx::tma_prefetch_desc(&tm_v);
      ptx::tma_prefetch_desc(&tm_o);
    }
  }
  __syncthreads();
  const int extent = static_cast<int>(misc[2]);

  // A block whose rows all lie at or past the last valid key has only masked
  // query rows: with zero_masked_queries its output is all zeros.
  if (kMask && args.zero_masked_queries && q0 >= extent) {
    if (warp < kSoftmaxWarps) {
      const int row = q0 + threadIdx.x;
      if (row < S) {
        uint4* dst = reinterpret_cast<uint4*>(
            reinterpret_cast<uint16_t*>(args.o) + static_cast<int64_t>(b) * args.o_sb +
            static_cast<int64_t>(h) * args.o_sh + static_cast<int64_t>(row) * args.o_ss);
#pragma unroll
        for (int c = 0; c < D / 8; ++c) dst[c] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    return;
  }

  if (warp == kMmaWarp) {
    ptx::tmem_alloc(sbase + C::kOffMisc, kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = misc[0];

  // Key tiles each query tile visits.
  const int n_kv = kMask ? max(1, (extent + kBlockN - 1) / kBlockN) : (S + kBlockN - 1) / kBlockN;
  int n_tiles[2];
#pragma unroll
  for (int i = 0; i < 2; ++i)
    n_tiles[i] = kCausal ? min(2 * qb + i + 1, n_kv) : n_kv;
  const int n_max = n_tiles[1];  // Q1 never needs fewer tiles than Q0

  if (warp == kLoadWarp) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      ptx::mbar_arrive_expect_tx(bar_q, 2u * C::kTileBytes);
#pragma unroll
      for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int c = 0; c < C::kChunks; ++c)
          ptx::tma_load_4d(sbase + C::kOffQ + i * C::kTileBytes + c * C::kChunkBytes, &tm_q, bar_q,
                           64 * c, q0 + kBlockM * i, h, b);
      uint32_t L = 0;
      bool ok = true;
      for (int j = 0; ok && j < n_max; ++j) {
        for (int kv = 0; kv < 2; ++kv) {
          const uint32_t s = L % NSLOT, r = L / NSLOT;
          if (!wait_bar(slot_empty(s), (r & 1u) ^ 1u, abort_flag, args.err)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_expect_tx(slot_full(s), C::kTileBytes);
          const CUtensorMap* tm = kv ? &tm_v : &tm_k;
#pragma unroll
          for (int c = 0; c < C::kChunks; ++c)
            ptx::tma_load_4d(sbase + C::kOffRing + s * C::kTileBytes + c * C::kChunkBytes, tm,
                             slot_full(s), 64 * c, kBlockN * j, h, b);
          ++L;
        }
      }
      if (!ok) {
        // Let copies already issued land before the CTA's shared memory goes away.
        const uint32_t first = L > NSLOT ? L - NSLOT : 0u;
        for (uint32_t x = first; x < L; ++x) {
          const uint64_t t0 = ptx::globaltimer_ns();
          while (!ptx::mbar_try_wait(slot_full(x % NSLOT), (x / NSLOT) & 1u) &&
                 ptx::globaltimer_ns() - t0 < kWaitTimeoutNs) {
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------ tcgen05 issuer
    if (lane == 0) {
      constexpr uint32_t id_qk = ptx::idesc_f16(kBF16, kBlockM, kBlockN, false);
      constexpr uint32_t id_pv = ptx::idesc_f16(kBF16, kBlockM, D, true);
      bool ok = wait_bar(bar_q, 0, abort_flag, args.err);
      for (int j = 0; ok && j <= n_max; ++j) {
        const uint32_t kL = 2u * j, vL = 2u * j - 1u;  // K(j), V(j-1) load indices
        const uint32_t ks = kL % NSLOT, vs = vL % NSLOT;
        if (j < n_max && !wait_bar(slot_full(ks), (kL / NSLOT) & 1u, abort_flag, args.err)) {
          ok = false;
          break;
        }
        if (j >= 1 && !wait_bar(slot_full(vs), (vL / NSLOT) & 1u, abort_flag, args.err)) {
          ok = false;
          break;
        }
        ptx::tc_fence_after();
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          if (j >= 1 && j - 1 < n_tiles[i]) {
            // O_i += P_i(j-1) V(j-1): A = P from TMEM, B = V (MN-major, D contiguous)
            if (!wait_bar(p_full(i), (j - 1) & 1, abort_flag, args.err)) {
              ok = false;
              break;
            }
            ptx::tc_fence_after();
            const uint32_t vaddr = sbase + C::kOffRing + vs * C::kTileBytes;
#pragma unroll
            for (int kk = 0; kk < kBlockN / 16; ++kk) {
              const uint64_t bdesc = ptx::smem_desc_sw128(vaddr + kk * 2048, C::kChunkBytes, 1024);
              ptx::tc_mma_ts(tmem + C::col_o(i), tmem + C::col_s(i) + 64 + kk * 8, bdesc, id_pv,
                             (j > 1 || kk > 0) ? 1u : 0u);
            }
            if (j - 1 == n_tiles[i] - 1) ptx::tc_commit(o_full(i));
            if (i == 1) ptx::tc_commit(slot_empty(vs));
          }
          if (j < n_tiles[i]) {
            // S_i = Q_i K(j)^T: A = Q (K-major), B = K (K-major)
            const uint32_t qaddr = sbase + C::kOffQ + i * C::kTileBytes;
            const uint32_t kaddr = sbase + C::kOffRing + ks * C::kTileBytes;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = (kk >> 2) * C::kChunkBytes + (kk & 3) * 32;
              ptx::tc_mma_ss(tmem + C::col_s(i), ptx::smem_desc_sw128(qaddr + off, 16, 1024),
                             ptx::smem_desc_sw128(kaddr + off, 16, 1024), id_qk, kk > 0 ? 1u : 0u);
            }
            ptx::tc_commit(s_full(i));
            if (i == 1) ptx::tc_commit(slot_empty(ks));
          }
        }
      }
      // Drain: every MMA this thread issued completes before TMEM is freed.
      ptx::tc_commit(bar_drain);
      const uint64_t t0 = ptx::globaltimer_ns();
      while (!ptx::mbar_try_wait(bar_drain, 0) && ptx::globaltimer_ns() - t0 < kWaitTimeoutNs) {
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    const int i = warp >> 2;                 // query tile
    const int quad = warp & 3;               // TMEM lane quadrant of this warp
    const int rl = quad * 32 + lane;         // row within the tile = TMEM lane
    const int row = q0 + kBlockM * i + rl;   // global query row
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + lane_off + C::col_s(i);
    const uint32_t tP = tS + 64;
    const uint32_t tO = tmem + lane_off + C::col_o(i);
    const float scale_log2 = args.scale_log2;
    const int n = n_tiles[i];
    const int diag = kCausal ? 2 * qb + i : -1;

    float m_run = -INFINITY;
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int key0 = j * kBlockN;
      uint32_t mw[4] = {~0u, ~0u, ~0u, ~0u};
      uint8_t mb[4] = {1, 1, 1, 1};
      if constexpr (kMask) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int key = key0 + 32 * q + lane;
          mb[q] = key < S ? mrow[static_cast<int64_t>(key) * args.mask_ss] : uint8_t(0);
        }
      }
      if (!warp_wait_bar(s_full(i), j & 1, abort_flag, args.err)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      uint32_t sr[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) ptx::tmem_ld_32x32b_x32(tS + 32 * c, sr[c]);
      ptx::tmem_wait_ld();

      const bool edge = (key0 + kBlockN > S);
      bool partial = edge || (kCausal && j == diag);
      if constexpr (kMask) {
#pragma unroll
        for (int q = 0; q < 4; ++q) mw[q] = __ballot_sync(0xffffffffu, mb[q] != 0);
        partial = partial || ((mw[0] & mw[1] & mw[2] & mw[3]) != ~0u);
      }
      if (partial) {
        int lim = S - 1 - key0;  // last in-range key of this tile
        if (kCausal && j == diag) lim = min(lim, rl);
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int k = 32 * c + e;
            const bool vis = (k <= lim) && (((mw[c] >> e) & 1u) != 0u);
            if (!vis) sr[c][e] = __float_as_uint(-INFINITY);
          }
      }

      if (n == 1) {
        // Every visible key of this query tile lies in this one key tile, so
        // the row sum is complete here: reproduce the reference's rounding
        // points exactly (model/triton_fused_attention.py:1272-1284): scores
        // rounded to the input dtype, the scale multiply rounded again, fp32
        // softmax normalised before P is rounded.  Rows with few keys (early
        // causal rows, short or heavily padded sequences) have large outputs,
        // where a different rounding order would show as whole output ulps.
        const float scale = args.scale;
        float cmx[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float m4 = -INFINITY;
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float v = round_to_input<kBF16>(round_to_input<kBF16>(__uint_as_float(sr[c][e])) * scale);
            sr[c][e] = __float_as_uint(v);
            m4 = fmaxf(m4, v);
          }
          cmx[c] = m4;
        }
        const float mx2 = fmaxf(fmaxf(cmx[0], cmx[1]), fmaxf(cmx[2], cmx[3]));
        const float sub = (mx2 == -INFINITY) ? 0.f : mx2;
        float tot = 0.f;
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const float pe = expf(__uint_as_float(sr[c][e]) - sub);
            sr[c][e] = __float_as_uint(pe);
            tot += pe;
          }
        const float inv = 1.f / tot;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e)
            pk[e] = pack2<kBF16>(__uint_as_float(sr[c][2 * e]) * inv,
                                 __uint_as_float(sr[c][2 * e + 1]) * inv);
#pragma unroll
          for (int e = 0; e < 16; ++e) sr[c >> 1][16 * (c & 1) + e] = pk[e];
          if (c & 1) ptx::tmem_st_32x32b_x32(tP + 32 * (c >> 1), sr[c >> 1]);
        }
        m_run = mx2;  // -inf only when the row has no visible key (NaN output)
        l_run = 1.f;  // P is already normalised
        ptx::tmem_wait_st();
        ptx::tc_fence_before();
        ptx::mbar_arrive(p_full(i));
        continue;
      }

      // Row max: a 3-input max tree (depth 5) instead of a 128-long chain.
      float cm[4];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float v[11];
#pragma unroll
        for (int t = 0; t < 10; ++t)
          v[t] = fmax3(__uint_as_float(sr[c][3 * t]), __uint_as_float(sr[c][3 * t + 1]),
                       __uint_as_float(sr[c][3 * t + 2]));
        v[10] = fmaxf(__uint_as_float(sr[c][30]), __uint_as_float(sr[c][31]));
        cm[c] = fmax3(fmax3(v[0], v[1], v[2]), fmax3(v[3], v[4], v[5]),
                      fmax3(v[6], v[7], fmax3(v[8], v[9], v[10])));
      }
      const float mx = fmaxf(fmaxf(cm[0], cm[1]), fmaxf(cm[2], cm[3]));
      const float m_cand = mx * scale_log2;
      const bool resc = m_cand > m_run + kRescaleLog2;
      const float m_new = resc ? m_cand : m_run;
      const float alpha = resc ? ptx::ex2_approx(m_run - m_new) : 1.f;
      l_run *= alpha;
      m_run = m_new;
      const float neg_m = (m_run == -INFINITY) ? 0.f : -m_run;

      // p = 2^(s*scale*log2e - m): most elements on the MUFU (ex2.approx),
      // kPolyPer8 of every 8 on the FMA pipe (ex2_poly), which balances the
      // two pipes; four independent partial sums.
      float sum[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float p2[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int k = 2 * e + h;
            const float x = fmaf(__uint_as_float(sr[c][k]), scale_log2, neg_m);
            p2[h] = ((k & 7) < kPolyPer8) ? ex2_poly(fmaxf(x, -126.f)) : ptx::ex2_approx(x);
          }
          sum[e & 3] += p2[0] + p2[1];
          pk[e] = pack2<kBF16>(p2[0], p2[1]);
        }
        // pack two 16-column groups into one 32-column store
#pragma unroll
        for (int e = 0; e < 16; ++e) sr[c >> 1][16 * (c & 1) + e] = pk[e];
        if (c & 1) ptx::tmem_st_32x32b_x32(tP + 32 * (c >> 1), sr[c >> 1]);
      }
      l_run += (sum[0] + sum[1]) + (sum[2] + sum[3]);

      if (j > 0 && __any_sync(0xffffffffu, resc)) {
        // O_i holds sum over tiles < j (its last MMA completed before S_i(j)).
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
      ptx::tmem_wait_st();
      ptx::tc_fence_before();
      ptx::mbar_arrive(p_full(i));
    }

    // ------------------------------------------------------------ epilogue
    if (ok) ok = warp_wait_bar(o_full(i), 0, abort_flag, args.err);
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
      const float inv_l = zero_row ? 0.f : (m_run == -INFINITY ? __int_as_float(0x7fc00000) : 1.f / l_run);
      const uint32_t stage = sbase + C::kOffQ + i * C::kTileBytes;  // Q_i is no longer read
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        ptx::tmem_ld_32x32b_x32(tO + 32 * c, o);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float a = __uint_as_float(o[8 * u + 2 * e]) * inv_l;
            float bb = __uint_as_float(o[8 * u + 2 * e + 1]) * inv_l;
            if (zero_row) a = bb = 0.f;
            w[e] = pack2<kBF16>(a, bb);
          }
          const int col = 32 * c + 8 * u;           // first element of this 16-byte chunk
          const int cb = col >> 6;                  // 64-column block
          const int lc = (col & 63) >> 3;           // logical 16-byte chunk within the row
          const uint32_t addr = stage + cb * C::kChunkBytes + rl * 128 + ((lc ^ (rl & 7)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w[0]),
                       "r"(w[1]), "r"(w[2]), "r"(w[3])
                       : "memory");
        }
      }
      ptx::fence_proxy_async_smem();
      ptx::named_barrier_sync(1 + i, kBlockM);
      if (rl == 0 && q0 + kBlockM * i < S) {
#pragma unroll
        for (int cb = 0; cb < C::kChunks; ++cb)
          ptx::tma_store_4d(&tm_o, stage + cb * C::kChunkBytes, 64 * cb, q0 + kBlockM * i, h, b);
        ptx::bulk_commit_group();
        ptx::bulk_wait_group_all();
      }
    }
  }

  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------- host
namespace {

thread_local char g_last_error[256] = {0};

void set_error(const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
}

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

bool supported_head_dim(int64_t d) { return d == 64 || d == 128; }

// Alignment rules of the 4-D TMA view {D, S, H, B}: 16-byte base, 16-byte
// multiples for every stride whose dimension has extent > 1.
bool tensor_aligned(const void* ptr, const int64_t st[3], const b200_attn_fwd_params* p) {
  if (reinterpret_cast<uintptr_t>(ptr) & 15u) return false;
  const int64_t ext[3] = {p->batch, p->heads, p->seq_len};
  for (int a = 0; a < 3; ++a) {
    if (ext[a] <= 1) continue;
    if (st[a] <= 0) return false;
    if ((st[a] * 2) % 16 != 0) return false;
  }
  return true;
}

int encode_map(CUtensorMap* m, const void* ptr, const int64_t st[3],
               const b200_attn_fwd_params* p) {
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled entry point unavailable");
    return B200_ATTN_ERR_LAUNCH;
  }
  const int64_t D = p->head_dim, S = p->seq_len, H = p->heads, B = p->batch;
  // Size-1 dimensions never move the address; give them a legal stride.
  const int64_t fill = D * 2 * 16;
  int64_t s_seq = S > 1 ? st[2] * 2 : fill;
  int64_t s_head = H > 1 ? st[1] * 2 : fill;
  int64_t s_batch = B > 1 ? st[0] * 2 : fill;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S),
                        static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(s_seq), static_cast<cuuint64_t>(s_head),
                           static_cast<cuuint64_t>(s_batch)};
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(kBlockM), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt =
      p->dtype == B200_ATTN_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(m, dt, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
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

template <int D, int NSLOT, bool C, bool M, bool BF>
int launch_one(const CUtensorMap maps[4], const KernelArgs& args, int device, cudaStream_t stream) {
  using Cf = Cfg<D, NSLOT>;
  auto kernel = attn_fwd_sm100_kernel<D, NSLOT, C, M, BF>;
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
  kernel<<<grid, kThreads, Cf::kSmemBytes, stream>>>(maps[0], maps[1], maps[2], maps[3], args);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error(cudaGetErrorString(e));
    return B200_ATTN_ERR_LAUNCH;
  }
  return B200_ATTN_OK;
}

template <int D, int NSLOT>
int dispatch_flags(const CUtensorMap maps[4], const KernelArgs& a, const b200_attn_fwd_params* p,
                   int dev, cudaStream_t s) {
  const bool c = p->causal != 0, m = p->key_mask != nullptr, bf = p->dtype == B200_ATTN_DTYPE_BF16;
  if (c) {
    if (m) return bf ? launch_one<D, NSLOT, true, true, true>(maps, a, dev, s)
                     : launch_one<D, NSLOT, true, true, false>(maps, a, dev, s);
    return bf ? launch_one<D, NSLOT, true, false, true>(maps, a, dev, s)
              : launch_one<D, NSLOT, true, false, false>(maps, a, dev, s);
  }
  if (m) return bf ? launch_one<D, NSLOT, false, true, true>(maps, a, dev, s)
                   : launch_one<D, NSLOT, false, true, false>(maps, a, dev, s);
  return bf ? launch_one<D, NSLOT, false, false, true>(maps, a, dev, s)
            : launch_one<D, NSLOT, false, false, false>(maps, a, dev, s);
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
  if (dtype != B200_ATTN_DTYPE_BF16 && dtype != B200_ATTN_DTYPE_FP16) return 0;
  return supported_head_dim(head_dim) ? 1 : 0;
}

extern "C" const char* b200_attn_error_string(int32_t code) {
  switch (code) {
    case B200_ATTN_OK: return "ok";
    case B200_ATTN_ERR_INVALID_ARGUMENT: return "invalid argument";
    case B200_ATTN_ERR_UNSUPPORTED: return "unsupported dtype or head_dim";
    case B200_ATTN_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
    case B200_ATTN_ERR_DEVICE: return "no sm_100 device for the given pointers";
    case B200_ATTN_ERR_LAUNCH: return "kernel launch failed";
    case B200_ATTN_ERR_TIMEOUT: return "device pipeline wait timed out";
    default: return "unknown error";
  }
}

extern "C" const char* b200_attn_last_error_detail(void) { return g_last_error; }

extern "C" int32_t b200_attn_check(const b200_attn_fwd_params* p) {
  if (!p || !p->q || !p->k || !p->v || !p->o) return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->batch < 1 || p->heads < 1 || p->seq_len < 1 || p->head_dim < 1)
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->batch * p->heads > (1ll << 24) || p->seq_len > (1ll << 30))
    return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (!(p->scale > 0.f) || !std::isfinite(p->scale)) return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (p->dtype != B200_ATTN_DTYPE_BF16 && p->dtype != B200_ATTN_DTYPE_FP16)
    return B200_ATTN_ERR_UNSUPPORTED;
  if (!supported_head_dim(p->head_dim)) return B200_ATTN_ERR_UNSUPPORTED;
  if (p->zero_masked_queries && !p->key_mask) return B200_ATTN_ERR_INVALID_ARGUMENT;
  if (!tensor_aligned(p->q, p->q_stride, p) || !tensor_aligned(p->k, p->k_stride, p) ||
      !tensor_aligned(p->v, p->v_stride, p) || !tensor_aligned(p->o, p->o_stride, p))
    return B200_ATTN_ERR_ALIGNMENT;
  return B200_ATTN_OK;
}

extern "C" int32_t b200_attn_launches_per_call(const b200_attn_fwd_params* p) {
  return b200_attn_check(p) == B200_ATTN_OK ? 1 : 0;
}

extern "C" int32_t b200_attn_fwd(const b200_attn_fwd_params* p, void* stream) {
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

  CUtensorMap maps[4];
  const void* ptrs[4] = {p->q, p->k, p->v, p->o};
  const int64_t* strides[4] = {p->q_stride, p->k_stride, p->v_stride, p->o_stride};
  for (int t = 0; t < 4; ++t)
    if ((rc = encode_map(&maps[t], ptrs[t], strides[t], p)) != B200_ATTN_OK) return rc;

  KernelArgs a;
  a.seq_len = static_cast<int32_t>(p->seq_len);
  a.heads = static_cast<int32_t>(p->heads);
  a.batch = static_cast<int32_t>(p->batch);
  a.num_q_blocks = static_cast<int32_t>((p->seq_len + kRowsPerCta - 1) / kRowsPerCta);
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
  a.err = p->error_word;
  if (static_cast<int64_t>(a.num_q_blocks) * p->batch * p->heads > 0x7fffffffll)
    return B200_ATTN_ERR_INVALID_ARGUMENT;

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (p->head_dim == 128) return dispatch_flags<128, 4>(maps, a, p, dev, s);
  return dispatch_flags<64, 6>(maps, a, p, dev, s);
}
