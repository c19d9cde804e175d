// Flash-attention backward on the 5th-generation tensor cores (sm_100a), as two kernels so that no
// partial gradient is ever accumulated with atomics.
//
// dK/dV kernel -- CTA = one 128-key block j of one KV head (all query heads of its GQA group); for
// every visible 128-query block i:
//   S^T  = K_j Q_i^T                 (SS MMA, keys on TMEM lanes, fp32, cols [0,128))
//   dP^T = V_j dO_i^T                (SS MMA, cols [128,256))
//   P^T  = exp2(S^T c - lse_i)       (compute warps: thread = key row; bf16 over S^T cols [0,64))
//   dS^T = P^T (dP^T - D_i) * scale  (bf16 over dP^T cols [128,192))
//   dV  += P^T dO_i, dK += dS^T Q_i  (TS MMAs: A from TMEM, B = dO_i / Q_i MN-major from smem)
// dK and dV leave TMEM once, after the last block.
//
// dQ kernel -- CTA = one 128-query block i of one head; for every visible 128-key block j:
//   S = Q_i K_j^T, dP = dO_i V_j^T  (S double-buffered in TMEM so the next block's S overlaps)
//   dS = P (dP - D_i) * scale       (thread = query row; bf16 over the S columns)
//   dQ += dS K_j                     (TS MMA: A = dS from TMEM, B = K_j MN-major)
// dQ leaves TMEM once, as bf16.
//
// Warps (both kernels): 0-7 compute (warp w: TMEM lanes 32 (w % 4).., column half w / 4), 8 MMA (one
// elected thread), 9 TMA (+ per-query scalars in the dK/dV kernel). Blocks that need no mask take a
// branch-free path. Every wait is bounded and records an error code on timeout.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include "kernels.h"
#include "sm100_primitives.cuh"

namespace mxk {
namespace fab100 {

constexpr int BM = 128;  // queries per block
constexpr int BN = 128;  // keys per CTA
// Both kernels: warps 0-15 compute (warp w: TMEM lanes 32 (w % 4).., block columns 32 (w / 4)..),
// 16 MMA, 17 TMA. Four compute warps per SM sub-partition hide the latency of each warp's
// dependent exp / scale / pack chain.
constexpr int kThreadsKV = 576;
constexpr int kMmaWarpKV = 16, kTmaWarpKV = 17;

struct BwdArgs {
  int B, S, H, Hkv, window;
  float scale, scale_log2;
  const int* seg;
  const float* lse;   // [T, H] natural-log logsumexp of the forward
  const float* dsum;  // [T, H] rowsum(dO * O)
  __nv_bfloat16* dq;  // [T, H, HD]
  __nv_bfloat16* dk;
  long dk_tok, dk_head;
  __nv_bfloat16* dv;
  long dv_tok, dv_head;
  int dv_accumulate;
  int* err;
  // Optional phase counters of the dK/dV kernel (cycles summed over warps / CTAs), else null:
  // compute warps: [0] waiting for S^T / dP^T, [1] TMEM loads, [2] math, [3] TMEM stores + release,
  // [4] blocks; MMA thread: [5] waiting for P^T / dS^T, [6] waiting for its own MMAs, [7] waiting
  // for Q / dO, [8] MMA loop total, [9] CTA total, [10] dK / dV write-out; TMA warp: [11] waiting
  // for a free Q / dO buffer, [12] issuing loads and staging the per-query scalars.
  unsigned long long* prof;
};

// A [128 rows x HD] bf16 operand tile as stored by the dK/dV kernel: head-dim columns 0-63 as one
// chunk in the 128-byte swizzle (rows of 128 B), then columns 64..HD-1 -- 32 of them for HD = 96,
// in the 64-byte swizzle (rows of 64 B), so the tile is not padded to 128 columns (24 KB instead of
// 32 KB for HD = 96), or 64 for HD = 128 in the 128-byte swizzle.
template <int HD, bool UNPAD = true>
struct TileFmt {
  // columns of the second chunk: 0, 32 or 64 (UNPAD = false pads HD = 96 to a second 64-column chunk)
  static constexpr int W1 = UNPAD || HD <= 64 ? HD - 64 : 64;
  static constexpr int P1 = 2 * W1;   // its row pitch in bytes
  static constexpr int kC0 = 128 * 128;
  static constexpr int kBytes = kC0 + 128 * P1;
  static constexpr uint32_t kLay1 = W1 == 32 ? 4u : 2u;  // descriptor layout of the second chunk
  static constexpr bool kNarrow = W1 == 32;
  // K-major descriptor of k-step ks (head-dim columns 16 ks..) for the rows from `row`
  static __device__ __forceinline__ uint64_t kmaj(uint32_t base, int ks, int row) {
    if (ks < 4) return make_sdesc(base + row * 128 + ks * 32, 16, 1024);
    return make_sdesc_l(base + kC0 + row * P1 + (ks - 4) * 32, 16, 8 * P1, kLay1);
  }
  // MN-major descriptor (head dim = N) of K rows [16 kr, 16 kr + 16): the whole tile as one operand
  // (N = HD, chunks at a 16 KB stride) when both chunks share the 128-byte swizzle, else chunk c
  static __device__ __forceinline__ uint64_t mnmaj(uint32_t base, int c, int kr) {
    if (c == 0) return make_sdesc(base + kr * 2048, kC0, 1024);
    return make_sdesc_l(base + kC0 + kr * 16 * P1, 128 * P1, 8 * P1, kLay1);
  }
};

template <int HD, bool UNPAD = true>
struct Smem {
  static constexpr int KCH = (HD + 63) / 64;
  static constexpr int kTile = TileFmt<HD, UNPAD>::kBytes;
  // Q / dO stages: three when they fit beside K and V (unpadded HD = 96 tiles: 8 x 24 KB)
  static constexpr int NQ = (2 + 6) * kTile + 3 * BM * 12 + 256 <= 227 * 1024 - 128 ? 3 : 2;
  // K, V, Q[NQ], dO[NQ], then per-query scalars and barriers. The tiles need 1024-byte alignment;
  // the dynamic shared memory base is expected to have it (the kernel checks and reports otherwise).
  static constexpr int kScal = NQ * BM * 12;  // [NQ buffers] x 128 x (lse2 f32, dsum f32, key-lo i32)
  static constexpr int kBars = 256;
  static constexpr int kUsed = (2 + 2 * NQ) * kTile + kScal + kBars;
  static constexpr int kBytes = kUsed + 128;
};

// TMEM columns of the dK/dV kernel
constexpr uint32_t kColS = 0, kColDP = 128;
template <int HD>
struct Cols {
  static constexpr uint32_t dV = 256;
  static constexpr uint32_t dK = 256 + HD;
};

// 2^x on the special-function unit (PTX ex2.approx.ftz.f32; -inf -> +0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// First key visible to query qi (window / segment start), and whether qi is a real position.
__device__ __forceinline__ int query_key_lo(int qi, int S, int window, const int* seg, int base) {
  if (qi >= S) return 1 << 30;
  int lo = 0;
  if (window > 0) lo = max(lo, qi - window + 1);
  if (seg) {
    const int sid = seg[base + qi];
    int a = 0, b = qi;
    while (a < b) {
      const int m = (a + b) >> 1;
      if (seg[base + m] == sid) b = m; else a = m + 1;
    }
    lo = max(lo, a);
  }
  return lo;
}

template <int HD, bool UNPAD>
__global__ void __launch_bounds__(kThreadsKV, 1)
    fa_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                        const __grid_constant__ CUtensorMap tmQn, const __grid_constant__ CUtensorMap tmKn,
                        const __grid_constant__ CUtensorMap tmVn, const __grid_constant__ CUtensorMap tmOn,
                        const BwdArgs a) {
  // tm*: 64-column boxes in the 128-byte swizzle; tm*n: 32-column boxes in the 64-byte swizzle
  // (the second chunk of an HD = 96 tile)
  using SM = Smem<HD, UNPAD>;
  using C = Cols<HD>;
  using TF = TileFmt<HD, UNPAD>;
  constexpr int NQ = SM::NQ;
  constexpr uint32_t tile = SM::kTile;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  if (pad + SM::kUsed > SM::kBytes) {  // misaligned base: report instead of overrunning shared memory
    if (threadIdx.x == 0) atomicExch(a.err, kErrBadArgs);
    return;
  }
  uint8_t* smem = smem_raw + pad;
  uint8_t* sK = smem;
  uint8_t* sV = smem + tile;
  uint8_t* sQ = smem + 2 * tile;         // [NQ]
  uint8_t* sO = smem + (2 + NQ) * tile;  // [NQ] (dO)
  float* sLse = reinterpret_cast<float*>(smem + (2 + 2 * NQ) * tile);  // [NQ][128] lse in log2 units
  float* sDsum = sLse + NQ * BM;                                       // [NQ][128]
  int* sKlo = reinterpret_cast<int*>(sDsum + NQ * BM);                 // [NQ][128] first visible key
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKlo + NQ * BM);
  uint64_t* kv_full = bars + 0;
  uint64_t* qd_full = bars + 1;            // [NQ]
  uint64_t* qd_empty = bars + 1 + NQ;      // [NQ]
  uint64_t* ld_full = bars + 1 + 2 * NQ;   // [NQ]
  uint64_t* sdp_full = bars + 1 + 3 * NQ;  // [2] per query half
  uint64_t* p_ready = sdp_full + 2;        // [2]
  uint64_t* mma_done = sdp_full + 4;       // [2]
  uint64_t* kv_done = sdp_full + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sdp_full + 7);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long cta_t0 = clock64();
  // Longest first (linear block order): key block j sees the queries after it, so small j first,
  // with heads and batches fastest.
  const int lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int nhb = gridDim.y * gridDim.z;
  const int j = lin / nhb, kh = (lin % nhb) % gridDim.y, b = (lin % nhb) / gridDim.y;
  const int rep = a.H / a.Hkv;
  const int base = b * a.S;
  const int k0 = j * BN;
  const int nqb = (a.S + BM - 1) / BM;
  int i_lo = k0 / BM;
  int i_hi = nqb - 1;
  if (a.window > 0) i_hi = min(i_hi, (k0 + BN - 1 + a.window - 1) / BM);
  const int n_i = k0 < a.S ? max(i_hi - i_lo + 1, 0) : 0;
  const int n_it = rep * n_i;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int t = 0; t < NQ; ++t) {
      mbar_init(&qd_full[t], 1);
      mbar_init(&qd_empty[t], 1);
      mbar_init(&ld_full[t], 32);
    }
    for (int hh = 0; hh < 2; ++hh) {
      mbar_init(&sdp_full[hh], 1);
      mbar_init(&p_ready[hh], 256);  // the eight compute warps of the half
      mbar_init(&mma_done[hh], 1);
    }
    mbar_init(kv_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarpKV) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kTmaWarpKV) {
    // ------------------------------------------------------------------ TMA + per-query scalars
    if (n_it > 0) {
      // chunk 0 (columns 0-63) through the 128-byte-swizzle maps, chunk 1 through the narrow maps
      // for HD = 96, else through the same maps
      auto load_tile = [&](const CUtensorMap* m, const CUtensorMap* mn, uint64_t* bar, uint8_t* dst, int col0,
                           int row0) {
        tma_load_2d(m, bar, dst, col0, row0);
        if constexpr (TF::W1 > 0) tma_load_2d(TF::kNarrow ? mn : m, bar, dst + TF::kC0, col0 + 64, row0);
      };
      if (lane == 0) {
        mbar_arrive_expect_tx(kv_full, 2 * tile);
        load_tile(&tmK, &tmKn, kv_full, sK, kh * HD, base + k0);
        load_tile(&tmV, &tmVn, kv_full, sV, kh * HD, base + k0);
      }
      for (int it = 0; it < n_it; ++it) {
        const int buf = it % NQ;
        const int h = kh * rep + it / n_i;
        const int q0 = (i_lo + it % n_i) * BM;
        bool ok = true;
        const long long pw0 = clock64();
        if (lane == 0) ok = mbar_wait(&qd_empty[buf], ((it / NQ) & 1) ^ 1, a.err, kErrTimeoutProducer, abort_flag);
        if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        const long long pw1 = clock64();
        if (lane == 0) {
          mbar_arrive_expect_tx(&qd_full[buf], 2 * tile);
          load_tile(&tmQ, &tmQn, &qd_full[buf], sQ + buf * tile, h * HD, base + q0);
          load_tile(&tmO, &tmOn, &qd_full[buf], sO + buf * tile, h * HD, base + q0);
        }
        // All global loads first (in flight together), then the shared-memory stores: interleaved,
        // the stores kept each next load waiting for the previous one.
        float lv[BM / 32], dv[BM / 32];
#pragma unroll
        for (int u = 0; u < BM / 32; ++u) {
          const int qi = q0 + u * 32 + lane;
          const long idx = (long)(base + qi) * a.H + h;
          lv[u] = qi < a.S ? __ldg(a.lse + idx) : 0.f;
          dv[u] = qi < a.S ? __ldg(a.dsum + idx) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < BM / 32; ++u) {
          const int q = u * 32 + lane, qi = q0 + q;
          const bool in = qi < a.S;
          // negated and pre-scaled: P^T = 2^(s c + nlse), dS^T = P^T (dP^T scale + nsd)
          sLse[buf * BM + q] = in ? -lv[u] * 1.4426950408889634f : -INFINITY;
          sDsum[buf * BM + q] = in ? -dv[u] * a.scale : 0.f;
          sKlo[buf * BM + q] = query_key_lo(qi, a.S, a.window, a.seg, base);
        }
        __syncwarp();
        mbar_arrive(&ld_full[buf]);
        if (a.prof && lane == 0) {
          atomicAdd(&a.prof[11], (unsigned long long)(pw1 - pw0));
          atomicAdd(&a.prof[12], (unsigned long long)(clock64() - pw1));
        }
      }
    }
  } else if (warp == kMmaWarpKV) {
    // ------------------------------------------------------------------------------ MMA issuer
    if (lane == 0 && n_it > 0) {
      // The two 64-query halves of a block are pipeline stages: S^T / dP^T of half h fill TMEM
      // columns [64 h, 64 h + 64) of their regions, so half h of block it + 1 is computed while
      // the other half's compute warps (and the dV / dK MMAs of half h) run. Issue order per
      // block: dV/dK(it, 0), S/dP(it + 1, 0), dV/dK(it, 1), S/dP(it + 1, 1).
      constexpr uint32_t idesc_s = make_idesc_bf16(BN, BM / 2, false, false);  // keys x 64 queries
      // keys x head_dim: one MMA over the whole tile, or (HD = 96) one per chunk, 64 + 32 columns
      constexpr uint32_t idesc_kv = make_idesc_bf16(BN, TF::kNarrow ? 64 : HD, false, true);
      constexpr uint32_t idesc_kv1 = make_idesc_bf16(BN, TF::kNarrow ? 32 : HD, false, true);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      auto issue_sdp = [&](int it, int hh) {
        const uint32_t q_addr = smem_u32(sQ + (it % NQ) * tile), o_addr = smem_u32(sO + (it % NQ) * tile);
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks)  // the half's 64 query rows start at row 64 hh
          umma_bf16(tmem + kColS + 64 * hh, TF::kmaj(k_addr, ks, 0), TF::kmaj(q_addr, ks, 64 * hh), idesc_s,
                    ks > 0 ? 1u : 0u);
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks)
          umma_bf16(tmem + kColDP + 64 * hh, TF::kmaj(v_addr, ks, 0), TF::kmaj(o_addr, ks, 64 * hh), idesc_s,
                    ks > 0 ? 1u : 0u);
        umma_commit(&sdp_full[hh]);
      };
      auto issue_dkdv = [&](int it, int hh) {
        const uint32_t q_addr = smem_u32(sQ + (it % NQ) * tile), o_addr = smem_u32(sO + (it % NQ) * tile);
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4) {
          const int ks = 4 * hh + k4;
          // queries 16 ks.. were packed by column quarter ks / 2 at the start of its S^T columns
          const uint32_t pc = (ks >> 1) * 32 + (ks & 1) * 8;
          const uint32_t acc = (it > 0 || ks > 0) ? 1u : 0u;
          umma_ts(tmem + C::dV, tmem + kColS + pc, TF::mnmaj(o_addr, 0, ks), idesc_kv, acc);
          umma_ts(tmem + C::dK, tmem + kColDP + pc, TF::mnmaj(q_addr, 0, ks), idesc_kv, acc);
          if constexpr (TF::kNarrow) {
            umma_ts(tmem + C::dV + 64, tmem + kColS + pc, TF::mnmaj(o_addr, 1, ks), idesc_kv1, acc);
            umma_ts(tmem + C::dK + 64, tmem + kColDP + pc, TF::mnmaj(q_addr, 1, ks), idesc_kv1, acc);
          }
        }
        umma_commit(&mma_done[hh]);
      };
      const long long loop0 = clock64();
      bool ok = mbar_wait(kv_full, 0, a.err, kErrTimeoutMma, abort_flag);
      ok = ok && mbar_wait(&qd_full[0], 0, a.err, kErrTimeoutMma, abort_flag);
      if (ok) {
        tc_fence_after();
        issue_sdp(0, 0);
        issue_sdp(0, 1);
      }
      for (int it = 0; it < n_it && ok; ++it) {
        const int buf = it % NQ;
        for (int hh = 0; hh < 2 && ok; ++hh) {
          long long w0 = clock64();
          if (!mbar_wait(&p_ready[hh], it & 1, a.err, kErrTimeoutMma, abort_flag)) { ok = false; break; }
          if (a.prof) atomicAdd(&a.prof[5], (unsigned long long)(clock64() - w0));
          tc_fence_after();
          issue_dkdv(it, hh);
          if (hh == 1) umma_commit(&qd_empty[buf]);
          if (it + 1 < n_it) {
            // the next block's Q / dO landed, and dV / dK of this half (readers of its P^T / dS^T
            // columns) are done
            w0 = clock64();
            if (hh == 0 && !mbar_wait(&qd_full[(it + 1) % NQ], ((it + 1) / NQ) & 1, a.err, kErrTimeoutMma,
                                      abort_flag)) {
              ok = false;
              break;
            }
            const long long w1 = clock64();
            if (!mbar_wait(&mma_done[hh], it & 1, a.err, kErrTimeoutMma, abort_flag)) { ok = false; break; }
            if (a.prof) {
              atomicAdd(&a.prof[7], (unsigned long long)(w1 - w0));
              atomicAdd(&a.prof[6], (unsigned long long)(clock64() - w1));
            }
            tc_fence_after();
            issue_sdp(it + 1, hh);
          }
        }
      }
      umma_commit(kv_done);
      if (a.prof) atomicAdd(&a.prof[8], (unsigned long long)(clock64() - loop0));
    }
  } else {
    // -------------------------------------------------------------------------- compute warps
    const int qt = warp >> 2;  // query-column quarter [32 qt, 32 qt + 32)
    const int kr = (warp & 3) * 32 + lane;
    const int kj = k0 + kr;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + kColS + lane_off + 32 * qt, t_dp = tmem + kColDP + lane_off + 32 * qt;
    const bool plain = a.seg == nullptr;
    bool alive = true;
    for (int it = 0; it < n_it; ++it) {
      const int buf = it % NQ;
      const int qb = (i_lo + it % n_i) * BM + 32 * qt;  // first query of this quarter
      const long long p_t0 = clock64();
      bool got = mbar_wait(&ld_full[buf], (it / NQ) & 1, a.err, kErrTimeoutEpilogue, abort_flag);
      got = got && mbar_wait(&sdp_full[qt >> 1], it & 1, a.err, kErrTimeoutEpilogue, abort_flag);
      if (!__all_sync(0xffffffffu, got)) { alive = false; break; }
      const long long p_t1 = clock64();
      tc_fence_after();
      const float* lse2 = sLse + buf * BM + 32 * qt;
      const float* dsq = sDsum + buf * BM + 32 * qt;
      const int* klo = sKlo + buf * BM + 32 * qt;
      // every (query, key) pair of this quarter visible: no masks
      const bool full = plain && qb >= k0 + BN - 1 && (a.window <= 0 || qb + 31 - k0 < a.window) && qb + 31 < a.S &&
                        k0 + BN <= a.S;
      float sv[32], dp[32];
      tmem_ld32(t_s, sv);
      tmem_ld32(t_dp, dp);
      tmem_wait_ld();
      const long long p_t2 = clock64();
      uint32_t pw[16], dw[16];
      if (full) {
        // fp32 pairs (f32x2): x = s c + nlse, t = dp scale + nsd, dS = P t
        const uint64_t c2 = f2_make(a.scale_log2, a.scale_log2), sc2 = f2_make(a.scale, a.scale);
#pragma unroll
        for (int u = 0; u < 32; u += 4) {
          const float4 L = *reinterpret_cast<const float4*>(lse2 + u);
          const float4 D = *reinterpret_cast<const float4*>(dsq + u);
          float x0, x1, x2, x3, d0, d1, d2, d3;
          f2_split(f2_fma(f2_make(sv[u], sv[u + 1]), c2, f2_make(L.x, L.y)), x0, x1);
          f2_split(f2_fma(f2_make(sv[u + 2], sv[u + 3]), c2, f2_make(L.z, L.w)), x2, x3);
          const float p0 = ex2(x0), p1 = ex2(x1), p2 = ex2(x2), p3 = ex2(x3);
          const uint64_t t01 = f2_fma(f2_make(dp[u], dp[u + 1]), sc2, f2_make(D.x, D.y));
          const uint64_t t23 = f2_fma(f2_make(dp[u + 2], dp[u + 3]), sc2, f2_make(D.z, D.w));
          f2_split(f2_mul(f2_make(p0, p1), t01), d0, d1);
          f2_split(f2_mul(f2_make(p2, p3), t23), d2, d3);
          pw[u / 2] = pack_bf16x2(p0, p1);
          pw[u / 2 + 1] = pack_bf16x2(p2, p3);
          dw[u / 2] = pack_bf16x2(d0, d1);
          dw[u / 2 + 1] = pack_bf16x2(d2, d3);
        }
      } else {
#pragma unroll
        for (int u = 0; u < 32; u += 2) {
          float pv[2], dv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int qq = u + e;
            const int qi = qb + qq;
            const bool vis = kj <= qi && kj >= klo[qq] && kj < a.S;
            const float p = vis ? ex2(fmaf(sv[u + e], a.scale_log2, lse2[qq])) : 0.f;
            pv[e] = p;
            dv[e] = p * fmaf(dp[u + e], a.scale, dsq[qq]);
          }
          pw[u / 2] = pack_bf16x2(pv[0], pv[1]);
          dw[u / 2] = pack_bf16x2(dv[0], dv[1]);
        }
      }
      const long long p_t3 = clock64();
      // P^T / dS^T (bf16 pairs) over the first 16 of this quarter's own S^T / dP^T columns
      tmem_st16(t_s, pw);
      tmem_st16(t_dp, dw);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_ready[qt >> 1]);
      if (a.prof && lane == 0) {
        const long long p_t4 = clock64();
        atomicAdd(&a.prof[0], (unsigned long long)(p_t1 - p_t0));
        atomicAdd(&a.prof[1], (unsigned long long)(p_t2 - p_t1));
        atomicAdd(&a.prof[2], (unsigned long long)(p_t3 - p_t2));
        atomicAdd(&a.prof[3], (unsigned long long)(p_t4 - p_t3));
        atomicAdd(&a.prof[4], 1ull);
      }
    }
    const int hf = qt;  // the write-out uses the first eight warps, one head-dim half each
    const long long out0 = clock64();
    // ---- dK, dV out (once per CTA); half hf writes head-dim columns [hf HD/2, (hf + 1) HD/2)
    if (hf < 2 && k0 < a.S) {
      bool have = n_it > 0 && alive;
      if (have) {
        const bool got = mbar_wait(kv_done, 0, a.err, kErrTimeoutEpilogue, abort_flag);
        have = __all_sync(0xffffffffu, got);
        tc_fence_after();
      }
      if (n_it == 0 || have) {
        __nv_bfloat16* dvr = a.dv + (long)(base + kj) * a.dv_tok + (long)kh * a.dv_head;
        __nv_bfloat16* dkr = a.dk + (long)(base + kj) * a.dk_tok + (long)kh * a.dk_head;
#pragma unroll 1
        for (int c = hf * (HD / 2); c < (hf + 1) * (HD / 2); c += 16) {
          float vv[16], kk[16];
          if (have) {
            tmem_ld16(tmem + C::dV + lane_off + c, vv);
            tmem_ld16(tmem + C::dK + lane_off + c, kk);
            tmem_wait_ld();
          } else {
#pragma unroll
            for (int u = 0; u < 16; ++u) vv[u] = kk[u] = 0.f;
          }
          if (kj < a.S) {
            uint32_t pv[8], pk[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              float v0 = vv[2 * u], v1 = vv[2 * u + 1];
              if (a.dv_accumulate) {
                const __nv_bfloat162 old = reinterpret_cast<const __nv_bfloat162*>(dvr + c)[u];
                v0 += __bfloat162float(old.x);
                v1 += __bfloat162float(old.y);
              }
              pv[u] = pack_bf16x2(v0, v1);
              pk[u] = pack_bf16x2(kk[2 * u], kk[2 * u + 1]);
            }
            reinterpret_cast<uint4*>(dvr + c)[0] = make_uint4(pv[0], pv[1], pv[2], pv[3]);
            reinterpret_cast<uint4*>(dvr + c)[1] = make_uint4(pv[4], pv[5], pv[6], pv[7]);
            reinterpret_cast<uint4*>(dkr + c)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            reinterpret_cast<uint4*>(dkr + c)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          }
        }
      }
    }
    if (a.prof && lane == 0 && warp < 8) atomicAdd(&a.prof[10], (unsigned long long)(clock64() - out0));
  }
  if (a.prof && threadIdx.x == 0) atomicAdd(&a.prof[9], (unsigned long long)(clock64() - cta_t0));
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarpKV) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------------------------ dQ kernel
template <int HD>
struct SmemQ {
  static constexpr int kTile = ((HD + 63) / 64) * 128 * 128;
  // Q, dO, K[3], V[2], barriers. K is held from S_t to dQ_t (the dQ MMA runs one block behind),
  // so it gets a third stage: K_{t+1} then loads while blocks t-1 and t are still in flight.
  static constexpr int kUsed = 7 * kTile + 256;
  static constexpr int kBytes = kUsed + 128;
};

template <int HD>
__global__ void __launch_bounds__(kThreadsKV, 1)
    fa_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                     const BwdArgs a) {
  using SM = SmemQ<HD>;
  constexpr int KCH = (HD + 63) / 64;
  constexpr uint32_t tile = SM::kTile;
  constexpr uint32_t kColSb = 0, kColDp = 256, kColDq = 384;  // S[2], dP, dQ
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t pad = (1024u - (smem_u32(smem_raw) & 1023u)) & 1023u;
  if (pad + SM::kUsed > SM::kBytes) {
    if (threadIdx.x == 0) atomicExch(a.err, kErrBadArgs);
    return;
  }
  uint8_t* smem = smem_raw + pad;
  uint8_t* sQ = smem;
  uint8_t* sO = smem + tile;
  uint8_t* sK = smem + 2 * tile;  // [3]
  uint8_t* sV = smem + 5 * tile;  // [2]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 7 * tile);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [3]
  uint64_t* k_empty = bars + 4;   // [3]
  uint64_t* v_full = bars + 7;    // [2]
  uint64_t* v_empty = bars + 9;   // [2]
  uint64_t* s_full = bars + 11;   // [2]
  uint64_t* dq_mma = bars + 13;   // [2]
  uint64_t* dp_free = bars + 15;
  uint64_t* ds_ready = bars + 16;
  uint64_t* dq_done = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Longest first (linear block order): query block i sees the keys up to it, so large i first,
  // with heads and batches fastest.
  const int lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int nhb = gridDim.y * gridDim.z;
  const int i = gridDim.x - 1 - lin / nhb, h = (lin % nhb) % gridDim.y, b = (lin % nhb) / gridDim.y;
  const int kh = h / (a.H / a.Hkv);
  const int base = b * a.S;
  const int q0 = i * BM;
  int j_lo = 0;
  if (a.window > 0) j_lo = max(0, q0 - a.window + 1) / BN;
  const int j_hi = min(i, (a.S + BN - 1) / BN - 1);
  const int nj = q0 < a.S ? max(j_hi - j_lo + 1, 0) : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int t = 0; t < 3; ++t) {
      mbar_init(&k_full[t], 1);
      mbar_init(&k_empty[t], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&v_full[t], 1);
      mbar_init(&v_empty[t], 1);
      mbar_init(&s_full[t], 1);
      mbar_init(&dq_mma[t], 1);
    }
    mbar_init(dp_free, 512);
    mbar_init(ds_ready, 512);
    mbar_init(dq_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarpKV) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kTmaWarpKV) {
    // ------------------------------------------------------------------------- TMA producer
    if (lane == 0 && nj > 0) {
      mbar_arrive_expect_tx(q_full, 2 * tile);
      for (int c = 0; c < KCH; ++c) {
        tma_load_2d(&tmQ, q_full, sQ + c * BM * 128, h * HD + c * 64, base + q0);
        tma_load_2d(&tmO, q_full, sO + c * BM * 128, h * HD + c * 64, base + q0);
      }
      for (int t = 0; t < nj; ++t) {
        const int ks = t % 3, vs = t & 1;
        const int kr = base + (j_lo + t) * BN;
        if (!mbar_wait(&k_empty[ks], ((t / 3) & 1) ^ 1, a.err, kErrTimeoutProducer, abort_flag)) break;
        mbar_arrive_expect_tx(&k_full[ks], tile);
        for (int c = 0; c < KCH; ++c)
          tma_load_2d(&tmK, &k_full[ks], sK + ks * tile + c * BN * 128, kh * HD + c * 64, kr);
        if (!mbar_wait(&v_empty[vs], ((t >> 1) & 1) ^ 1, a.err, kErrTimeoutProducer, abort_flag)) break;
        mbar_arrive_expect_tx(&v_full[vs], tile);
        for (int c = 0; c < KCH; ++c)
          tma_load_2d(&tmV, &v_full[vs], sV + vs * tile + c * BN * 128, kh * HD + c * 64, kr);
      }
    }
  } else if (warp == kMmaWarpKV) {
    // ------------------------------------------------------------------------------ MMA issuer
    if (lane == 0 && nj > 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idesc_q = make_idesc_bf16(BM, HD, false, true);
      const uint32_t q_addr = smem_u32(sQ), o_addr = smem_u32(sO);
      bool ok = mbar_wait(q_full, 0, a.err, kErrTimeoutMma, abort_flag);
      // software pipeline: S/dP of block t are issued before the dQ MMA of block t-1
      for (int t = 0; t <= nj && ok; ++t) {
        if (t < nj) {
          const int st = t & 1;
          const uint32_t k_addr = smem_u32(sK + (t % 3) * tile), v_addr = smem_u32(sV + st * tile);
          if (!mbar_wait(&k_full[t % 3], (t / 3) & 1, a.err, kErrTimeoutMma, abort_flag)) break;
          if (t >= 2 && !mbar_wait(&dq_mma[st], ((t - 2) >> 1) & 1, a.err, kErrTimeoutMma, abort_flag)) break;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < HD / 16; ++ks) {
            const uint32_t off = (ks / 4) * 128 * 128 + (ks % 4) * 32;
            umma_bf16(tmem + kColSb + st * 128, make_sdesc(q_addr + off, 16, 1024), make_sdesc(k_addr + off, 16, 1024),
                      idesc_s, ks > 0 ? 1u : 0u);
          }
          if (t >= 1) {
            if (!mbar_wait(dp_free, (t - 1) & 1, a.err, kErrTimeoutMma, abort_flag)) break;
          }
          if (!mbar_wait(&v_full[st], (t >> 1) & 1, a.err, kErrTimeoutMma, abort_flag)) break;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < HD / 16; ++ks) {
            const uint32_t off = (ks / 4) * 128 * 128 + (ks % 4) * 32;
            umma_bf16(tmem + kColDp, make_sdesc(o_addr + off, 16, 1024), make_sdesc(v_addr + off, 16, 1024), idesc_s,
                      ks > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[st]);
          umma_commit(&v_empty[st]);  // V_t is read by dP_t only
        }
        if (t >= 1) {
          const int pt = t - 1, ps = pt & 1;
          const uint32_t k_addr = smem_u32(sK + (pt % 3) * tile);
          if (!mbar_wait(ds_ready, pt & 1, a.err, kErrTimeoutMma, abort_flag)) break;
          tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < BN / 16; ++ks)
            umma_ts(tmem + kColDq, tmem + kColSb + ps * 128 + (ks >> 1) * 32 + (ks & 1) * 8,
                    make_sdesc(k_addr + ks * 2048, BN * 128, 1024), idesc_q, (pt > 0 || ks > 0) ? 1u : 0u);
          umma_commit(&dq_mma[ps]);
          umma_commit(&k_empty[pt % 3]);
        }
      }
      umma_commit(dq_done);
    }
  } else if (warp < kMmaWarpKV) {
    // -------------------------------------------------------------------------- compute warps
    const int qt = warp >> 2;  // key-column quarter [32 qt, 32 qt + 32) of each block
    const int q = (warp & 3) * 32 + lane;
    const int qi = q0 + q;
    const bool in = qi < a.S;
    const long sidx = (long)(base + qi) * a.H + h;
    const float lse2 = in ? a.lse[sidx] * 1.4426950408889634f : INFINITY;
    const float dq_sum = in ? a.dsum[sidx] : 0.f;
    const int klo = query_key_lo(qi, a.S, a.window, a.seg, base);
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const bool plain = a.seg == nullptr;
    // fp32 pairs: x = s c - lse, t = dp scale - D scale, dS = P t
    const uint64_t c2 = f2_make(a.scale_log2, a.scale_log2), nl2 = f2_make(-lse2, -lse2);
    const uint64_t sc2 = f2_make(a.scale, a.scale), nd2 = f2_make(-dq_sum * a.scale, -dq_sum * a.scale);
    bool alive = true;
    for (int t = 0; t < nj; ++t) {
      const int st = t & 1;
      const int kb = (j_lo + t) * BN + 32 * qt;  // first key of this quarter
      const bool got = mbar_wait(&s_full[st], (t >> 1) & 1, a.err, kErrTimeoutEpilogue, abort_flag);
      if (!__all_sync(0xffffffffu, got)) { alive = false; break; }
      tc_fence_after();
      const uint32_t t_s = tmem + kColSb + st * 128 + lane_off + 32 * qt;
      float dp[32], sv[32];
      tmem_ld32(tmem + kColDp + lane_off + 32 * qt, dp);
      tmem_ld32(t_s, sv);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(dp_free);
      const bool full = plain && q0 >= kb + 31 && (a.window <= 0 || q0 + BM - 1 - kb < a.window) &&
                        q0 + BM <= a.S && kb + 32 <= a.S;
      uint32_t dw[16];
      if (full) {
#pragma unroll
        for (int u = 0; u < 32; u += 2) {
          float x0, x1, d0, d1;
          f2_split(f2_fma(f2_make(sv[u], sv[u + 1]), c2, nl2), x0, x1);
          const float p0 = ex2(x0), p1 = ex2(x1);
          f2_split(f2_mul(f2_make(p0, p1), f2_fma(f2_make(dp[u], dp[u + 1]), sc2, nd2)), d0, d1);
          dw[u / 2] = pack_bf16x2(d0, d1);
        }
      } else {
#pragma unroll
        for (int u = 0; u < 32; u += 2) {
          float dv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int kj = kb + u + e;
            const bool vis = kj <= qi && kj >= klo && kj < a.S;
            const float p = vis ? ex2(fmaf(sv[u + e], a.scale_log2, -lse2)) : 0.f;
            dv[e] = p * (dp[u + e] - dq_sum) * a.scale;
          }
          dw[u / 2] = pack_bf16x2(dv[0], dv[1]);
        }
      }
      // dS (bf16 pairs) over the first 16 of this quarter's own S columns
      tmem_st16(t_s, dw);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(ds_ready);
    }
    const int hf = qt;  // the write-out uses the first eight warps, one head-dim half each
    if (hf < 2 && alive && nj > 0) {
      const bool got = mbar_wait(dq_done, 0, a.err, kErrTimeoutEpilogue, abort_flag);
      if (__all_sync(0xffffffffu, got)) {
        tc_fence_after();
        __nv_bfloat16* row = a.dq + sidx * HD;
#pragma unroll 1
        for (int c = hf * (HD / 2); c < (hf + 1) * (HD / 2); c += 16) {
          float v[16];
          tmem_ld16(tmem + kColDq + lane_off + c, v);
          tmem_wait_ld();
          if (in) {
            uint32_t pk[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) pk[u] = pack_bf16x2(v[2 * u], v[2 * u + 1]);
            reinterpret_cast<uint4*>(row + c)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            reinterpret_cast<uint4*>(row + c)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarpKV) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace fab100

bool make_tmap_bf16_2d(CUtensorMap* m, const void* ptr, int64_t inner, int64_t outer, int64_t ld, int box_inner,
                       int box_outer);
bool make_tmap_bf16_2d_sw64(CUtensorMap* m, const void* ptr, int64_t inner, int64_t outer, int64_t ld,
                            int box_inner, int box_outer);

template <int HD>
static int run_fa_bwd_sm100(const AttnLaunch& L, int* err, cudaStream_t st) {
  using namespace fab100;
  CUtensorMap tq, tk, tv, to, tqn, tkn, tvn, ton;
  const long T = (long)L.B * L.S;
  if (!make_tmap_bf16_2d(&tq, L.q, (long)L.H * HD, T, L.q_tok, 64, BM)) return kErrBadArgsHost;
  if (!make_tmap_bf16_2d(&tk, L.k, (long)L.Hkv * HD, T, L.k_tok, 64, BN)) return kErrBadArgsHost;
  if (!make_tmap_bf16_2d(&tv, L.v, (long)L.Hkv * HD, T, L.v_tok, 64, BN)) return kErrBadArgsHost;
  if (!make_tmap_bf16_2d(&to, L.dout, (long)L.H * HD, T, (long)L.H * HD, 64, BM)) return kErrBadArgsHost;
  // HD = 96 tiles stay padded to 128 columns (two Q / dO stages) unless MXK_ATTN_BWD_UNPAD=1: the
  // unpadded three-stage form measured 8 % slower on one B200 (0.766 vs 0.707 ms for 8 x 2048 x 16 x 96
  // causal): splitting each dV / dK product into N = 64 and N = 32 MMAs costs more than the third
  // stage saves
  static const bool unpad = [] {
    const char* e = getenv("MXK_ATTN_BWD_UNPAD");
    return e && e[0] == '1';
  }();
  if (TileFmt<HD>::kNarrow) {  // 32-column boxes for the second chunk of an unpadded HD = 96 tile
    if (!make_tmap_bf16_2d_sw64(&tqn, L.q, (long)L.H * HD, T, L.q_tok, 32, BM)) return kErrBadArgsHost;
    if (!make_tmap_bf16_2d_sw64(&tkn, L.k, (long)L.Hkv * HD, T, L.k_tok, 32, BN)) return kErrBadArgsHost;
    if (!make_tmap_bf16_2d_sw64(&tvn, L.v, (long)L.Hkv * HD, T, L.v_tok, 32, BN)) return kErrBadArgsHost;
    if (!make_tmap_bf16_2d_sw64(&ton, L.dout, (long)L.H * HD, T, (long)L.H * HD, 32, BM)) return kErrBadArgsHost;
  } else {
    tqn = tq; tkn = tk; tvn = tv; ton = to;
  }
  BwdArgs a{};
  a.B = L.B; a.S = L.S; a.H = L.H; a.Hkv = L.Hkv; a.window = L.window;
  a.scale = L.scale;
  a.scale_log2 = L.scale * 1.4426950408889634f;
  a.seg = L.seg;
  a.lse = L.lse;
  a.dsum = L.dsum;
  a.dq = (__nv_bfloat16*)L.dq;
  a.dk = (__nv_bfloat16*)L.dk; a.dk_tok = L.dk_tok; a.dk_head = L.dk_head;
  a.dv = (__nv_bfloat16*)L.dv; a.dv_tok = L.dv_tok; a.dv_head = L.dv_head;
  a.dv_accumulate = L.dv_accumulate;
  a.err = err;
  a.prof = (unsigned long long*)L.prof;
  constexpr int smem_kv = Smem<HD, true>::kBytes, smem_kv_pad = Smem<HD, false>::kBytes;
  constexpr int smem_q = SmemQ<HD>::kBytes;
  static_assert(smem_kv <= 232448 && smem_kv_pad <= 232448 && smem_q <= 232448, "shared memory budget");
  static bool init = false;
  if (!init) {
    if (cudaFuncSetAttribute(fa_bwd_dkdv_kernel<HD, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_kv) !=
            cudaSuccess ||
        cudaFuncSetAttribute(fa_bwd_dkdv_kernel<HD, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             smem_kv_pad) != cudaSuccess ||
        cudaFuncSetAttribute(fa_bwd_dq_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_q) != cudaSuccess)
      return kErrBadArgsHost;
    init = true;
  }
  count_launch();
  const dim3 grid_kv((L.S + BN - 1) / BN, L.Hkv, L.B);
  if (unpad || !TileFmt<HD>::kNarrow)
    fa_bwd_dkdv_kernel<HD, true><<<grid_kv, kThreadsKV, smem_kv, st>>>(tq, tk, tv, to, tqn, tkn, tvn, ton, a);
  else
    fa_bwd_dkdv_kernel<HD, false><<<grid_kv, kThreadsKV, smem_kv_pad, st>>>(tq, tk, tv, to, tq, tk, tv, to, a);
  count_launch();
  fa_bwd_dq_kernel<HD><<<dim3((L.S + BM - 1) / BM, L.H, L.B), kThreadsKV, smem_q, st>>>(tq, tk, tv, to, a);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrBadArgsHost;
}

// Same contract as launch_flash_bwd (the dsum pass is shared with it); dq is written directly, so the
// fp32 dq accumulator is not used.
int launch_flash_bwd_sm100(const AttnLaunch& L, int* err, cudaStream_t st) {
  if (L.q_head != L.hd || L.k_head != L.hd || L.v_head != L.hd) return kErrBadArgsHost;
  if ((L.q_tok * 2) % 16 || (L.k_tok * 2) % 16 || (L.v_tok * 2) % 16) return kErrBadArgsHost;
  if ((reinterpret_cast<uintptr_t>(L.q) | reinterpret_cast<uintptr_t>(L.k) | reinterpret_cast<uintptr_t>(L.v) |
       reinterpret_cast<uintptr_t>(L.dout)) & 15)
    return kErrBadArgsHost;
  if ((L.dk_tok | L.dk_head | L.dv_tok | L.dv_head) % 8) return kErrBadArgsHost;  // 16-byte row stores
  AttnLaunch P = L;
  P.dq_acc = nullptr;  // dsum only
  int r = launch_flash_bwd_prep(P, st);
  if (r) return r;
  switch (L.hd) {
    case 64: r = run_fa_bwd_sm100<64>(L, err, st); break;
    case 96: r = run_fa_bwd_sm100<96>(L, err, st); break;
    case 128: r = run_fa_bwd_sm100<128>(L, err, st); break;
    default: return kErrBadArgsHost;
  }
  return r;
}

}  // namespace mxk
