// Flash attention forward on the 5th-generation tensor cores (sm_100a).
//
// CTA = two 128-query tiles of one head, ping-ponged: softmax warps (thread = query row = TMEM
// lane; in the default split-row kernel two warps per row, 64 key columns each), one MMA warp
// (one elected thread issues tcgen05.mma), one TMA warp. For each 128-key block j:
//   S_j = Q K_j^T            (SS MMA: Q, K_j from 128B-swizzled smem; S_j in TMEM, fp32)
//   P_j = exp2(S_j*c - m)    (softmax warps: tcgen05.ld S, tcgen05.st P as bf16 into TMEM)
//   O  += P_j V_j            (TS MMA: A = P_j from TMEM, B = V_j MN-major from smem; O in TMEM)
// The running max is only raised (and O, l rescaled) when a row max grows by more than 2^8, so
// most blocks skip the O correction. The two tiles' softmax phases alternate so that one tile's
// exponentials overlap the other tile's MMAs. All waits are bounded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include <string>

#include "kernels.h"
#include "sm100_primitives.cuh"

namespace mxk {
namespace fa100 {

constexpr int BM = 128;  // queries per CTA
constexpr int BN = 128;  // keys per block
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct FwdArgs {
  int B, S, H, Hkv, hd;
  int window;
  float scale_log2;
  const int* seg;
  __nv_bfloat16* o;  // [T, H, hd]
  float* lse;        // [T, H]
  int q_x0, k_x0, v_x0;  // column offsets (elements) of head 0 in the Q / K / V tensor maps
  int* err;
  // Optional phase-timing counters (cycles, summed over CTAs): [0] softmax wait s_full, [1] pass 1,
  // [2] pass 2, [3] O rescale, [4] MMA wait p_full, [5] MMA wait kv_full, [6] MMA wait o_done,
  // [7] softmax blocks, [8] rescales.
  unsigned long long* prof;
};

__device__ __forceinline__ void umma_ts_bf16(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ bool visible(int qi, int kj, int S, int window, const int* seg, int base) {
  if (kj > qi || kj >= S || qi >= S) return false;
  if (window > 0 && qi - kj >= window) return false;
  if (seg && seg[base + qi] != seg[base + kj]) return false;
  return true;
}

template <int HD>
struct Smem {
  static constexpr int KCH = (HD + 63) / 64;        // 64-element (128 B) chunks along head_dim
  static constexpr int kTile = KCH * BM * 128;       // one [128 rows x HD] operand tile
  // Q0, Q1, K[2 stages], V[2 stages]
  static constexpr int kBytes = 6 * kTile + 1024 + 512;
};

// Visible key range of query qi: [lo, hi] (segments are contiguous runs of equal ids).
__device__ __forceinline__ void key_range(int qi, int S, int window, const int* seg, int base, int& lo, int& hi) {
  hi = qi < S ? qi : -1;
  lo = 0;
  if (window > 0) lo = max(lo, qi - window + 1);
  if (seg && qi < S) {
    // first position of qi's segment: binary search on the non-decreasing run boundary
    const int sid = seg[base + qi];
    int a = 0, b = qi;
    while (a < b) {
      const int m = (a + b) >> 1;
      if (seg[base + m] == sid) b = m; else a = m + 1;
    }
    lo = max(lo, a);
  }
}

// Ping-pong forward: CTA = two 128-query tiles (rows q0..q0+255) of one head.
// warps 0-3: softmax of tile 0, warps 4-7: softmax of tile 1, warp 8: MMA, warp 9: TMA.
// TMEM: S0 [0,128) S1 [128,256) O0 [256,256+HD) O1 [384,384+HD).
constexpr int kThreadsPP = 320;

template <int HD>
__global__ void __launch_bounds__(kThreadsPP, 1)
    fa_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const FwdArgs a) {
  using SM = Smem<HD>;
  constexpr int KCH = SM::KCH;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                    // [2][tile]
  uint8_t* sK = smem + 2 * SM::kTile;    // [2 stages][tile]
  uint8_t* sV = smem + 4 * SM::kTile;    // [2 stages][tile]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * SM::kTile);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2] per tile
  uint64_t* p_full = bars + 7;    // [2] per tile
  uint64_t* o_done = bars + 9;    // [2] per tile
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Longest first: CTAs start in linear block order, so the tile index is the slowest-varying
  // one and descending (a causal tile's work grows with its index), heads and batches fastest;
  // the last wave then holds the shortest tiles instead of a tail of the longest.
  const int lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int nhb = gridDim.y * gridDim.z;
  const int h = (lin % nhb) % gridDim.y, b = (lin % nhb) / gridDim.y;
  const int kh = h / (a.H / a.Hkv);
  const int q0 = (gridDim.x - 1 - lin / nhb) * 2 * BM;
  const int base = b * a.S;
  // key blocks for the two tiles; tile 0 stops one block earlier (causal)
  int kb_lo = 0;
  if (a.window > 0) kb_lo = max(0, q0 - a.window + 1) / BN;
  const int kb_hi1 = (min(a.S, q0 + 2 * BM) + BN - 1) / BN;
  const int kb_hi0 = (min(a.S, q0 + BM) + BN - 1) / BN;
  const int nb = max(kb_hi1 - kb_lo, 0);
  // tile t uses blocks j in [lo_t, nb_t); tile 1 may skip early blocks outside its window
  int lo_t[2], nb_t[2];
  nb_t[0] = max(kb_hi0 - kb_lo, 0);
  nb_t[1] = nb;
  lo_t[0] = 0;
  lo_t[1] = 0;
  if (a.window > 0) lo_t[1] = max(0, (q0 + BM - a.window + 1) / BN - kb_lo);
  if (q0 + BM >= a.S) nb_t[1] = 0;  // tile 1 entirely past the sequence

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 9) {
    // ------------------------------------------------------------------------ TMA producer
    if (lane == 0 && nb > 0) {
      constexpr uint32_t tile = SM::kTile;
      mbar_arrive_expect_tx(q_full, 2 * tile);
      for (int t = 0; t < 2; ++t)
        for (int c = 0; c < KCH; ++c)
          tma_load_2d(&tmQ, q_full, sQ + t * tile + c * BM * 128, a.q_x0 + h * HD + c * 64, base + q0 + t * BM);
      for (int j = 0; j < nb; ++j) {
        const int st = j & 1;
        const int kr = base + (kb_lo + j) * BN;
        if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1, a.err, kErrTimeoutProducer, abort_flag)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * tile);
        for (int c = 0; c < KCH; ++c) {
          tma_load_2d(&tmK, &kv_full[st], sK + st * tile + c * BN * 128, a.k_x0 + kh * HD + c * 64, kr);
          tma_load_2d(&tmV, &kv_full[st], sV + st * tile + c * BN * 128, a.v_x0 + kh * HD + c * 64, kr);
        }
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------------------ MMA issuer
    if (lane == 0 && nb > 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(BM, HD, false, true);
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      int s_cnt[2] = {0, 0};  // S/PV issue counters per tile (barrier phases)
      bool ok = mbar_wait(q_full, 0, a.err, kErrTimeoutMma, abort_flag);
      auto issue_qk = [&](int t, int st) {
        const uint32_t qa = q_addr + t * SM::kTile, ka = k_addr + st * SM::kTile;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
          const uint32_t off = (ks / 4) * BM * 128 + (ks % 4) * 32;
          umma_bf16(tmem + t * 128, make_sdesc(qa + off, 16, 1024), make_sdesc(ka + off, 16, 1024), idesc_s,
                    ks > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int st, bool acc) {
        const uint32_t va = v_addr + st * SM::kTile;
#pragma unroll
        for (int ks = 0; ks < BN / 16; ++ks)
          umma_ts_bf16(tmem + 256 + t * 128, tmem + t * 128 + ks * 8, make_sdesc(va + ks * 2048, BN * 128, 1024),
                       idesc_o, (acc || ks > 0) ? 1u : 0u);
        umma_commit(&o_done[t]);
      };
      // Issue order per key block j: PV0_j, S0_{j+1}, PV1_j, S1_{j+1}. Tile 0's softmax of block
      // j+1 then runs while the tensor core does PV1_j and S1_{j+1}, and tile 1's while it does
      // PV0_{j+1} and S0_{j+2}: the two softmax groups alternate instead of contending for the
      // SFU at the same time. S_{j+1} overwrites P_j (aliased in TMEM), so it waits for PV_j.
      unsigned long long wp = 0, wkv = 0, wo = 0;
      auto active = [&](int t, int j) { return j >= lo_t[t] && j < nb_t[t]; };
      if (ok) {
        long long c0 = clock64();
        ok = mbar_wait(&kv_full[0], 0, a.err, kErrTimeoutMma, abort_flag);
        wkv += clock64() - c0;
        tc_fence_after();
        for (int t = 0; t < 2 && ok; ++t)
          if (active(t, 0)) issue_qk(t, 0);
      }
      for (int j = 0; j < nb && ok; ++j) {
        const int st = j & 1;
        bool next_ready = false;  // K/V of block j + 1 landed
        for (int t = 0; t < 2 && ok; ++t) {
          if (active(t, j)) {
            long long c2 = clock64();
            if (!mbar_wait(&p_full[t], s_cnt[t] & 1, a.err, kErrTimeoutMma, abort_flag)) { ok = false; break; }
            wp += clock64() - c2;
            tc_fence_after();
            issue_pv(t, st, s_cnt[t] > 0);
            ++s_cnt[t];
          }
          if (j + 1 < nb && active(t, j + 1)) {
            if (!next_ready) {
              long long c0 = clock64();
              if (!mbar_wait(&kv_full[st ^ 1], ((j + 1) >> 1) & 1, a.err, kErrTimeoutMma, abort_flag)) {
                ok = false;
                break;
              }
              wkv += clock64() - c0;
              next_ready = true;
            }
            if (s_cnt[t] > 0) {
              long long c1 = clock64();
              if (!mbar_wait(&o_done[t], (s_cnt[t] - 1) & 1, a.err, kErrTimeoutMma, abort_flag)) { ok = false; break; }
              wo += clock64() - c1;
            }
            tc_fence_after();
            issue_qk(t, st ^ 1);
          }
        }
        if (!ok) break;
        umma_commit(&kv_empty[st]);
      }
      if (a.prof) {
        atomicAdd(&a.prof[4], wp);
        atomicAdd(&a.prof[5], wkv);
        atomicAdd(&a.prof[6], wo);
      }
    }
  } else {
    // ------------------------------------------------------------------------ softmax warps
    const int t = warp >> 2;              // tile
    const int row = (warp & 3) * 32 + lane;
    const int qi = q0 + t * BM + row;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + t * 128 + lane_off;
    const uint32_t t_o = tmem + 256 + t * 128 + lane_off;
    int klo, khi;
    key_range(qi, a.S, a.window, a.seg, base, klo, khi);
    float m_run = -INFINITY, l_run = 0.f;
    bool alive = true;
    int cnt = 0;
    unsigned long long pw = 0, p1 = 0, p2 = 0, p3 = 0, nres = 0;
    for (int j = lo_t[t]; j < nb_t[t]; ++j, ++cnt) {
      long long c_a = clock64();
      const bool got = mbar_wait(&s_full[t], cnt & 1, a.err, kErrTimeoutEpilogue, abort_flag);
      long long c_b = clock64();
      pw += c_b - c_a;
      if (!__all_sync(0xffffffffu, got)) { alive = false; break; }
      tc_fence_after();
      const int k0 = (kb_lo + j) * BN;
      const int lo = klo - k0, hi = khi - k0;  // visible columns [lo, hi] of this block
      const bool full = lo <= 0 && hi >= BN - 1;
      // S row (128 fp32 columns) into registers with all four loads in flight, one wait
      float s0[32], s1[32], s2[32], s3[32];
      tmem_ld32(t_s + 0, s0);
      tmem_ld32(t_s + 32, s1);
      tmem_ld32(t_s + 64, s2);
      tmem_ld32(t_s + 96, s3);
      tmem_wait_ld();
      if (!full) {
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          if (c < lo || c > hi) s0[c] = -INFINITY;
          if (c + 32 < lo || c + 32 > hi) s1[c] = -INFINITY;
          if (c + 64 < lo || c + 64 > hi) s2[c] = -INFINITY;
          if (c + 96 < lo || c + 96 > hi) s3[c] = -INFINITY;
        }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 32; ++c) mx = fmaxf(mx, fmaxf(fmaxf(s0[c], s1[c]), fmaxf(s2[c], s3[c])));
      mx *= a.scale_log2;
      long long c_c = clock64();
      p1 += c_c - c_b;
      float alpha = 1.f;
      bool rescale = false;
      if (mx > m_run + kRescaleThreshold || (m_run == -INFINITY && mx > -INFINITY)) {
        if (m_run != -INFINITY) {
          alpha = exp2f(m_run - mx);
          rescale = true;
        }
        m_run = mx;
        l_run *= alpha;
      }
      const float mb = m_run == -INFINITY ? 0.f : m_run;
      const float sc = a.scale_log2;
      float rs = 0.f;
      // P = exp2(s*c - m) as bf16 pairs into the first 64 columns of S (all reads are done).
      // Arguments and the row sum use packed fp32 pairs; columns 32-63 take the FMA-pipe
      // exponential, the rest the special-function unit.
      {
        const uint64_t sc2 = f2_make(sc, sc), nm2 = f2_make(-mb, -mb);
        uint64_t rs2 = f2_make(0.f, 0.f);
        auto emit = [&](const float (&sv)[32], uint32_t col, bool poly) {
          uint32_t w[16];
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const uint64_t x = f2_fma(f2_make(sv[c], sv[c + 1]), sc2, nm2);
            float x0, x1, e0, e1;
            f2_split(x, x0, x1);
            if (poly) {
              ex2_poly2(x0, x1, e0, e1);
            } else {
              e0 = ex2_sfu(x0);
              e1 = ex2_sfu(x1);
            }
            rs2 = f2_add(rs2, f2_make(e0, e1));
            w[c / 2] = pack_bf16x2(e0, e1);
          }
          tmem_st16(t_s + col, w);
        };
        emit(s0, 0, false);
        emit(s1, 16, true);
        emit(s2, 32, false);
        emit(s3, 48, false);
        float r0, r1;
        f2_split(rs2, r0, r1);
        rs = r0 + r1;
      }
      l_run += rs;
      long long c_d = clock64();
      p2 += c_d - c_c;
      if (__any_sync(0xffffffffu, rescale)) {
        ++nres;
        const bool g2 = mbar_wait(&o_done[t], (cnt - 1) & 1, a.err, kErrTimeoutEpilogue, abort_flag);
        if (!__all_sync(0xffffffffu, g2)) { alive = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < HD; c += 16) {
          float o[16];
          tmem_ld16(t_o + c, o);
          tmem_wait_ld();
          uint32_t ou[16];
#pragma unroll
          for (int u = 0; u < 16; ++u) ou[u] = __float_as_uint(o[u] * alpha);
          tmem_st16(t_o + c, ou);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
      p3 += clock64() - c_d;
    }
    if (a.prof && lane == 0) {
      atomicAdd(&a.prof[0], pw);
      atomicAdd(&a.prof[1], p1);
      atomicAdd(&a.prof[2], p2);
      atomicAdd(&a.prof[3], p3);
      atomicAdd(&a.prof[7], (unsigned long long)cnt);
      atomicAdd(&a.prof[8], nres);
    }
    if (alive && cnt > 0) {
      const bool got = mbar_wait(&o_done[t], (cnt - 1) & 1, a.err, kErrTimeoutEpilogue, abort_flag);
      if (__all_sync(0xffffffffu, got)) {
        tc_fence_after();
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        __nv_bfloat16* orow = a.o + ((long)(base + qi) * a.H + h) * HD;
#pragma unroll 1
        for (int c = 0; c < HD; c += 16) {
          float o[16];
          tmem_ld16(t_o + c, o);
          tmem_wait_ld();
          if (qi < a.S) {
            uint32_t pkd[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) pkd[u] = pack_bf16x2(o[2 * u] * inv, o[2 * u + 1] * inv);
            reinterpret_cast<uint4*>(orow + c)[0] = make_uint4(pkd[0], pkd[1], pkd[2], pkd[3]);
            reinterpret_cast<uint4*>(orow + c)[1] = make_uint4(pkd[4], pkd[5], pkd[6], pkd[7]);
          }
        }
        if (qi < a.S)
          a.lse[(long)(base + qi) * a.H + h] = l_run > 0.f ? (m_run + log2f(l_run)) * 0.6931471805599453f : INFINITY;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Split-row forward: the same two-tile ping-pong, with each tile's softmax spread over eight warps
// -- two per TMEM subpartition, each owning 64 of a block's 128 key columns for its 32 rows -- so
// the per-block softmax latency, which bounds the tensor core's duty cycle (a tile's next S waits
// for its P), roughly halves. The two halves of a row agree on the block's row max through a
// shared-memory exchange gated by a per-subpartition mbarrier (64 arrivals per block, bounded
// waits); their partial row sums are combined once at the end. P of keys 0-63 goes to TMEM
// columns 0-31 of the tile's S region and P of keys 64-127 to columns 64-95, so each half only
// overwrites S columns it has already read itself.
constexpr int kThreadsSR = 576;  // softmax warps 0-15 (tile = warp / 8), MMA warp 16, TMA warp 17

template <int HD>
struct SmemSR {
  static constexpr int KCH = (HD + 63) / 64;
  static constexpr int kTile = KCH * BM * 128;
  static constexpr int kBarOff = 6 * kTile;                      // Q0, Q1, K[2], V[2] before it
  static constexpr int kMaxOff = kBarOff + 256;                  // float [2 parity][2 tiles][2 halves][BM]
  static constexpr int kSumOff = kMaxOff + 2 * 2 * 2 * BM * 4;   // float [2 tiles][2 halves][BM]
  static constexpr int kBytes = kSumOff + 2 * 2 * BM * 4 + 1024;  // + base alignment slack
};

// 2^x of 32 scores as bf16 pairs into 16 TMEM columns; the first NP pairs on the FMA pipe.
template <int NP>
__device__ __forceinline__ void softmax_emit32(const float (&sv)[32], uint32_t taddr, uint64_t sc2, uint64_t nm2,
                                               uint64_t& acc0, uint64_t& acc1) {
  uint32_t w[16];
#pragma unroll
  for (int c = 0; c < 32; c += 2) {
    const uint64_t x = f2_fma(f2_make(sv[c], sv[c + 1]), sc2, nm2);
    float x0, x1, e0, e1;
    f2_split(x, x0, x1);
    if (c / 2 < NP) {
      ex2_poly2(x0, x1, e0, e1);
    } else {
      e0 = ex2_sfu(x0);
      e1 = ex2_sfu(x1);
    }
    if ((c / 2) & 1) acc1 = f2_add(acc1, f2_make(e0, e1));
    else acc0 = f2_add(acc0, f2_make(e0, e1));
    w[c / 2] = pack_bf16x2(e0, e1);
  }
  tmem_st16(taddr, w);
}

template <int HD, int NP0, int NP1>
__global__ void __launch_bounds__(kThreadsSR, 1)
    fa_fwd_sm100_split_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                              const __grid_constant__ CUtensorMap tmV, const FwdArgs a) {
  using SM = SmemSR<HD>;
  constexpr int KCH = SM::KCH;
  constexpr int HH = HD / 2;  // O columns per half
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + 2 * SM::kTile;
  uint8_t* sV = smem + 4 * SM::kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::kBarOff);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2] per tile
  uint64_t* p_full = bars + 7;    // [2] per tile, 256 arrivals
  uint64_t* o_done = bars + 9;    // [2] per tile
  uint64_t* xbar = bars + 11;     // [2 tiles][4 subpartitions], 64 arrivals
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xmax = reinterpret_cast<float*>(smem + SM::kMaxOff);
  float* xsum = reinterpret_cast<float*>(smem + SM::kSumOff);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Longest first (see fa_fwd_sm100_kernel).
  const int lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int nhb = gridDim.y * gridDim.z;
  const int h = (lin % nhb) % gridDim.y, b = (lin % nhb) / gridDim.y;
  const int kh = h / (a.H / a.Hkv);
  const int q0 = (gridDim.x - 1 - lin / nhb) * 2 * BM;
  const int base = b * a.S;
  int kb_lo = 0;
  if (a.window > 0) kb_lo = max(0, q0 - a.window + 1) / BN;
  const int kb_hi1 = (min(a.S, q0 + 2 * BM) + BN - 1) / BN;
  const int kb_hi0 = (min(a.S, q0 + BM) + BN - 1) / BN;
  const int nb = max(kb_hi1 - kb_lo, 0);
  int lo_t[2], nb_t[2];
  nb_t[0] = max(kb_hi0 - kb_lo, 0);
  nb_t[1] = nb;
  lo_t[0] = 0;
  lo_t[1] = 0;
  if (a.window > 0) lo_t[1] = max(0, (q0 + BM - a.window + 1) / BN - kb_lo);
  if (q0 + BM >= a.S) nb_t[1] = 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 256);
      mbar_init(&o_done[i], 1);
    }
    for (int i = 0; i < 8; ++i) mbar_init(&xbar[i], 64);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 16) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 17) {
    // ------------------------------------------------------------------------ TMA producer
    if (lane == 0 && nb > 0) {
      constexpr uint32_t tile = SM::kTile;
      mbar_arrive_expect_tx(q_full, 2 * tile);
      for (int t = 0; t < 2; ++t)
        for (int c = 0; c < KCH; ++c)
          tma_load_2d(&tmQ, q_full, sQ + t * tile + c * BM * 128, a.q_x0 + h * HD + c * 64, base + q0 + t * BM);
      for (int j = 0; j < nb; ++j) {
        const int st = j & 1;
        const int kr = base + (kb_lo + j) * BN;
        if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1, a.err, kErrTimeoutProducer, abort_flag)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * tile);
        for (int c = 0; c < KCH; ++c) {
          tma_load_2d(&tmK, &kv_full[st], sK + st * tile + c * BN * 128, a.k_x0 + kh * HD + c * 64, kr);
          tma_load_2d(&tmV, &kv_full[st], sV + st * tile + c * BN * 128, a.v_x0 + kh * HD + c * 64, kr);
        }
      }
    }
  } else if (warp == 16) {
    // ------------------------------------------------------------------------ MMA issuer
    if (lane == 0 && nb > 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BM, BN, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(BM, HD, false, true);
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      int s_cnt[2] = {0, 0};
      bool ok = mbar_wait(q_full, 0, a.err, kErrTimeoutMma, abort_flag);
      auto issue_qk = [&](int t, int st) {
        const uint32_t qa = q_addr + t * SM::kTile, ka = k_addr + st * SM::kTile;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
          const uint32_t off = (ks / 4) * BM * 128 + (ks % 4) * 32;
          umma_bf16(tmem + t * 128, make_sdesc(qa + off, 16, 1024), make_sdesc(ka + off, 16, 1024), idesc_s,
                    ks > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int st, bool acc) {
        const uint32_t va = v_addr + st * SM::kTile;
#pragma unroll
        for (int ks = 0; ks < BN / 16; ++ks)  // P of keys 16ks.. at column 8ks, +32 for the upper half
          umma_ts_bf16(tmem + 256 + t * 128, tmem + t * 128 + ks * 8 + (ks >= 4 ? 32 : 0),
                       make_sdesc(va + ks * 2048, BN * 128, 1024), idesc_o, (acc || ks > 0) ? 1u : 0u);
        umma_commit(&o_done[t]);
      };
      unsigned long long wp = 0, wkv = 0, wo = 0;
      auto active = [&](int t, int j) { return j >= lo_t[t] && j < nb_t[t]; };
      if (ok) {
        long long c0 = clock64();
        ok = mbar_wait(&kv_full[0], 0, a.err, kErrTimeoutMma, abort_flag);
        wkv += clock64() - c0;
        tc_fence_after();
        for (int t = 0; t < 2 && ok; ++t)
          if (active(t, 0)) issue_qk(t, 0);
      }
      for (int j = 0; j < nb && ok; ++j) {
        const int st = j & 1;
        bool next_ready = false;
        for (int t = 0; t < 2 && ok; ++t) {
          if (active(t, j)) {
            long long c2 = clock64();
            if (!mbar_wait(&p_full[t], s_cnt[t] & 1, a.err, kErrTimeoutMma, abort_flag)) { ok = false; break; }
            wp += clock64() - c2;
            tc_fence_after();
            issue_pv(t, st, s_cnt[t] > 0);
            ++s_cnt[t];
          }
          if (j + 1 < nb && active(t, j + 1)) {
            if (!next_ready) {
              long long c0 = clock64();
              if (!mbar_wait(&kv_full[st ^ 1], ((j + 1) >> 1) & 1, a.err, kErrTimeoutMma, abort_flag)) {
                ok = false;
                break;
              }
              wkv += clock64() - c0;
              next_ready = true;
            }
            if (s_cnt[t] > 0) {
              long long c1 = clock64();
              if (!mbar_wait(&o_done[t], (s_cnt[t] - 1) & 1, a.err, kErrTimeoutMma, abort_flag)) { ok = false; break; }
              wo += clock64() - c1;
            }
            tc_fence_after();
            issue_qk(t, st ^ 1);
          }
        }
        if (!ok) break;
        umma_commit(&kv_empty[st]);
      }
      if (a.prof) {
        atomicAdd(&a.prof[4], wp);
        atomicAdd(&a.prof[5], wkv);
        atomicAdd(&a.prof[6], wo);
      }
    }
  } else {
    // ------------------------------------------------------------------------ softmax warps
    const int t = warp >> 3, sp = warp & 3, hf = (warp >> 2) & 1;
    const int row = sp * 32 + lane;
    const int qi = q0 + t * BM + row;
    const uint32_t lane_off = (uint32_t)(sp * 32) << 16;
    const uint32_t t_s = tmem + t * 128 + lane_off;
    const uint32_t t_o = tmem + 256 + t * 128 + lane_off + hf * HH;
    uint64_t* xb = &xbar[t * 4 + sp];
    int klo, khi;
    key_range(qi, a.S, a.window, a.seg, base, klo, khi);
    float m_run = -INFINITY, l_run = 0.f;
    bool alive = true;
    int cnt = 0;
    unsigned long long pw = 0, p1 = 0, p2 = 0, p3 = 0, nres = 0;
    for (int j = lo_t[t]; j < nb_t[t]; ++j, ++cnt) {
      long long c_a = clock64();
      const bool got = mbar_wait(&s_full[t], cnt & 1, a.err, kErrTimeoutEpilogue, abort_flag);
      long long c_b = clock64();
      pw += c_b - c_a;
      if (!__all_sync(0xffffffffu, got)) { alive = false; break; }
      tc_fence_after();
      const int k0 = (kb_lo + j) * BN + hf * 64;
      const int lo = klo - k0, hi = khi - k0;  // visible columns [lo, hi] of this half-block
      const bool full = lo <= 0 && hi >= 63;
      float s0[32], s1[32];
      tmem_ld32(t_s + hf * 64, s0);
      tmem_ld32(t_s + hf * 64 + 32, s1);
      tmem_wait_ld();
      if (!full) {
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          if (c < lo || c > hi) s0[c] = -INFINITY;
          if (c + 32 < lo || c + 32 > hi) s1[c] = -INFINITY;
        }
      }
      float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        mxa = fmaxf(mxa, fmaxf(s0[c], s1[c]));
        mxb = fmaxf(mxb, fmaxf(s0[c + 1], s1[c + 1]));
      }
      float mx = fmaxf(mxa, mxb);
      const int par = cnt & 1;
      xmax[((par * 2 + t) * 2 + hf) * BM + row] = mx;
      mbar_arrive(xb);
      const bool gx = mbar_wait(xb, par, a.err, kErrTimeoutEpilogue, abort_flag);
      if (!__all_sync(0xffffffffu, gx)) { alive = false; break; }
      mx = fmaxf(mx, xmax[((par * 2 + t) * 2 + (hf ^ 1)) * BM + row]) * a.scale_log2;
      long long c_c = clock64();
      p1 += c_c - c_b;
      float alpha = 1.f;
      bool rescale = false;
      if (mx > m_run + kRescaleThreshold || (m_run == -INFINITY && mx > -INFINITY)) {
        if (m_run != -INFINITY) {
          alpha = exp2f(m_run - mx);
          rescale = true;
        }
        m_run = mx;
        l_run *= alpha;
      }
      const float mb = m_run == -INFINITY ? 0.f : m_run;
      {
        const uint64_t sc2 = f2_make(a.scale_log2, a.scale_log2), nm2 = f2_make(-mb, -mb);
        uint64_t acc0 = f2_make(0.f, 0.f), acc1 = f2_make(0.f, 0.f);
        softmax_emit32<NP0>(s0, t_s + hf * 64, sc2, nm2, acc0, acc1);
        softmax_emit32<NP1>(s1, t_s + hf * 64 + 16, sc2, nm2, acc0, acc1);
        float r0, r1, r2, r3;
        f2_split(acc0, r0, r1);
        f2_split(acc1, r2, r3);
        l_run += (r0 + r1) + (r2 + r3);
      }
      long long c_d = clock64();
      p2 += c_d - c_c;
      if (__any_sync(0xffffffffu, rescale)) {
        ++nres;
        const bool g2 = mbar_wait(&o_done[t], (cnt - 1) & 1, a.err, kErrTimeoutEpilogue, abort_flag);
        if (!__all_sync(0xffffffffu, g2)) { alive = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < HH; c += 16) {
          float o[16];
          tmem_ld16(t_o + c, o);
          tmem_wait_ld();
          uint32_t ou[16];
#pragma unroll
          for (int u = 0; u < 16; ++u) ou[u] = __float_as_uint(o[u] * alpha);
          tmem_st16(t_o + c, ou);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
      p3 += clock64() - c_d;
    }
    if (a.prof && lane == 0) {
      atomicAdd(&a.prof[0], pw);
      atomicAdd(&a.prof[1], p1);
      atomicAdd(&a.prof[2], p2);
      atomicAdd(&a.prof[3], p3);
      atomicAdd(&a.prof[7], (unsigned long long)cnt);
      atomicAdd(&a.prof[8], nres);
    }
    if (alive && cnt > 0) {
      xsum[(t * 2 + hf) * BM + row] = l_run;
      mbar_arrive(xb);
      bool got = mbar_wait(xb, cnt & 1, a.err, kErrTimeoutEpilogue, abort_flag);
      got = got && mbar_wait(&o_done[t], (cnt - 1) & 1, a.err, kErrTimeoutEpilogue, abort_flag);
      if (__all_sync(0xffffffffu, got)) {
        tc_fence_after();
        const float l_tot = l_run + xsum[(t * 2 + (hf ^ 1)) * BM + row];
        const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
        __nv_bfloat16* orow = a.o + ((long)(base + qi) * a.H + h) * HD + hf * HH;
#pragma unroll 1
        for (int c = 0; c < HH; c += 16) {
          float o[16];
          tmem_ld16(t_o + c, o);
          tmem_wait_ld();
          if (qi < a.S) {
            uint32_t pkd[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) pkd[u] = pack_bf16x2(o[2 * u] * inv, o[2 * u + 1] * inv);
            reinterpret_cast<uint4*>(orow + c)[0] = make_uint4(pkd[0], pkd[1], pkd[2], pkd[3]);
            reinterpret_cast<uint4*>(orow + c)[1] = make_uint4(pkd[4], pkd[5], pkd[6], pkd[7]);
          }
        }
        if (qi < a.S && hf == 0)
          a.lse[(long)(base + qi) * a.H + h] = l_tot > 0.f ? (m_run + log2f(l_tot)) * 0.6931471805599453f : INFINITY;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 16) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Separate-P forward (HD <= 96): keys in blocks of BNS = 96, so that each tile's S (96 columns)
// and P (48 columns of bf16 pairs) no longer share TMEM columns. The softmax releases S as soon as
// it has loaded it, the MMA thread then computes the tile's next S while the exponentials still run,
// and only the P buffer waits for the previous PV. Per tile the chain becomes
//   softmax_j (S_{j+1} computed meanwhile) -> softmax_{j+1} ...
// instead of softmax_j -> PV_j -> S_{j+1} -> softmax_{j+1}.
// TMEM: S0 [0, 96), S1 [128, 224), O0 [256, 256 + HD), O1 [384, 384 + HD); P_t in the spare columns
// (k-steps 0-3 of P0 at 96.., 4-5 at 224..; of P1 at 352.., 480..). Warps 0-3 / 4-7 softmax of tile
// 0 / 1 (thread = query row), warp 8 MMA, warp 9 TMA; three K / V stages.
constexpr int BNS = 96;
constexpr int kStagesSP = 3;

template <int HD>
struct SmemSP {
  static constexpr int KCH = (HD + 63) / 64;
  static constexpr int kTileQ = KCH * BM * 128;   // [128 rows x HD] in 64-column chunks
  static constexpr int kTileKV = KCH * BNS * 128;  // [96 rows x HD]
  static constexpr int kBarOff = 2 * kTileQ + 2 * kStagesSP * kTileKV;
  static constexpr int kBytes = kBarOff + 256 + 1024;
};

// TMEM column of P's k-step ks (16 keys = 8 columns of bf16 pairs) for tile t
__device__ __forceinline__ uint32_t p_col(int t, int ks) {
  const uint32_t b0 = t ? 352u : 96u, b1 = t ? 480u : 224u;
  return ks < 4 ? b0 + ks * 8 : b1 + (ks - 4) * 8;
}

template <int NP>
__device__ __forceinline__ void softmax_pack32(const float (&sv)[32], uint32_t (&w)[16], uint64_t sc2, uint64_t nm2,
                                               uint64_t& acc0, uint64_t& acc1) {
#pragma unroll
  for (int c = 0; c < 32; c += 2) {
    const uint64_t x = f2_fma(f2_make(sv[c], sv[c + 1]), sc2, nm2);
    float x0, x1, e0, e1;
    f2_split(x, x0, x1);
    if (c / 2 < NP) {
      ex2_poly2(x0, x1, e0, e1);
    } else {
      e0 = ex2_sfu(x0);
      e1 = ex2_sfu(x1);
    }
    if ((c / 2) & 1) acc1 = f2_add(acc1, f2_make(e0, e1));
    else acc0 = f2_add(acc0, f2_make(e0, e1));
    w[c / 2] = pack_bf16x2(e0, e1);
  }
}

template <int HD>
__global__ void __launch_bounds__(kThreadsPP, 1)
    fa_fwd_sm100_sp_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const FwdArgs a) {
  static_assert(HD <= 96, "separate-P layout needs O to fit 96 columns per tile");
  using SM = SmemSP<HD>;
  constexpr int KCH = SM::KCH;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                    // [2][tileQ]
  uint8_t* sK = smem + 2 * SM::kTileQ;   // [stages][tileKV]
  uint8_t* sV = sK + kStagesSP * SM::kTileKV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::kBarOff);
  uint64_t* q_full = bars + 0;
  uint64_t* kv_full = bars + 1;                 // [stages]
  uint64_t* kv_empty = bars + 1 + kStagesSP;    // [stages]
  uint64_t* s_full = bars + 1 + 2 * kStagesSP;  // [2] per tile
  uint64_t* s_free = s_full + 2;                // [2] per tile, 128 arrivals
  uint64_t* p_full = s_full + 4;                // [2] per tile, 128 arrivals
  uint64_t* o_done = s_full + 6;                // [2] per tile
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Longest first (see fa_fwd_sm100_kernel).
  const int lin = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  const int nhb = gridDim.y * gridDim.z;
  const int h = (lin % nhb) % gridDim.y, b = (lin % nhb) / gridDim.y;
  const int kh = h / (a.H / a.Hkv);
  const int q0 = (gridDim.x - 1 - lin / nhb) * 2 * BM;
  const int base = b * a.S;
  int kb_lo = 0;
  if (a.window > 0) kb_lo = max(0, q0 - a.window + 1) / BNS;
  const int kb_hi1 = (min(a.S, q0 + 2 * BM) + BNS - 1) / BNS;
  const int kb_hi0 = (min(a.S, q0 + BM) + BNS - 1) / BNS;
  const int nb = max(kb_hi1 - kb_lo, 0);
  int lo_t[2], nb_t[2];
  nb_t[0] = max(kb_hi0 - kb_lo, 0);
  nb_t[1] = nb;
  lo_t[0] = 0;
  lo_t[1] = 0;
  if (a.window > 0) lo_t[1] = max(0, (q0 + BM - a.window + 1) / BNS - kb_lo);
  if (q0 + BM >= a.S) nb_t[1] = 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kStagesSP; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 9) {
    // ------------------------------------------------------------------------ TMA producer
    if (lane == 0 && nb > 0) {
      mbar_arrive_expect_tx(q_full, 2 * SM::kTileQ);
      for (int t = 0; t < 2; ++t)
        for (int c = 0; c < KCH; ++c)
          tma_load_2d(&tmQ, q_full, sQ + t * SM::kTileQ + c * BM * 128, a.q_x0 + h * HD + c * 64,
                      base + q0 + t * BM);
      for (int j = 0; j < nb; ++j) {
        const int st = j % kStagesSP;
        const int kr = base + (kb_lo + j) * BNS;
        if (!mbar_wait(&kv_empty[st], ((j / kStagesSP) & 1) ^ 1, a.err, kErrTimeoutProducer, abort_flag)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * SM::kTileKV);
        for (int c = 0; c < KCH; ++c) {
          tma_load_2d(&tmK, &kv_full[st], sK + st * SM::kTileKV + c * BNS * 128, a.k_x0 + kh * HD + c * 64, kr);
          tma_load_2d(&tmV, &kv_full[st], sV + st * SM::kTileKV + c * BNS * 128, a.v_x0 + kh * HD + c * 64, kr);
        }
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------------------ MMA issuer
    if (lane == 0 && nb > 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BM, BNS, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(BM, HD, false, true);
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      auto issue_s = [&](int t, int st) {
        const uint32_t qa = q_addr + t * SM::kTileQ, ka = k_addr + st * SM::kTileKV;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
          const uint32_t oq = (ks / 4) * BM * 128 + (ks % 4) * 32, ok_ = (ks / 4) * BNS * 128 + (ks % 4) * 32;
          umma_bf16(tmem + t * 128, make_sdesc(qa + oq, 16, 1024), make_sdesc(ka + ok_, 16, 1024), idesc_s,
                    ks > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int st, bool acc) {
        const uint32_t va = v_addr + st * SM::kTileKV;
#pragma unroll
        for (int ks = 0; ks < BNS / 16; ++ks)
          umma_ts_bf16(tmem + 256 + t * 128, tmem + p_col(t, ks), make_sdesc(va + ks * 2048, BNS * 128, 1024),
                       idesc_o, (acc || ks > 0) ? 1u : 0u);
        umma_commit(&o_done[t]);
      };
      // Event loop: each pass issues every product whose inputs are ready, so neither tile waits
      // behind the other. Tile t's S for block j needs K_j and its S of block j - 1 loaded by the
      // softmax (s_free); its PV for block j needs P_j (p_full). A K / V stage is released once
      // every active tile has issued its PV for that block. Each barrier can run at most one phase
      // ahead of the parity tested here (a softmax cannot load an S or store a P that was not
      // issued or whose previous PV is outstanding), so the parity tests are unambiguous.
      unsigned long long wp = 0, wkv = 0, ws = 0;
      bool ok = mbar_wait(q_full, 0, a.err, kErrTimeoutMma, abort_flag);
      int ns[2] = {lo_t[0], lo_t[1]}, np[2] = {lo_t[0], lo_t[1]};
      int rel = 0;
      long long t_last = clock64(), t_iter = t_last;
      while (ok) {
        bool prog = false;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (ns[t] < nb_t[t]) {
            const int j = ns[t];
            bool ready = mbar_test(&kv_full[j % kStagesSP], (j / kStagesSP) & 1);
            if (ready && j > lo_t[t]) ready = mbar_test(&s_free[t], (j - 1 - lo_t[t]) & 1);
            if (ready) {
              tc_fence_after();
              issue_s(t, j % kStagesSP);
              ++ns[t];
              prog = true;
            }
          }
          if (np[t] < ns[t]) {
            const int j = np[t];
            if (mbar_test(&p_full[t], (j - lo_t[t]) & 1)) {
              tc_fence_after();
              issue_pv(t, j % kStagesSP, j > lo_t[t]);
              ++np[t];
              prog = true;
            }
          }
        }
        while (rel < nb) {
          bool done = true;
#pragma unroll
          for (int t = 0; t < 2; ++t)
            if (rel >= lo_t[t] && rel < nb_t[t] && np[t] <= rel) done = false;
          if (!done) break;
          umma_commit(&kv_empty[rel % kStagesSP]);
          ++rel;
        }
        if (rel >= nb && np[0] >= nb_t[0] && np[1] >= nb_t[1]) break;
        const long long now = clock64();
        if (prog) {
          t_last = now;
        } else {
          wp += now - t_iter;  // cycles spent polling with nothing ready
          if (*abort_flag) break;
          if (now - t_last > kWaitCycles) {
            atomicExch(a.err, kErrTimeoutMma);
            *abort_flag = 1;
            break;
          }
        }
        t_iter = now;
      }
      if (a.prof) {
        atomicAdd(&a.prof[4], wp);
        atomicAdd(&a.prof[5], wkv);
        atomicAdd(&a.prof[6], ws);
      }
    }
  } else {
    // ------------------------------------------------------------------------ softmax warps
    const int t = warp >> 2;
    const int row = (warp & 3) * 32 + lane;
    const int qi = q0 + t * BM + row;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + t * 128 + lane_off;
    const uint32_t t_o = tmem + 256 + t * 128 + lane_off;
    int klo, khi;
    key_range(qi, a.S, a.window, a.seg, base, klo, khi);
    float m_run = -INFINITY, l_run = 0.f;
    bool alive = true;
    int cnt = 0;
    unsigned long long pw = 0, p1 = 0, p2 = 0, p3 = 0, nres = 0;
    for (int j = lo_t[t]; j < nb_t[t]; ++j, ++cnt) {
      long long c_a = clock64();
      const bool got = mbar_wait(&s_full[t], cnt & 1, a.err, kErrTimeoutEpilogue, abort_flag);
      long long c_b = clock64();
      pw += c_b - c_a;
      if (!__all_sync(0xffffffffu, got)) { alive = false; break; }
      tc_fence_after();
      float s0[32], s1[32], s2[32];
      tmem_ld32(t_s + 0, s0);
      tmem_ld32(t_s + 32, s1);
      tmem_ld32(t_s + 64, s2);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_free[t]);  // the MMA thread may now overwrite S with the next block's
      const int k0 = (kb_lo + j) * BNS;
      const int lo = klo - k0, hi = khi - k0;  // visible columns [lo, hi] of this block
      if (!(lo <= 0 && hi >= BNS - 1)) {
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          if (c < lo || c > hi) s0[c] = -INFINITY;
          if (c + 32 < lo || c + 32 > hi) s1[c] = -INFINITY;
          if (c + 64 < lo || c + 64 > hi) s2[c] = -INFINITY;
        }
      }
      float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
      for (int c = 0; c < 32; c += 2) {
        mxa = fmaxf(mxa, fmaxf(fmaxf(s0[c], s1[c]), s2[c]));
        mxb = fmaxf(mxb, fmaxf(fmaxf(s0[c + 1], s1[c + 1]), s2[c + 1]));
      }
      const float mx = fmaxf(mxa, mxb) * a.scale_log2;
      long long c_c = clock64();
      p1 += c_c - c_b;
      float alpha = 1.f;
      bool rescale = false;
      if (mx > m_run + kRescaleThreshold || (m_run == -INFINITY && mx > -INFINITY)) {
        if (m_run != -INFINITY) {
          alpha = exp2f(m_run - mx);
          rescale = true;
        }
        m_run = mx;
        l_run *= alpha;
      }
      const float mb = m_run == -INFINITY ? 0.f : m_run;
      uint32_t w0[16], w1[16], w2[16];
      {
        const uint64_t sc2 = f2_make(a.scale_log2, a.scale_log2), nm2 = f2_make(-mb, -mb);
        uint64_t acc0 = f2_make(0.f, 0.f), acc1 = f2_make(0.f, 0.f);
        softmax_pack32<4>(s0, w0, sc2, nm2, acc0, acc1);
        softmax_pack32<4>(s1, w1, sc2, nm2, acc0, acc1);
        softmax_pack32<4>(s2, w2, sc2, nm2, acc0, acc1);
        float r0, r1, r2, r3;
        f2_split(acc0, r0, r1);
        f2_split(acc1, r2, r3);
        l_run += (r0 + r1) + (r2 + r3);
      }
      long long c_d = clock64();
      p2 += c_d - c_c;
      // P's buffer and O are free once the previous block's PV has completed
      if (cnt > 0) {
        const bool g2 = mbar_wait(&o_done[t], (cnt - 1) & 1, a.err, kErrTimeoutEpilogue, abort_flag);
        if (!__all_sync(0xffffffffu, g2)) { alive = false; break; }
        tc_fence_after();
      }
      if (__any_sync(0xffffffffu, rescale)) {
        ++nres;
#pragma unroll 1
        for (int c = 0; c < HD; c += 16) {
          float o[16];
          tmem_ld16(t_o + c, o);
          tmem_wait_ld();
          uint32_t ou[16];
#pragma unroll
          for (int u = 0; u < 16; ++u) ou[u] = __float_as_uint(o[u] * alpha);
          tmem_st16(t_o + c, ou);
        }
      }
      tmem_st16(tmem + lane_off + p_col(t, 0), w0);
      tmem_st16(tmem + lane_off + p_col(t, 2), w1);
      tmem_st16(tmem + lane_off + p_col(t, 4), w2);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&p_full[t]);
      p3 += clock64() - c_d;
    }
    if (a.prof && lane == 0) {
      atomicAdd(&a.prof[0], pw);
      atomicAdd(&a.prof[1], p1);
      atomicAdd(&a.prof[2], p2);
      atomicAdd(&a.prof[3], p3);
      atomicAdd(&a.prof[7], (unsigned long long)cnt);
      atomicAdd(&a.prof[8], nres);
    }
    if (alive && cnt > 0) {
      const bool got = mbar_wait(&o_done[t], (cnt - 1) & 1, a.err, kErrTimeoutEpilogue, abort_flag);
      if (__all_sync(0xffffffffu, got)) {
        tc_fence_after();
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        __nv_bfloat16* orow = a.o + ((long)(base + qi) * a.H + h) * HD;
#pragma unroll 1
        for (int c = 0; c < HD; c += 16) {
          float o[16];
          tmem_ld16(t_o + c, o);
          tmem_wait_ld();
          if (qi < a.S) {
            uint32_t pkd[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) pkd[u] = pack_bf16x2(o[2 * u] * inv, o[2 * u + 1] * inv);
            reinterpret_cast<uint4*>(orow + c)[0] = make_uint4(pkd[0], pkd[1], pkd[2], pkd[3]);
            reinterpret_cast<uint4*>(orow + c)[1] = make_uint4(pkd[4], pkd[5], pkd[6], pkd[7]);
          }
        }
        if (qi < a.S)
          a.lse[(long)(base + qi) * a.H + h] = l_run > 0.f ? (m_run + log2f(l_run)) * 0.6931471805599453f : INFINITY;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Persistent separate-P forward: one CTA per SM loops over work items (a pair of 128-query tiles of
// one head), so a CTA's start-up -- TMEM allocation, barrier set-up, the Q load and the first K / V
// loads -- is paid once, and each item's epilogue (O normalised and stored by the softmax warps)
// overlaps the next item's Q / K / V loads and first S products. Items are taken round-robin in the
// longest-first order. Measured slower than the one-item-per-CTA kernel (0.222 vs 0.201 ms on
// 8 x 2048 x 16 x 96 causal): the static round-robin of causal items of very different lengths
// leaves some SMs with more work than others, which the hardware's dynamic CTA scheduling avoids;
// kept opt-in (MXK_ATTN_FWD=spp). Every barrier keeps counting phases across items: the MMA issuer and the
// softmax warps track global S / PV / block counts per tile; O is reused by the next item's first PV
// only after the softmax warps have read it (o_free), and Q only after the item's last S (q_empty).
struct SpItem {
  int h, b, kh, q0, base, kb_lo, nb, lo_t[2], nb_t[2];
};

__device__ __forceinline__ SpItem sp_item(int item, const FwdArgs& a, int nqt) {
  SpItem w;
  const int nhb = a.H * a.B;
  w.h = (item % nhb) % a.H;
  w.b = (item % nhb) / a.H;
  w.kh = w.h / (a.H / a.Hkv);
  w.q0 = (nqt - 1 - item / nhb) * 2 * BM;
  w.base = w.b * a.S;
  w.kb_lo = 0;
  if (a.window > 0) w.kb_lo = max(0, w.q0 - a.window + 1) / BNS;
  const int kb_hi1 = (min(a.S, w.q0 + 2 * BM) + BNS - 1) / BNS;
  const int kb_hi0 = (min(a.S, w.q0 + BM) + BNS - 1) / BNS;
  w.nb = max(kb_hi1 - w.kb_lo, 0);
  w.nb_t[0] = max(kb_hi0 - w.kb_lo, 0);
  w.nb_t[1] = w.nb;
  w.lo_t[0] = 0;
  w.lo_t[1] = 0;
  if (a.window > 0) w.lo_t[1] = max(0, (w.q0 + BM - a.window + 1) / BNS - w.kb_lo);
  if (w.q0 + BM >= a.S) w.nb_t[1] = 0;
  return w;
}

template <int HD>
__global__ void __launch_bounds__(kThreadsPP, 1)
    fa_fwd_sm100_spp_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, const FwdArgs a, int n_items) {
  static_assert(HD <= 96, "separate-P layout needs O to fit 96 columns per tile");
  using SM = SmemSP<HD>;
  constexpr int KCH = SM::KCH;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + 2 * SM::kTileQ;
  uint8_t* sV = sK + kStagesSP * SM::kTileKV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM::kBarOff);
  uint64_t* q_full = bars + 0;
  uint64_t* q_empty = bars + 1;
  uint64_t* kv_full = bars + 2;                 // [stages]
  uint64_t* kv_empty = bars + 2 + kStagesSP;    // [stages]
  uint64_t* s_full = bars + 2 + 2 * kStagesSP;  // [2] per tile
  uint64_t* s_free = s_full + 2;                // [2], 128 arrivals
  uint64_t* p_full = s_full + 4;                // [2], 128 arrivals
  uint64_t* o_done = s_full + 6;                // [2]
  uint64_t* o_free = s_full + 8;                // [2], 128 arrivals
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(s_full + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nqt = (a.S + 2 * BM - 1) / (2 * BM);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < kStagesSP; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
      mbar_init(&o_free[i], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 8) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 9) {
    // ------------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int qi = 0;
      long kvc = 0;  // global K / V block count: stage and phase
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const SpItem w = sp_item(item, a, nqt);
        if (w.nb == 0) continue;
        if (!mbar_wait(q_empty, (qi & 1) ^ 1, a.err, kErrTimeoutProducer, abort_flag)) break;
        mbar_arrive_expect_tx(q_full, 2 * SM::kTileQ);
        for (int t = 0; t < 2; ++t)
          for (int c = 0; c < KCH; ++c)
            tma_load_2d(&tmQ, q_full, sQ + t * SM::kTileQ + c * BM * 128, a.q_x0 + w.h * HD + c * 64,
                        w.base + w.q0 + t * BM);
        ++qi;
        for (int j = 0; j < w.nb; ++j, ++kvc) {
          const int st = (int)(kvc % kStagesSP);
          const int kr = w.base + (w.kb_lo + j) * BNS;
          if (!mbar_wait(&kv_empty[st], ((kvc / kStagesSP) & 1) ^ 1, a.err, kErrTimeoutProducer, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[st], 2 * SM::kTileKV);
          for (int c = 0; c < KCH; ++c) {
            tma_load_2d(&tmK, &kv_full[st], sK + st * SM::kTileKV + c * BNS * 128, a.k_x0 + w.kh * HD + c * 64, kr);
            tma_load_2d(&tmV, &kv_full[st], sV + st * SM::kTileKV + c * BNS * 128, a.v_x0 + w.kh * HD + c * 64, kr);
          }
        }
      }
    }
  } else if (warp == 8) {
    // ------------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16(BM, BNS, false, false);
      constexpr uint32_t idesc_o = make_idesc_bf16(BM, HD, false, true);
      const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      long gs[2] = {0, 0}, gp[2] = {0, 0};  // global S / PV counts per tile
      int oi[2] = {0, 0};                    // items whose O tile t has drained
      int qi = 0;
      long kvc0 = 0;  // global index of the item's first K / V block
      bool ok = true;
      unsigned long long wp = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const SpItem w = sp_item(item, a, nqt);
        if (w.nb == 0) continue;
        if (!mbar_wait(q_full, qi & 1, a.err, kErrTimeoutMma, abort_flag)) break;
        ++qi;
        auto issue_s = [&](int t, long kb) {
          const int st = (int)(kb % kStagesSP);
          const uint32_t qa = q_addr + t * SM::kTileQ, ka = k_addr + st * SM::kTileKV;
#pragma unroll
          for (int ks = 0; ks < HD / 16; ++ks) {
            const uint32_t oq = (ks / 4) * BM * 128 + (ks % 4) * 32, ok_ = (ks / 4) * BNS * 128 + (ks % 4) * 32;
            umma_bf16(tmem + t * 128, make_sdesc(qa + oq, 16, 1024), make_sdesc(ka + ok_, 16, 1024), idesc_s,
                      ks > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[t]);
        };
        auto issue_pv = [&](int t, long kb, bool acc) {
          const uint32_t va = v_addr + (int)(kb % kStagesSP) * SM::kTileKV;
#pragma unroll
          for (int ks = 0; ks < BNS / 16; ++ks)
            umma_ts_bf16(tmem + 256 + t * 128, tmem + p_col(t, ks), make_sdesc(va + ks * 2048, BNS * 128, 1024),
                         idesc_o, (acc || ks > 0) ? 1u : 0u);
          umma_commit(&o_done[t]);
        };
        int ns[2] = {w.lo_t[0], w.lo_t[1]}, np[2] = {w.lo_t[0], w.lo_t[1]};
        int rel = 0;
        long long t_last = clock64(), t_iter = t_last;
        while (true) {
          bool prog = false;
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (ns[t] < w.nb_t[t]) {
              const long kb = kvc0 + ns[t];
              bool ready = mbar_test(&kv_full[kb % kStagesSP], (kb / kStagesSP) & 1);
              if (ready && gs[t] > 0) ready = mbar_test(&s_free[t], (gs[t] - 1) & 1);
              if (ready) {
                tc_fence_after();
                issue_s(t, kb);
                ++ns[t];
                ++gs[t];
                prog = true;
              }
            }
            if (np[t] < ns[t]) {
              const bool first = np[t] == w.lo_t[t];
              bool ready = mbar_test(&p_full[t], gp[t] & 1);
              if (ready && first && oi[t] > 0) ready = mbar_test(&o_free[t], (oi[t] - 1) & 1);
              if (ready) {
                tc_fence_after();
                issue_pv(t, kvc0 + np[t], !first);
                ++np[t];
                ++gp[t];
                prog = true;
              }
            }
          }
          while (rel < w.nb) {
            bool done = true;
#pragma unroll
            for (int t = 0; t < 2; ++t)
              if (rel >= w.lo_t[t] && rel < w.nb_t[t] && np[t] <= rel) done = false;
            if (!done) break;
            umma_commit(&kv_empty[(kvc0 + rel) % kStagesSP]);
            ++rel;
          }
          if (rel >= w.nb && np[0] >= w.nb_t[0] && np[1] >= w.nb_t[1]) break;
          const long long now = clock64();
          if (prog) {
            t_last = now;
          } else {
            wp += now - t_iter;
            if (*abort_flag) {
              ok = false;
              break;
            }
            if (now - t_last > kWaitCycles) {
              atomicExch(a.err, kErrTimeoutMma);
              *abort_flag = 1;
              ok = false;
              break;
            }
          }
          t_iter = now;
        }
        umma_commit(q_empty);  // Q is free once this item's S products have completed
        kvc0 += w.nb;
        for (int t = 0; t < 2; ++t)
          if (w.nb_t[t] > w.lo_t[t]) ++oi[t];
      }
      if (a.prof) atomicAdd(&a.prof[4], wp);
    }
  } else {
    // ------------------------------------------------------------------------ softmax warps
    const int t = warp >> 2;
    const int row = (warp & 3) * 32 + lane;
    const uint32_t lane_off = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t t_s = tmem + t * 128 + lane_off;
    const uint32_t t_o = tmem + 256 + t * 128 + lane_off;
    long gcnt = 0;  // global blocks of this tile
    bool alive = true;
    unsigned long long pw = 0, p1 = 0, p2 = 0, p3 = 0, nblk = 0;
    for (int item = blockIdx.x; item < n_items && alive; item += gridDim.x) {
      const SpItem w = sp_item(item, a, nqt);
      if (w.nb == 0 || w.nb_t[t] <= w.lo_t[t]) continue;
      const int qi = w.q0 + t * BM + row;
      int klo, khi;
      key_range(qi, a.S, a.window, a.seg, w.base, klo, khi);
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = w.lo_t[t]; j < w.nb_t[t]; ++j, ++gcnt) {
        long long c_a = clock64();
        const bool got = mbar_wait(&s_full[t], gcnt & 1, a.err, kErrTimeoutEpilogue, abort_flag);
        long long c_b = clock64();
        pw += c_b - c_a;
        if (!__all_sync(0xffffffffu, got)) { alive = false; break; }
        tc_fence_after();
        float s0[32], s1[32], s2[32];
        tmem_ld32(t_s + 0, s0);
        tmem_ld32(t_s + 32, s1);
        tmem_ld32(t_s + 64, s2);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&s_free[t]);
        const int k0 = (w.kb_lo + j) * BNS;
        const int lo = klo - k0, hi = khi - k0;
        if (!(lo <= 0 && hi >= BNS - 1)) {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            if (c < lo || c > hi) s0[c] = -INFINITY;
            if (c + 32 < lo || c + 32 > hi) s1[c] = -INFINITY;
            if (c + 64 < lo || c + 64 > hi) s2[c] = -INFINITY;
          }
        }
        float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
        for (int c = 0; c < 32; c += 2) {
          mxa = fmaxf(mxa, fmaxf(fmaxf(s0[c], s1[c]), s2[c]));
          mxb = fmaxf(mxb, fmaxf(fmaxf(s0[c + 1], s1[c + 1]), s2[c + 1]));
        }
        const float mx = fmaxf(mxa, mxb) * a.scale_log2;
        long long c_c = clock64();
        p1 += c_c - c_b;
        float alpha = 1.f;
        bool rescale = false;
        if (mx > m_run + kRescaleThreshold || (m_run == -INFINITY && mx > -INFINITY)) {
          if (m_run != -INFINITY) {
            alpha = exp2f(m_run - mx);
            rescale = true;
          }
          m_run = mx;
          l_run *= alpha;
        }
        const float mb = m_run == -INFINITY ? 0.f : m_run;
        uint32_t w0[16], w1[16], w2[16];
        {
          const uint64_t sc2 = f2_make(a.scale_log2, a.scale_log2), nm2 = f2_make(-mb, -mb);
          uint64_t acc0 = f2_make(0.f, 0.f), acc1 = f2_make(0.f, 0.f);
          softmax_pack32<4>(s0, w0, sc2, nm2, acc0, acc1);
          softmax_pack32<4>(s1, w1, sc2, nm2, acc0, acc1);
          softmax_pack32<4>(s2, w2, sc2, nm2, acc0, acc1);
          float r0, r1, r2, r3;
          f2_split(acc0, r0, r1);
          f2_split(acc1, r2, r3);
          l_run += (r0 + r1) + (r2 + r3);
        }
        long long c_d = clock64();
        p2 += c_d - c_c;
        // P's buffer (and O for a rescale) are free once the previous PV of this tile completed
        if (gcnt > 0) {
          const bool g2 = mbar_wait(&o_done[t], (gcnt - 1) & 1, a.err, kErrTimeoutEpilogue, abort_flag);
          if (!__all_sync(0xffffffffu, g2)) { alive = false; break; }
          tc_fence_after();
        }
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
          for (int c = 0; c < HD; c += 16) {
            float o[16];
            tmem_ld16(t_o + c, o);
            tmem_wait_ld();
            uint32_t ou[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) ou[u] = __float_as_uint(o[u] * alpha);
            tmem_st16(t_o + c, ou);
          }
        }
        tmem_st16(tmem + lane_off + p_col(t, 0), w0);
        tmem_st16(tmem + lane_off + p_col(t, 2), w1);
        tmem_st16(tmem + lane_off + p_col(t, 4), w2);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[t]);
        p3 += clock64() - c_d;
        ++nblk;
      }
      if (!alive) break;
      // epilogue: the item's last PV, then O normalised and stored; O is then free for the next item
      const bool got = mbar_wait(&o_done[t], (gcnt - 1) & 1, a.err, kErrTimeoutEpilogue, abort_flag);
      if (!__all_sync(0xffffffffu, got)) { alive = false; break; }
      tc_fence_after();
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      __nv_bfloat16* orow = a.o + ((long)(w.base + qi) * a.H + w.h) * HD;
#pragma unroll 1
      for (int c = 0; c < HD; c += 16) {
        float o[16];
        tmem_ld16(t_o + c, o);
        tmem_wait_ld();
        if (qi < a.S) {
          uint32_t pkd[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) pkd[u] = pack_bf16x2(o[2 * u] * inv, o[2 * u + 1] * inv);
          reinterpret_cast<uint4*>(orow + c)[0] = make_uint4(pkd[0], pkd[1], pkd[2], pkd[3]);
          reinterpret_cast<uint4*>(orow + c)[1] = make_uint4(pkd[4], pkd[5], pkd[6], pkd[7]);
        }
      }
      tc_fence_before();
      mbar_arrive(&o_free[t]);
      if (qi < a.S)
        a.lse[(long)(w.base + qi) * a.H + w.h] = l_run > 0.f ? (m_run + log2f(l_run)) * 0.6931471805599453f : INFINITY;
    }
    if (a.prof && lane == 0) {
      atomicAdd(&a.prof[0], pw);
      atomicAdd(&a.prof[1], p1);
      atomicAdd(&a.prof[2], p2);
      atomicAdd(&a.prof[3], p3);
      atomicAdd(&a.prof[7], nblk);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace fa100

bool make_tmap_bf16_2d(CUtensorMap* m, const void* ptr, int64_t inner, int64_t outer, int64_t ld, int box_inner,
                       int box_outer);

template <int HD>
static int run_fa_fwd_sm100(const AttnLaunch& L, int* err, cudaStream_t st) {
  using namespace fa100;
  CUtensorMap tq, tk, tv;
  const long T = (long)L.B * L.S;
  // 2-D maps over [tokens, row elements]; a head's 64-wide chunk starts at x = head * hd + 64 c
  // inner extent = the heads actually present (columns past it read as zero, never past the buffer)
  if (!make_tmap_bf16_2d(&tq, L.q, (long)L.H * HD, T, L.q_tok, 64, BM)) return kErrBadArgsHost;
  if (!make_tmap_bf16_2d(&tk, L.k, (long)L.Hkv * HD, T, L.k_tok, 64, BN)) return kErrBadArgsHost;
  if (!make_tmap_bf16_2d(&tv, L.v, (long)L.Hkv * HD, T, L.v_tok, 64, BN)) return kErrBadArgsHost;
  FwdArgs a{};
  a.B = L.B; a.S = L.S; a.H = L.H; a.Hkv = L.Hkv; a.hd = HD; a.window = L.window;
  a.scale_log2 = L.scale * 1.4426950408889634f;
  a.seg = L.seg;
  a.o = (__nv_bfloat16*)L.o;
  a.lse = L.lse;
  a.q_x0 = 0; a.k_x0 = 0; a.v_x0 = 0;
  a.err = err;
  a.prof = (unsigned long long*)L.prof;
  dim3 grid((L.S + 2 * BM - 1) / (2 * BM), L.H, L.B);
  // MXK_ATTN_FWD: "sp" (default for head dimensions <= 96: 96-key blocks with S and P in separate
  // TMEM columns; 0.193-0.198 ms against 0.205 ms for "split" on 8 x 2048 x 16 x 96 causal),
  // "split" (eight softmax warps per tile; the default above 96) or "pp" (four per tile)
  static const int variant = [] {
    const char* e = getenv("MXK_ATTN_FWD");
    const std::string v = e ? e : "sp";
    return v == "pp" ? 0 : v == "split" ? 1 : v == "spp" ? 3 : 2;
  }();
  if constexpr (HD <= 96) {
    if (variant == 3) {  // persistent separate-P: one CTA per SM looping over the work items
      CUtensorMap tk96, tv96;
      if (!make_tmap_bf16_2d(&tk96, L.k, (long)L.Hkv * HD, T, L.k_tok, 64, BNS)) return kErrBadArgsHost;
      if (!make_tmap_bf16_2d(&tv96, L.v, (long)L.Hkv * HD, T, L.v_tok, 64, BNS)) return kErrBadArgsHost;
      constexpr int smem = SmemSP<HD>::kBytes;
      static bool init = false;
      static int sms = 0;
      if (!init) {
        if (cudaFuncSetAttribute(fa_fwd_sm100_spp_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
          return kErrBadArgsHost;
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        init = true;
      }
      const int n_items = (int)(grid.x * grid.y * grid.z);
      count_launch();
      fa_fwd_sm100_spp_kernel<HD><<<min(n_items, sms), kThreadsPP, smem, st>>>(tq, tk96, tv96, a, n_items);
      return cudaGetLastError() == cudaSuccess ? 0 : kErrBadArgsHost;
    }
    if (variant == 2) {
      CUtensorMap tk96, tv96;
      if (!make_tmap_bf16_2d(&tk96, L.k, (long)L.Hkv * HD, T, L.k_tok, 64, BNS)) return kErrBadArgsHost;
      if (!make_tmap_bf16_2d(&tv96, L.v, (long)L.Hkv * HD, T, L.v_tok, 64, BNS)) return kErrBadArgsHost;
      constexpr int smem = SmemSP<HD>::kBytes;
      static bool init = false;
      if (!init) {
        if (cudaFuncSetAttribute(fa_fwd_sm100_sp_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
            cudaSuccess)
          return kErrBadArgsHost;
        init = true;
      }
      count_launch();
      fa_fwd_sm100_sp_kernel<HD><<<grid, kThreadsPP, smem, st>>>(tq, tk96, tv96, a);
      return cudaGetLastError() == cudaSuccess ? 0 : kErrBadArgsHost;
    }
  }
  const bool split = variant != 0;
  if (split) {
    // share of the exponentials on the FMA pipe (MXK_ATTN_POLY: 25, 50 or 75 percent). Measured on
    // one B200 (8 x 2048, 16 x 96, causal): 0.206 / 0.218 / 0.219 ms -- the special-function unit
    // is not the limiter (27 % busy), so a quarter stays the default
    static const int poly = [] {
      const char* e = getenv("MXK_ATTN_POLY");
      return e ? atoi(e) : 25;
    }();
    constexpr int smem = SmemSR<HD>::kBytes;
    static bool init = false;
    if (!init) {
      if (cudaFuncSetAttribute(fa_fwd_sm100_split_kernel<HD, 0, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               smem) != cudaSuccess ||
          cudaFuncSetAttribute(fa_fwd_sm100_split_kernel<HD, 8, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               smem) != cudaSuccess ||
          cudaFuncSetAttribute(fa_fwd_sm100_split_kernel<HD, 16, 8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               smem) != cudaSuccess)
        return kErrBadArgsHost;
      init = true;
    }
    count_launch();
    if (poly >= 75)
      fa_fwd_sm100_split_kernel<HD, 16, 8><<<grid, kThreadsSR, smem, st>>>(tq, tk, tv, a);
    else if (poly >= 50)
      fa_fwd_sm100_split_kernel<HD, 8, 8><<<grid, kThreadsSR, smem, st>>>(tq, tk, tv, a);
    else
      fa_fwd_sm100_split_kernel<HD, 0, 8><<<grid, kThreadsSR, smem, st>>>(tq, tk, tv, a);
    return cudaGetLastError() == cudaSuccess ? 0 : kErrBadArgsHost;
  }
  constexpr int smem = Smem<HD>::kBytes;
  static bool init = false;
  if (!init) {
    if (cudaFuncSetAttribute(fa_fwd_sm100_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return kErrBadArgsHost;
    init = true;
  }
  count_launch();
  fa_fwd_sm100_kernel<HD><<<grid, kThreadsPP, smem, st>>>(tq, tk, tv, a);
  return cudaGetLastError() == cudaSuccess ? 0 : kErrBadArgsHost;
}

// q / k / v: row-major [tokens, row] bf16 with the head's hd elements at column head*hd (q: H
// heads, k / v: Hkv heads; v may start at an offset inside a wider row, passed via L.v).
int launch_flash_fwd_sm100(const AttnLaunch& L, int* err, cudaStream_t st) {
  if (L.q_head != L.hd || L.k_head != L.hd || L.v_head != L.hd) return kErrBadArgsHost;
  if ((L.q_tok * 2) % 16 || (L.k_tok * 2) % 16 || (L.v_tok * 2) % 16) return kErrBadArgsHost;
  if ((reinterpret_cast<uintptr_t>(L.q) | reinterpret_cast<uintptr_t>(L.k) | reinterpret_cast<uintptr_t>(L.v)) & 15)
    return kErrBadArgsHost;
  switch (L.hd) {
    case 64: return run_fa_fwd_sm100<64>(L, err, st);
    case 96: return run_fa_fwd_sm100<96>(L, err, st);
    case 128: return run_fa_fwd_sm100<128>(L, err, st);
    default: return kErrBadArgsHost;
  }
}

}  // namespace mxk
