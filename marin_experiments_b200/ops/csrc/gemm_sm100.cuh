// Persistent, warp-specialised bf16 GEMM for sm_100a on the 5th-generation tensor cores.
//
//   C[g] (M x N) = A'[g] (M x K) * B'[g] (N x K)^T        fp32 accumulation in TMEM
//
// A' / B' are each either K-major (stored rows x K, K contiguous) or MN-major (stored K x rows,
// rows contiguous); TMA brings 128-byte-swizzled tiles into shared memory and the UMMA
// descriptors encode the matching canonical layout, so every transpose the forward and backward
// passes need is a descriptor choice instead of a copy.
//
// Grouping: G independent problems that share N and K. Group g reads A rows starting at outer
// coordinate g*a_grp, B rows at g*b_grp and writes C rows starting at g*c_grp. A device array of
// per-group counts makes either M (expert token counts) or K (weight-gradient contraction over
// the tokens an expert received) ragged; tiles past the count are never scheduled.
//
// CTA = 6 warps:  warp 0 = TMA producer, warp 1 = MMA issuer (+ TMEM owner),
//                 warps 2..5 = epilogue (TMEM lane quadrant = warp % 4).
// Accumulators are double-buffered in TMEM (2 x BN fp32 columns) so the epilogue of tile i
// overlaps the main loop of tile i+1. One CTA per SM, grid = min(#tiles, #SMs).
#pragma once
#include "gemm_params.h"
#include "sm100_primitives.cuh"

namespace mxk {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kGemmThreads = 192;
constexpr int kMaxGroups = 512;

enum EpiKind : int {
  EPI_STORE = 0,   // C = alpha*acc (bf16 or f32), or C += alpha*acc (f32, accumulate)
  EPI_SWIGLU = 1,  // BN=256 tile = [gate 128 | up 128]: H = acc (bf16), Act = silu(gate)*up (bf16)
  EPI_RESID = 2,   // C = acc + R (bf16); R may alias C
  EPI_GATE_MUL = 3,  // C = X * sigmoid(acc) (bf16), X given in R (GatedNorm up projection)
  EPI_SILU = 4,    // C = silu(acc) (bf16) and H = acc (bf16) (GatedNorm down projection)
  EPI_ROWSCALE = 5,  // C = acc * row_scale[row] (bf16)
  EPI_CE = 6,      // logits tile: C = acc (bf16) and per-(row, n-tile) max / sum(exp(x - max))
  EPI_ACT = 7,     // non-GLU MLP: H = acc (bf16), C = act(acc) (bf16); act in `act_kind`
};

template <int BN>
struct GemmSmem {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
};

__device__ __forceinline__ int group_count(const GemmParams& p, int g) {
  if (p.counts) return p.counts[g];
  return p.ragged == 2 ? p.K : p.M;
}

// Number of output tiles of group g.
template <int BN>
__device__ __forceinline__ int group_tiles(const GemmParams& p, int g) {
  const int n_tiles = (p.N + BN - 1) / BN;
  if (p.ragged == 1) {
    int cnt = min(group_count(p, g), p.M);
    return ((cnt + kBM - 1) / kBM) * n_tiles;
  }
  int m_tiles = (p.M + kBM - 1) / kBM;
  if (p.ragged == 2) return group_count(p, g) > 0 ? m_tiles * n_tiles : 0;
  return m_tiles * n_tiles;
}

struct TileCoord {
  int g, mt, nt, nkb;
};

template <int BN>
__device__ __forceinline__ TileCoord decode_tile(const GemmParams& p, const int* prefix, int tile) {
  // binary search: largest g with prefix[g] <= tile
  int lo = 0, hi = p.G - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  TileCoord tc;
  tc.g = lo;
  int local = tile - prefix[lo];
  int m_tiles;
  if (p.ragged == 1) {
    int cnt = min(group_count(p, lo), p.M);
    m_tiles = (cnt + kBM - 1) / kBM;
  } else {
    m_tiles = (p.M + kBM - 1) / kBM;
  }
  tc.mt = local % m_tiles;
  tc.nt = local / m_tiles;
  int kext = (p.ragged == 2) ? group_count(p, lo) : p.K;
  tc.nkb = (kext + kBK - 1) / kBK;
  return tc;
}

__device__ __forceinline__ float apply_act(float x, int kind) {
  if (kind == 1) return fmaxf(x, 0.f);
  if (kind == 2) {
    float u = 0.7978845608f * (x + 0.044715f * x * x * x);
    return 0.5f * x * (1.f + tanhf(u));
  }
  return silu_f(x);
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const GemmParams p) {
  using S = GemmSmem<BN>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Align the dynamic smem base to 1024 B (required by the 128-B swizzle atoms).
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::kABytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * S::kStageBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* prefix = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr uint32_t kTmemCols = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128
                               : (2 * BN <= 256) ? 256 : 512;

  // Tile prefix sums over groups (every thread needs the schedule).
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int g = 0; g < p.G; ++g) {
      prefix[g] = acc;
      acc += group_tiles<BN>(p, g);
    }
    prefix[p.G] = acc;
    *abort_flag = 0;
  }
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 128);
    }
    mbar_init(drain_bar, 1);
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total_tiles = prefix[p.G];

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x) {
        TileCoord tc = decode_tile<BN>(p, prefix, tile);
        const int bgrp = p.b_mod ? tc.g % p.b_mod : tc.g;
        for (int kb = 0; kb < tc.nkb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty_bar[s], ph ^ 1, p.err, kErrTimeoutProducer, abort_flag)) { ok = false; break; }
          mbar_arrive_expect_tx(&full_bar[s], S::kStageBytes);
          uint8_t* a_dst = sA + s * S::kABytes;
          uint8_t* b_dst = sB + s * S::kBBytes;
          if constexpr (!A_MN) {
            tma_load_2d(&tmA, &full_bar[s], a_dst, kb * kBK, tc.g * p.a_grp + tc.mt * kBM);
          } else {
#pragma unroll
            for (int j = 0; j < kBM / 64; ++j)
              tma_load_2d(&tmA, &full_bar[s], a_dst + j * kBK * 128, tc.mt * kBM + j * 64, tc.g * p.a_grp + kb * kBK);
          }
          if constexpr (!B_MN) {
            tma_load_2d(&tmB, &full_bar[s], b_dst, kb * kBK, bgrp * p.b_grp + tc.nt * BN);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_2d(&tmB, &full_bar[s], b_dst + j * kBK * 128, tc.nt * BN + j * 64, bgrp * p.b_grp + kb * kBK);
          }
        }
      }
      if (!ok) {
        // Drain: wait (bounded) for the loads of the last STAGES issued iterations to land, so no
        // TMA write targets this CTA's shared memory after it exits.
        for (int i = (it > STAGES ? it - STAGES : 0); i < it; ++i) {
          long long t0 = clock64();
          while (!mbar_try_wait(&full_bar[i % STAGES], (i / STAGES) & 1) && clock64() - t0 < (1ll << 26)) {}
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(kBM, BN, A_MN, B_MN);
      int it = 0, tcount = 0;
      bool ok = true;
      bool issued = false;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += gridDim.x, ++tcount) {
        TileCoord tc = decode_tile<BN>(p, prefix, tile);
        const int buf = tcount & 1;
        const uint32_t tph = (tcount >> 1) & 1;
        if (!mbar_wait(&tempty_bar[buf], tph ^ 1, p.err, kErrTimeoutMma, abort_flag)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int kb = 0; kb < tc.nkb; ++kb, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full_bar[s], ph, p.err, kErrTimeoutMma, abort_flag)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + s * S::kABytes);
          const uint32_t b_base = smem_u32(sB + s * S::kBBytes);
#pragma unroll
          for (int ks = 0; ks < kBK / 16; ++ks) {
            uint64_t adesc, bdesc;
            if constexpr (!A_MN) adesc = make_sdesc(a_base + ks * 32, 16, 1024);
            else adesc = make_sdesc(a_base + ks * 2048, kBK * 128, 1024);
            if constexpr (!B_MN) bdesc = make_sdesc(b_base + ks * 32, 16, 1024);
            else bdesc = make_sdesc(b_base + ks * 2048, kBK * 128, 1024);
            umma_bf16(d_tmem, adesc, bdesc, idesc, (kb | ks) != 0 ? 1u : 0u);
          }
          issued = true;
          umma_commit(&empty_bar[s]);
        }
        if (!ok) break;
        umma_commit(&tfull_bar[buf]);
      }
      if (!ok && issued) {
        // Drain: wait (bounded) until every MMA issued so far has completed before TMEM is freed.
        umma_commit(drain_bar);
        long long t0 = clock64();
        while (!mbar_try_wait(drain_bar, 0) && clock64() - t0 < (1ll << 26)) {}
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue warps
    const int q = warp & 3;  // TMEM lane quadrant accessible by this warp
    const int r_in_tile = q * 32 + lane;
    int tcount = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++tcount) {
      TileCoord tc = decode_tile<BN>(p, prefix, tile);
      const int buf = tcount & 1;
      const uint32_t tph = (tcount >> 1) & 1;
      const bool got = mbar_wait(&tfull_bar[buf], tph, p.err, kErrTimeoutEpilogue, abort_flag);
      if (!__all_sync(0xffffffffu, got)) break;  // keep the warp converged for tcgen05.ld
      tc_fence_after();
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN;
      const int row = tc.mt * kBM + r_in_tile;
      const bool row_ok = row < p.M;
      const long crow = (long)(p.c_mod ? tc.g % p.c_mod : tc.g) * p.c_grp + row;
      const int col0 = tc.nt * BN;

      if constexpr (EPI == EPI_SWIGLU) {
        static_assert(BN == 256, "SwiGLU epilogue expects [gate 128 | up 128] tiles");
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          float gv[32], uv[32];
          tmem_ld32(taddr + c, gv);
          tmem_ld32(taddr + 128 + c, uv);
          tmem_wait_ld();
          if (row_ok) {
            __nv_bfloat16* H = reinterpret_cast<__nv_bfloat16*>(p.C) + crow * p.ldc + col0;
            __nv_bfloat16* A2 = reinterpret_cast<__nv_bfloat16*>(p.C2) + crow * p.ldc2 + tc.nt * 128;
            uint32_t hg[16], hu[16], ha[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              hg[i] = pack_bf16x2(gv[2 * i], gv[2 * i + 1]);
              hu[i] = pack_bf16x2(uv[2 * i], uv[2 * i + 1]);
              // activation from the bf16-rounded pre-activations so backward sees the same inputs
              float2 g2 = unpack_bf16x2(hg[i]);
              float2 u2 = unpack_bf16x2(hu[i]);
              ha[i] = pack_bf16x2(silu_f(g2.x) * u2.x, silu_f(g2.y) * u2.y);
            }
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              reinterpret_cast<uint4*>(H + c)[v] = make_uint4(hg[4 * v], hg[4 * v + 1], hg[4 * v + 2], hg[4 * v + 3]);
              reinterpret_cast<uint4*>(H + 128 + c)[v] =
                  make_uint4(hu[4 * v], hu[4 * v + 1], hu[4 * v + 2], hu[4 * v + 3]);
              reinterpret_cast<uint4*>(A2 + c)[v] = make_uint4(ha[4 * v], ha[4 * v + 1], ha[4 * v + 2], ha[4 * v + 3]);
            }
          }
        }
      } else if constexpr (EPI == EPI_CE) {
        // Logits tile (bf16) plus per-row (max, sum exp(x - max)) over this tile's valid columns.
        float m = -INFINITY, ssum = 0.f;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          tmem_ld32(taddr + c, v);
          tmem_wait_ld();
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
          float cm = -INFINITY;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float2 f = unpack_bf16x2(pk[i]);
            v[2 * i] = (col0 + c + 2 * i < p.N) ? f.x : -INFINITY;
            v[2 * i + 1] = (col0 + c + 2 * i + 1 < p.N) ? f.y : -INFINITY;
            cm = fmaxf(cm, fmaxf(v[2 * i], v[2 * i + 1]));
          }
          float nm = fmaxf(m, cm);
          if (nm > -INFINITY) {
            float acc = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) acc += __expf(v[i] - nm);
            ssum = ssum * __expf(m - nm) + acc;
            m = nm;
          }
          if (row_ok && col0 + c < p.N) {
            __nv_bfloat16* Cp = reinterpret_cast<__nv_bfloat16*>(p.C) + crow * p.ldc + col0 + c;
#pragma unroll
            for (int vv = 0; vv < 4; ++vv)
              reinterpret_cast<uint4*>(Cp)[vv] = make_uint4(pk[4 * vv], pk[4 * vv + 1], pk[4 * vv + 2], pk[4 * vv + 3]);
          }
        }
        if (row_ok) {
          // stats row stride ldc2 is in floats; entry nt holds (max, sumexp)
          float2* st = reinterpret_cast<float2*>(reinterpret_cast<float*>(p.C2) + crow * p.ldc2 + 2 * tc.nt);
          *st = make_float2(m, ssum);
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          float v[32];
          tmem_ld32(taddr + c, v);
          tmem_wait_ld();
          const int col = col0 + c;
          if (!row_ok || col >= p.N) continue;
          if constexpr (EPI == EPI_STORE) {
            if (p.c_f32) {
              float* Cp = reinterpret_cast<float*>(p.C) + crow * p.ldc + col;
              if (p.c_accum == 2) {
#pragma unroll
                for (int vv = 0; vv < 8; ++vv)
                  atomicAdd(reinterpret_cast<float4*>(Cp) + vv,
                            make_float4(p.alpha * v[4 * vv], p.alpha * v[4 * vv + 1], p.alpha * v[4 * vv + 2],
                                        p.alpha * v[4 * vv + 3]));
              } else if (p.c_accum) {
#pragma unroll
                for (int vv = 0; vv < 8; ++vv) {
                  float4 o = reinterpret_cast<float4*>(Cp)[vv];
                  o.x += p.alpha * v[4 * vv];
                  o.y += p.alpha * v[4 * vv + 1];
                  o.z += p.alpha * v[4 * vv + 2];
                  o.w += p.alpha * v[4 * vv + 3];
                  reinterpret_cast<float4*>(Cp)[vv] = o;
                }
              } else {
#pragma unroll
                for (int vv = 0; vv < 8; ++vv)
                  reinterpret_cast<float4*>(Cp)[vv] = make_float4(p.alpha * v[4 * vv], p.alpha * v[4 * vv + 1],
                                                                  p.alpha * v[4 * vv + 2], p.alpha * v[4 * vv + 3]);
              }
            } else {
              __nv_bfloat16* Cp = reinterpret_cast<__nv_bfloat16*>(p.C) + crow * p.ldc + col;
              uint32_t pk[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(p.alpha * v[2 * i], p.alpha * v[2 * i + 1]);
#pragma unroll
              for (int vv = 0; vv < 4; ++vv)
                reinterpret_cast<uint4*>(Cp)[vv] = make_uint4(pk[4 * vv], pk[4 * vv + 1], pk[4 * vv + 2], pk[4 * vv + 3]);
            }
          } else if constexpr (EPI == EPI_RESID || EPI == EPI_GATE_MUL) {
            const __nv_bfloat16* Rp = reinterpret_cast<const __nv_bfloat16*>(p.R) + crow * p.ldr + col;
            __nv_bfloat16* Cp = reinterpret_cast<__nv_bfloat16*>(p.C) + crow * p.ldc + col;
            uint4 rv[4];
#pragma unroll
            for (int vv = 0; vv < 4; ++vv) rv[vv] = reinterpret_cast<const uint4*>(Rp)[vv];
            const uint32_t* ru = reinterpret_cast<const uint32_t*>(rv);
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float2 r2 = unpack_bf16x2(ru[i]);
              if constexpr (EPI == EPI_RESID)
                pk[i] = pack_bf16x2(v[2 * i] + r2.x, v[2 * i + 1] + r2.y);
              else
                pk[i] = pack_bf16x2(r2.x * sigmoid_f(v[2 * i]), r2.y * sigmoid_f(v[2 * i + 1]));
            }
#pragma unroll
            for (int vv = 0; vv < 4; ++vv)
              reinterpret_cast<uint4*>(Cp)[vv] = make_uint4(pk[4 * vv], pk[4 * vv + 1], pk[4 * vv + 2], pk[4 * vv + 3]);
          } else if constexpr (EPI == EPI_SILU || EPI == EPI_ACT) {
            __nv_bfloat16* Cp = reinterpret_cast<__nv_bfloat16*>(p.C) + crow * p.ldc + col;
            __nv_bfloat16* Hp = reinterpret_cast<__nv_bfloat16*>(p.C2) + crow * p.ldc2 + col;
            uint32_t ph[16], pa[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              ph[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
              float2 h2 = unpack_bf16x2(ph[i]);
              const int kind = (EPI == EPI_SILU) ? 0 : p.act_kind;
              pa[i] = pack_bf16x2(apply_act(h2.x, kind), apply_act(h2.y, kind));
            }
#pragma unroll
            for (int vv = 0; vv < 4; ++vv) {
              reinterpret_cast<uint4*>(Cp)[vv] = make_uint4(pa[4 * vv], pa[4 * vv + 1], pa[4 * vv + 2], pa[4 * vv + 3]);
              reinterpret_cast<uint4*>(Hp)[vv] = make_uint4(ph[4 * vv], ph[4 * vv + 1], ph[4 * vv + 2], ph[4 * vv + 3]);
            }
          } else if constexpr (EPI == EPI_ROWSCALE) {
            const float sc = p.row_scale[crow];
            __nv_bfloat16* Cp = reinterpret_cast<__nv_bfloat16*>(p.C) + crow * p.ldc + col;
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(sc * v[2 * i], sc * v[2 * i + 1]);
#pragma unroll
            for (int vv = 0; vv < 4; ++vv)
              reinterpret_cast<uint4*>(Cp)[vv] = make_uint4(pk[4 * vv], pk[4 * vv + 1], pk[4 * vv + 2], pk[4 * vv + 3]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <int BN, int STAGES>
constexpr int gemm_smem_bytes() {
  // stages + barriers/scalars + prefix table + 1 KB alignment slack
  return STAGES * GemmSmem<BN>::kStageBytes + 1024 + (kMaxGroups + 1) * 4 + 256;
}

}  // namespace mxk
