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
// coordinate g*a_grp, B rows at (b_mod ? g % b_mod : g)*b_grp and writes C rows starting at
// (c_mod ? g % c_mod : g)*c_grp. A device array of per-group counts makes either M (expert token
// counts) or K (weight-gradient contraction over the tokens an expert received) ragged; tiles
// past the count are never scheduled. Non-grouped GEMMs can split K over CTAs (``ksplit``).
//
// CTA = 6 warps:  warp 0 = TMA producer, warp 1 = MMA issuer (+ TMEM owner),
//                 warps 2..5 = epilogue (TMEM lane quadrant = warp % 4).
// Accumulators are double-buffered in TMEM (2 x BN fp32 columns) so the epilogue of tile i
// overlaps the main loop of tile i+1. Epilogue warps stage 32-row x 64-byte boxes of their rows
// in 64B-swizzled shared memory (a 4-deep ring per warp) and write them with TMA bulk stores;
// fp32 accumulation into an existing C (weight gradients, split-K partials) uses the TMA bulk
// reduce-add, which is element-wise atomic. One CTA per SM, grid = min(#tiles, #SMs).
#pragma once
#include "gemm_params.h"
#include "sm100_primitives.cuh"

namespace mxk {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kEpiWarps = 8;  // two per TMEM lane quadrant, each on one half of the tile's columns
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;
constexpr int kMaxGroups = 4096;
// Tile-prefix table in shared memory: entry j holds the first tile of group j * gpb, where
// gpb = ceil(G / kPrefixSlots) groups share a slot (one per slot up to 256 groups); decoding a
// tile walks at most gpb groups from its slot's first group.
constexpr int kPrefixSlots = 256;
constexpr int kStageBufs = 2;    // minimum epilogue staging ring depth per warp
constexpr int kStageBox = 2048;  // 32 rows x 64 bytes

enum EpiKind : int {
  EPI_STORE = 0,     // C = alpha*acc (bf16 or f32), or C += alpha*acc (f32, TMA reduce-add)
  EPI_SWIGLU = 1,    // BN=256 tile = [gate 128 | up 128]: H = acc (bf16), Act = silu(gate)*up (bf16)
  EPI_RESID = 2,     // C = acc + R (bf16); R may alias C
  EPI_GATE_MUL = 3,  // C = X * sigmoid(acc) (bf16), X given in R (GatedNorm up projection)
  EPI_SILU = 4,      // C = silu(acc) (bf16) and H = acc (bf16) (GatedNorm down projection)
  EPI_ROWSCALE = 5,  // C = acc * row_scale[row] (bf16)
  EPI_CE = 6,        // logits tile: C = acc (bf16) and per-(row, n-tile half) max / sum(exp(x - max))
  EPI_ACT = 7,       // non-GLU MLP: H = acc (bf16), C = act(acc) (bf16); act in `act_kind`
  EPI_SWIGLU_BWD = 8,  // acc = dAct [rows, I]; R = SwiGLU pre-activations H [rows, 2I] (blocked
                       // [gate 128 | up 128] per 256 columns); C = dH [rows, 2I] (bf16), SiLU gate
};

// Shared-memory plan of one CTA. PAIR: the tile is 256 x BN over a CTA pair; each CTA stages its
// 128 rows of A and BN / 2 rows of B.
template <int BN, bool PAIR = false>
struct GemmSmem {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = (PAIR ? BN / 2 : BN) * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiBytes = kEpiWarps * kStageBufs * kStageBox;
};

// Epilogue shared memory. Most epilogues use a per-warp staging ring of kStageBufs store boxes.
// The SwiGLU backward epilogue instead gives each warp kSlots slots of two boxes (gate, up): H
// chunks are loaded into a slot by TMA, overwritten in place with the gradients and stored from
// there; one mbarrier per slot follows the loads. Its slot count is what the shared memory left
// after the operand stages holds (at most 3).
constexpr int kSmemLimit = 232448;
constexpr int kSwbSlotBytes = 2 * kStageBox;

template <int BN, int STAGES, bool PAIR>
constexpr int smem_fixed_bytes() {
  // operand stages + 1 KB alignment slack + barriers/scalars + tile prefix table
  return STAGES * GemmSmem<BN, PAIR>::kStageBytes + 1024 + 256 + (kPrefixSlots + 1) * 4;
}

// Store-ring depth per epilogue warp: as many 2 KB boxes as the shared memory left after the
// operand stages holds (at least kStageBufs, at most 8). More boxes in flight keep more TMA stores /
// reduce-adds outstanding per SM, which is what an fp32-accumulating epilogue is bound by.
template <int BN, int STAGES, bool PAIR>
constexpr int epi_ring() {
  constexpr int n = (kSmemLimit - smem_fixed_bytes<BN, STAGES, PAIR>()) / (kEpiWarps * kStageBox);
  return n < kStageBufs ? kStageBufs : (n > 8 ? 8 : n);
}

template <int BN, int STAGES, bool PAIR, int EPI>
constexpr int epi_slots() {
  if (EPI != EPI_SWIGLU_BWD) return epi_ring<BN, STAGES, PAIR>();
  constexpr int n = (kSmemLimit - smem_fixed_bytes<BN, STAGES, PAIR>()) / (kEpiWarps * (kSwbSlotBytes + 8));
  return n > 3 ? 3 : n;
}

template <int BN, int STAGES, bool PAIR, int EPI>
constexpr int epi_bytes() {
  if (EPI != EPI_SWIGLU_BWD) return kEpiWarps * epi_ring<BN, STAGES, PAIR>() * kStageBox;
  return kEpiWarps * epi_slots<BN, STAGES, PAIR, EPI>() * (kSwbSlotBytes + 8);
}

__device__ __forceinline__ int group_count(const GemmParams& p, int g) {
  if (p.counts) return p.counts[g];
  return p.ragged == 2 ? p.K : p.M;
}

// Number of scheduled tiles (output tiles of TM x BN, x K splits) of group g.
template <int BN, int TM = kBM>
__device__ __forceinline__ int group_tiles(const GemmParams& p, int g) {
  const int n_tiles = (p.N + BN - 1) / BN;
  if (p.ragged == 1) {
    int cnt = min(group_count(p, g), p.M);
    return ((cnt + TM - 1) / TM) * n_tiles;
  }
  int m_tiles = (p.M + TM - 1) / TM;
  if (p.ragged == 2) return group_count(p, g) > 0 ? m_tiles * n_tiles : 0;
  return m_tiles * n_tiles * max(p.ksplit, 1);
}

struct TileCoord {
  int g, mt, nt, kb0, nkb;
};

__device__ __forceinline__ int prefix_gpb(int G) { return (G + kPrefixSlots - 1) / kPrefixSlots; }
__device__ __forceinline__ int prefix_slots(int G) {
  const int gpb = prefix_gpb(G);
  return (G + gpb - 1) / gpb;
}

template <int BN, int TM = kBM>
__device__ __forceinline__ TileCoord decode_tile(const GemmParams& p, const int* prefix, int tile) {
  const int gpb = prefix_gpb(p.G);
  int lo = 0, hi = prefix_slots(p.G) - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= tile) lo = mid; else hi = mid - 1;
  }
  // walk the slot's groups (zero-tile groups are skipped like the binary search above skips them)
  int grp = lo * gpb, acc = prefix[lo];
  const int gend = min(p.G, grp + gpb);
  while (grp + 1 < gend) {
    const int nt = group_tiles<BN, TM>(p, grp);
    if (acc + nt > tile) break;
    acc += nt;
    ++grp;
  }
  TileCoord tc;
  tc.g = grp;
  lo = grp;
  int local = tile - acc;
  int m_tiles;
  if (p.ragged == 1) {
    int cnt = min(group_count(p, lo), p.M);
    m_tiles = (cnt + TM - 1) / TM;
  } else {
    m_tiles = (p.M + TM - 1) / TM;
  }
  const int n_tiles = (p.N + BN - 1) / BN;
  const int kext = (p.ragged == 2) ? group_count(p, lo) : p.K;
  const int nkb = (kext + kBK - 1) / kBK;
  const int ks = (p.ragged == 0) ? max(p.ksplit, 1) : 1;
  int split = 0;
  if (ks > 1) {
    split = local / (m_tiles * n_tiles);
    local = local % (m_tiles * n_tiles);
  }
  // raster_n: consecutive tiles walk N first, so the tiles in flight share a few A row blocks
  // (problems with few N tiles); otherwise M first, so they share B column blocks.
  if (p.raster_n) {
    tc.nt = local % n_tiles;
    tc.mt = local / n_tiles;
  } else {
    tc.mt = local % m_tiles;
    tc.nt = local / m_tiles;
  }
  const int per = (nkb + ks - 1) / ks;
  tc.kb0 = split * per;
  tc.nkb = max(0, min(nkb, tc.kb0 + per) - tc.kb0);
  return tc;
}

__device__ __forceinline__ float apply_act(float x, int kind) {
  if (kind == 1) return fmaxf(x, 0.f);
  if (kind == 2) {
    // tanh-approximated GELU, 0.5 x (1 + tanh(u)) = x * sigmoid(2u)
    const float u = 0.7978845608f * (x + 0.044715f * x * x * x);
    return x * sigmoid_f(2.f * u);
  }
  return silu_f(x);
}

// Epilogue staging ring of one warp: 32-row x 64-byte boxes in 64B-swizzled smem (16-byte chunk k
// of row r lives at chunk k ^ ((r >> 1) & 3)), written to global by TMA (only lane 0 issues and
// tracks the bulk groups; the ring slot is warp-uniform).
template <int DEPTH>
struct EpiRing {
  uint8_t* base;
  int slot;

  __device__ __forceinline__ uint8_t* acquire(int lane) {
    if (lane == 0) bulk_wait_read<DEPTH - 1>();
    __syncwarp();
    return base + slot * kStageBox;
  }
  __device__ __forceinline__ static void put_row(uint8_t* buf, int r, uint4 c0, uint4 c1, uint4 c2, uint4 c3) {
    const int sw = (r >> 1) & 3;
    uint8_t* row = buf + r * 64;
    *reinterpret_cast<uint4*>(row + ((0 ^ sw) << 4)) = c0;
    *reinterpret_cast<uint4*>(row + ((1 ^ sw) << 4)) = c1;
    *reinterpret_cast<uint4*>(row + ((2 ^ sw) << 4)) = c2;
    *reinterpret_cast<uint4*>(row + ((3 ^ sw) << 4)) = c3;
  }
  __device__ __forceinline__ void issue(const CUtensorMap* tm, uint8_t* buf, int x, int y, bool reduce, int lane) {
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      if (reduce) tma_reduce_add_2d(tm, buf, x, y);
      else tma_store_2d(tm, buf, x, y);
      bulk_commit();
    }
    slot = (slot + 1) % DEPTH;
  }
  // 32 fp32 values of this lane's row -> one bf16 box (32 columns) at (x, y)
  __device__ __forceinline__ void bf16_box(const CUtensorMap* tm, const float (&v)[32], int x, int y, int lane) {
    uint8_t* buf = acquire(lane);
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) pk[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
    put_row(buf, lane, make_uint4(pk[0], pk[1], pk[2], pk[3]), make_uint4(pk[4], pk[5], pk[6], pk[7]),
            make_uint4(pk[8], pk[9], pk[10], pk[11]), make_uint4(pk[12], pk[13], pk[14], pk[15]));
    issue(tm, buf, x, y, false, lane);
  }
  // 32 fp32 values -> two fp32 boxes of 16 columns each (store, or reduce-add into C)
  __device__ __forceinline__ void f32_boxes(const CUtensorMap* tm, const float (&v)[32], int x, int y, bool reduce,
                                            int lane) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint8_t* buf = acquire(lane);
      const float* w = v + 16 * h;
      put_row(buf, lane,
              make_uint4(__float_as_uint(w[0]), __float_as_uint(w[1]), __float_as_uint(w[2]), __float_as_uint(w[3])),
              make_uint4(__float_as_uint(w[4]), __float_as_uint(w[5]), __float_as_uint(w[6]), __float_as_uint(w[7])),
              make_uint4(__float_as_uint(w[8]), __float_as_uint(w[9]), __float_as_uint(w[10]), __float_as_uint(w[11])),
              make_uint4(__float_as_uint(w[12]), __float_as_uint(w[13]), __float_as_uint(w[14]),
                         __float_as_uint(w[15])));
      issue(tm, buf, x + 16 * h, y, reduce, lane);
    }
  }
};

// PAIR: launched as (2, 1, 1) clusters; a cluster computes a 256 x BN tile with cta_group::2
// MMAs issued by its even CTA (rank 0). Each CTA loads its 128 rows of A and rows
// [rank * BN / 2, (rank + 1) * BN / 2) of B's tile; both CTAs' loads complete rank 0's full
// barrier; MMA completion is multicast to both CTAs' empty / TMEM-full barriers; both CTAs'
// epilogues release rank 0's TMEM-empty barrier.
template <int BN, int STAGES, bool A_MN, bool B_MN, int EPI, bool PAIR>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmC2,
                      const GemmParams p) {
  using S = GemmSmem<BN, PAIR>;
  constexpr int TM = PAIR ? 2 * kBM : kBM;  // output rows of a tile
  constexpr int BNL = PAIR ? BN / 2 : BN;  // B rows staged by this CTA
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * S::kABytes;
  uint8_t* sEpi = smem + STAGES * S::kStageBytes;  // 1024-aligned (stage sizes are multiples of 1 KB)
  constexpr int kSlots = epi_slots<BN, STAGES, PAIR, EPI>();
  static_assert(EPI != EPI_SWIGLU_BWD || kSlots >= 2, "SwiGLU backward epilogue needs two H slots per warp");
  // SwiGLU backward: H-slot barriers after all warps' slots
  uint64_t* h_bar = reinterpret_cast<uint64_t*>(sEpi + kEpiWarps * kSlots * kSwbSlotBytes);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(sEpi + epi_bytes<BN, STAGES, PAIR, EPI>());
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;
  uint64_t* tempty_bar = tfull_bar + 2;
  uint64_t* drain_bar = tempty_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* prefix = reinterpret_cast<int*>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int tile0 = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;  // first tile of this CTA / pair
  const int tstep = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  constexpr uint32_t kTmemCols = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128
                               : (2 * BN <= 256) ? 256 : 512;

  if (threadIdx.x == 0) {
    const int gpb = prefix_gpb(p.G);
    int acc = 0;
    for (int g = 0; g < p.G; ++g) {
      if (g % gpb == 0) prefix[g / gpb] = acc;
      acc += group_tiles<BN, TM>(p, g);
    }
    prefix[prefix_slots(p.G)] = acc;
    *abort_flag = 0;
  }
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], (PAIR ? 2 : 1) * 32 * kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    if constexpr (EPI == EPI_SWIGLU_BWD) {
      for (int i = 0; i < kEpiWarps * kSlots; ++i) mbar_init(&h_bar[i], 1);
    }
    fence_barrier_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if constexpr (EPI == EPI_SWIGLU_BWD) prefetch_tmap(&tmC2);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) cluster_sync();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int total_tiles = prefix[prefix_slots(p.G)];

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      // one TMA load: PAIR loads count their bytes on rank 0's full barrier
      auto load = [&](const CUtensorMap* tm, int s, void* dst, int x, int y) {
        if constexpr (PAIR) tma_load_2d_pair(tm, mapa_shared(&full_bar[s], 0), dst, x, y);
        else tma_load_2d(tm, &full_bar[s], dst, x, y);
      };
      for (int tile = tile0; tile < total_tiles && ok; tile += tstep) {
        TileCoord tc = decode_tile<BN, TM>(p, prefix, tile);
        const int bgrp = p.b_mod ? tc.g % p.b_mod : tc.g;
        const int arow = tc.mt * TM + (int)rank * kBM;  // this CTA's first A row (or M column)
        const int brow = tc.nt * BN + (int)rank * BNL;  // this CTA's first B row (or N column)
        for (int i = 0; i < tc.nkb; ++i, ++it) {
          const int kb = tc.kb0 + i;
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty_bar[s], ph ^ 1, p.err, kErrTimeoutProducer, abort_flag)) { ok = false; break; }
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[s], (PAIR ? 2 : 1) * S::kStageBytes);
          uint8_t* a_dst = sA + s * S::kABytes;
          uint8_t* b_dst = sB + s * S::kBBytes;
          if constexpr (!A_MN) {
            load(&tmA, s, a_dst, kb * kBK, tc.g * p.a_grp + arow);
          } else {
#pragma unroll
            for (int j = 0; j < kBM / 64; ++j)
              load(&tmA, s, a_dst + j * kBK * 128, arow + j * 64, tc.g * p.a_grp + kb * kBK);
          }
          if constexpr (!B_MN) {
            load(&tmB, s, b_dst, kb * kBK, bgrp * p.b_grp + brow);
          } else {
#pragma unroll
            for (int j = 0; j < BNL / 64; ++j)
              load(&tmB, s, b_dst + j * kBK * 128, brow + j * 64, bgrp * p.b_grp + kb * kBK);
          }
        }
      }
      if (!ok && PAIR && rank != 0) {
        // The peer cannot observe rank 0's full barrier: give its loads in flight a fixed
        // (bounded) time to land before this CTA's shared memory is released.
        long long t0 = clock64();
        while (clock64() - t0 < (1ll << 24)) {}
      } else if (!ok) {
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
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = make_idesc_bf16(TM, BN, A_MN, B_MN);
      int it = 0, tcount = 0;
      bool ok = true;
      bool issued = false;
      for (int tile = tile0; tile < total_tiles && ok; tile += tstep) {
        TileCoord tc = decode_tile<BN, TM>(p, prefix, tile);
        if (tc.nkb == 0) continue;  // (host never schedules empty splits; kept consistent anyway)
        const int buf = tcount & 1;
        const uint32_t tph = (tcount >> 1) & 1;
        const bool freed = PAIR ? mbar_wait_cluster(&tempty_bar[buf], tph ^ 1, p.err, kErrTimeoutMma, abort_flag)
                                : mbar_wait(&tempty_bar[buf], tph ^ 1, p.err, kErrTimeoutMma, abort_flag);
        if (!freed) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * BN;
        for (int i = 0; i < tc.nkb; ++i, ++it) {
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
            if constexpr (PAIR) umma_bf16_pair(d_tmem, adesc, bdesc, idesc, (i | ks) != 0 ? 1u : 0u);
            else umma_bf16(d_tmem, adesc, bdesc, idesc, (i | ks) != 0 ? 1u : 0u);
          }
          issued = true;
          if constexpr (PAIR) umma_commit_pair(&empty_bar[s], 0x3);
          else umma_commit(&empty_bar[s]);
        }
        if (!ok) break;
        if constexpr (PAIR) umma_commit_pair(&tfull_bar[buf], 0x3);
        else umma_commit(&tfull_bar[buf]);
        ++tcount;
      }
      if (!ok && issued) {
        // Drain: wait (bounded) until every MMA issued so far has completed before TMEM is freed.
        if constexpr (PAIR) umma_commit_pair(drain_bar, 0x1);
        else umma_commit(drain_bar);
        long long t0 = clock64();
        while (!mbar_try_wait(drain_bar, 0) && clock64() - t0 < (1ll << 26)) {}
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue warps
    const int q = warp & 3;  // TMEM lane quadrant accessible by this warp
    const int half = (warp - 2) >> 2;  // which half of the tile's columns this warp drains
    constexpr int kHalf = BN / 2;
    constexpr int kRing = epi_ring<BN, STAGES, PAIR>();
    EpiRing<kRing> ring{sEpi + (warp - 2) * kRing * kStageBox, 0};
    const bool reduce = p.c_f32 && p.c_accum != 0;
    int tcount = 0;
    const uint32_t tempty_c0 = PAIR ? mapa_shared(&tempty_bar[0], 0) : 0u;
    const uint32_t tempty_c1 = PAIR ? mapa_shared(&tempty_bar[1], 0) : 0u;
    // SwiGLU backward: this warp's stream of H chunks (4 chunks of 32 activation columns per tile,
    // in tile order) is loaded by TMA kSlots - 1 chunks ahead of its use, across tile boundaries,
    // so the loads overlap the previous chunks' math and the wait for the next accumulator.
    uint8_t* h_slots = sEpi + (warp - 2) * kSlots * kSwbSlotBytes;
    uint64_t* h_bars = h_bar + (warp - 2) * kSlots;
    int h_issued = 0, h_used = 0;
    int la_tile = total_tiles, la_c = 0, la_x = 0, la_y = 0;  // next chunk to load
    bool h_fail = false;
    auto la_seek = [&](int t) {  // first tile >= t of this worker that has work: its H box origin
      for (; t < total_tiles; t += tstep) {
        const TileCoord lc = decode_tile<BN, TM>(p, prefix, t);
        if (lc.nkb == 0) continue;
        la_y = (p.c_mod ? lc.g % p.c_mod : lc.g) * p.c_grp + lc.mt * TM + (int)rank * kBM + q * 32;
        la_x = (((lc.nt * BN) >> 7) + half) * 256;
        break;
      }
      la_tile = t;
      la_c = 0;
    };
    auto h_issue = [&]() {
      if (la_tile >= total_tiles) return;
      const int slot = h_issued % kSlots;
      if (lane == 0) {
        // the slot last held chunk h_issued - kSlots; only the stores of the chunk consumed since
        // then may still be reading shared memory
        bulk_wait_read<1>();
        uint8_t* dst = h_slots + slot * kSwbSlotBytes;
        mbar_arrive_expect_tx(&h_bars[slot], kSwbSlotBytes);
        tma_load_2d(&tmC2, &h_bars[slot], dst, la_x + la_c * 32, la_y);
        tma_load_2d(&tmC2, &h_bars[slot], dst + kStageBox, la_x + 128 + la_c * 32, la_y);
      }
      ++h_issued;
      if (++la_c == 4) la_seek(la_tile + tstep);
    };
    if constexpr (EPI == EPI_SWIGLU_BWD) {
      la_seek(tile0);
      for (int i = 0; i < kSlots - 1; ++i) h_issue();
    }
    // Residual / gate epilogues: this lane's R row segment (the warp's column half of a tile) is
    // prefetched into L2 one tile ahead -- when the tile before it starts draining -- so the drain's
    // R loads hit L2 instead of waiting on DRAM. Bounds as in the loads themselves.
    auto prefetch_r = [&](int t) {
      if constexpr (EPI == EPI_RESID || EPI == EPI_GATE_MUL) {
        if (t >= total_tiles) return;
        const TileCoord pc = decode_tile<BN, TM>(p, prefix, t);
        if (pc.nkb == 0 || pc.mt * TM + (int)rank * kBM + q * 32 + lane >= p.M) return;
        const long pr = (long)((p.c_mod ? pc.g % p.c_mod : pc.g) * p.c_grp + pc.mt * TM + (int)rank * kBM + q * 32) +
                        lane;
        const int c0 = pc.nt * BN + half * kHalf;
        const __nv_bfloat16* rp = reinterpret_cast<const __nv_bfloat16*>(p.R) + pr * p.ldr + c0;
#pragma unroll
        for (int off = 0; off < kHalf; off += 64) {
          if (c0 + off < p.N) prefetch_l2(rp + off);
        }
      }
    };
    prefetch_r(tile0);
    for (int tile = tile0; tile < total_tiles; tile += tstep) {
      TileCoord tc = decode_tile<BN, TM>(p, prefix, tile);
      if (tc.nkb == 0) continue;
      const int buf = tcount & 1;
      const uint32_t tph = (tcount >> 1) & 1;
      ++tcount;
      const bool got = mbar_wait(&tfull_bar[buf], tph, p.err, kErrTimeoutEpilogue, abort_flag);
      if (!__all_sync(0xffffffffu, got)) break;  // keep the warp converged for tcgen05.ld
      tc_fence_after();
      prefetch_r(tile + tstep);
      const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN;
      const int row = tc.mt * TM + (int)rank * kBM + q * 32 + lane;
      const bool row_ok = row < p.M;
      const int y0 = (p.c_mod ? tc.g % p.c_mod : tc.g) * p.c_grp + tc.mt * TM + (int)rank * kBM + q * 32;  // warp's first C row
      const long crow = (long)y0 + lane;
      const int col0 = tc.nt * BN;

      if constexpr (EPI == EPI_SWIGLU) {
        static_assert(BN == 256, "SwiGLU epilogue expects [gate 128 | up 128] tiles");
#pragma unroll 1
        for (int c = half * 64; c < half * 64 + 64; c += 32) {
          float gv[32], uv[32];
          tmem_ld32(taddr + c, gv);
          tmem_ld32(taddr + 128 + c, uv);
          tmem_wait_ld();
          float av[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            // activation from the bf16-rounded pre-activations so backward sees the same inputs
            const float g = __bfloat162float(__float2bfloat16(gv[i]));
            const float u = __bfloat162float(__float2bfloat16(uv[i]));
            av[i] = silu_f(g) * u;
          }
          ring.bf16_box(&tmC, gv, col0 + c, y0, lane);
          ring.bf16_box(&tmC, uv, col0 + 128 + c, y0, lane);
          ring.bf16_box(&tmC2, av, tc.nt * 128 + c, y0, lane);
        }
      } else if constexpr (EPI == EPI_SWIGLU_BWD) {
        // Activation-gradient tile -> gate / up gradients: the half of the tile drained by this warp
        // is one 128-column activation block ab, whose gate and up columns are H[:, 256 ab + ..]
        // and H[:, 256 ab + 128 + ..]. Each 32-column chunk's H boxes arrive in a slot (64B
        // swizzle: 16-byte piece k of row r at piece k ^ ((r >> 1) & 3)); every lane overwrites its
        // row with dG / dU and the slot's two boxes are stored to C's matching columns.
        static_assert(BN == 256, "SwiGLU backward epilogue drains 128-column activation blocks");
        const int ab = (col0 >> 7) + half;
        const bool blk_ok = ab * 128 < p.N;  // warp-uniform
        const int sw = (lane >> 1) & 3;
#pragma unroll 1
        for (int c = 0; c < 128; c += 32) {
          const int slot = h_used % kSlots;
          const uint32_t hph = (h_used / kSlots) & 1;
          float v[32];
          tmem_ld32(taddr + half * 128 + c, v);
          const bool hok = mbar_wait(&h_bars[slot], hph, p.err, kErrTimeoutEpilogue, abort_flag);
          tmem_wait_ld();
          if (!__all_sync(0xffffffffu, hok)) {
            h_fail = true;
            break;
          }
          ++h_used;
          uint8_t* gbuf = h_slots + slot * kSwbSlotBytes;
          uint8_t* grow = gbuf + lane * 64;
          uint8_t* urow = grow + kStageBox;
          if (blk_ok) {
#pragma unroll
            for (int vv = 0; vv < 4; ++vv) {
              uint4* gp = reinterpret_cast<uint4*>(grow + ((vv ^ sw) << 4));
              uint4* up = reinterpret_cast<uint4*>(urow + ((vv ^ sw) << 4));
              const uint4 g4 = *gp, u4 = *up;
              const uint32_t gw[4] = {g4.x, g4.y, g4.z, g4.w};
              const uint32_t uw[4] = {u4.x, u4.y, u4.z, u4.w};
              uint32_t dgw[4], duw[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const float2 g2 = unpack_bf16x2(gw[k]), u2 = unpack_bf16x2(uw[k]);
                const int i = vv * 8 + 2 * k;
                const float s0 = sigmoid_f(g2.x), s1 = sigmoid_f(g2.y);
                // d silu(g) / dg = s (1 + g (1 - s)); d(silu(g) u) = (u silu'(g), silu(g))
                dgw[k] = pack_bf16x2(v[i] * u2.x * s0 * (1.f + g2.x * (1.f - s0)),
                                     v[i + 1] * u2.y * s1 * (1.f + g2.y * (1.f - s1)));
                duw[k] = pack_bf16x2(v[i] * g2.x * s0, v[i + 1] * g2.y * s1);
              }
              *gp = make_uint4(dgw[0], dgw[1], dgw[2], dgw[3]);
              *up = make_uint4(duw[0], duw[1], duw[2], duw[3]);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              tma_store_2d(&tmC, gbuf, ab * 256 + c, y0);
              tma_store_2d(&tmC, gbuf + kStageBox, ab * 256 + 128 + c, y0);
            }
          }
          if (lane == 0) bulk_commit();
          __syncwarp();
          h_issue();
        }
        if (h_fail) break;
      } else if constexpr (EPI == EPI_CE) {
        // Logits tile (bf16) plus per-row (max, sum exp(x - max)) over this tile's valid columns.
        float m = -INFINITY, ssum = 0.f;
#pragma unroll 1
        for (int c = half * kHalf; c < (half + 1) * kHalf; c += 32) {
          float v[32];
          tmem_ld32(taddr + c, v);
          tmem_wait_ld();
          if (col0 + c >= p.N) continue;
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = __bfloat162float(__float2bfloat16(v[i]));
          ring.bf16_box(&tmC, v, col0 + c, y0, lane);
          float cm = -INFINITY;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (col0 + c + i >= p.N) v[i] = -INFINITY;
            cm = fmaxf(cm, v[i]);
          }
          const float nm = fmaxf(m, cm);
          if (nm > -INFINITY) {
            float acc = 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) acc += __expf(v[i] - nm);
            ssum = ssum * __expf(m - nm) + acc;
            m = nm;
          }
        }
        if (row_ok) {
          // stats row stride ldc2 is in floats; entry 2 nt + half holds (max, sumexp) of the
          // tile's column half drained by this warp
          float2* st = reinterpret_cast<float2*>(reinterpret_cast<float*>(p.C2) + crow * p.ldc2) + 2 * tc.nt + half;
          *st = make_float2(m, ssum);
        }
      } else if constexpr (EPI == EPI_RESID || EPI == EPI_GATE_MUL) {
        // R (residual / gate input) rows are read with the next chunk's loads issued before this
        // chunk's TMEM read, so their latency overlaps the epilogue math (two chunks in flight).
        const __nv_bfloat16* Rrow = reinterpret_cast<const __nv_bfloat16*>(p.R) + crow * p.ldr;
        auto load_r = [&](int col, uint4 (&u)[4]) {
          if (row_ok && col < p.N) {
            const uint4* Rp = reinterpret_cast<const uint4*>(Rrow + col);
#pragma unroll
            for (int vv = 0; vv < 4; ++vv) u[vv] = Rp[vv];
          } else {
#pragma unroll
            for (int vv = 0; vv < 4; ++vv) u[vv] = make_uint4(0, 0, 0, 0);
          }
        };
        auto finish = [&](int c, const uint4 (&u)[4]) {
          float v[32];
          tmem_ld32(taddr + c, v);
          tmem_wait_ld();
          const int col = col0 + c;
          if (col >= p.N) return;
          float o[32];
#pragma unroll
          for (int vv = 0; vv < 4; ++vv) {
            const uint32_t w4[4] = {u[vv].x, u[vv].y, u[vv].z, u[vv].w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float2 f = unpack_bf16x2(w4[k]);
              const int i = vv * 8 + 2 * k;
              o[i] = (EPI == EPI_RESID) ? v[i] + f.x : f.x * sigmoid_f(v[i]);
              o[i + 1] = (EPI == EPI_RESID) ? v[i + 1] + f.y : f.y * sigmoid_f(v[i + 1]);
            }
          }
          if (p.c_f32) ring.f32_boxes(&tmC, o, col, y0, reduce, lane);
          else ring.bf16_box(&tmC, o, col, y0, lane);
        };
        uint4 ra[4], rb[4];
        static_assert(kHalf % 64 == 0, "residual epilogue drains 64-column steps");
        const int c_lo = half * kHalf, c_hi = c_lo + kHalf;
        load_r(col0 + c_lo, ra);
#pragma unroll 1
        for (int c = c_lo; c < c_hi; c += 64) {
          load_r(col0 + c + 32, rb);
          finish(c, ra);
          if (c + 64 < c_hi) load_r(col0 + c + 64, ra);
          finish(c + 32, rb);
        }
      } else {
#pragma unroll 1
        for (int c = half * kHalf; c < (half + 1) * kHalf; c += 32) {
          float v[32];
          tmem_ld32(taddr + c, v);
          tmem_wait_ld();
          const int col = col0 + c;
          if (col >= p.N) continue;  // warp-uniform; the box would be clipped anyway
          float o[32];
          if constexpr (EPI == EPI_STORE) {
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = p.alpha * v[i];
          } else if constexpr (EPI == EPI_SILU || EPI == EPI_ACT) {
            const int kind = (EPI == EPI_SILU) ? 0 : p.act_kind;
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = apply_act(__bfloat162float(__float2bfloat16(v[i])), kind);
          } else if constexpr (EPI == EPI_ROWSCALE) {
            const float sc = row_ok ? p.row_scale[crow] : 0.f;
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = sc * v[i];
          }
          bool stored = false;
          if constexpr (EPI == EPI_STORE) {
            if (p.peer_maps != nullptr) {
              // the tile's rows belong to source rank g / peer_epl: store them into its buffer
              const CUtensorMap* pm = reinterpret_cast<const CUtensorMap*>(p.peer_maps) + tc.g / p.peer_epl;
              const int yp = (p.peer_my * p.peer_epl + tc.g % p.peer_epl) * p.peer_cap + (y0 - tc.g * p.c_grp);
              ring.bf16_box(pm, o, col, yp, lane);
              stored = true;
            }
          }
          if (!stored) {
            if (p.c_f32) ring.f32_boxes(&tmC, o, col, y0, reduce, lane);
            else ring.bf16_box(&tmC, o, col, y0, lane);
          }
          if constexpr (EPI == EPI_SILU || EPI == EPI_ACT) ring.bf16_box(&tmC2, v, col, y0, lane);
        }
      }
      tc_fence_before();
      if constexpr (PAIR) mbar_arrive_remote(buf ? tempty_c1 : tempty_c0);
      else mbar_arrive(&tempty_bar[buf]);
    }
    if constexpr (EPI == EPI_SWIGLU_BWD) {
      // H loads issued but never consumed (an aborted run): let them land (bounded) before exit
      for (int j = h_used; j < h_issued; ++j) {
        long long t0 = clock64();
        while (!mbar_try_wait(&h_bars[j % kSlots], (j / kSlots) & 1) && clock64() - t0 < (1ll << 26)) {}
      }
    }
    if (lane == 0) {
      bulk_wait_all();  // every TMA store / reduce of this warp has landed
      // stores into other GPUs' memory: ordered before anything this GPU signals to them afterwards
      if (p.peer_maps != nullptr) __threadfence_system();
    }
  }

  tc_fence_before();
  __syncthreads();
  // PAIR: neither CTA leaves while the other may still arrive on its barriers or while rank 0's
  // MMAs may read its shared memory
  if constexpr (PAIR) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, kTmemCols);
    else tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <int BN, int STAGES, bool PAIR = false, int EPI = EPI_STORE>
constexpr int gemm_smem_bytes() {
  // stages + epilogue staging + 1 KB alignment slack + barriers/scalars + tile prefix table
  return smem_fixed_bytes<BN, STAGES, PAIR>() + epi_bytes<BN, STAGES, PAIR, EPI>();
}

}  // namespace mxk
