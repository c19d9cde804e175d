// Expert-parallel token exchange over NVLink peer memory (no NCCL on this path).
//
// Every rank of an expert-parallel group maps the same-sized "heap" of every peer (CUDA IPC), so a
// buffer at heap offset `off` exists on every rank and rank r can address rank p's copy directly.
// Token rows move with 16-byte loads/stores issued by the kernels that produce or consume them:
//
//   dispatch (forward):  the permute kernel of source s writes each routed row straight into the
//                        receive buffer of the expert's owner, layout [source][local expert][cap][D];
//   combine (forward):   the combine kernel of source s reads its K expert outputs per token from
//                        the owners' output buffers and forms sum_k w_k * y_k + residual;
//   backward:            the combine-backward kernel pushes w * dout rows to the owners; the
//                        unpermute kernel pulls the input-gradient rows back and sums them.
//
// Ordering: a producer kernel fences its stores at system scope; the last CTA to finish (found with
// an atomic counter) then writes `epoch` into the flag slot [purpose][source] of every peer with a
// release store. A consumer waits with acquire loads until its W flags reach `epoch` before any
// kernel reads the exchanged rows. Every wait is bounded (a per-call wall-time limit, 20 s by
// default); on timeout the waiter records kErrTimeoutPeer in the error flag and returns, so the host
// sees the failure instead of a hung GPU. Rows are never read through TMA or any cluster-multicast
// path from peer memory.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstring>

#include <cstdlib>
#include <string>

#include "kernels.h"
#include "sm100_primitives.cuh"

namespace mxk {

namespace {

// Default limit of a wait for peers' flags: 20 s of wall time (peers may lag by a whole layer).
constexpr long long kPeerWaitNs = 20ll * 1000 * 1000 * 1000;

__device__ __forceinline__ long long global_ns() {
  long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ char* peer_ptr(const PeerTable& pt, int rank, size_t off) {
  return static_cast<char*>(pt.base[rank]) + off;
}

// Flag slot of (purpose, source) inside a rank's flag area.
__device__ __forceinline__ int* flag_slot(const PeerTable& pt, int rank, size_t flags_off, int purpose, int src) {
  return reinterpret_cast<int*>(peer_ptr(pt, rank, flags_off)) + purpose * kMaxPeers + src;
}

// Called by every CTA of a producer kernel after its last store: publishes `epoch` to every peer's
// flag (purpose, my) once all CTAs are done.
__device__ void publish(const PeerTable& pt, int world, int my, size_t flags_off, int purpose, int epoch,
                        unsigned int* counter) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned int prev = atomicAdd(counter, 1u);
    if (prev == gridDim.x - 1) {
      __threadfence_system();
      for (int p = 0; p < world; ++p) st_release_sys(flag_slot(pt, p, flags_off, purpose, my), epoch);
      *counter = 0u;  // ready for the next launch (stream order)
    }
  }
}

__device__ __forceinline__ int round128(int c) { return (c + 127) & ~127; }

__device__ __forceinline__ void acc8(float (&a)[8], uint4 u, float w) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    a[2 * i] += w * f.x;
    a[2 * i + 1] += w * f.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&a)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(a[2 * i], a[2 * i + 1]);
  return u;
}

// Row r = e * cap + s of the source-side [E][cap] layout lives on rank e / E_loc at row
// ((my * E_loc) + e % E_loc) * cap + s of that rank's [W][E_loc][cap] buffer.
__device__ __forceinline__ long remote_row(int e, int s, int e_loc, int cap, int my) {
  return ((long)my * e_loc + (e % e_loc)) * cap + s;
}

// Push order: every source walks the [E][cap] rows starting at the first row of the next rank's
// experts (rank my + 1), so at any moment the sources write to different destinations. In expert
// order all eight sources would write to rank 0's experts first, then rank 1's: one destination's
// NVLink ingress at a time (measured at 8 GPUs: the pushes reached half of the pulls' rate).
__device__ __forceinline__ long push_rotation(const EpArgs& a) {
  return (long)((a.my + 1) % a.world) * a.e_loc * a.cap;
}

// ------------------------------------------------------------------------------------ kernels
// Forward dispatch: x[perm] rows (zeros on pad rows up to round128(count)) -> owners' receive buffers;
// counts -> owners' count arrays.
__global__ void ep_dispatch_push_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ perm,
                                        const int* __restrict__ counts, EpArgs a) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int E = a.e_loc * a.world;
  if (blockIdx.x == 0 && a.s_lo == 0)
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      int* dst = reinterpret_cast<int*>(peer_ptr(a.peers, e / a.e_loc, a.counts_off));
      dst[a.my * a.e_loc + e % a.e_loc] = counts[e];
    }
  const long total = (long)E * a.cap, rot = push_rotation(a);
  for (long q = blockIdx.x * (long)warps + (threadIdx.x >> 5); q < total; q += (long)gridDim.x * warps) {
    const long r = (q + rot) % total;
    const int e = (int)(r / a.cap), s = (int)(r % a.cap);
    const int c = counts[e];
    if (s >= round128(c) || s < a.s_lo || s >= a.s_hi) continue;
    uint4* dst = reinterpret_cast<uint4*>(peer_ptr(a.peers, e / a.e_loc, a.buf_off)) +
                 remote_row(e, s, a.e_loc, a.cap, a.my) * (a.D / 8);
    if (s < c) {
      const uint4* src = reinterpret_cast<const uint4*>(x + (long)perm[r] * a.D);
      for (int i = lane; i < a.D / 8; i += 32) dst[i] = src[i];
    } else {
      for (int i = lane; i < a.D / 8; i += 32) dst[i] = make_uint4(0, 0, 0, 0);
    }
  }
  publish(a.peers, a.world, a.my, a.flags_off, a.purpose, a.epoch, a.counter);
}

// Backward of the combine, pushed: dY rows = w * dout[perm] (zeros on pad rows) -> owners' buffers.
__global__ void ep_combine_bwd_push_kernel(const __nv_bfloat16* __restrict__ dout, const int* __restrict__ perm,
                                           const float* __restrict__ wperm, const int* __restrict__ counts, EpArgs a) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int E = a.e_loc * a.world;
  const long total = (long)E * a.cap, rot = push_rotation(a);
  for (long q = blockIdx.x * (long)warps + (threadIdx.x >> 5); q < total; q += (long)gridDim.x * warps) {
    const long r = (q + rot) % total;
    const int e = (int)(r / a.cap), s = (int)(r % a.cap);
    const int c = counts[e];
    if (s >= round128(c) || s < a.s_lo || s >= a.s_hi) continue;
    uint4* dst = reinterpret_cast<uint4*>(peer_ptr(a.peers, e / a.e_loc, a.buf_off)) +
                 remote_row(e, s, a.e_loc, a.cap, a.my) * (a.D / 8);
    if (s < c) {
      const float w = wperm[r];
      const uint4* src = reinterpret_cast<const uint4*>(dout + (long)perm[r] * a.D);
      for (int i = lane; i < a.D / 8; i += 32) {
        float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        acc8(v, src[i], w);
        dst[i] = pack8(v);
      }
    } else {
      for (int i = lane; i < a.D / 8; i += 32) dst[i] = make_uint4(0, 0, 0, 0);
    }
  }
  publish(a.peers, a.world, a.my, a.flags_off, a.purpose, a.epoch, a.counter);
}

// Forward combine, pulled: out[t] = residual[t] + sum_k w[t,k] * Y_owner[row(t,k)]; the pulled rows
// are also stored to y_local in the source layout [E][cap][D] for the backward's weight gradient.
__global__ void ep_combine_pull_kernel(const int* __restrict__ sel, const int* __restrict__ slot,
                                       const float* __restrict__ comb, const __nv_bfloat16* __restrict__ residual,
                                       __nv_bfloat16* __restrict__ out, __nv_bfloat16* __restrict__ y_local, int T,
                                       int K, EpArgs a) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    for (int c = lane; c < a.D / 8; c += 32) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (residual) acc8(acc, reinterpret_cast<const uint4*>(residual + (long)t * a.D)[c], 1.f);
      for (int k = 0; k < K; ++k) {
        const int s = slot[(long)t * K + k];
        if (s < 0) continue;
        const int e = sel[(long)t * K + k];
        const uint4* src = reinterpret_cast<const uint4*>(peer_ptr(a.peers, e / a.e_loc, a.buf_off)) +
                           remote_row(e, s, a.e_loc, a.cap, a.my) * (a.D / 8);
        const uint4 v = __ldcv(src + c);
        if (y_local) reinterpret_cast<uint4*>(y_local + ((long)e * a.cap + s) * a.D)[c] = v;
        acc8(acc, v, comb[(long)t * K + k]);
      }
      reinterpret_cast<uint4*>(out + (long)t * a.D)[c] = pack8(acc);
    }
  }
}

// Backward unpermute, pulled: dx[t] = sum_k dXp_owner[row(t,k)].
__global__ void ep_unpermute_pull_kernel(const int* __restrict__ sel, const int* __restrict__ slot,
                                         __nv_bfloat16* __restrict__ dx, int T, int K, EpArgs a) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    for (int c = lane; c < a.D / 8; c += 32) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int k = 0; k < K; ++k) {
        const int s = slot[(long)t * K + k];
        if (s < 0) continue;
        const int e = sel[(long)t * K + k];
        const uint4* src = reinterpret_cast<const uint4*>(peer_ptr(a.peers, e / a.e_loc, a.buf_off)) +
                           remote_row(e, s, a.e_loc, a.cap, a.my) * (a.D / 8);
        acc8(acc, __ldcv(src + c), 1.f);
      }
      reinterpret_cast<uint4*>(dx + (long)t * a.D)[c] = pack8(acc);
    }
  }
}

// Pushes with two rows per warp in flight: both rows' source indices, then all of both rows' 16-byte
// loads, then the peer stores (the generic kernels above load and store one chunk at a time).
// V = D / 256 chunks per lane.
template <int V, bool SCALED>
__global__ void ep_push_v2_kernel(const __nv_bfloat16* __restrict__ x, const int* __restrict__ perm,
                                  const float* __restrict__ wperm, const int* __restrict__ counts, EpArgs a) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  const int E = a.e_loc * a.world;
  if (!SCALED && blockIdx.x == 0 && a.s_lo == 0)
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      int* dst = reinterpret_cast<int*>(peer_ptr(a.peers, e / a.e_loc, a.counts_off));
      dst[a.my * a.e_loc + e % a.e_loc] = counts[e];
    }
  const long rows = (long)E * a.cap, rot = push_rotation(a);
  const long stride = (long)gridDim.x * warps;
  for (long q0 = blockIdx.x * (long)warps + (threadIdx.x >> 5); q0 < rows; q0 += 2 * stride) {
    long r[2] = {q0, q0 + stride};
#pragma unroll
    for (int u = 0; u < 2; ++u)
      if (r[u] < rows) r[u] = (r[u] + rot) % rows;
    uint4* dst[2] = {nullptr, nullptr};
    const uint4* src[2] = {nullptr, nullptr};
    float w[2] = {1.f, 1.f};
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (r[u] >= rows) continue;
      const int e = (int)(r[u] / a.cap), s = (int)(r[u] % a.cap);
      const int c = counts[e];
      if (s >= round128(c) || s < a.s_lo || s >= a.s_hi) continue;
      dst[u] = reinterpret_cast<uint4*>(peer_ptr(a.peers, e / a.e_loc, a.buf_off)) +
               remote_row(e, s, a.e_loc, a.cap, a.my) * (a.D / 8);
      if (s < c) {
        src[u] = reinterpret_cast<const uint4*>(x + (long)perm[r[u]] * a.D);
        if (SCALED) w[u] = wperm[r[u]];
      }
    }
    uint4 v[2][V];
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int k = 0; k < V; ++k) v[u][k] = src[u] ? src[u][lane + 32 * k] : make_uint4(0, 0, 0, 0);
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      if (!dst[u]) continue;
#pragma unroll
      for (int k = 0; k < V; ++k) {
        if (SCALED && src[u]) {
          float f[8] = {0, 0, 0, 0, 0, 0, 0, 0};
          acc8(f, v[u][k], w[u]);
          dst[u][lane + 32 * k] = pack8(f);
        } else {
          dst[u][lane + 32 * k] = v[u][k];
        }
      }
    }
  }
  publish(a.peers, a.world, a.my, a.flags_off, a.purpose, a.epoch, a.counter);
}

// Pushes through the copy engine, by tiles of 32 consecutive capacity slots of one expert: the
// warp's 32 lanes each issue one row's bulk load (x[perm[r]], local) into the tile's shared-memory
// slot, pad rows are zero-filled in place, and one bulk store moves the whole tile (up to 96 KB,
// contiguous in the owner's buffer) over NVLink. Two tile slots alternate, so a tile's loads run
// while the previous tile is being stored; a handful of CTAs keeps NVLink busy, which is what a
// dispatch running beside a GEMM on few SMs needs. SCALED: the warp multiplies each row by its
// combine weight in shared memory between the loads and the store.
constexpr int kTileRows = 32;

template <bool SCALED>
__global__ void __launch_bounds__(32) ep_push_bulk_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const int* __restrict__ perm,
                                                          const float* __restrict__ wperm,
                                                          const int* __restrict__ counts, EpArgs a) {
  extern __shared__ __align__(128) uint8_t sm_push[];
  __shared__ uint64_t full[2];
  __shared__ int abort_sm;
  const int lane = threadIdx.x;
  const uint32_t rb = (uint32_t)a.D * 2;                     // row bytes, a multiple of 16
  const size_t tile_bytes = (size_t)kTileRows * rb;
  const int E = a.e_loc * a.world;
  if (!SCALED && blockIdx.x == 0 && a.s_lo == 0)
    for (int e = lane; e < E; e += 32) {
      int* dst = reinterpret_cast<int*>(peer_ptr(a.peers, e / a.e_loc, a.counts_off));
      dst[a.my * a.e_loc + e % a.e_loc] = counts[e];
    }
  if (lane == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    abort_sm = 0;
    fence_barrier_init();
  }
  __syncwarp();
  // tiles of expert e: slots [lo, hi) = [s_lo, min(s_hi, round128(count))) in steps of 32; the CTA
  // takes global tile indices blockIdx.x, blockIdx.x + gridDim.x, ... (walking the experts once)
  int e = 0, t0 = 0;  // expert of the next tile, global index of that expert's first tile
  auto tiles_of = [&](int ee) {
    const int hi = min(a.s_hi, round128(counts[ee])), lo = a.s_lo;
    return hi > lo ? (hi - lo + kTileRows - 1) / kTileRows : 0;
  };
  int nt_e = E > 0 ? tiles_of(0) : 0;
  bool ok = true;
  int it = 0;
  int pend_e = -1, pend_s0 = 0, pend_n = 0, pend_c = 0;  // the tile whose loads are in flight
  for (int t = blockIdx.x;; t += gridDim.x, ++it) {
    // locate global tile t (t only grows, so the expert walk is shared by the whole loop)
    bool have = false;
    int te = 0, s0 = 0, n = 0, c = 0;
    while (e < E) {
      if (t < t0 + nt_e) {
        te = e;
        c = counts[e];
        s0 = a.s_lo + (t - t0) * kTileRows;
        n = min(kTileRows, min(a.s_hi, round128(c)) - s0);
        have = true;
        break;
      }
      t0 += nt_e;
      ++e;
      if (e < E) nt_e = tiles_of(e);
    }
    if (have) {
      const int slot = it & 1;
      uint8_t* buf = sm_push + slot * tile_bytes;
      if (lane == 0) {
        if (it >= 2) bulk_wait_read<0>();  // the slot's previous tile has been read by its store
        uint32_t real = 0;
        for (int i = 0; i < n; ++i) real += (s0 + i < c) ? rb : 0;
        mbar_arrive_expect_tx(&full[slot], real);
      }
      __syncwarp();
      const int s = s0 + lane;
      if (lane < n) {
        uint8_t* row = buf + (size_t)lane * rb;
        if (s < c) {
          bulk_load(row, x + (long)perm[(long)te * a.cap + s] * a.D, rb, &full[slot]);
        } else {
          for (uint32_t i = 0; i < rb / 16; ++i) reinterpret_cast<uint4*>(row)[i] = make_uint4(0, 0, 0, 0);
        }
      }
    }
    // store the tile loaded in the previous iteration
    if (pend_e >= 0) {
      const int slot = (it - 1) & 1;
      uint8_t* buf = sm_push + slot * tile_bytes;
      // every lane observes the phase (the scaling reads the loaded rows)
      const bool got = mbar_wait(&full[slot], ((it - 1) >> 1) & 1, nullptr, kErrTimeoutPeer, &abort_sm);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      if (SCALED) {
        for (int i = 0; i < pend_n; ++i) {
          if (pend_s0 + i >= pend_c) break;
          const float w = wperm[(long)pend_e * a.cap + pend_s0 + i];
          uint4* row = reinterpret_cast<uint4*>(buf + (size_t)i * rb);
          for (uint32_t k = lane; k < rb / 16; k += 32) {
            float f[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            acc8(f, row[k], w);
            row[k] = pack8(f);
          }
        }
      }
      fence_proxy_async_smem();  // zero-filled pad rows (and scaled rows) are read by the bulk store
      __syncwarp();
      if (lane == 0) {
        uint4* dst = reinterpret_cast<uint4*>(peer_ptr(a.peers, pend_e / a.e_loc, a.buf_off)) +
                     remote_row(pend_e, pend_s0, a.e_loc, a.cap, a.my) * (a.D / 8);
        bulk_store(dst, buf, (uint32_t)pend_n * rb);
        bulk_commit();
      }
    }
    if (!have) break;
    pend_e = te;
    pend_s0 = s0;
    pend_n = n;
    pend_c = c;
  }
  if (lane == 0) bulk_wait_all();  // every store has landed in the peers' memory
  __syncwarp();
  if (ok) publish(a.peers, a.world, a.my, a.flags_off, a.purpose, a.epoch, a.counter);
}

// Pulls with all of a token's K rows in flight at once. The kernels above walk k inside the chunk
// loop, so each 16-byte peer load waits for the previous one (and the slot / expert lookups are
// repeated per chunk): a chain of K dependent NVLink round trips per chunk. Here lanes 0..K-1 read
// the token's K (slot, expert, weight) once and broadcast them, the K row pointers are formed once,
// and every chunk issues its K loads back to back before accumulating.
template <int KMAX>
__device__ __forceinline__ int token_rows(const int* sel, const int* slot, const float* comb, long t, int K,
                                          const EpArgs& a, const uint4* (&src)[KMAX], float (&w)[KMAX],
                                          long (&lrow)[KMAX]) {
  const int lane = threadIdx.x & 31;
  int s = -1, e = 0;
  float wk = 0.f;
  if (lane < K) {
    s = slot[t * K + lane];
    e = sel[t * K + lane];
    if (comb) wk = comb[t * K + lane];
  }
  int n = 0;
#pragma unroll
  for (int k = 0; k < KMAX; ++k) {
    const int sk = __shfl_sync(0xffffffffu, s, k), ek = __shfl_sync(0xffffffffu, e, k);
    w[k] = __shfl_sync(0xffffffffu, wk, k);
    src[k] = nullptr;
    lrow[k] = -1;
    if (k < K && sk >= 0) {
      src[k] = reinterpret_cast<const uint4*>(peer_ptr(a.peers, ek / a.e_loc, a.buf_off)) +
               remote_row(ek, sk, a.e_loc, a.cap, a.my) * (a.D / 8);
      lrow[k] = (long)ek * a.cap + sk;
      ++n;
    }
  }
  return n;
}

template <int KMAX>
__global__ void ep_combine_pull_v2_kernel(const int* __restrict__ sel, const int* __restrict__ slot,
                                          const float* __restrict__ comb, const __nv_bfloat16* __restrict__ residual,
                                          __nv_bfloat16* __restrict__ out, __nv_bfloat16* __restrict__ y_local, int T,
                                          int K, EpArgs a) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    const uint4* src[KMAX];
    float w[KMAX];
    long lrow[KMAX];
    token_rows<KMAX>(sel, slot, comb, t, K, a, src, w, lrow);
    for (int c = lane; c < a.D / 8; c += 32) {
      uint4 v[KMAX];
#pragma unroll
      for (int k = 0; k < KMAX; ++k)
        if (src[k]) v[k] = __ldcv(src[k] + c);
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (residual) acc8(acc, reinterpret_cast<const uint4*>(residual + (long)t * a.D)[c], 1.f);
#pragma unroll
      for (int k = 0; k < KMAX; ++k)
        if (src[k]) {
          if (y_local) reinterpret_cast<uint4*>(y_local + lrow[k] * a.D)[c] = v[k];
          acc8(acc, v[k], w[k]);
        }
      reinterpret_cast<uint4*>(out + (long)t * a.D)[c] = pack8(acc);
    }
  }
}

template <int KMAX>
__global__ void ep_unpermute_pull_v2_kernel(const int* __restrict__ sel, const int* __restrict__ slot,
                                            __nv_bfloat16* __restrict__ dx, int T, int K, EpArgs a) {
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  for (int t = blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += gridDim.x * warps) {
    const uint4* src[KMAX];
    float w[KMAX];
    long lrow[KMAX];
    token_rows<KMAX>(sel, slot, nullptr, t, K, a, src, w, lrow);
    for (int c = lane; c < a.D / 8; c += 32) {
      uint4 v[KMAX];
#pragma unroll
      for (int k = 0; k < KMAX; ++k)
        if (src[k]) v[k] = __ldcv(src[k] + c);
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int k = 0; k < KMAX; ++k)
        if (src[k]) acc8(acc, v[k], 1.f);
      reinterpret_cast<uint4*>(dx + (long)t * a.D)[c] = pack8(acc);
    }
  }
}

// Publish `epoch` for (purpose, my) to every peer once the previous work on the stream is done
// (e.g. after the expert GEMMs that wrote the buffer the peers will pull).
__global__ void ep_signal_kernel(PeerTable peers, int world, int my, size_t flags_off, int purpose, int epoch) {
  __threadfence_system();
  if (threadIdx.x < world) st_release_sys(flag_slot(peers, threadIdx.x, flags_off, purpose, my), epoch);
}

// Wait until every source's flag for `purpose` reached `epoch` (bounded).
// The limit is wall time (the global timer), so it does not depend on the SM clock.
__global__ void ep_wait_kernel(PeerTable peers, int world, int my, size_t flags_off, int purpose, int epoch,
                               int* err, long long limit_ns) {
  if (threadIdx.x < world) {
    const int* f = flag_slot(peers, my, flags_off, purpose, threadIdx.x);
    const long long t0 = global_ns();
    while (ld_acquire_sys(f) < epoch) {
      if (global_ns() - t0 > limit_ns) {
        atomicExch(err, kErrTimeoutPeer);
        break;
      }
      __nanosleep(128);
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------- ZeRO over peer memory
// Reduce-scatter fused with the mean: out[k] = scale * sum_r grad_r[k] for k in [lo, hi), reading
// every rank's gradient buffer (heap offset grad_off) over NVLink. 16-byte loads; lo, hi and the
// buffers are 16-byte aligned (the store pads its shards to 64 elements).
__global__ void zero_rs_kernel(PeerTable peers, int world, size_t grad_off, long long lo, long long hi,
                               float* __restrict__ out, float scale) {
  const long long n4 = (hi - lo) >> 2;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const long long k = lo + (i << 2);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < world; ++r) {
      const float4 v = __ldcv(reinterpret_cast<const float4*>(peer_ptr(peers, r, grad_off)) + (k >> 2));
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    acc.x *= scale; acc.y *= scale; acc.z *= scale; acc.w *= scale;
    reinterpret_cast<float4*>(out)[k >> 2] = acc;
  }
}

// All-gather fused with the bf16 cast: for k in [0, end), rank k / per owns element k; the other
// ranks' elements are read from their master buffers (heap offset master_off) into `master`, and
// every element's bf16 copy is written to `compute`.
__global__ void zero_ag_kernel(PeerTable peers, int world, int my, size_t master_off, long long per, long long end,
                               float* __restrict__ master, __nv_bfloat16* __restrict__ compute) {
  const long long n4 = end >> 2;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const long long k = i << 2;
    const int owner = (int)(k / per);
    float4 v;
    if (owner == my || owner >= world) {
      v = reinterpret_cast<const float4*>(master)[i];
    } else {
      v = __ldcv(reinterpret_cast<const float4*>(peer_ptr(peers, owner, master_off)) + i);
      reinterpret_cast<float4*>(master)[i] = v;
    }
    __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<uint32_t*>(&a);
    u.y = *reinterpret_cast<uint32_t*>(&b);
    reinterpret_cast<uint2*>(compute)[i] = u;
  }
}

inline int grid_rows(long work) {
  long g = (work + 7) / 8;
  if (g > 148 * 8) g = 148 * 8;
  return g < 1 ? 1 : (int)g;
}

}  // namespace

// MXK_EP_XCHG=v1 selects the one-chunk-at-a-time exchange kernels (kept as the baseline)
static bool xchg_v2() {
  static const bool v2 = [] {
    const char* e = std::getenv("MXK_EP_XCHG");
    return !(e && std::string(e) == "v1");
  }();
  return v2;
}

// MXK_EP_PUSH=bulk: copy-engine pushes for the single-exchange path too (chunked dispatches, which
// run beside a GEMM on few CTAs, always use them)
static bool push_bulk_default() {
  static const bool on = [] {
    const char* e = std::getenv("MXK_EP_PUSH");
    return e && std::string(e) == "bulk";
  }();
  return on;
}

template <bool SCALED>
static bool launch_push_bulk(const void* x, const int* perm, const float* wperm, const int* counts, const EpArgs& a,
                             cudaStream_t st) {
  if (!(a.max_blocks > 0 || push_bulk_default()) || a.D % 8) return false;
  const size_t rb = (size_t)a.D * 2;
  const size_t smem = 2 * kTileRows * rb;  // two 32-row tile slots
  if (smem > 220 * 1024) return false;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(ep_push_bulk_kernel<SCALED>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024) !=
        cudaSuccess)
      return false;
    attr = true;
  }
  const int g = a.max_blocks > 0 ? a.max_blocks : 32;
  ep_push_bulk_kernel<SCALED><<<g, 32, smem, st>>>((const __nv_bfloat16*)x, perm, wperm, counts, a);
  return true;
}

template <bool SCALED>
static bool launch_push_v2(const void* x, const int* perm, const float* wperm, const int* counts, const EpArgs& a,
                           cudaStream_t st) {
  if (launch_push_bulk<SCALED>(x, perm, wperm, counts, a, st)) return true;
  if (!xchg_v2() || a.D % 256) return false;
  int g = grid_rows((long)a.e_loc * a.world * a.cap);
  if (a.max_blocks > 0 && g > a.max_blocks) g = a.max_blocks;
  const auto* xb = (const __nv_bfloat16*)x;
  switch (a.D / 256) {
    case 2: ep_push_v2_kernel<2, SCALED><<<g, 256, 0, st>>>(xb, perm, wperm, counts, a); return true;
    case 3: ep_push_v2_kernel<3, SCALED><<<g, 256, 0, st>>>(xb, perm, wperm, counts, a); return true;
    case 4: ep_push_v2_kernel<4, SCALED><<<g, 256, 0, st>>>(xb, perm, wperm, counts, a); return true;
    case 6: ep_push_v2_kernel<6, SCALED><<<g, 256, 0, st>>>(xb, perm, wperm, counts, a); return true;
    case 8: ep_push_v2_kernel<8, SCALED><<<g, 256, 0, st>>>(xb, perm, wperm, counts, a); return true;
    default: return false;
  }
}

void launch_ep_dispatch_push(const void* x, const int* perm, const int* counts, const EpArgs& a, cudaStream_t st) {
  count_launch();
  if (launch_push_v2<false>(x, perm, nullptr, counts, a, st)) return;
  int g = grid_rows((long)a.e_loc * a.world * a.cap);
  if (a.max_blocks > 0 && g > a.max_blocks) g = a.max_blocks;
  ep_dispatch_push_kernel<<<g, 256, 0, st>>>((const __nv_bfloat16*)x, perm, counts, a);
}

void launch_ep_combine_bwd_push(const void* dout, const int* perm, const float* wperm, const int* counts,
                                const EpArgs& a, cudaStream_t st) {
  count_launch();
  if (launch_push_v2<true>(dout, perm, wperm, counts, a, st)) return;
  int g = grid_rows((long)a.e_loc * a.world * a.cap);
  if (a.max_blocks > 0 && g > a.max_blocks) g = a.max_blocks;
  ep_combine_bwd_push_kernel<<<g, 256, 0, st>>>((const __nv_bfloat16*)dout, perm, wperm, counts, a);
}

static bool pull_v2() { return xchg_v2(); }

void launch_ep_combine_pull(const int* sel, const int* slot, const float* comb, const void* residual, void* out,
                            void* y_local, int T, int K, const EpArgs& a, cudaStream_t st) {
  count_launch();
  const auto* r = (const __nv_bfloat16*)residual;
  auto* o = (__nv_bfloat16*)out;
  auto* y = (__nv_bfloat16*)y_local;
  if (pull_v2() && K <= 4)
    ep_combine_pull_v2_kernel<4><<<grid_rows(T), 256, 0, st>>>(sel, slot, comb, r, o, y, T, K, a);
  else if (pull_v2() && K <= 8)
    ep_combine_pull_v2_kernel<8><<<grid_rows(T), 256, 0, st>>>(sel, slot, comb, r, o, y, T, K, a);
  else
    ep_combine_pull_kernel<<<grid_rows(T), 256, 0, st>>>(sel, slot, comb, r, o, y, T, K, a);
}

void launch_ep_unpermute_pull(const int* sel, const int* slot, void* dx, int T, int K, const EpArgs& a,
                              cudaStream_t st) {
  count_launch();
  auto* d = (__nv_bfloat16*)dx;
  if (pull_v2() && K <= 4)
    ep_unpermute_pull_v2_kernel<4><<<grid_rows(T), 256, 0, st>>>(sel, slot, d, T, K, a);
  else if (pull_v2() && K <= 8)
    ep_unpermute_pull_v2_kernel<8><<<grid_rows(T), 256, 0, st>>>(sel, slot, d, T, K, a);
  else
    ep_unpermute_pull_kernel<<<grid_rows(T), 256, 0, st>>>(sel, slot, d, T, K, a);
}

void launch_zero_rs(const PeerTable& peers, int world, size_t grad_off, long long lo, long long hi, float* out,
                    float scale, cudaStream_t st) {
  count_launch();
  zero_rs_kernel<<<148 * 8, 256, 0, st>>>(peers, world, grad_off, lo, hi, out, scale);
}

void launch_zero_ag(const PeerTable& peers, int world, int my, size_t master_off, long long per, long long end,
                    float* master, void* compute, cudaStream_t st) {
  count_launch();
  zero_ag_kernel<<<148 * 8, 256, 0, st>>>(peers, world, my, master_off, per, end, master, (__nv_bfloat16*)compute);
}

void launch_ep_signal(const EpArgs& a, cudaStream_t st) {
  count_launch();
  ep_signal_kernel<<<1, 32, 0, st>>>(a.peers, a.world, a.my, a.flags_off, a.purpose, a.epoch);
}

void launch_ep_wait(const EpArgs& a, int* err, long long limit_ns, cudaStream_t st) {
  count_launch();
  ep_wait_kernel<<<1, 32, 0, st>>>(a.peers, a.world, a.my, a.flags_off, a.purpose, a.epoch, err,
                                   limit_ns > 0 ? limit_ns : kPeerWaitNs);
}

// ----------------------------------------------------------------------------------- host IPC
int ipc_alloc(size_t bytes, void** ptr, void* handle_out) {
  if (cudaMalloc(ptr, bytes) != cudaSuccess) return 1;
  if (cudaMemset(*ptr, 0, bytes) != cudaSuccess) return 2;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, *ptr) != cudaSuccess) return 3;
  memcpy(handle_out, &h, sizeof(h));
  return 0;
}

int ipc_open(const void* handle, void** ptr) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? 0 : 1;
}

int ipc_close(void* ptr) { return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? 0 : 1; }

int ipc_free(void* ptr) { return cudaFree(ptr) == cudaSuccess ? 0 : 1; }

}  // namespace mxk
