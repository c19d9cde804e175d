// Argument block of the sm_100a GEMM kernel (plain C++: shared by device and host code).
#pragma once
#include <stdint.h>

namespace mxk {

struct GemmParams {
  int G, M, N, K;
  const int* counts;  // per-group ragged extent (device), or nullptr
  int ragged;         // 0: none, 1: M ragged, 2: K ragged
  int a_grp, b_grp, c_grp;
  // Group index used for B / C offsets: (b_mod ? g % b_mod : g), likewise c_mod. Lets
  // (source rank, expert) activation groups share one expert's weights and weight gradient.
  int b_mod, c_mod;
  int ksplit;  // K splits per output tile (non-grouped, accumulating fp32 C only)
  int raster_n;  // tile order: 1 = N tiles fastest, 0 = M tiles fastest (set by the launcher)
  void* C;
  int ldc;
  int c_f32;
  int c_accum;  // 0: store, 1: C += acc, 2: C += acc with atomics (groups share C rows)
  void* C2;  // EPI_SWIGLU: activation output; EPI_SILU/EPI_ACT: pre-activation copy; EPI_CE: stats
  int ldc2;
  const void* R;  // bf16 residual / gate input
  int ldr;
  const float* row_scale;
  float alpha;
  int act_kind;  // 0 silu, 1 relu, 2 gelu(tanh)
  int* err;
  // Peer-store epilogue (EPI_STORE, bf16 C, grouped): when peer_maps is set, group g's rows go to
  // rank g / peer_epl through the g / peer_epl-th tensor map of the device array peer_maps (one
  // 64-byte-aligned CUtensorMap per rank over that rank's [E][cap][N] buffer), at row
  // (peer_my * peer_epl + g % peer_epl) * peer_cap + (row within the group).
  const void* peer_maps;
  int peer_epl, peer_my, peer_cap;
};

}  // namespace mxk
