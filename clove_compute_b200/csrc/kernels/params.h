// params.h -- plain parameter structs shared by the kernels and the host launchers.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace clove {
namespace kern {

enum EpiMode : int {
  kEpiF16AlphaBeta = 0,  // C = half(alpha*acc + beta*C)
  kEpiI8Tensor = 1,      // C = half(float(acc') * scale)
  kEpiI8RowCol = 2,      // C = half(float(acc) * row_scale[m] * col_scale[n])
  kEpiI32Raw = 3,        // C(int32) = acc'  (acc' = zero-point corrected acc)
};

// Replicated output of an N-split GEMM: every fp16 tile the kernel finishes is
// also TMA-stored, from the same staged shared-memory tile as the local store,
// into the row-major C of each rank (this rank's own and its peers', mapped
// through CUDA IPC; NVLink carries the remote stores), at columns col0 + n. Map d
// spans columns [0, col0 + N) of rank d's C, so the box clips at this rank's last
// column. count == 0: no replicated output.
//
// Receiver-ready handshake: rank d's C may still be read by rank d's consumers of
// the previous call when this call starts, so no remote store leaves before every
// rank has reached this call on its stream. `epoch` counts this rank's completed
// replicated calls (the completion-signal kernel that follows each call bumps it);
// at its start the call publishes epoch + 1 into slot `rank` of every rank's
// ready array (ready_slot[d] = &ready_d[rank], system-scope release) and its
// epilogue waits until every slot of its own array (ready_in) has reached
// epoch + 1 before the first remote store (bounded, like every wait here).
//
// mc != 0: the ranks' C are bound to one NVLink multicast object and mc is its
// address in this process (row pitch ldc elements). Each staged tile then leaves
// once, as multimem stores that the NVSwitch fabric delivers to every rank's C
// (this rank's included); the maps are unused.
constexpr int kMaxPeers = 8;
struct PeerOut {
  int count;
  int col0;
  int rank;
  int ldc;
  unsigned long long mc;
  unsigned long long* ready_slot[kMaxPeers];
  const unsigned long long* ready_in;
  const unsigned long long* epoch;
  CUtensorMap maps[kMaxPeers];
};

// Epilogue of the tensor-core tile kernels.
struct EpiParams {
  int mode;
  float alpha, beta;        // kEpiF16AlphaBeta
  const __half* c_in;       // beta source, row-major [M,N] (may alias C)
  float scale;              // kEpiI8Tensor: A_scale * B_scale
  const float* row_scale;   // kEpiI8RowCol
  const float* col_scale;
  int za, zb;               // int8 zero points
  const int32_t* row_sum;   // sum_k A[m,k]   (required when zb != 0)
  const int32_t* col_sum;   // sum_k B[k,n]   (required when za != 0)
  void* c_out;              // C itself (split-K tiles store rows directly)
  PeerOut peer;             // replicated output (fp16 C only)
};

// Stream-K schedule of the CTA-pair kernel. Tiles [0, dp_tiles) go round-robin to
// the pairs with their whole K range. The K blocks of tiles [dp_tiles, dp_tiles +
// sk_tiles), taken tile after tile, are cut into one contiguous range per pair of
// equal length, so every pair ends at the same time; a tile cut between several
// pairs is summed by whichever contributor finishes last (an atomic ticket), from
// 32-bit partial accumulators in `partials`. Each pair works through its stream-K
// range before its whole-K tiles. sk_tiles == 0: plain persistent tiles.
struct SkParams {
  int dp_tiles;
  int sk_tiles;
  int max_contrib;          // partial slots per stream-K tile
  uint32_t* partials;       // [sk_tiles][max_contrib][2 CTAs][64 column quads][128 rows][4]
  int* tickets;             // [sk_tiles][2 CTAs], zero at launch; the tile's last
                            // contributor sets its ticket back to zero
};

// Epilogue of the int8 GEMV (modes as EpiMode 1..3).
struct GemvI8Epi {
  int mode;
  float scale;
  const float* row_scale;   // [rows]
  const float* col_scale;   // [NC]
  int za, zb;
};

// Epilogue of the SIMT fallback (modes as EpiMode 0..3).
struct SimtEpi {
  int mode;
  float alpha, beta;
  float scale;
  const float* row_scale;
  const float* col_scale;
  int za, zb;
};

}  // namespace kern
}  // namespace clove
