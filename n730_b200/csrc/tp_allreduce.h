// One-shot allreduce of a row-split projection's partial sums over peer
// memory (tensor-parallel decode), fused with the residual add.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace n730 {

constexpr int AR_MAX_RANKS = 8;
constexpr int AR_SLICES = 32;  // CTAs of one allreduce; slice s of the vector is CTA s's

// The exchange region of one rank (one cudaMalloc, exported with cudaIpcGetMemHandle):
//   flags [2 parity][ranks][AR_SLICES] int    - epoch of the last slice each rank pushed here
//   recv  [2 parity][ranks][cap] float        - the partial sums each rank pushed here
//   xcnt  int                                 - cross-GPU barrier counter of the persistent
//                                               tensor-parallel decode kernel (which reuses recv)
// plus, not shared: epoch (int, ops done) and done (int, CTAs finished in the current op).
struct ArRegion {
  int* flags = nullptr;
  float* recv = nullptr;
  int* xcnt = nullptr;
};

struct ArArgs {
  const float* part;                      // [n] this rank's partial sums
  float* x;                               // [n] residual stream, x += sum over ranks (rank order)
  int n;                                  // elements (batch x hidden), n <= cap, n % 4 == 0
  int rank, size;
  int64_t cap;                            // recv floats per (parity, rank)
  ArRegion local;                         // this rank's region
  ArRegion peer[AR_MAX_RANKS];            // every rank's region mapped here (peer[rank] = local)
  int* epoch;                             // this rank's op counter
  int* done;                              // CTAs finished in the current op
  int* err;                               // device error word (DEV_ERR_TIMEOUT when a peer never arrives)
  uint64_t wait_ns = 0;                   // limit of the wait for a peer's slice (0: AR_WAIT_NS, 2 s)
};

// Bytes of the shared part of a region for `size` ranks and `cap` floats per slot.
size_t ar_region_bytes(int size, int64_t cap);
// Carve a region out of `base` (ar_region_bytes bytes).
ArRegion ar_region_at(void* base, int size);
// x += sum_r part_r (rank order): push this rank's slices into every rank's
// region, raise the slice flags, wait (bounded) for every rank's slice, sum.
int ar_launch(const ArArgs& a, cudaStream_t st);

}  // namespace n730
