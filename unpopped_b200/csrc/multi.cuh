// multi.cuh — what scan.cu and comm.cu share for scans sharded over the GPUs of one node.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace up {

// The cross-GPU part of a scan sharded block-cyclically over the ranks of a communicator (the MULTI form of the
// persistent scan). The global array is a sequence of stripes of kStripeTiles tiles of 8192 elements (one tile per
// CTA of the persistent grid); stripe s lives on rank s % G as that rank's local stripe s / G. Each rank's CTA 0
// publishes the aggregate of each of its local stripes into every other rank's stripe words (peer stores over
// NVLink); the look-back adds, to the local chain of tile aggregates, the aggregates of the other ranks' stripes
// that sit between a CTA's previous tile and its next one in the global order.
constexpr int kMaxRanks = 8;
constexpr int kStripeTiles = 148;  // the persistent grid of the block-cyclic form (one CTA per SM of a B200)
constexpr int64_t kStripeElems = (int64_t)kStripeTiles * 8192;

struct MultiScan {
  const uint64_t* sflags;      // this rank's stripe words, by global stripe (written by the other ranks)
  uint64_t* peers[kMaxRanks];  // every rank's stripe words, for publishing (this rank's own is not written)
  int G, r;                    // ranks, this rank
  uint32_t tag;                // the communicator's launch tag (the same on every rank)
};

// scan.cu: one rank's pass of the block-cyclic scan, and the stripe words it needs per rank.
int scan_i32_block_cyclic(const int32_t* x, int32_t* y, int64_t k, int op, int exclusive, const int32_t* carry_in,
                          void* workspace, size_t workspace_bytes, const MultiScan& m, cudaStream_t s);
int64_t block_cyclic_stripe_words(int64_t k, int G);

}  // namespace up
