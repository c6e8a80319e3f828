// exchange.cuh -- state exchange of the sharded dense groupby over peer memory (exchange.cu).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "tambear_gb.h"

namespace tbgb {

constexpr int kMaxRanks = 8;  // GPUs of one node

struct PeerPtrs {
  void* p[kMaxRanks];
};

// The fold kernel's push into the peers (the fused exchange): where this rank's slot lies in
// every buffer (its own included), every buffer's flag of this rank, and a block counter in the
// own buffer (the last block to finish raises the flags).  world == 0: no push.
struct PushArgs {
  double* slot[kMaxRanks];
  unsigned long long* flag[kMaxRanks];
  unsigned int* counter;
  int world;
  int rank;
  unsigned long long epoch;
};
PushArgs exchange_push_args(const PeerPtrs& peers, int world, int rank, int G, unsigned long long epoch);

// Doubles of one rank's slot (a state table of G groups).
long long exchange_slot_words(int G);
// Bytes of an exchange buffer: [2 parities][world slots] state tables, then world u64 flags.
size_t exchange_bytes(int world, int G);
// Byte offset of slot (parity, rank) and of the flags inside an exchange buffer.
size_t exchange_slot_offset(int world, int G, int parity, int rank);
size_t exchange_flags_offset(int world, int G);

// Copies this rank's slot (already written in its own buffer) into the same slot of every
// peer's buffer, then raises flag[rank] = epoch in every buffer (release, system scope).
cudaError_t exchange_push_launch(const PeerPtrs& peers, int world, int rank, int G, unsigned long long epoch,
                                 cudaStream_t s, uint64_t* launches);

// Waits (bounded) until every flag of the own buffer is >= epoch, then folds the slots of
// the epoch's parity in rank order into `out`.
cudaError_t exchange_merge_launch(const void* own, int world, int G, unsigned long long epoch, uint32_t* err,
                                  const tbgb_moments* out, cudaStream_t s, uint64_t* launches);

}  // namespace tbgb
