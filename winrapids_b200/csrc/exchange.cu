// exchange.cu -- the exchange step of the sharded dense groupby over NVLink peer memory.
//
// Each GPU reduces its row shard to a mergeable state table (ST_COUNT x G doubles: the Chan /
// Pébay state of descriptive.rs:216-253, intermediates.rs:352-377), and every GPU needs every
// table to fold them in rank order.  Instead of a library all-gather, each rank writes its table
// straight into its slot of every peer's exchange buffer (plain stores to memory mapped from the
// peer with CUDA IPC; no multicast), fences at system scope and raises its flag in every buffer;
// each rank then waits for all flags of its own buffer and folds the slots, reading only local
// memory.
//
// Buffer: [2][world] slots (the slot parity is the epoch's, so a rank one step ahead never writes
// the slots a slower rank is still folding) followed by world u64 flags.  A flag holds the last
// epoch its rank pushed; waiting for flag >= epoch tolerates a rank that already moved on.  A rank
// can run at most one epoch ahead of another's fold: its next push needs that rank's flag of the
// current epoch, which that rank raises only after its own fold of the previous epoch.  The wait
// is bounded (about 2 s of wall time): past it the kernel reports KERR_TIMEOUT and returns.
#include <cstdint>

#include "common.cuh"
#include "dense.cuh"
#include "errbits.hpp"
#include "exchange.cuh"
#include "gstate.cuh"

namespace tbgb {

namespace {

constexpr int XNT = 256;

size_t round256(size_t x) { return (x + 255) / 256 * 256; }

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// One block: copy the own slot to every peer's slot, fence, raise the flags.
__global__ void __launch_bounds__(1024) exchange_push_kernel(PeerPtrs peers, int world, int rank,
                                                             long long slot_off_words, long long words,
                                                             long long flags_off_words, unsigned long long epoch) {
  const double* src = static_cast<const double*>(peers.p[rank]) + slot_off_words;
  for (int q = 0; q < world; ++q) {
    if (q == rank) continue;
    double* dst = static_cast<double*>(peers.p[q]) + slot_off_words;
    for (long long i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < world) {
    unsigned long long* flags = reinterpret_cast<unsigned long long*>(static_cast<double*>(peers.p[threadIdx.x]) +
                                                                       flags_off_words);
    st_release_sys(flags + rank, epoch);
  }
}

__global__ void __launch_bounds__(XNT) exchange_merge_kernel(const double* own, long long slots_off_words,
                                                             long long slot_words, const unsigned long long* flags,
                                                             int world, int G, unsigned long long epoch,
                                                             uint32_t* err, tbgb_moments out) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int q = 0; q < world && ok; ++q) {
      while (ld_acquire_sys(flags + q) < epoch) {
        if (globaltimer_ns() - t0 > 2000000000ull) {
          atomicOr(err, KERR_TIMEOUT);
          ok = 0;
          break;
        }
        __nanosleep(200);
      }
    }
  }
  __syncthreads();
  const int g = blockIdx.x * XNT + threadIdx.x;
  if (!ok || g >= G) return;
  GState A = gstate_empty();
  for (int r = 0; r < world; ++r) {
    const GState B = gstate_load(own + slots_off_words + static_cast<long long>(r) * slot_words, G, g);
    gstate_fold(A, B);
  }
  gstate_finalize(A, g, out);
}

}  // namespace

long long exchange_slot_words(int G) { return static_cast<long long>(ST_COUNT) * G; }

size_t exchange_slot_offset(int world, int G, int parity, int rank) {
  return static_cast<size_t>(parity * world + rank) * static_cast<size_t>(exchange_slot_words(G)) * 8;
}

size_t exchange_flags_offset(int world, int G) {
  return round256(static_cast<size_t>(2 * world) * static_cast<size_t>(exchange_slot_words(G)) * 8);
}

size_t exchange_bytes(int world, int G) {
  return exchange_flags_offset(world, G) + round256(static_cast<size_t>(world + 1) * 8);
}

PushArgs exchange_push_args(const PeerPtrs& peers, int world, int rank, int G, unsigned long long epoch) {
  PushArgs a{};
  const int parity = static_cast<int>(epoch & 1ull);
  const size_t slot_off = exchange_slot_offset(world, G, parity, rank);
  const size_t flags_off = exchange_flags_offset(world, G);
  for (int q = 0; q < world; ++q) {
    char* base = static_cast<char*>(peers.p[q]);
    a.slot[q] = reinterpret_cast<double*>(base + slot_off);
    a.flag[q] = reinterpret_cast<unsigned long long*>(base + flags_off) + rank;
  }
  // the word after the world flags of the own buffer (inside its 256-byte rounding; zeroed at
  // allocation, and returned to zero by the block that uses it)
  a.counter = reinterpret_cast<unsigned int*>(reinterpret_cast<unsigned long long*>(
      static_cast<char*>(peers.p[rank]) + flags_off) + world);
  a.world = world;
  a.rank = rank;
  a.epoch = epoch;
  return a;
}

cudaError_t exchange_push_launch(const PeerPtrs& peers, int world, int rank, int G, unsigned long long epoch,
                                 cudaStream_t s, uint64_t* launches) {
  const int parity = static_cast<int>(epoch & 1ull);
  const long long slot_off = static_cast<long long>(exchange_slot_offset(world, G, parity, rank) / 8);
  const long long flags_off = static_cast<long long>(exchange_flags_offset(world, G) / 8);
  exchange_push_kernel<<<1, 1024, 0, s>>>(peers, world, rank, slot_off, exchange_slot_words(G), flags_off, epoch);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) (*launches)++;
  return e;
}

cudaError_t exchange_merge_launch(const void* own, int world, int G, unsigned long long epoch, uint32_t* err,
                                  const tbgb_moments* out, cudaStream_t s, uint64_t* launches) {
  const int parity = static_cast<int>(epoch & 1ull);
  const double* base = static_cast<const double*>(own);
  const long long slots_off = static_cast<long long>(exchange_slot_offset(world, G, parity, 0) / 8);
  const auto* flags = reinterpret_cast<const unsigned long long*>(static_cast<const char*>(own) +
                                                                  exchange_flags_offset(world, G));
  exchange_merge_kernel<<<(G + XNT - 1) / XNT, XNT, 0, s>>>(base, slots_off, exchange_slot_words(G), flags, world, G,
                                                            epoch, err, *out);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) (*launches)++;
  return e;
}

}  // namespace tbgb
