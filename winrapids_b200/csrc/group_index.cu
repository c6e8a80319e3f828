// group_index.cu -- key factorisation on the device.
//
// GroupIndex::build (crates/tambear/src/group_index.rs:117-204) builds, on the host, for a
// dense int32 key column with keys in [0, max_key]:
//   row_to_group[i] = keys[i]; group_counts[g]; group_offsets = exclusive prefix of the
//   counts with group_offsets[max_key + 1] = n; rows_by_group = row ids ordered by group,
//   row order kept inside a group; n_active = groups with a row.
// Here: one pass writes row_to_group and the counts (shared-memory histograms when the
// counts fit), one block scans the offsets, and a stable radix sort of (key, row) pairs
// produces rows_by_group.
//
// Dictionary (crates/tambear/src/dictionary.rs:40-75) assigns codes to values in the order
// they are first seen.  For int64 keys the same codes come from a device hash table: each
// slot keeps its key's first row; the distinct keys are compacted, sorted by first row
// (stable radix sort), numbered, and every row is given its key's number.
#include <cstdint>

#include "common.cuh"
#include "group_index.cuh"
#include "rowops.cuh"
#include "sort.cuh"

namespace tbgb {

namespace {

constexpr int GNT = 256;
constexpr int kSmemCounts = 12288;  // groups whose counts are privatised in shared memory

__global__ void __launch_bounds__(GNT) gi_count_kernel(const int32_t* __restrict__ keys, long long n, int G,
                                                       uint32_t* row_to_group, uint32_t* counts, uint32_t* err) {
  extern __shared__ unsigned int sc[];
  const bool priv = G <= kSmemCounts;
  if (priv) {
    for (int g = threadIdx.x; g < G; g += GNT) sc[g] = 0;
    __syncthreads();
  }
  for (long long i = blockIdx.x * static_cast<long long>(GNT) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * GNT) {
    const int k = __ldcs(keys + i);
    row_to_group[i] = static_cast<uint32_t>(k);
    if (static_cast<unsigned>(k) >= static_cast<unsigned>(G)) {
      atomicOr(err, KERR_KEY_RANGE);
      continue;
    }
    if (priv) atomicAdd(sc + k, 1u);
    else atomicAdd(counts + k, 1u);
  }
  if (priv) {
    __syncthreads();
    for (int g = threadIdx.x; g < G; g += GNT)
      if (sc[g]) atomicAdd(counts + g, sc[g]);
  }
}

// offsets[g] = sum of counts[0..g), offsets[G] = total; n_active = groups with a row.
__global__ void __launch_bounds__(1024) gi_offsets_kernel(const uint32_t* __restrict__ counts, int G,
                                                          uint32_t* offsets, int64_t* n_active) {
  __shared__ unsigned int warp_sums[32];
  __shared__ unsigned int warp_act[32];
  __shared__ unsigned int carry, active;
  if (threadIdx.x == 0) { carry = 0; active = 0; }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int b = 0; b < G; b += 1024) {
    const int g = b + threadIdx.x;
    const unsigned int x = g < G ? counts[g] : 0u;
    unsigned int inc = x;
    for (int d = 1; d < 32; d <<= 1) {
      const unsigned int y = __shfl_up_sync(0xffffffffu, inc, d);
      if (lane >= d) inc += y;
    }
    const unsigned int act = __popc(__ballot_sync(0xffffffffu, x != 0));
    if (lane == 31) { warp_sums[warp] = inc; warp_act[warp] = act; }
    __syncthreads();
    if (warp == 0) {
      unsigned int w = warp_sums[lane];
      for (int d = 1; d < 32; d <<= 1) {
        const unsigned int y = __shfl_up_sync(0xffffffffu, w, d);
        if (lane >= d) w += y;
      }
      warp_sums[lane] = w;
    }
    __syncthreads();
    const unsigned int before = carry + (warp > 0 ? warp_sums[warp - 1] : 0u) + inc - x;
    if (g < G) offsets[g] = before;
    __syncthreads();
    if (threadIdx.x == 1023) carry = before + x;
    if (threadIdx.x == 0) {
      unsigned int a = 0;
      for (int w = 0; w < 32; ++w) a += warp_act[w];
      active += a;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    offsets[G] = carry;
    *n_active = static_cast<int64_t>(active);
  }
}

// ---- int64 keys: first-seen codes --------------------------------------------------------
// Slot: key (INT64_MIN when free), first row, code, unused.  The key INT64_MIN itself lives in
// the sentinel slot after the table, which counts as used once its first row is set.
constexpr unsigned long long kFree = 0x8000000000000000ull;
constexpr int kFzMaxProbe = 4096;
enum { FZ_KEY = 0, FZ_FIRST, FZ_CODE, FZ_PAD, FZ_WORDS };

__global__ void fz_init_kernel(unsigned long long* T, unsigned long long nslots) {
  for (unsigned long long s = blockIdx.x * static_cast<unsigned long long>(blockDim.x) + threadIdx.x; s < nslots;
       s += static_cast<unsigned long long>(gridDim.x) * blockDim.x) {
    ulonglong2* p = reinterpret_cast<ulonglong2*>(T + s * FZ_WORDS);
    p[0] = make_ulonglong2(kFree, ~0ull);
    p[1] = make_ulonglong2(~0ull, 0ull);
  }
}

// Slot of `key` (inserted when absent and `insert`), or -1.
__device__ __forceinline__ long long fz_slot(unsigned long long* T, unsigned long long slots, unsigned long long key,
                                             bool insert, uint32_t* err) {
  if (key == kFree) return static_cast<long long>(slots);
  unsigned long long h = fmix64(key) & (slots - 1);
  for (int probe = 0; probe < kFzMaxProbe; ++probe) {
    const unsigned long long cur = __ldcg(T + h * FZ_WORDS);
    if (cur == key) return static_cast<long long>(h);
    if (cur == kFree) {
      if (!insert) return -1;
      const unsigned long long old = atomicCAS(T + h * FZ_WORDS, kFree, key);
      if (old == kFree || old == key) return static_cast<long long>(h);
    }
    h = (h + 1) & (slots - 1);
  }
  if (insert) atomicOr(err, KERR_TABLE_FULL);
  return -1;
}

__global__ void __launch_bounds__(GNT) fz_insert_kernel(const int64_t* __restrict__ keys, long long n,
                                                        unsigned long long* T, unsigned long long slots,
                                                        uint32_t* err) {
  for (long long i = blockIdx.x * static_cast<long long>(GNT) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * GNT) {
    const long long s = fz_slot(T, slots, static_cast<unsigned long long>(__ldcs(keys + i)), true, err);
    if (s < 0) continue;
    unsigned long long* f = T + static_cast<unsigned long long>(s) * FZ_WORDS + FZ_FIRST;
    if (static_cast<unsigned long long>(i) < __ldcg(f)) atomicMin(f, static_cast<unsigned long long>(i));
  }
}

// Used slots -> (first row, slot index) pairs, in slot order: per-block counts, one block
// scanning them, then each block writing its pairs from its offset.
constexpr int FZ_CHUNK = GNT * 16;

__device__ __forceinline__ bool fz_used(const unsigned long long* T, unsigned long long i, unsigned long long slots) {
  return i < slots ? T[i * FZ_WORDS + FZ_KEY] != kFree : T[i * FZ_WORDS + FZ_FIRST] != ~0ull;
}

__global__ void __launch_bounds__(GNT) fz_count_kernel(const unsigned long long* __restrict__ T,
                                                       unsigned long long slots, unsigned int* counts) {
  const unsigned long long total = slots + 1;
  unsigned int c = 0;
  for (int k = 0; k < FZ_CHUNK / GNT; ++k) {
    const unsigned long long i = static_cast<unsigned long long>(blockIdx.x) * FZ_CHUNK +
                                 static_cast<unsigned long long>(k) * GNT + threadIdx.x;
    if (i < total && fz_used(T, i, slots)) ++c;
  }
  for (int o = 16; o > 0; o >>= 1) c += __shfl_down_sync(0xffffffffu, c, o);
  __shared__ unsigned int ws[GNT / 32];
  if ((threadIdx.x & 31) == 0) ws[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned int t = 0;
    for (int w = 0; w < GNT / 32; ++w) t += ws[w];
    counts[blockIdx.x] = t;
  }
}

__global__ void __launch_bounds__(1024) fz_scan_kernel(unsigned int* counts, long long len, long long max_groups,
                                                       int64_t* n_uniques, unsigned long long* n_dev, uint32_t* err) {
  __shared__ unsigned int warp_sums[32];
  __shared__ unsigned int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (long long b = 0; b < len; b += 1024) {
    const long long i = b + threadIdx.x;
    const unsigned int x = i < len ? counts[i] : 0u;
    unsigned int inc = x;
    for (int d = 1; d < 32; d <<= 1) {
      const unsigned int y = __shfl_up_sync(0xffffffffu, inc, d);
      if (lane >= d) inc += y;
    }
    if (lane == 31) warp_sums[warp] = inc;
    __syncthreads();
    if (warp == 0) {
      unsigned int w = warp_sums[lane];
      for (int d = 1; d < 32; d <<= 1) {
        const unsigned int y = __shfl_up_sync(0xffffffffu, w, d);
        if (lane >= d) w += y;
      }
      warp_sums[lane] = w;
    }
    __syncthreads();
    const unsigned int before = carry + (warp > 0 ? warp_sums[warp - 1] : 0u) + inc - x;
    if (i < len) counts[i] = before;
    __syncthreads();
    if (threadIdx.x == 1023) carry = before + x;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    *n_dev = carry;
    *n_uniques = static_cast<int64_t>(carry < static_cast<unsigned long long>(max_groups) ? carry : max_groups);
    if (carry > static_cast<unsigned long long>(max_groups)) atomicOr(err, KERR_TABLE_FULL);
  }
}

__global__ void __launch_bounds__(GNT) fz_pairs_kernel(const unsigned long long* __restrict__ T,
                                                       unsigned long long slots,
                                                       const unsigned int* __restrict__ offsets,
                                                       unsigned long long* first, uint32_t* slot_of) {
  const unsigned long long total = slots + 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __shared__ unsigned int wc[GNT / 32];
  unsigned int pos = offsets[blockIdx.x];
  for (int k = 0; k < FZ_CHUNK / GNT; ++k) {
    const unsigned long long i = static_cast<unsigned long long>(blockIdx.x) * FZ_CHUNK +
                                 static_cast<unsigned long long>(k) * GNT + threadIdx.x;
    const bool used = i < total && fz_used(T, i, slots);
    const unsigned bal = __ballot_sync(0xffffffffu, used);
    if (lane == 0) wc[warp] = __popc(bal);
    __syncthreads();
    unsigned int before = 0, all = 0;
    for (int w = 0; w < GNT / 32; ++w) {
      before += w < warp ? wc[w] : 0u;
      all += wc[w];
    }
    if (used) {
      const unsigned int j = pos + before + __popc(bal & ((1u << lane) - 1u));
      first[j] = T[i * FZ_WORDS + FZ_FIRST];
      slot_of[j] = static_cast<uint32_t>(i);
    }
    pos += all;
    __syncthreads();
  }
}

// After the sort by first row: distinct key j (in first-seen order) gets code j.
__global__ void fz_codes_kernel(unsigned long long* T, const uint32_t* __restrict__ slot_of,
                                const unsigned long long* __restrict__ n_dev, long long max_groups,
                                int64_t* uniques) {
  const unsigned long long u = *n_dev;
  for (unsigned long long j = blockIdx.x * static_cast<unsigned long long>(blockDim.x) + threadIdx.x; j < u;
       j += static_cast<unsigned long long>(gridDim.x) * blockDim.x) {
    unsigned long long* p = T + static_cast<unsigned long long>(slot_of[j]) * FZ_WORDS;
    p[FZ_CODE] = j;
    if (j < static_cast<unsigned long long>(max_groups)) uniques[j] = static_cast<int64_t>(p[FZ_KEY]);
  }
}

__global__ void __launch_bounds__(GNT) fz_lookup_kernel(const int64_t* __restrict__ keys, long long n,
                                                        unsigned long long* T, unsigned long long slots,
                                                        int32_t* codes, uint32_t* err) {
  for (long long i = blockIdx.x * static_cast<long long>(GNT) + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * GNT) {
    const long long s = fz_slot(T, slots, static_cast<unsigned long long>(__ldcs(keys + i)), false, err);
    codes[i] = s < 0 ? -1 : static_cast<int32_t>(T[static_cast<unsigned long long>(s) * FZ_WORDS + FZ_CODE]);
  }
}

int grid_of(long long n, int num_sms) {
  long long b = (n + GNT - 1) / GNT;
  const long long cap = static_cast<long long>(num_sms) * 8;
  if (b > cap) b = cap;
  return b < 1 ? 1 : static_cast<int>(b);
}

// Radix bits covering values up to maxval, in whole 8-bit passes (at least one).
int bits_for(unsigned long long maxval) {
  int b = 0;
  while (b < 64 && (maxval >> b) != 0) ++b;
  b = (b + 7) / 8 * 8;
  return b < 8 ? 8 : b;
}

}  // namespace

size_t group_index_scratch_bytes(long long n) {
  return (static_cast<size_t>(n) * 4 * 3 + 255) / 256 * 256 + (sort_counts_bytes(n) + 255) / 256 * 256;
}

cudaError_t group_index_launch(const int32_t* keys, long long n, int G, uint32_t* row_to_group, uint32_t* counts,
                               uint32_t* offsets, uint32_t* rows_by_group, int64_t* n_active, void* scratch,
                               uint32_t* err, int num_sms, cudaStream_t s, uint64_t* launches) {
  cudaError_t e = cudaMemsetAsync(counts, 0, static_cast<size_t>(G) * 4, s);
  if (e != cudaSuccess) return e;
  const size_t smem = G <= kSmemCounts ? static_cast<size_t>(G) * 4 : 0;
  if (smem > 48 * 1024) {
    e = cudaFuncSetAttribute(gi_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  gi_count_kernel<<<grid_of(n, num_sms), GNT, smem, s>>>(keys, n, G, row_to_group, counts, err);
  gi_offsets_kernel<<<1, 1024, 0, s>>>(counts, G, offsets, n_active);
  *launches += 2;
  // rows_by_group: a stable sort of (key, row) by key
  char* w = static_cast<char*>(scratch);
  const size_t nb = (static_cast<size_t>(n) * 4 + 255) / 256 * 256;
  uint32_t* skeys = reinterpret_cast<uint32_t*>(w);
  uint32_t* ktmp = reinterpret_cast<uint32_t*>(w + nb);
  uint32_t* vtmp = reinterpret_cast<uint32_t*>(w + 2 * nb);
  unsigned int* cnt = reinterpret_cast<unsigned int*>(w + 3 * nb);
  e = cudaMemcpyAsync(skeys, row_to_group, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToDevice, s);
  if (e != cudaSuccess) return e;
  e = sort_pairs_u32(skeys, rows_by_group, n, bits_for(static_cast<unsigned long long>(G - 1)), ktmp, vtmp, cnt, s,
                     launches, true);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

size_t factorize_scratch_bytes(long long n, long long max_groups) {
  const unsigned long long slots = factorize_slots(max_groups);
  const size_t table = ((slots + 1) * FZ_WORDS * 8 + 255) / 256 * 256;
  const size_t nblk = (slots + 1 + FZ_CHUNK - 1) / FZ_CHUNK;
  const size_t cnts = (nblk * 4 + 255) / 256 * 256 + 256;
  const size_t pairs = ((slots + 1) * 8 + 255) / 256 * 256 * 2 + ((slots + 1) * 4 + 255) / 256 * 256 * 2;
  return table + cnts + pairs + (sort_counts_bytes(static_cast<long long>(slots + 1)) + 255) / 256 * 256;
}

unsigned long long factorize_slots(long long max_groups) {
  unsigned long long want = static_cast<unsigned long long>(max_groups) * 2, p = 1024;
  while (p < want) p <<= 1;
  return p;
}

cudaError_t factorize_launch(const int64_t* keys, long long n, long long max_groups, int32_t* codes,
                             int64_t* uniques, int64_t* n_uniques, void* scratch, uint32_t* err, int num_sms,
                             cudaStream_t s, uint64_t* launches) {
  const unsigned long long slots = factorize_slots(max_groups);
  const unsigned long long nslots = slots + 1;
  char* w = static_cast<char*>(scratch);
  unsigned long long* T = reinterpret_cast<unsigned long long*>(w);
  w += (nslots * FZ_WORDS * 8 + 255) / 256 * 256;
  const unsigned long long nblk = (nslots + FZ_CHUNK - 1) / FZ_CHUNK;
  unsigned int* bcounts = reinterpret_cast<unsigned int*>(w);
  w += (nblk * 4 + 255) / 256 * 256;
  unsigned long long* n_dev = reinterpret_cast<unsigned long long*>(w);
  w += 256;
  const size_t f_bytes = (nslots * 8 + 255) / 256 * 256, s_bytes = (nslots * 4 + 255) / 256 * 256;
  unsigned long long* first = reinterpret_cast<unsigned long long*>(w);
  unsigned long long* first_tmp = reinterpret_cast<unsigned long long*>(w + f_bytes);
  uint32_t* slot_of = reinterpret_cast<uint32_t*>(w + 2 * f_bytes);
  uint32_t* slot_tmp = reinterpret_cast<uint32_t*>(w + 2 * f_bytes + s_bytes);
  unsigned int* scnt = reinterpret_cast<unsigned int*>(w + 2 * f_bytes + 2 * s_bytes);

  unsigned long long ib = (nslots + 255) / 256;
  if (ib > 65536) ib = 65536;
  fz_init_kernel<<<static_cast<unsigned int>(ib), 256, 0, s>>>(T, nslots);
  if (n > 0) fz_insert_kernel<<<grid_of(n, num_sms), GNT, 0, s>>>(keys, n, T, slots, err);
  fz_count_kernel<<<static_cast<unsigned int>(nblk), GNT, 0, s>>>(T, slots, bcounts);
  fz_scan_kernel<<<1, 1024, 0, s>>>(bcounts, static_cast<long long>(nblk), max_groups, n_uniques, n_dev, err);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  *launches += n > 0 ? 4 : 3;
  // Sort the distinct keys by first row.  The pair count is only known on the device, so the
  // sort runs over every slot's worth of pairs with the unused tail holding first row ~0
  // (after every real row), which keeps the real pairs at the front in first-seen order.
  e = cudaMemsetAsync(first, 0xFF, nslots * 8, s);  // placeholder rows sort last
  if (e != cudaSuccess) return e;
  fz_pairs_kernel<<<static_cast<unsigned int>(nblk), GNT, 0, s>>>(T, slots, bcounts, first, slot_of);
  (*launches)++;
  e = sort_pairs_u64(first, slot_of, static_cast<long long>(nslots), bits_for(n > 0 ? static_cast<unsigned long long>(n) : 1),
                     first_tmp, slot_tmp, scnt, s, launches, false);
  if (e != cudaSuccess) return e;
  fz_codes_kernel<<<grid_of(static_cast<long long>(nslots), num_sms), GNT, 0, s>>>(T, slot_of, n_dev, max_groups,
                                                                                  uniques);
  if (n > 0) fz_lookup_kernel<<<grid_of(n, num_sms), GNT, 0, s>>>(keys, n, T, slots, codes, err);
  e = cudaGetLastError();
  if (e == cudaSuccess) *launches += n > 0 ? 2 : 1;
  return e;
}

}  // namespace tbgb
