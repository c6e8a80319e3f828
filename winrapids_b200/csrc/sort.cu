// sort.cu -- stable LSD radix sort of (key, value) pairs, 8 bits per pass.
//
// Used to build the row inversion of a group index (rows_by_group: row ids sorted by
// group, row order kept inside a group) and to order distinct keys by their first row.
// Each pass: per-tile digit histograms, one block scanning the [digit][tile] counts into
// write offsets, and a stable scatter.  Inside a tile rows are taken 1024 at a time (one
// per thread): __match_any_sync ranks a row among the lanes of its warp with the same
// digit, per-warp digit counts are turned into prefixes over the block's warps, and a
// running offset per digit carries the order from step to step and tile to tile.
#include <cstdint>

#include "common.cuh"
#include "sort.cuh"

namespace tbgb {

namespace {

constexpr int SNT = 1024;             // threads per block
constexpr int SNW = SNT / 32;
constexpr int RADIX = 256;
constexpr long long STILE = 32768;    // rows per tile
constexpr int SSTEPS = STILE / SNT;

template <class K>
__global__ void __launch_bounds__(SNT) radix_hist_kernel(const K* __restrict__ keys, long long n, int shift,
                                                         long long ntiles, unsigned int* counts) {
  __shared__ unsigned int h[RADIX];
  for (int d = threadIdx.x; d < RADIX; d += SNT) h[d] = 0;
  __syncthreads();
  const long long base = static_cast<long long>(blockIdx.x) * STILE;
  for (int s = 0; s < SSTEPS; ++s) {
    const long long i = base + static_cast<long long>(s) * SNT + threadIdx.x;
    if (i < n) atomicAdd(h + static_cast<int>((keys[i] >> shift) & (RADIX - 1)), 1u);
  }
  __syncthreads();
  for (int d = threadIdx.x; d < RADIX; d += SNT) counts[static_cast<long long>(d) * ntiles + blockIdx.x] = h[d];
}

// Exclusive scan of `len` u32 counts in one block (in place).
__global__ void __launch_bounds__(SNT) radix_scan_kernel(unsigned int* counts, long long len) {
  __shared__ unsigned int warp_sums[SNW];
  __shared__ unsigned int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (long long b = 0; b < len; b += SNT) {
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
    if (threadIdx.x == SNT - 1) carry = before + x;
    __syncthreads();
  }
}

template <class K>
__global__ void __launch_bounds__(SNT) radix_scatter_kernel(const K* __restrict__ keys_in,
                                                            const uint32_t* __restrict__ vals_in, long long n,
                                                            int shift, long long ntiles,
                                                            const unsigned int* __restrict__ offsets, K* keys_out,
                                                            uint32_t* vals_out) {
  __shared__ unsigned int wcnt[SNW][RADIX];  // rows of each digit per warp in this step, then their prefix
  __shared__ unsigned int running[RADIX];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long t = blockIdx.x;
  for (int d = threadIdx.x; d < RADIX; d += SNT) running[d] = offsets[static_cast<long long>(d) * ntiles + t];
  const unsigned lt = (1u << lane) - 1u;
  const long long base = t * STILE;
  for (int s = 0; s < SSTEPS; ++s) {
    if (base + static_cast<long long>(s) * SNT >= n) break;  // uniform across the block
    for (int d = lane; d < RADIX; d += 32) wcnt[warp][d] = 0;
    const long long i = base + static_cast<long long>(s) * SNT + threadIdx.x;
    const bool live = i < n;
    K key = 0;
    uint32_t val = 0;
    int dig = RADIX;  // out-of-range rows get a digit no live row has
    if (live) {
      key = keys_in[i];
      val = vals_in ? vals_in[i] : static_cast<uint32_t>(i);
      dig = static_cast<int>((key >> shift) & (RADIX - 1));
    }
    const unsigned peers = __match_any_sync(0xffffffffu, dig);
    const unsigned rank = __popc(peers & lt);
    __syncwarp();
    if (live && rank == 0) wcnt[warp][dig] = __popc(peers);
    __syncthreads();
    // digits d: exclusive prefix over the warps, and the step's total
    unsigned int tot = 0;
    if (threadIdx.x < RADIX) {
      const int d = threadIdx.x;
      for (int w = 0; w < SNW; ++w) {
        const unsigned int c = wcnt[w][d];
        wcnt[w][d] = tot;
        tot += c;
      }
    }
    __syncthreads();
    if (live) {
      const unsigned int pos = running[dig] + wcnt[warp][dig] + rank;
      keys_out[pos] = key;
      vals_out[pos] = val;
    }
    __syncthreads();
    if (threadIdx.x < RADIX) running[threadIdx.x] += tot;
    __syncthreads();
  }
}

template <class K>
cudaError_t sort_pairs_impl(K* keys, uint32_t* vals, long long n, int bits, K* keys_tmp, uint32_t* vals_tmp,
                            unsigned int* counts, cudaStream_t s, uint64_t* launches, bool vals_are_rows) {
  if (n <= 0) return cudaSuccess;
  const long long ntiles = (n + STILE - 1) / STILE;
  K* kin = keys;
  uint32_t* vin = vals;
  K* kout = keys_tmp;
  uint32_t* vout = vals_tmp;
  int passes = 0;
  for (int shift = 0; shift < bits; shift += 8, ++passes) {
    radix_hist_kernel<K><<<static_cast<unsigned int>(ntiles), SNT, 0, s>>>(kin, n, shift, ntiles, counts);
    radix_scan_kernel<<<1, SNT, 0, s>>>(counts, ntiles * RADIX);
    radix_scatter_kernel<K><<<static_cast<unsigned int>(ntiles), SNT, 0, s>>>(
        kin, (passes == 0 && vals_are_rows) ? nullptr : vin, n, shift, ntiles, counts, kout, vout);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    *launches += 3;
    K* tk = kin; kin = kout; kout = tk;
    uint32_t* tv = vin; vin = vout; vout = tv;
  }
  if (passes % 2 == 1) {  // the result is in the scratch buffers: copy it back
    cudaError_t e = cudaMemcpyAsync(keys, kin, static_cast<size_t>(n) * sizeof(K), cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(vals, vin, static_cast<size_t>(n) * sizeof(uint32_t), cudaMemcpyDeviceToDevice, s);
    return e;
  }
  return cudaSuccess;
}

}  // namespace

size_t sort_counts_bytes(long long n) {
  const long long ntiles = (n + STILE - 1) / STILE;
  return static_cast<size_t>(ntiles > 0 ? ntiles : 1) * RADIX * sizeof(unsigned int);
}

cudaError_t sort_pairs_u32(uint32_t* keys, uint32_t* vals, long long n, int bits, uint32_t* keys_tmp,
                           uint32_t* vals_tmp, unsigned int* counts, cudaStream_t s, uint64_t* launches,
                           bool vals_are_rows) {
  return sort_pairs_impl<uint32_t>(keys, vals, n, bits, keys_tmp, vals_tmp, counts, s, launches, vals_are_rows);
}

cudaError_t sort_pairs_u64(unsigned long long* keys, uint32_t* vals, long long n, int bits,
                           unsigned long long* keys_tmp, uint32_t* vals_tmp, unsigned int* counts, cudaStream_t s,
                           uint64_t* launches, bool vals_are_rows) {
  return sort_pairs_impl<unsigned long long>(keys, vals, n, bits, keys_tmp, vals_tmp, counts, s, launches,
                                             vals_are_rows);
}

}  // namespace tbgb
