// noalloc.cu -- dense-key groupby that allocates no device memory per call.
//
// Some callers cannot let a library allocate device memory while they run: a
// host engine that has already reserved (nearly) all of HBM for its own buffer
// store and hands out only input and output buffers, or a latency-critical loop
// in which cudaMalloc's implicit device-wide synchronisation is not acceptable.
// For them, tbgb_groupby_dense_noalloc runs the same dense moments kernels as
// tbgb_groupby_dense, but its scratch (per-CTA partial states, spill states,
// first-zero trackers, the device error word) lives in one file-scope device
// array.  That array is part of this library's image: every GPU that loads the
// library holds it (about 10.5 MB) until the process exits.
#include <cuda_runtime.h>

#include <mutex>

#include "dense.cuh"
#include "errbits.hpp"
#include "tambear_gb.h"

namespace {

constexpr int kNoAllocMaxGroups = 256;  // largest n_groups this entry point accepts
constexpr int kNoAllocMaxCtas = 160;    // CTAs used at most (B200 has 148 SMs)
constexpr int kMaxDevices = 64;

// Word counts of the scratch regions at the largest accepted size.
constexpr size_t kPartWords = static_cast<size_t>(tbgb::ST_COUNT) * kNoAllocMaxCtas * 2 * 256;
constexpr size_t kSpillWords = static_cast<size_t>(tbgb::kDenseSpillFields) * kNoAllocMaxCtas * kNoAllocMaxGroups;
constexpr size_t kZeroWords = kNoAllocMaxGroups;
constexpr size_t kErrWords = 32;
constexpr size_t kScratchWords = kPartWords + kSpillWords + kZeroWords + kErrWords;

// The scratch array.  In host code this name is only a host-side stand-in for the
// symbol, never a device address: the device address is obtained per device with
// cudaGetSymbolAddress and passed to the kernels.
static __device__ __align__(256) unsigned long long g_noalloc_scratch[kScratchWords];

struct DeviceInfo {
  int sms = 0;
  bool ready = false;
};

std::mutex g_setup_mutex;
DeviceInfo g_info_of[kMaxDevices];

// The scratch address on the current device and that device's SM count.  The address is
// looked up on every call, with the device current: a reset of the device or another
// context made current reloads this library's module there, and a cached address would
// then point at memory that is no longer ours.  Only the SM count (a property of the
// hardware) is cached.  The first lookup on a device loads the module and maps the array
// (with CUDA's default lazy module loading), which can fail with TBGB_ERR_BACKEND when
// the device has no free memory left.
tbgb_status device_scratch(int dev, unsigned long long** base, int* sms_out) {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return TBGB_ERR_BACKEND;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  DeviceInfo& d = g_info_of[dev];
  if (!d.ready) {
    int sms = 0, major = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return TBGB_ERR_BACKEND;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return TBGB_ERR_BACKEND;
    if (major != 10) return TBGB_ERR_BACKEND;  // built for sm_100a only
    d.sms = sms;
    d.ready = true;
  }
  *base = static_cast<unsigned long long*>(p);
  *sms_out = d.sms;
  return TBGB_OK;
}

}  // namespace

extern "C" tbgb_status tbgb_groupby_dense_noalloc(const int32_t* d_keys, const double* d_vals, const uint64_t* d_mask,
                                                  int64_t n, int32_t n_groups, const tbgb_moments* out, void* stream) {
  if (n < 0 || !out) return TBGB_ERR_INVALID_ARGUMENT;
  if (n_groups < 1 || n_groups > kNoAllocMaxGroups) return TBGB_ERR_INVALID_ARGUMENT;
  if (n > 0 && (!d_keys || !d_vals)) return TBGB_ERR_INVALID_ARGUMENT;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return TBGB_ERR_BACKEND;
  unsigned long long* base = nullptr;
  int sms = 0;
  tbgb_status st = device_scratch(dev, &base, &sms);
  if (st != TBGB_OK) return st;

  const int ctas = sms < kNoAllocMaxCtas ? sms : kNoAllocMaxCtas;
  const tbgb::DenseLaunch L = tbgb::dense_plan(n_groups, ctas);
  if (L.part_doubles > kPartWords || L.spill_words > kSpillWords) return TBGB_ERR_INVALID_ARGUMENT;
  double* part = reinterpret_cast<double*>(base);
  unsigned long long* spill = base + kPartWords;
  unsigned long long* zfirst = spill + kSpillWords;
  uint32_t* err = reinterpret_cast<uint32_t*>(zfirst + kZeroWords);

  // The scratch keeps the previous call's contents: the first-zero trackers must
  // start at all-ones and the error word at zero (partial and spill states are
  // rewritten by the kernel itself).
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(zfirst, 0xFF, static_cast<size_t>(n_groups) * 8, s) != cudaSuccess) return TBGB_ERR_DISPATCH;
  if (cudaMemsetAsync(err, 0, sizeof(uint32_t), s) != cudaSuccess) return TBGB_ERR_DISPATCH;
  uint64_t launches = 0;
  if (tbgb::dense_moments_launch(L, d_keys, d_vals, d_mask, n, 0, n_groups, part, spill, zfirst, err, out, nullptr, s,
                                 &launches) != cudaSuccess)
    return TBGB_ERR_DISPATCH;

  // Device-side errors are read back before returning, so the call completes
  // synchronously with respect to `stream`.
  uint32_t bits = 0;
  if (cudaMemcpyAsync(&bits, err, sizeof(bits), cudaMemcpyDeviceToHost, s) != cudaSuccess) return TBGB_ERR_TRANSFER;
  if (cudaStreamSynchronize(s) != cudaSuccess) return TBGB_ERR_DISPATCH;
  if (bits & tbgb::KERR_KEY_RANGE) return TBGB_ERR_KEY_OUT_OF_RANGE;
  if (bits & tbgb::KERR_TIMEOUT) return TBGB_ERR_TIMEOUT;
  if (bits != 0) return TBGB_ERR_BACKEND;
  return TBGB_OK;
}
