// phi.cuh -- launchers of the phi-scatter and extremum primitives.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "tambear_gb.h"

namespace tbgb {

constexpr int kMaxPhi = 5;  // compute_engine.rs:118: at most five phi expressions per call

size_t phi_smem_bytes(int n_phi, int G);
// out: n_phi * G doubles (row j = phis[j]); zeroed, then accumulated.
cudaError_t phi_scatter_launch(const int* phis, int n_phi, const int32_t* keys, const double* vals,
                               const double* refs, const uint64_t* mask, long long n, int G, double* out,
                               uint32_t* err, int num_sms, cudaStream_t s, uint64_t* launches);
// scratch: 2 * G u64.
cudaError_t extremum_launch(int is_max, const int32_t* keys, const double* vals, long long n, int G, double* out,
                            unsigned long long* scratch, uint32_t* err, int num_sms, cudaStream_t s,
                            uint64_t* launches);

}  // namespace tbgb
