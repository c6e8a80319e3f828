// phi.cu -- the reference's scatter primitives over dense int32 keys, as kernels:
//   scatter_phi / scatter_multi_phi / scatter_phi_masked: out_j[k[i]] += phi_j(v[i], refs[k[i]])
//     (ComputeEngine, crates/tambear/src/compute_engine.rs:109-154; CPU :252-302;
//      ScatterJit::scatter_multi_phi_masked, scatter_jit.rs:402-495)
//   scatter_extremum: per-group min or max, +-inf when empty, NaN never wins
//     (compute_engine.rs:165-178, CPU :304-322)
// with the CPU path's semantics: every sum is over the finite, nonzero phi terms (the
// reference's CPU accumulator is exact and skips +-0, NaN and +-inf), here accumulated in
// f64; extrema follow the strict `<` / `>` scan, +-0 ties to the first zero in row order.
//
// Small tables (all n_phi x n_groups sums plus the refs fit in 160 KB) are accumulated per
// CTA in shared memory and flushed once with global atomics; larger ones go to global
// atomics directly.  Extrema update a u64 order-preserving image of the doubles with
// atomicMin / atomicMax after a plain read shows the row can win.
#include <cstdint>

#include "common.cuh"
#include "gstate.cuh"
#include "phi.cuh"

namespace tbgb {

namespace {

constexpr int FNT = 512;
constexpr size_t kPhiSmemBytes = 160 * 1024;

// phi_scatter_eval (compute_engine.rs:593-609): each operation rounded separately.
__device__ __forceinline__ double phi_eval(int phi, double v, double r) {
  switch (phi) {
    case TBGB_PHI_V: return v;
    case TBGB_PHI_VV: return __dmul_rn(v, v);
    case TBGB_PHI_ONE: return 1.0;
    case TBGB_PHI_VMR: return __dsub_rn(v, r);
    case TBGB_PHI_VMR2: { const double d = __dsub_rn(v, r); return __dmul_rn(d, d); }
    case TBGB_PHI_ABS_VMR: return fabs(__dsub_rn(v, r));
    case TBGB_PHI_VMR3: { const double d = __dsub_rn(v, r); return __dmul_rn(__dmul_rn(d, d), d); }
    case TBGB_PHI_VMR4: { const double d = __dsub_rn(v, r); const double d2 = __dmul_rn(d, d); return __dmul_rn(d2, d2); }
    case TBGB_PHI_VR: return __dmul_rn(v, r);
    case TBGB_PHI_LOG: return log(v);
    case TBGB_PHI_RECIP: return __ddiv_rn(1.0, v);
    default: return qnan();
  }
}

struct PhiArgs {
  const int32_t* keys;
  const double* vals;
  const double* refs;    // nullable: r = 0
  const uint64_t* mask;  // nullable
  long long n;
  int G;
  int n_phi;
  int phis[kMaxPhi];
  double* out;           // [n_phi][G], zeroed before the launch
  uint32_t* err;
};

template <bool SMEM>
__global__ void __launch_bounds__(FNT) phi_scatter_kernel(PhiArgs a) {
  extern __shared__ __align__(16) unsigned char sm[];
  double* acc = reinterpret_cast<double*>(sm);                    // [n_phi][G]
  double* rs = acc + static_cast<size_t>(a.n_phi) * a.G;          // [G]
  const int G = a.G, np = a.n_phi;
  if constexpr (SMEM) {
    for (int i = threadIdx.x; i < np * G; i += FNT) acc[i] = 0.0;
    for (int g = threadIdx.x; g < G; g += FNT) rs[g] = a.refs ? a.refs[g] : 0.0;
    __syncthreads();
  }
  for (long long row = blockIdx.x * static_cast<long long>(FNT) + threadIdx.x; row < a.n;
       row += static_cast<long long>(gridDim.x) * FNT) {
    if (a.mask && !((__ldg(a.mask + (row >> 6)) >> (row & 63)) & 1ull)) continue;
    const int k = __ldcs(a.keys + row);
    if (static_cast<unsigned>(k) >= static_cast<unsigned>(G)) {
      atomicOr(a.err, KERR_KEY_RANGE);
      continue;
    }
    const double v = __ldcs(a.vals + row);
    double r;
    if constexpr (SMEM) r = rs[k];
    else r = a.refs ? __ldg(a.refs + k) : 0.0;
    for (int j = 0; j < np; ++j) {
      const double p = phi_eval(a.phis[j], v, r);
      if (is_finite(p) && p != 0.0) {
        if constexpr (SMEM) atomicAdd(acc + j * G + k, p);
        else atomicAdd(a.out + static_cast<size_t>(j) * G + k, p);
      }
    }
  }
  if constexpr (SMEM) {
    __syncthreads();
    for (int i = threadIdx.x; i < np * G; i += FNT)
      if (acc[i] != 0.0) atomicAdd(a.out + i, acc[i]);
  }
}

__global__ void __launch_bounds__(FNT) extremum_kernel(const int32_t* __restrict__ keys,
                                                       const double* __restrict__ vals, long long n, int G,
                                                       int is_max, unsigned long long* ord,
                                                       unsigned long long* zf, uint32_t* err) {
  for (long long row = blockIdx.x * static_cast<long long>(FNT) + threadIdx.x; row < n;
       row += static_cast<long long>(gridDim.x) * FNT) {
    const int k = __ldcs(keys + row);
    if (static_cast<unsigned>(k) >= static_cast<unsigned>(G)) {
      atomicOr(err, KERR_KEY_RANGE);
      continue;
    }
    const double v = __ldcs(vals + row);
    if (is_nan(v)) continue;
    const unsigned long long o = f2o(v);
    if (is_max) {
      if (o > __ldcg(ord + k)) atomicMax(ord + k, o);
    } else {
      if (o < __ldcg(ord + k)) atomicMin(ord + k, o);
    }
    if (v == 0.0) atomicMin(zf + k, zero_code(row, v));
  }
}

__global__ void extremum_init_kernel(unsigned long long* ord, unsigned long long* zf, int G, int is_max) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g < G) {
    ord[g] = is_max ? f2o(neg_inf()) : f2o(pos_inf());
    zf[g] = ~0ull;
  }
}

__global__ void extremum_final_kernel(const unsigned long long* ord, const unsigned long long* zf, int G,
                                      double* out) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= G) return;
  double x = o2f(ord[g]);
  if (x == 0.0 && zf[g] != ~0ull) x = (zf[g] & 1ull) ? -0.0 : 0.0;
  out[g] = x;
}

int grid_for(long long n, int num_sms) {
  long long b = (n + FNT - 1) / FNT;
  const long long cap = static_cast<long long>(num_sms) * 4;
  if (b > cap) b = cap;
  return b < 1 ? 1 : static_cast<int>(b);
}

}  // namespace

size_t phi_smem_bytes(int n_phi, int G) { return static_cast<size_t>(n_phi + 1) * G * 8; }

cudaError_t phi_scatter_launch(const int* phis, int n_phi, const int32_t* keys, const double* vals,
                               const double* refs, const uint64_t* mask, long long n, int G, double* out,
                               uint32_t* err, int num_sms, cudaStream_t s, uint64_t* launches) {
  cudaError_t e = cudaMemsetAsync(out, 0, static_cast<size_t>(n_phi) * G * 8, s);
  if (e != cudaSuccess || n == 0) return e;
  PhiArgs a{};
  a.keys = keys; a.vals = vals; a.refs = refs; a.mask = mask; a.n = n; a.G = G; a.n_phi = n_phi;
  for (int j = 0; j < n_phi; ++j) a.phis[j] = phis[j];
  a.out = out; a.err = err;
  const size_t smem = phi_smem_bytes(n_phi, G);
  if (smem <= kPhiSmemBytes) {
    e = cudaFuncSetAttribute(phi_scatter_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    phi_scatter_kernel<true><<<num_sms, FNT, smem, s>>>(a);
  } else {
    phi_scatter_kernel<false><<<grid_for(n, num_sms), FNT, 0, s>>>(a);
  }
  e = cudaGetLastError();
  if (e == cudaSuccess) (*launches)++;
  return e;
}

cudaError_t extremum_launch(int is_max, const int32_t* keys, const double* vals, long long n, int G, double* out,
                            unsigned long long* scratch, uint32_t* err, int num_sms, cudaStream_t s,
                            uint64_t* launches) {
  unsigned long long* ord = scratch;
  unsigned long long* zf = scratch + G;
  const int gb = (G + 255) / 256;
  extremum_init_kernel<<<gb, 256, 0, s>>>(ord, zf, G, is_max);
  if (n > 0) extremum_kernel<<<grid_for(n, num_sms), FNT, 0, s>>>(keys, vals, n, G, is_max, ord, zf, err);
  extremum_final_kernel<<<gb, 256, 0, s>>>(ord, zf, G, out);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) *launches += n > 0 ? 3 : 2;
  return e;
}

}  // namespace tbgb
