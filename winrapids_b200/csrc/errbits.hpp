// errbits.hpp -- deferred device error bits (kernel -> host), shared by host and device code.
#pragma once
#include <cstdint>

namespace tbgb {

// Error bits written by kernels into the per-context status word; tbgb_sync maps
// them onto tbgb_status codes (include/tambear_gb.h).
enum : uint32_t {
  KERR_KEY_RANGE = 1u << 0,   // a key outside [0, n_groups)
  KERR_TIMEOUT = 1u << 1,     // a bounded wait gave up
  KERR_TABLE_FULL = 1u << 2,  // hash table probe limit reached
  KERR_MISALIGNED = 1u << 3,  // staged copy source not 16-byte aligned
  KERR_BOUNDARIES = 1u << 4,  // bin boundaries not non-decreasing within [0, n_ticks]
};

}  // namespace tbgb
