// nc_errors.h -- thread-local error reporting for the C ABI.
#pragma once

#include <cuda_runtime.h>

#include "neurocell_b200.h"

namespace nc {

// Usable dynamic shared memory per CTA assumed by the layout policy (B200: 227 KB opt-in).
constexpr size_t kSmemBudget = 225 * 1024;

nc_status set_error(nc_status st, const char* fmt, ...);
nc_status cuda_error(cudaError_t e, const char* what);
void clear_error();
// Counts one successful kernel launch (reported by nc_launch_count).
void note_launch();

}  // namespace nc

#define NC_CUDA_CHECK(expr)                                   \
  do {                                                        \
    cudaError_t e_ = (expr);                                  \
    if (e_ != cudaSuccess) return ::nc::cuda_error(e_, #expr); \
  } while (0)

#define NC_CHECK(expr)                 \
  do {                                 \
    nc_status s_ = (expr);             \
    if (s_ != NC_OK) return s_;        \
  } while (0)
