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

// Launch configuration with programmatic dependent launch: the grid may be scheduled
// before the kernel it follows on the stream has finished, once every CTA of that kernel
// has run pdl_trigger(); it must call pdl_wait() (nc_common.cuh) before it reads anything
// an earlier kernel wrote.  Use in place (cfg.attrs points into the object):
//   PdlLaunch L(grid, block, smem, st);  cudaLaunchKernelEx(&L.cfg, kernel, args...);
struct PdlLaunch {
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[1];
  PdlLaunch(dim3 grid, dim3 block, size_t smem, cudaStream_t st) : cfg(), attr() {
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  PdlLaunch(const PdlLaunch&) = delete;
  PdlLaunch& operator=(const PdlLaunch&) = delete;
};

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
