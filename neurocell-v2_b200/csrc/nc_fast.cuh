// nc_fast.cuh -- register-tiled fused kernels for M = 16 (see nc_fast.cu).
#pragma once

#include <stddef.h>

#include "nc_internal.h"

namespace nc {

// Opt-in dynamic shared memory per CTA on B200 (227 KB).
constexpr size_t kFastSmemMax = 232448;

namespace fastc {
constexpr int M = 16;     // directions handled by the specialisation
constexpr int MP = 8;     // direction pairs
constexpr int NW = 16;    // warps per CTA
constexpr int RH = 4;     // rows per forward / epilogue strip
constexpr int CWX = 10;   // columns per dX strip
constexpr int RG = 4;     // row groups of the dG reduction
}  // namespace fastc

// Shared-memory carve-up of the fast backward kernel; offsets in floats.  Strides are
// picked on the host so that the dG loads of one warp hit distinct banks.
struct FastBwdLayout {
  int fs;       // field row stride (floats)
  int rs;       // plane-gradient row stride (float2 units)
  int ps;       // plane-pair stride (float2 units)
  int vs;       // filter-pair row stride (float2 units, >= kw, even)
  size_t gx, f, gz, gy, red, stats;
  size_t bytes;
};

struct FastKernels {
  const void* fwd;
  const void* bwd;
  size_t fwd_smem, bwd_smem;
  int fwd_threads;
  FastBwdLayout bl;
};

// Specialised forward for this geometry (fn == nullptr when none applies).
struct FastFwd {
  const void* fn;
  size_t smem;
  int threads;
};
FastFwd fast_fwd_select(const Geo& g);
FastBwdLayout fast_bwd_layout(const Geo& g, int kh, int kw);
FastKernels fast_kernels(const Geo& g);

}  // namespace nc
