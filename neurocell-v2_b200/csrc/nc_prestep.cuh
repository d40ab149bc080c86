// nc_prestep.cuh -- the per-cell body of the pre-step fusion, shared by prestep_kernel
// (nc_aux.cu) and the fused-FFT launch that also builds the pair spectra (nc_fftf.cu).
#pragma once

#include "nc_common.cuh"
#include "nc_kernels.cuh"

namespace nc {

// Pre-step fusion (neurocell/params.py:220-322 with Codd gating :31-80) of grid cell i
// (i < H*W): Codd probabilities and their surrogate derivative, the pinned weights, the
// border template, and the ROI's w_eff, s_eff, b_roi.
__device__ __forceinline__ void prestep_cell(const Geo& g, const StepParams& sp, const float* __restrict__ cell,
                                             const uint8_t* __restrict__ io, const uint8_t* __restrict__ owm,
                                             const uint8_t* __restrict__ bmask, const nc_codd& codd, int i) {
  const int HW = g.H * g.W;
  const float Wv = cell[i], Bv = cell[HW + i], Sv = cell[2 * HW + i];
  float ds;
  const float s = codd_prob(Sv, io[i] != 0, g.hard_pin, codd.mode, codd_tau(codd),
                            codd.active_threshold, &ds);
  const float wp = owm[i] ? 1.0f : Wv;
  sp.sprob[i] = s;
  sp.dsprob[i] = ds;
  sp.wpinned[i] = wp;
  sp.border[i] = bmask[i] ? act_fwd(g.act, Bv, g.slope) * s : 0.0f;
  const int r = i / g.W, c = i - (i / g.W) * g.W;
  const int rr = r - g.pad_h, cc = c - g.pad_w;
  if (rr >= 0 && rr < g.roi_h && cc >= 0 && cc < g.roi_w) {
    const int p = rr * g.roi_w + cc;
    const float inv_m = 1.0f / (float)g.M;
    sp.weff[p] = inv_m * wp * (1.0f - s);
    sp.seff[p] = inv_m * s;
    sp.broi[p] = Bv;
  }
}

// Effective filter tap j (propagator.py:262-264: sigmoid when gated_filters).
__device__ __forceinline__ float geff_tap(const Geo& g, const float* __restrict__ filters, int j) {
  const float f = filters[j];
  return g.gated ? sigmoidf_(f) : f;
}

}  // namespace nc
