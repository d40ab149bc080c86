// nc_common.cuh -- device helpers shared by the VNN kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "neurocell_b200.h"

namespace nc {

// Programmatic dependent launch (PdlLaunch, nc_errors.h): pdl_wait() returns once the
// kernels this grid follows on the stream have finished and their writes are visible;
// pdl_trigger() lets the next kernel be scheduled.  Kernels call both at their start, so
// at most one dependent grid waits at a time.  Both do nothing in an ordinary launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_enter() {
  pdl_wait();
  pdl_trigger();
}

constexpr float kNormEps = 1e-5f;      // neurocell/kernels_pallas.py:204 (rsqrt(var + 1e-5))
constexpr float kTauMin = 1e-4f;       // neurocell/params.py:63
constexpr float kGeluC = 0.7978845608028654f;   // sqrt(2/pi), kernels_pallas.py:130

// Activation value (neurocell/kernels_pallas.py:111-126).  CUDA's own tanhf / expf are
// used unchanged so that results stay within a few ulp of the reference's float32 math.
__device__ __forceinline__ float act_fwd(int act, float x, float slope) {
  switch (act) {
    case NC_ACT_TANH: return tanhf(x);
    case NC_ACT_SIGMOID: return 1.0f / (1.0f + expf(-x));
    case NC_ACT_RELU: return fmaxf(x, 0.0f);
    case NC_ACT_LEAKY_RELU: return x >= 0.0f ? x : slope * x;
    case NC_ACT_GELU: {
      const float u = kGeluC * (x + 0.044715f * x * x * x);
      return 0.5f * x * (1.0f + tanhf(u));
    }
    default: return x;
  }
}

// Activation value and derivative (neurocell/kernels_pallas.py:129-156).
__device__ __forceinline__ float act_fwd_deriv(int act, float x, float slope, float* dy) {
  switch (act) {
    case NC_ACT_TANH: {
      const float y = tanhf(x);
      *dy = 1.0f - y * y;
      return y;
    }
    case NC_ACT_SIGMOID: {
      const float y = 1.0f / (1.0f + expf(-x));
      *dy = y * (1.0f - y);
      return y;
    }
    case NC_ACT_RELU:
      *dy = x > 0.0f ? 1.0f : 0.0f;
      return fmaxf(x, 0.0f);
    case NC_ACT_LEAKY_RELU:
      *dy = x >= 0.0f ? 1.0f : slope;
      return x >= 0.0f ? x : slope * x;
    case NC_ACT_GELU: {
      const float x2 = x * x;
      const float th = tanhf(kGeluC * (x + 0.044715f * x2 * x));
      const float du = kGeluC * (1.0f + 3.0f * 0.044715f * x2);
      *dy = 0.5f * (1.0f + th) + 0.5f * x * (1.0f - th * th) * du;
      return 0.5f * x * (1.0f + th);
    }
    default:
      *dy = 1.0f;
      return x;
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// Codd temperature of a call: the device scalar when given (read at run time), else the
// value passed by the host.
__device__ __forceinline__ float codd_tau(const nc_codd& c) {
  return c.temperature_dev ? *c.temperature_dev : c.temperature;
}

// Codd gating of one cell (neurocell/params.py:31-80).  Returns s_prob and writes the
// derivative of the surrogate used in backward (sigmoid' / tau for the STE modes).
__device__ __forceinline__ float codd_prob(float s_raw, bool io, int hard_pin, int mode,
                                           float tau, float thr, float* ds) {
  const float s_base = (!hard_pin && io) ? 1.0f : s_raw;
  const float dbase = (!hard_pin && io) ? 0.0f : 1.0f;
  float s, d;
  if (mode == NC_CODD_CONTINUOUS) {
    s = sigmoidf_(s_base);
    d = s * (1.0f - s);
  } else {
    const float inv_tau = 1.0f / fmaxf(tau, kTauMin);
    const float soft = sigmoidf_(s_base * inv_tau);
    d = soft * (1.0f - soft) * inv_tau;
    if (mode == NC_CODD_ANNEALED) {
      s = soft;
    } else if (mode == NC_CODD_STE_BINARY) {
      // soft + (hard - soft) is exactly `hard` in binary floating point (Sterbenz)
      s = s_base >= 0.0f ? 1.0f : 0.0f;
    } else {
      s = s_base >= thr ? 1.0f : (s_base > 0.0f ? 0.5f : 0.0f);
    }
  }
  d *= dbase;
  if (hard_pin && io) {
    s = 1.0f;
    d = 0.0f;
  }
  *ds = d;
  return s;
}

}  // namespace nc
