// nc_fast_dev.cuh -- device helpers shared by the specialised fused kernels.
#pragma once

#include <cuda_runtime.h>

#include "nc_common.cuh"
#include "nc_fast.cuh"
#include "nc_kernels.cuh"

namespace nc {
namespace fast {

using namespace fastc;

// Phase timestamps of CTA 0 for performance work (compiled in only with
// -DNC_PHASE_TIMING=1; read back with nc_debug_phase_times).
#if NC_PHASE_TIMING
static __device__ long long g_nc_phase[8][8];
static __device__ long long g_nc_warp[8][32][2];
#define NC_PHASE_MARK(t, k) \
  do { if (blockIdx.x == 0 && threadIdx.x == 0) g_nc_phase[(t)][(k)] = clock64(); } while (0)
#define NC_WARP_MARK(t, k) \
  do { if (blockIdx.x == 0 && (threadIdx.x & 31) == 0) g_nc_warp[(t)][threadIdx.x >> 5][(k)] = clock64(); } while (0)
#else
#define NC_PHASE_MARK(t, k) do {} while (0)
#define NC_WARP_MARK(t, k) do {} while (0)
#endif
constexpr int NT = kFusedThreads;   // 512

__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 dup2(float x) { return make_float2(x, x); }

// out[m] = scale * sum over the CTA of v[m], m < 16.
__device__ __forceinline__ void sum16_block(float (&v)[M], float* red, float* out, float scale) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int m = 0; m < M; ++m) v[m] = warp_sum(v[m]);
  if (lane == 0) {
#pragma unroll
    for (int m = 0; m < M; ++m) red[warp * M + m] = v[m];
  }
  __syncthreads();
  if (threadIdx.x < M) {
    float s = 0.f;
    for (int w = 0; w < NW; ++w) s += red[w * M + threadIdx.x];
    out[threadIdx.x] = s * scale;
  }
  __syncthreads();
}

// Step t=0 field (zeros + the sample's inputs), row stride `fs`, `rows` rows.
inline __device__ void inject(const Geo& g, float* F, int fs, int rows, const int32_t* in_index,
                       const float* inp) {
  for (int i = threadIdx.x; i < rows * fs; i += blockDim.x) F[i] = 0.f;
  __syncthreads();
  for (int j = threadIdx.x; j < g.n_in; j += blockDim.x) {
    const int idx = in_index[j];
    if (idx < 0) continue;
    const int r = idx / g.W, c = idx - (idx / g.W) * g.W;
    F[(r + g.gr) * fs + c + g.gc] = inp[j];
  }
  __syncthreads();
}

inline __device__ void wrap_ring(const Geo& g, float* F, int fs) {
  const int n = g.Fh * g.Fw;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int fr = i / g.Fw, fc = i - fr * g.Fw;
    const int r = fr - g.oh, c = fc - g.ow;
    if (r >= 0 && r < g.roi_h && c >= 0 && c < g.roi_w) continue;
    int sr = r % g.roi_h; if (sr < 0) sr += g.roi_h;
    int sc = c % g.roi_w; if (sc < 0) sc += g.roi_w;
    F[fr * fs + fc] = F[(sr + g.oh) * fs + sc + g.ow];
  }
}

inline __device__ void border_ring(const Geo& g, float* F, int fs, const float* border) {
  const int n = g.Fh * g.Fw;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int fr = i / g.Fw, fc = i - fr * g.Fw;
    const int r = fr - g.oh, c = fc - g.ow;
    if (r >= 0 && r < g.roi_h && c >= 0 && c < g.roi_w) continue;
    F[fr * fs + fc] = border[fr * g.W + fc];
  }
}

// ROI pixel of an output cell, -1 outside the ROI (border outputs: universe mode only).
__device__ __forceinline__ int out_pixel(const Geo& g, int idx) {
  const int r = idx / g.W - g.pad_h, c = idx - (idx / g.W) * g.W - g.pad_w;
  return (r >= 0 && r < g.roi_h && c >= 0 && c < g.roi_w) ? r * g.roi_w + c : -1;
}

// ---------------------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------------------

}  // namespace fast
}  // namespace nc
