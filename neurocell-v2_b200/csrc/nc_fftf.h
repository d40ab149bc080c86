// nc_fftf.h -- per-sample fused FFT propagation for 64 x 64 FFT grids (nc_fftf.cu).
#pragma once

#include <cuda_runtime.h>

#include "nc_kernels.cuh"

namespace nc {

constexpr int kFftfN = 64;                     // the FFT side these kernels are built for
constexpr int kFftfPlane = 64 * 66;            // float2 per stored plane (row stride 66)
constexpr size_t kFftfSmemMax = 227 * 1024;    // opt-in dynamic shared memory per CTA

struct FftfArgs {
  Geo g;
  StepParams sp;
  const int32_t* in_index;
  const int32_t* out_index;
  const float* inputs;        // (B, n_in)
  const float2* H;            // (M/2, 64, 66) pair spectra conj(G^_2j) + i conj(G^_2j+1), / 64^2,
                              // rows padded to the on-chip plane layout (columns 64, 65 zero)
  float* out;                 // forward: (B, n_out)
  float* zhat;                // train: (B, d, M, P)
  float* rstd;                // train: (B, d, M)
  float* xsave;               // train: (B, d-1, P)
  int train;
  int batch;
  const float* gout;          // backward: (B, n_out)
  float* gpix;                // backward: (B, 3, P) per-sample pixel-parameter gradients
  float* gdpart;              // backward: (B, M*K) per-sample filter gradients
  float* gring;               // backward: (B, Fh*Fw) per-sample ring gradients (VALID, d>1) or null
  float* uroi;                // universe mode forward: (B, P) last-step ROI cells, else null
  const float* guroi;         // universe mode backward: (B, P) their gradient, else null
  float2* xspec;              // train: (B, d, 64 x 66) field spectra the forward computed
  int stage;                  // set by fftf_forward / fftf_backward: bulk-copy staging on
};

// True when the fused kernels serve this geometry (FFT side 64, even M, fits on chip).
bool fftf_fits(const Geo& g);
// Dynamic shared memory of the kernels; `stage` adds the bulk-copy staging buffers.
size_t fftf_fwd_smem(const Geo& g, bool stage);
size_t fftf_bwd_smem(const Geo& g, bool ring, bool stage);
// One launch: the pre-step fusion (step parameters, gated filters) and H_j (the filter-pair
// spectra, gated from `filters` directly).
nc_status fftf_prestep_spectra(const Geo& g, const StepParams& sp, const float* cell, const float* filters,
                               const uint8_t* io, const uint8_t* owm, const uint8_t* bmask,
                               const nc_codd& codd, float2* H, cudaStream_t st);
nc_status fftf_forward(const FftfArgs& a, cudaStream_t st);
nc_status fftf_backward(const FftfArgs& a, cudaStream_t st);

}  // namespace nc
