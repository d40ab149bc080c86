// nc_fftconv.h -- FFT-regime propagation (host orchestration of nc_fftconv.cu).
#pragma once

#include <cuda_runtime.h>

#include "nc_kernels.cuh"

namespace nc {

// Everything one forward or backward call of the FFT regime touches.
struct FftCall {
  Geo g;
  int batch;
  bool train;
  StepParams sp;
  const int32_t* in_index;
  const int32_t* out_index;
  const float* inputs;        // (B, n_in)
  const float2* tw_w;         // plan twiddles of the Nw transform
  const float2* tw_h;         // plan twiddles of the Nh transform
  // workspace
  float* field;               // (B, Fh, Fw)
  float2* xhat;               // (B/2, Nh, Nw)
  float2* tmp;                // intermediate lines
  float2* gspec;              // (M, Nh, Nw)
  float* mean;                // (B, M)
  float* rstd;                // (B, M)
  float2* rowstats;           // (B, M, roi_h) per-row (mean, M2) of the forward planes
  float* gzpart;              // train: (ceil(P/256), B, M, 2) per-CTA sums of gz, gz*zhat
  float4* ncoef;              // train: (B, M) standardisation-adjoint coefficients
  float* zscr;                // (B, M, P) inference planes
  float* zhat;                // train: (B, d, M, P) raw planes z of every step
  float* rstd_save;           // train: (B, d, M) their 1 / sqrt(var + eps)
  float* mean_save;           // train: (B, d, M) their means (zhat = (z - mean) * rstd)
  float* xsave;               // train: (B, d-1, P)
  float2* q;                  // train: (B/2, M, Nh, Nw)
  float2* dgacc;              // train: (M, Nh, Nw)
  float* gz;                  // train: (B, M, P)
  float* dx;                  // train: (B, Fh, Fw)
  float* gpart;               // train: (kRedChunks, 3, P)
  float* gsum;                // train: (3, P)
  float* gdsum;               // train: (M*K)
  float* gborder;             // train: (H*W), VALID with d > 1 only
  // call arguments
  const float* gout;          // backward: (B, n_out)
  float* out;                 // forward: (B, n_out)
  float* uroi;                // universe mode forward: (B, P) last-step ROI cells, else null
  const float* guroi;         // universe mode backward: (B, P) their gradient, else null
};

// Filter spectra G^_m / (Nh*Nw) into c.gspec (uses c.tmp).
nc_status fft_filter_spectra(const FftCall& c, cudaStream_t st);
// Forward d-step loop with FFT convolution (filter spectra included).  Launch count is
// reported through note_launch().
nc_status fft_forward(const FftCall& c, cudaStream_t st);
// Backward of the same call; leaves gsum, gdsum and gborder for prestep_bwd_kernel.
nc_status fft_backward(const FftCall& c, cudaStream_t st);

}  // namespace nc
