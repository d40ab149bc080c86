// nc_kernels.cuh -- argument blocks of the VNN kernels.
#pragma once

#include "nc_internal.h"

namespace nc {

constexpr int kFusedThreads = 512;

struct StepParams {           // pre-step fusion output (neurocell/params.py:104-135)
  float* weff;                // (P)  (1/M) * W_pinned * (1 - s)      on the ROI
  float* seff;                // (P)  (1/M) * s                       on the ROI
  float* broi;                // (P)  B                               on the ROI
  float* border;              // (H*W) act(B) * s  (VALID ring values)
  float* sprob;               // (H*W) s_prob
  float* dsprob;              // (H*W) d s_prob / d S_raw (surrogate)
  float* wpinned;             // (H*W) W with the output port pinned to 1
  float* geff;                // (M*K) filters (sigmoid-gated when requested)
  int* status;                // workspace status word: cleared by the forward's pre-step
                              // kernel, set to 1 when a kernel's bounded wait gives up
};

// Segments of one nc_stage_from_host call (device addresses).
struct StageSegs {
  void* dst[NC_MAX_STAGE_SEGS];
  const void* src[NC_MAX_STAGE_SEGS];
  size_t bytes[NC_MAX_STAGE_SEGS];
  int n;
};

struct FwdArgs {
  Geo g;
  StepParams sp;
  const int32_t* in_index;    // (n_in) flat grid index, -1 = dropped
  const int32_t* out_index;   // (n_out) flat grid index
  const float* inputs;        // (B, n_in)
  float* out;                 // (B, n_out)
  float* xsave;               // train: (B, d-1, P) field interior entering step t>=1
  float* zhat;                // train: (B, d, M, P) standardised planes
  float* rstd;                // train: (B, d, M)
  float* fscr;                // (B, F_elems) field scratch when F is not on-chip
  float* zscr;                // (B, M, P) plane scratch when z is not on-chip (inference)
  float* uroi;                // universe mode: (B, P) last-step ROI cells (ROI epilogue with
                              // the final activation) instead of the port outputs; else null
  int train, g_smem, f_smem, z_smem;
  int batch;
};

struct BwdArgs {
  Geo g;
  StepParams sp;
  const int32_t* in_index;
  const int32_t* out_index;
  const float* inputs;
  const float* gout;          // (B, n_out)
  const float* xsave;
  float* zhat;                // the specialised kernels overwrite consumed planes with gz
  const float* rstd;
  float* fscr;
  float* gzscr;               // (B, M, P) when gz is not on-chip
  float* gpix;                // (B, 3, P) per-sample partials + (B, P) dX plane after them
  float* gdpart;              // (B, M*K) per-sample filter-gradient partials
  float* gdelta;              // (B, M, P) per-sample sum over t>=1 of gz (VALID, d>1)
  const float* guroi;         // universe mode: (B, P) gradient of the last-step ROI cells
  int g_smem, f_smem, gz_smem;
  int batch;
};

// Up to three (batch, n_s) per-sample partial arrays, summed over sample chunks into one
// (chunks, total) partial array (seg_batch_sum1_kernel).
struct SegSum {
  const float* in[3];
  int n[3];
  int nseg, total;
};

// Grid window of an adaptive sub-ROI call inside the full chip: top-left grid cell and size.
struct UniWindow {
  int r0, c0, h, w;
};

}  // namespace nc
