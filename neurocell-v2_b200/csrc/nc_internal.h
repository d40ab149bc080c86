// nc_internal.h -- host/device shared geometry and workspace layout.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include "neurocell_b200.h"

namespace nc {

// Derived geometry passed by value to every kernel.
//
// The per-sample "field" F is the padded plane the Green's convolution reads:
//   VALID:        F is the full H x W grid; the ROI is its interior at (pad_h, pad_w).
//   SAME/CIRCULAR: F is the ROI (== grid) with a ((kh-1)/2, (kw-1)/2) halo that holds
//                 zeros (SAME) or the wrapped interior (CIRCULAR).
// conv_VALID(F, G) then equals conv_SAME(roi, G) + Delta_border of the reference
// (neurocell/propagator.py:1-12 identity) when F's ring holds border_2d.
struct Geo {
  int H, W, kh, kw, K, M, d, padding;
  int pad_h, pad_w;        // grid -> ROI offset (topology.pad_h / pad_w)
  int roi_h, roi_w, P;     // ROI size and pixel count
  int Fh, Fw, Fs;          // field height, width, row stride (floats)
  int oh, ow;              // ROI origin inside F
  int gr, gc;              // grid origin inside F (VALID: 0,0; else oh,ow)
  int n_in, n_out;
  int act, fact;
  float slope, fslope;
  int norm, hard_pin, gated;
  int F_elems;             // floats of one field buffer (incl. slack rows)
  int algo;                // resolved nc_conv_algo: NC_CONV_DIRECT or NC_CONV_FFT
  int Nh, Nw;              // FFT grid: sides >= Fh, Fw (powers of two to 64, then 64 R)
};

// Largest FFT side the on-chip line transforms handle.
constexpr int kFftMaxN = 1024;

nc_status make_geo(const nc_topo* t, Geo* g);

// Offsets (bytes) of the plan buffer sections.
struct PlanLayout {
  size_t in_index, out_index, io_mask, out_w_mask, border_mask;
  size_t twid_w, twid_h;   // FFT stage twiddles for the Nw and Nh transforms (FFT only)
  size_t total;
};
PlanLayout plan_layout(const nc_topo* t);

// Offsets (bytes) of the workspace sections; 0-sized sections have offset SIZE_MAX.
struct WsLayout {
  // status word of the call (always at offset 0; nc_workspace_status)
  size_t status;
  // step parameters (pre-step fusion output)
  size_t weff, seff, broi, border, sprob, dsprob, wpinned, geff;
  // universe mode: last-step ROI cells (B, P), their gradient (B, P), ring gradient (H*W)
  size_t uroi, guroi, gringf;
  // forward residuals (train)
  size_t xsave, zhat, rstd;
  // scratch when on-chip buffers do not fit
  size_t fscr, zscr, gzscr;
  // backward partials and reductions
  size_t gpix, gdpart, gdelta, gsum, gdsum, gdeltasum, gborder;
  size_t redscr;          // partial rows of the two-stage batch reductions
  // FFT convolution (complex sections hold float2)
  size_t f_field;         // (B, Fh, Fw) field of the current step
  size_t f_xhat;          // (B/2, Nh, Nw) spectra of sample-pair fields
  size_t f_tmp;           // row-pass / column-pass intermediate lines
  size_t f_gspec;         // (M, Nh, Nw) filter spectra / (Nh*Nw)
  size_t f_mean, f_rstd;  // (B, M) plane statistics of the current step
  size_t f_mean_save;     // train: (B, d, M) per-step plane means (the saved planes stay
                          // raw; the backward standardises them on the fly)
  size_t f_rowstats;      // (B, M, roi_h) per-row (mean, M2) of the current step's planes
  size_t f_gzpart;        // train: (ceil(P/256), B, M, 2) per-CTA sums of gz and gz*zhat
  size_t f_ncoef;         // train: (B, M) float4 (rstd, mean gz, mean gz*zhat, 0) of the
                          // standardisation adjoint applied by the next row pass
  size_t f_q;             // (B/2, M, Nh, Nw) plane-gradient spectra (train)
  size_t f_dgacc;         // (M, Nh, Nw) filter-gradient spectrum accumulator (train)
  size_t f_gz;            // (B, M, P) plane gradients (train)
  size_t f_dx;            // (B, Fh, Fw) field gradient (train)
  size_t f_gpart;         // (kRedChunks, 3, P) per-chunk pixel-gradient partials (train)
  size_t f_h;             // fused small-grid kernels: (M/2, 64, 64) pair spectra
  size_t f_gring;         // fused small-grid kernels: (B, Fh*Fw) ring gradients (train)
  size_t f_xspec;         // fused small-grid kernels: (B, d, 64 x 66) field spectra (train)
  size_t total;
};

// Sample chunks of the two-stage batch-and-step reductions.
constexpr int kRedChunks = 16;
WsLayout ws_layout(const Geo& g, int batch, uint32_t flags, bool* f_smem, bool* z_smem,
                   bool* gz_smem);

}  // namespace nc
