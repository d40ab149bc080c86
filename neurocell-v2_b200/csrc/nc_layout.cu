// nc_layout.cu -- geometry derivation, validation and buffer layouts (host code).
#include <stdio.h>
#include <string.h>

#include "nc_internal.h"
#include "nc_errors.h"
#include "nc_fft.cuh"
#include "nc_fftf.h"

namespace nc {

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

static int next_pow2(int x) {
  int n = 2;
  while (n < x) n <<= 1;
  return n;
}

// FFT side for a field side F: a power of two up to 64 (radix-4 plans), else the smallest
// N = 64 R >= F whose first-stage radix R the two-stage transforms have (nc_fft.cuh); a
// size above 1024 is refused by the caller.  The result of the convolution does not depend
// on the transform size as long as N >= F.
static int fft_side(int F) {
  if (F <= 64) return next_pow2(F);
  for (int R = 2; R <= kFftMaxN / 64; ++R)
    if (fft::stage_a_radix(R) && 64 * R >= F) return 64 * R;
  return next_pow2(F);
}

nc_status make_geo(const nc_topo* t, Geo* g) {
  if (!t) return set_error(NC_ERR_INVALID, "topology pointer is null");
  if (t->H <= 0 || t->W <= 0) return set_error(NC_ERR_INVALID, "grid must be positive, got %dx%d", t->H, t->W);
  if (t->kh <= 0 || t->kw <= 0 || (t->kh % 2) == 0 || (t->kw % 2) == 0)
    return set_error(NC_ERR_INVALID, "Green's function kernel_size must be odd, got (%d, %d)", t->kh, t->kw);
  if (t->M <= 0) return set_error(NC_ERR_INVALID, "directions must be >= 1, got %d", t->M);
  if (t->depth <= 0) return set_error(NC_ERR_INVALID, "depth must be >= 1, got %d", t->depth);
  if (t->padding < NC_PAD_VALID || t->padding > NC_PAD_CIRCULAR)
    return set_error(NC_ERR_INVALID, "unsupported padding_mode id %d", t->padding);
  if (t->act < NC_ACT_NONE || t->act > NC_ACT_GELU || t->final_act < NC_ACT_NONE || t->final_act > NC_ACT_GELU)
    return set_error(NC_ERR_INVALID, "unsupported activation id (%d, %d)", t->act, t->final_act);
  if (t->n_in < 0 || t->n_out <= 0) return set_error(NC_ERR_INVALID, "bad port sizes n_in=%d n_out=%d", t->n_in, t->n_out);
  memset(g, 0, sizeof(*g));
  g->H = t->H; g->W = t->W; g->kh = t->kh; g->kw = t->kw; g->K = t->kh * t->kw;
  g->M = t->M; g->d = t->depth; g->padding = t->padding;
  if (t->padding == NC_PAD_VALID) {
    g->pad_h = (t->kh - 1) / 2;
    g->pad_w = (t->kw - 1) / 2;
  }
  g->roi_h = t->H - 2 * g->pad_h;
  g->roi_w = t->W - 2 * g->pad_w;
  if (g->roi_h <= 0 || g->roi_w <= 0)
    return set_error(NC_ERR_INVALID, "grid (%d, %d) is too small for kernel (%d, %d)", t->H, t->W, t->kh, t->kw);
  g->P = g->roi_h * g->roi_w;
  g->Fh = g->roi_h + t->kh - 1;
  g->Fw = g->roi_w + t->kw - 1;
  g->Fs = ((g->Fw + 4) + 3) & ~3;   // >= 4 floats of slack per row for strip over-reads
  g->oh = (t->kh - 1) / 2;
  g->ow = (t->kw - 1) / 2;
  if (t->padding == NC_PAD_VALID) { g->gr = 0; g->gc = 0; } else { g->gr = g->oh; g->gc = g->ow; }
  g->n_in = t->n_in; g->n_out = t->n_out;
  g->act = t->act; g->fact = t->final_act;
  g->slope = t->act_slope; g->fslope = t->final_act_slope;
  g->norm = t->norm ? 1 : 0; g->hard_pin = t->hard_pin_io ? 1 : 0; g->gated = t->gated_filters ? 1 : 0;
  g->F_elems = (g->Fh + 1) * g->Fs;   // one slack row
  const double total_px = (double)g->M * (double)g->P;
  if (total_px > 2.0e9) return set_error(NC_ERR_UNSUPPORTED, "plane too large (%g values)", total_px);
  // Green's convolution algorithm (reference auto rule: propagator.py:68-85)
  g->Nh = fft_side(g->Fh);
  g->Nw = fft_side(g->Fw);
  const bool fft_fits = g->Nh <= kFftMaxN && g->Nw <= kFftMaxN;
  if (t->conv_algo < NC_CONV_AUTO || t->conv_algo > NC_CONV_FFT)
    return set_error(NC_ERR_INVALID, "unsupported conv_algo id %d", t->conv_algo);
  if (t->conv_algo == NC_CONV_FFT && !fft_fits)
    return set_error(NC_ERR_UNSUPPORTED, "FFT grid %dx%d exceeds %d per side", g->Nh, g->Nw, kFftMaxN);
  if (t->conv_algo == NC_CONV_AUTO) {
    // the reference's rule (large kernels) plus: mid-size kernels whose response planes do
    // not fit on chip, where the direct kernels would stream every plane through HBM
    const size_t on_chip = sizeof(float) * ((size_t)g->M * g->K + 4 * (size_t)g->M + 128 +
                                            (size_t)g->F_elems + (size_t)g->M * g->P);
    const bool planes_on_chip = on_chip <= kSmemBudget;   // the direct kernels' policy
    const bool large_k = t->kh * t->kw > 512;
    const bool mid_k = t->kh * t->kw >= 81 && !planes_on_chip;
    // 64 x 64 FFT grids run the fused per-sample FFT kernels, which beat the direct
    // kernels from about 11 x 11 taps on (ALU chip: 0.49 vs 0.82 ms per train step)
    const bool small_fused = fftf_fits(*g) && t->kh * t->kw >= 121;
    g->algo = (fft_fits && (large_k || mid_k || small_fused)) ? NC_CONV_FFT : NC_CONV_DIRECT;
  } else {
    g->algo = t->conv_algo;
  }
  return NC_OK;
}

PlanLayout plan_layout(const nc_topo* t) {
  PlanLayout L;
  size_t o = 0;
  L.in_index = o; o = align256(o + sizeof(int32_t) * (size_t)(t->n_in > 0 ? t->n_in : 1));
  L.out_index = o; o = align256(o + sizeof(int32_t) * (size_t)t->n_out);
  L.io_mask = o; o = align256(o + (size_t)t->H * t->W);
  L.out_w_mask = o; o = align256(o + (size_t)t->H * t->W);
  L.border_mask = o; o = align256(o + (size_t)t->H * t->W);
  Geo g;
  if (make_geo(t, &g) == NC_OK && g.algo == NC_CONV_FFT) {
    L.twid_w = o; o = align256(o + 8 * (size_t)fft::plan_twiddle_len(g.Nw));
    L.twid_h = o; o = align256(o + 8 * (size_t)fft::plan_twiddle_len(g.Nh));
  } else {
    L.twid_w = L.twid_h = SIZE_MAX;
  }
  L.total = o;
  return L;
}

WsLayout ws_layout(const Geo& g, int batch, uint32_t flags, bool* f_smem, bool* z_smem,
                   bool* gz_smem) {
  const bool train = (flags & NC_FLAG_TRAIN) != 0;
  const size_t B = (size_t)batch, P = (size_t)g.P, M = (size_t)g.M, HW = (size_t)g.H * g.W;
  const size_t fl = sizeof(float);
  // on-chip policy (fixed budget so workspace sizes do not depend on the device)
  const size_t budget = kSmemBudget;
  const size_t base = fl * ((size_t)g.M * g.K + 4 * (size_t)g.M + 128);
  const size_t fbytes = fl * (size_t)g.F_elems;
  const bool fs = base + fbytes <= budget;
  const bool zs = fs && base + fbytes + fl * M * P <= budget;
  const bool gzs = fs && base + fbytes + fl * M * P <= budget;
  if (f_smem) *f_smem = fs;
  if (z_smem) *z_smem = zs;
  if (gz_smem) *gz_smem = gzs;

  WsLayout L;
  size_t o = 0;
  auto take = [&](size_t bytes) { size_t r = o; o = align256(o + (bytes ? bytes : 1)); return r; };
  L.status = take(sizeof(int));   // offset 0 in every layout
  L.weff = take(fl * P);
  L.seff = take(fl * P);
  L.broi = take(fl * P);
  L.border = take(fl * HW);
  L.sprob = take(fl * HW);
  L.dsprob = take(fl * HW);
  L.wpinned = take(fl * HW);
  L.geff = take(fl * M * g.K);
  L.uroi = take(fl * B * P);
  L.guroi = train ? take(fl * B * P) : SIZE_MAX;
  L.gringf = train ? take(fl * HW) : SIZE_MAX;
  const size_t dm1 = (size_t)(g.d > 1 ? g.d - 1 : 0);
  L.xsave = train ? take(fl * B * (dm1 ? dm1 : 1) * P) : SIZE_MAX;
  L.zhat = train ? take(fl * B * g.d * M * P) : SIZE_MAX;
  L.rstd = train ? take(fl * B * g.d * M) : SIZE_MAX;
  L.f_field = L.f_xhat = L.f_tmp = L.f_gspec = L.f_mean = L.f_rstd = L.f_rowstats = L.f_gzpart = L.f_ncoef = SIZE_MAX;
  L.f_mean_save = SIZE_MAX;
  L.f_q = L.f_dgacc = L.f_gz = L.f_dx = L.f_gpart = L.f_h = L.f_gring = L.f_xspec = SIZE_MAX;
  if (g.algo == NC_CONV_FFT && fftf_fits(g)) {
    // fused per-sample FFT kernels: spectra tables + per-sample partials only
    if (f_smem) *f_smem = true;
    if (z_smem) *z_smem = true;
    if (gz_smem) *gz_smem = true;
    const size_t c64 = 2 * fl, NN = (size_t)g.Nh * g.Nw;
    L.f_h = take(c64 * (M / 2) * (size_t)kFftfPlane);   // planes in the on-chip layout
    L.fscr = L.zscr = L.gzscr = L.gdelta = L.gdeltasum = L.redscr = SIZE_MAX;
    if (train) {
      L.gpix = take(fl * B * 3 * P);
      L.gdpart = take(fl * B * M * g.K);
      L.f_xspec = take(c64 * B * (size_t)g.d * kFftfPlane);   // the forward's field spectra
      const bool ringp = g.padding == NC_PAD_VALID && g.d > 1;
      L.f_gring = ringp ? take(fl * B * (size_t)g.Fh * g.Fw) : SIZE_MAX;
      L.redscr = take(fl * kRedChunks * (3 * P + M * g.K + (ringp ? (size_t)g.Fh * g.Fw : 0)));
      L.gsum = L.gdsum = L.gborder = SIZE_MAX;   // summed inside the pre-step adjoint
    } else {
      L.gpix = L.gdpart = L.gsum = L.gdsum = L.gborder = SIZE_MAX;
    }
    L.total = o;
    return L;
  }
  if (g.algo == NC_CONV_FFT) {
    // FFT convolution: per-step planes live in HBM, nothing per sample on chip
    if (f_smem) *f_smem = false;
    if (z_smem) *z_smem = false;
    if (gz_smem) *gz_smem = false;
    const size_t pairs = (B + 1) / 2, c64 = 2 * fl;
    const size_t FF = (size_t)g.Fh * g.Fw, NN = (size_t)g.Nh * g.Nw;
    size_t lines = pairs * M * (size_t)g.roi_h;
    if (pairs * (size_t)g.Fh > lines) lines = pairs * (size_t)g.Fh;
    if (M * (size_t)g.kh > lines) lines = M * (size_t)g.kh;
    L.f_field = take(fl * B * FF);
    L.f_xhat = take(c64 * pairs * NN * (train ? g.d : 1));   // train: one slot per step
    L.f_tmp = take(c64 * lines * (size_t)g.Nw);
    L.f_gspec = take(c64 * M * NN);
    L.f_mean = take(fl * B * M);
    L.f_rstd = take(fl * B * M);
    L.f_rowstats = take(c64 * B * M * (size_t)g.roi_h);
    L.fscr = SIZE_MAX;
    L.zscr = train ? SIZE_MAX : take(fl * B * M * P);
    L.gzscr = L.gpix = L.gdpart = L.gdelta = L.gdeltasum = L.redscr = SIZE_MAX;
    if (train) {
      L.f_q = take(c64 * pairs * M * NN);
      L.f_dgacc = take(c64 * M * NN);
      L.f_gz = take(fl * B * M * P);
      L.f_dx = take(fl * B * FF);
      L.f_gpart = take(fl * kRedChunks * 3 * P);
      L.f_gzpart = take(fl * ((P + 255) / 256) * B * M * 2);
      L.f_ncoef = take(fl * 4 * B * M);
      L.f_mean_save = take(fl * B * g.d * M);
      L.gsum = take(fl * 3 * P);
      L.gdsum = take(fl * M * g.K);
      L.gborder = take(fl * HW);
    } else {
      L.gsum = L.gdsum = L.gborder = SIZE_MAX;
    }
    L.total = o;
    return L;
  }
  L.fscr = fs ? SIZE_MAX : take(fl * B * g.F_elems);
  L.zscr = (!train && !zs) ? take(fl * B * M * P) : SIZE_MAX;
  if (train) {
    L.gzscr = gzs ? SIZE_MAX : take(fl * B * M * P);
    // per-sample pixel partials: (B, d, 3, P) per-step slots (specialised kernels) or
    // (B, 3, P) followed by a (B, P) field-adjoint plane (generic kernels)
    L.gpix = take(fl * B * (3 * (size_t)g.d + 1) * P);
    L.gdpart = take(fl * B * M * g.K);
    L.gdelta = (g.padding == NC_PAD_VALID && g.d > 1) ? take(fl * B * M * P) : SIZE_MAX;
    L.gsum = take(fl * 3 * P);
    L.gdsum = take(fl * M * g.K);
    L.gdeltasum = (g.padding == NC_PAD_VALID && g.d > 1) ? take(fl * M * P) : SIZE_MAX;
    L.gborder = take(fl * HW);
    L.redscr = take(fl * kRedChunks * (3 * P > M * P ? 3 * P : M * P));
  } else {
    L.gzscr = L.gpix = L.gdpart = L.gdelta = L.gsum = L.gdsum = L.gdeltasum = L.gborder = SIZE_MAX;
    L.redscr = SIZE_MAX;
  }
  L.total = o;
  return L;
}

}  // namespace nc
