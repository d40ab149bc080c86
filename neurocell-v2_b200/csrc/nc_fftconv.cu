// nc_fftconv.cu -- the d-step VNN loop with FFT Green's convolution (sm_100a).
//
// The reference's large-kernel regime ("pallas_sram": rfft2_pruned / irfft2_pruned and the
// Plancherel VJP of neurocell/kernels_greens.py:25-66, 278-400 and
// neurocell/kernels_pallas.py:1759-1826) rebuilt around complex power-of-two transforms:
//
//  * two samples share one complex transform (real parts = sample 2p, imaginary = 2p+1).
//    The filter spectra are spectra of real signals, so a product with them keeps the two
//    samples apart: IFFT(X^ . conj(G^_m)) = z_{2p,m} + i z_{2p+1,m} (forward) and
//    IFFT(sum_m Q^_m . G^_m) = dX_{2p} + i dX_{2p+1} (field adjoint), and
//    Re IFFT(X^ . conj(Q^_m)) = sum over the pair of corr(X_b, gz_{b,m}) (filter adjoint),
//  * the forward transforms leave spectra in a fixed permuted order (digit-reversed for the
//    radix-4 plans, frequency k1 + R k2 at position 64 k1 + k2 for the two-stage plans) and
//    the inverse transforms take them back (nc_fft.cuh), so no pass reorders data,
//  * the transforms are pruned to the rows that hold data (field rows < Fh, plane rows
//    < roi_h) and to the rows and columns that are kept (ROI outputs, kh x kw filter lags),
//  * the filter-gradient spectrum is accumulated over samples and steps in a fixed order
//    and transformed back once per call (the reference's "dK reduced over B and d before one
//    M-irfft2"); every other batch reduction is a fixed-order loop as well, so the backward
//    is deterministic.
// The per-step epilogues have the semantics of neurocell/epilogue.py:28-56 / :82-128 with
// the centred variance of neurocell/kernels_pallas.py:202-205: per-row centred statistics
// merged per plane with the two-stage formula of the reference's tiled path
// (kernels_pallas.py:740-837).
#include <cuda_runtime.h>

#include <type_traits>

#include "nc_common.cuh"
#include "nc_errors.h"
#include "nc_fft.cuh"
#include "nc_fftconv.h"

namespace nc {

using fft::cadd;
using fft::cmul;
using fft::cmulc;
using fft::line_stride;
using fft::pidx;

namespace {

constexpr int kFftThreads = 256;
constexpr int kEpiThreads = 256;
constexpr int kStatThreads = 512;      // per-plane statistics kernels

// Real planes addressed as  base + b*sstride + m*plane + r*rs + e.
struct Planes {
  float* ptr;
  size_t sstride;
  int nsamp, ms, rows, cols, plane, rs;
  int pack;     // 1: a line holds samples (2g, 2g+1) as (re, im); 0: one sample, im = 0
  int units;    // lines / rows = (nsamp or pairs) * ms
  float scale;
  float2* rowstats;   // rows_inv: per stored row (mean, M2) of its `cols` values, or null
  // rows_fwd: with coef set, the pass reads the standardisation adjoint of the planes,
  // coef.x * (v - coef.y - zh * coef.z) per (sample, m) plane, from the planes v and the
  // forward's raw planes zh (same layout, sample stride zstride; the coefficients fold in
  // their standardisation, see norm_coef_kernel)
  const float* zh;
  size_t zstride;
  const float4* coef;
};

// Where one line of a row pass lives: the offsets of its row in a.ptr for sample 2g (or g)
// and, on packed lines, sample 2g+1 (o[1] = -1 when that sample does not exist), the same
// rows in a.zh, and the standardisation-adjoint coefficients of those planes (rows_fwd with
// a.coef).  A CTA computes them once per line (line_refs), so its element loops do no
// index divisions.
struct LineRef {
  long long o[2];
  long long z[2];
  float4 k[2];
};
constexpr int kLineRefF2 = sizeof(LineRef) / sizeof(float2);   // float2 words per LineRef

__device__ __forceinline__ void line_refs(const Planes& a, int line0, int nl, LineRef* refs, int tid,
                                          int nt) {
  for (int l = tid; l < nl; l += nt) {
    const int line = line0 + l;
    const int u = line / a.rows, r = line - u * a.rows;
    const int gs = u / a.ms, m = u - gs * a.ms;
    const int b1 = a.pack ? 2 * gs : gs;
    const size_t off = (size_t)m * a.plane + (size_t)r * a.rs;
    LineRef R;
#pragma unroll
    for (int s = 0; s < 2; ++s) {
      const int b = b1 + s;
      const bool ok = s == 0 || (a.pack && b < a.nsamp);
      R.o[s] = ok ? (long long)((size_t)b * a.sstride + off) : -1;
      R.z[s] = (ok && a.coef) ? (long long)((size_t)b * a.zstride + off) : 0;
      float4 k = make_float4(0.f, 0.f, 0.f, 0.f);
      if (ok && a.coef) {
        k = a.coef[(size_t)b * a.ms + m];
        k.x *= a.scale;
      }
      R.k[s] = k;
    }
    refs[l] = R;
  }
}

// L2 prefetch of [p, p + bytes) rounded inward to 16-byte boundaries: a hint that takes no
// registers and has no completion to wait for.
__device__ __forceinline__ void prefetch_l2(const void* p, size_t bytes) {
  const uintptr_t lo = ((uintptr_t)p + 15) & ~(uintptr_t)15;
  const uintptr_t hi = ((uintptr_t)p + bytes) & ~(uintptr_t)15;
  if (hi > lo)
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(lo), "r"((unsigned)(hi - lo)) : "memory");
}

// The row passes are bound by the latency of their loads (64 registers cap the loads a
// thread keeps in flight), so a CTA first asks L2 for all the rows it is about to read,
// in a few large requests, before it copies its twiddles and line references: the
// element loads then hit L2 or join requests already in flight.  rows_fwd: one prefetch
// per (line, sample, planes or zh) row of CTA blk.  (Measured against prefetching the
// CTAs a quarter, half or whole wave ahead: 67.8 vs 69.1 / 69.9 / 73.6 ms at config 4.)
__device__ __forceinline__ void prefetch_rows(const Planes& a, int blk, int L, int tid) {
  const int total = a.units * a.rows;
  if ((long long)blk * L >= total) return;
  const int line0 = blk * L;
  const int nl = min(L, total - line0);
  const int per = a.coef ? 4 : 2;
  if (tid >= nl * per) return;
  const int l = tid / per, k = tid - l * per, s = k & 1;
  const int line = line0 + l;
  const int u = line / a.rows, r = line - u * a.rows;
  const int gs = u / a.ms, m = u - gs * a.ms;
  const int b = (a.pack ? 2 * gs : gs) + s;
  if (s == 1 && !(a.pack && b < a.nsamp)) return;
  const size_t off = (size_t)m * a.plane + (size_t)r * a.rs;
  const float* base = k < 2 ? a.ptr + (size_t)b * a.sstride : a.zh + (size_t)b * a.zstride;
  prefetch_l2(base + off, sizeof(float) * (size_t)a.cols);
}

// Element e of sample s of a line as the row pass reads it (COEF: a.coef is set, see
// Planes::coef; line_refs folds a.scale into k.x).
template <bool COEF>
__device__ __forceinline__ float line_in(const Planes& a, const LineRef& R, int s, int e) {
  const float v = a.ptr[R.o[s] + e];
  if (!COEF) return v * a.scale;
  const float4 k = R.k[s];
  return k.x * (v - k.y - a.zh[R.z[s] + e] * k.z);
}

__device__ __forceinline__ int even_up(int x) { return (x + 1) & ~1; }

// Line l and element e of a flat index over lines of N elements: N = 64 RA is a compile-time
// constant when RA > 0; the other variants only see powers of two (N <= 64 for RA = 0,
// N = 1024 for RA = -1, see kernel_ra), so shifts.
template <int RA>
__device__ __forceinline__ void line_elem(int idx, int N, int lgN, int& l, int& e) {
  if constexpr (RA > 0) {
    l = idx / (64 * RA);
    e = idx - l * (64 * RA);
  } else {
    l = idx >> lgN;
    e = idx & (N - 1);
  }
}

// line_elem over element pairs (N even): idx runs over N / 2 pairs per line, e is even.
// Elements e and e + 1 sit next to each other in a line's shared-memory layout
// (pidx(e + 1) = pidx(e) + 1 for even e).
template <int RA>
__device__ __forceinline__ void line_pair(int idx, int N, int lgN, int& l, int& e) {
  if constexpr (RA > 0) {
    l = idx / (32 * RA);
    e = 2 * (idx - l * (32 * RA));
  } else {
    l = idx >> (lgN - 1);
    e = 2 * (idx & ((N >> 1) - 1));
  }
}

// Variants of the transform kernels: RA = N / 64 (2, 4, 8) specialises the radix-R stage that
// runs on global memory; RA = -1 chooses at run time between that stage (any R) and the
// shared-memory plan (used for N = 1024: measured faster than the radix-16
// specialisation); RA = 0 is the shared-memory plan alone (N <= 64 or N > 1024).  fft_ctas: CTAs per SM each variant is compiled for (registers per thread
// <= 64K / (256 * that)): five (48 registers, no spills) for the specialisations, four for
// the run-time variant and the column pass that sums over the directions (`heavy`); the
// shared-memory plans leave the choice to the compiler.
constexpr int fft_ctas(int RA, bool heavy = false) { return RA == 0 ? 1 : (RA < 0 || heavy) ? 4 : 5; }
// Threads of a column-pass CTA.  The sum over the directions (M loads per element) runs
// one CTA of 1024 threads per SM over 16 columns for every two-stage size (config 2:
// 12.24 -> 11.70 ms).  The other N = 1024 passes run two CTAs of 512 threads over 8
// columns each (shared memory holds 16 lines of N = 1024 per SM either way; one radix-16
// task per thread keeps more loads in flight; one 1024-thread CTA measured slower for
// them: its barrier phases stall the whole SM); the other sizes keep 256 threads (512
// measured slower).
constexpr bool cols_big(int MODE, int RA) { return RA != 0 && MODE == 2; }
constexpr int cols_threads(int MODE, int RA) {
  return cols_big(MODE, RA) ? 1024 : RA < 0 ? 512 : kFftThreads;
}

// Forward row transforms of real planes -> dst (lines, N) complex.  For N > 64 (RA = N/64)
// the radix-R stage reads the planes directly (fft::fwd_a_global).  Dynamic shared memory:
// L line references, the plan's twiddles, L lines (rows_smem).
template <int RA>
__global__ void __launch_bounds__(kFftThreads, fft_ctas(RA)) rows_fwd_kernel(Planes a, float2* __restrict__ dst,
                                                                int N, const float2* __restrict__ tw,
                                                                int L) {
  extern __shared__ __align__(16) float2 sm[];
  const int TN = fft::plan_twiddle_len(N);
  LineRef* refs = reinterpret_cast<LineRef*>(sm);
  float2* stw = sm + kLineRefF2 * L;
  float2* s = stw + even_up(TN);
  const int LS = line_stride(N), lgN = fft::ilog2(N);
  const int total = a.units * a.rows;
  const int line0 = blockIdx.x * L;
  const int nl = min(L, total - line0);
  const int tid = threadIdx.x, nt = blockDim.x;
  prefetch_rows(a, blockIdx.x, L, tid);
  for (int i = tid; i < TN; i += nt) stw[i] = tw[i];
  line_refs(a, line0, nl, refs, tid, nt);
  __syncthreads();
  // the transform, compiled once with and once without the standardisation adjoint on the
  // loads (a.coef is the same for the whole launch)
  auto run = [&](auto with_coef) {
    constexpr bool kCoef = decltype(with_coef)::value;
    auto ld = [&](int l, int e) -> float2 {
      if (e >= a.cols) return make_float2(0.f, 0.f);
      const LineRef& R = refs[l];
      const float re = line_in<kCoef>(a, R, 0, e);
      const float im = R.o[1] >= 0 ? line_in<kCoef>(a, R, 1, e) : 0.f;
      return make_float2(re, im);
    };
    if (RA > 0 || (RA < 0 && fft::a_global(N))) {
      if constexpr (RA > 0) fft::fwd_a_global<RA, false>(s, nl, 0, LS, stw, tid, nt, ld);
      else fft::fwd_a_global_plan<false>(s, nl, 0, LS, N, stw, tid, nt, ld);
    } else {
#pragma unroll 4
      for (int idx = tid; idx < nl * N; idx += nt) {
        int l, e;
        line_elem<RA>(idx, N, lgN, l, e);
        s[l * LS + pidx(e)] = ld(l, e);
      }
      fft::transform_lines_plan<false>(s, nl, N, stw, tid, nt);
    }
  };
  if (a.coef) run(std::true_type{});
  else run(std::false_type{});
  // two elements per 16-byte store (lines of even N, 16-byte aligned)
#pragma unroll 4
  for (int idx = tid; idx < nl * (N >> 1); idx += nt) {
    int l, e;
    line_pair<RA>(idx, N, lgN, l, e);
    const float2 v0 = s[l * LS + pidx(e)], v1 = s[l * LS + pidx(e) + 1];
    __stcs(reinterpret_cast<float4*>(&dst[(size_t)(line0 + l) * N + e]), make_float4(v0.x, v0.y, v1.x, v1.y));   // read once
  }
}

// Inverse row transforms of src (lines, N) -> real planes (re -> sample 2g, im -> 2g+1).
// For N > 64 (RA = N/64) the radix-R stage writes the planes directly (fft::inv_a_global).
// Shared memory as rows_fwd_kernel.
template <int RA>
__global__ void __launch_bounds__(kFftThreads, fft_ctas(RA)) rows_inv_kernel(const float2* __restrict__ src,
                                                                Planes a, int N,
                                                                const float2* __restrict__ tw,
                                                                int L) {
  extern __shared__ __align__(16) float2 sm[];
  const int TN = fft::plan_twiddle_len(N);
  LineRef* refs = reinterpret_cast<LineRef*>(sm);
  float2* stw = sm + kLineRefF2 * L;
  float2* s = stw + even_up(TN);
  const int LS = line_stride(N), lgN = fft::ilog2(N);
  const int total = a.units * a.rows;
  const int line0 = blockIdx.x * L;
  const int nl = min(L, total - line0);
  const int tid = threadIdx.x, nt = blockDim.x;
  if (tid == 0) prefetch_l2(src + (size_t)line0 * N, sizeof(float2) * (size_t)nl * N);   // see prefetch_rows
  for (int i = tid; i < TN; i += nt) stw[i] = tw[i];
  line_refs(a, line0, nl, refs, tid, nt);
  // two elements per 16-byte load (lines of even N, 16-byte aligned)
#pragma unroll 4
  for (int idx = tid; idx < nl * (N >> 1); idx += nt) {
    int l, e;
    line_pair<RA>(idx, N, lgN, l, e);
    const float4 v = __ldcs(reinterpret_cast<const float4*>(&src[(size_t)(line0 + l) * N + e]));   // last use
    s[l * LS + pidx(e)] = make_float2(v.x, v.y);
    s[l * LS + pidx(e) + 1] = make_float2(v.z, v.w);
  }
  if (RA > 0 || (RA < 0 && fft::a_global(N))) {
    __syncthreads();
    const bool keep = a.rowstats != nullptr;   // the row statistics read the lines back
    auto st = [&](int l, int e, float2 v) {
      if (e < a.cols) {
        const long long o0 = refs[l].o[0], o1 = refs[l].o[1];
        a.ptr[o0 + e] = v.x * a.scale;
        if (o1 >= 0) a.ptr[o1 + e] = v.y * a.scale;
      }
      if (keep) s[l * LS + pidx(e)] = v;       // in place: the positions this thread read
    };
    if constexpr (RA > 0) fft::inv_a_global<RA, false>(s, nl, 0, LS, stw, tid, nt, st);
    else fft::inv_a_global_plan<false>(s, nl, 0, LS, N, stw, tid, nt, st);
    if (keep) __syncthreads();
  } else {
    fft::transform_lines_plan<true>(s, nl, N, stw, tid, nt);
#pragma unroll 4
    for (int idx = tid; idx < nl * a.cols; idx += nt) {
      const int l = idx / a.cols, e = idx - l * a.cols;
      const float2 v = s[l * LS + pidx(e)];
      const long long o0 = refs[l].o[0], o1 = refs[l].o[1];
      a.ptr[o0 + e] = v.x * a.scale;
      if (o1 >= 0) a.ptr[o1 + e] = v.y * a.scale;
    }
  }
  if (a.rowstats) {
    // centred statistics of each stored row, two passes over the row in shared memory (one
    // warp per row): the first stage of the plane statistics (plane_stats_rows_kernel)
    const int warp = tid >> 5, lane = tid & 31, nw = nt >> 5;
    const float inv_c = 1.0f / (float)a.cols;
    for (int l = warp; l < nl; l += nw) {
      const float2* sl = s + l * LS;
      float sx = 0.f, sy = 0.f;
      for (int e = lane; e < a.cols; e += 32) {
        const float2 v = sl[pidx(e)];
        sx += v.x * a.scale;
        sy += v.y * a.scale;
      }
      const float mx = warp_sum(sx) * inv_c, my = warp_sum(sy) * inv_c;
      float qx = 0.f, qy = 0.f;
      for (int e = lane; e < a.cols; e += 32) {
        const float2 v = sl[pidx(e)];
        const float dx = v.x * a.scale - mx, dy = v.y * a.scale - my;
        qx = fmaf(dx, dx, qx);
        qy = fmaf(dy, dy, qy);
      }
      qx = warp_sum(qx);
      qy = warp_sum(qy);
      if (lane == 0) {
        const int line = line0 + l;
        const int u = line / a.rows, r = line - u * a.rows;
        const int gs = u / a.ms, m = u - gs * a.ms;
        const int b1 = a.pack ? 2 * gs : gs;
        a.rowstats[((size_t)b1 * a.ms + m) * a.rows + r] = make_float2(mx, qx);
        if (a.pack && b1 + 1 < a.nsamp) a.rowstats[((size_t)(b1 + 1) * a.ms + m) * a.rows + r] = make_float2(my, qy);
      }
    }
  }
}

enum ColMode { COL_FWD = 0, COL_INV_MULCONJ = 1, COL_INV_SUM = 2, COL_INV_PLAIN = 3 };

struct ColArgs {
  const float2* src;    // FWD / PLAIN: (units, rows_in, Nw); MULCONJ: x^ (pairs, Nh, Nw);
                        // SUM: q^ (pairs, M, Nh, Nw)
  const float2* spec;   // (M, Nh, Nw) filter spectra (MULCONJ, SUM)
  float2* dst;          // FWD: (units, Nh, Nw); inverse modes: (units, rows_out, Nw)
  int Nh, Nw, rows_in, rows_out, M;
  float scale;          // FWD only
};

// Line stride of the column tiles (see fft::line_stride_cols).
__host__ __device__ inline int col_line_stride(int N) {
  return fft::a_global(N) ? fft::line_stride_cols(N) : line_stride(N);
}

// Column transforms of C adjacent columns per CTA (blockIdx.y = unit).  For N > 64
// (RA = N/64) the radix-R stage reads (forward) or writes (inverse) global memory directly.
template <int MODE, int RA>
__global__ void __launch_bounds__(cols_threads(MODE, RA), cols_big(MODE, RA) ? 1 : RA < 0 ? 2 : fft_ctas(RA, MODE == 2)) cols_kernel(ColArgs a, const float2* __restrict__ tw,
                                                            int C) {
  extern __shared__ __align__(16) float2 sm[];
  const int N = a.Nh;
  const int TN = fft::plan_twiddle_len(N);
  float2* stw = sm;
  float2* s = sm + even_up(TN);
  const int LS = col_line_stride(N), lgC = fft::ilog2(C);
  const int c0 = blockIdx.x * C;
  int u = blockIdx.y;
  if (MODE == COL_INV_MULCONJ) {
    // blockIdx.y runs over the pairs first, so the CTAs in flight share one filter spectrum
    // (the M spectra together exceed L2); the unit (and output) order stays p * M + m
    const int pairs = gridDim.y / a.M, m = u / pairs;
    u = (u - m * pairs) * a.M + m;
  }
  const int tid = threadIdx.x, nt = blockDim.x;
  const size_t NN = (size_t)a.Nh * a.Nw;
  for (int i = tid; i < TN; i += nt) stw[i] = tw[i];
  if (MODE == COL_FWD && (RA > 0 || (RA < 0 && fft::a_global(N)))) {
    __syncthreads();
    auto ld = [&](int l, int r) -> float2 {
      if (r >= a.rows_in) return make_float2(0.f, 0.f);
      float2 v = __ldcs(&a.src[((size_t)u * a.rows_in + r) * a.Nw + c0 + l]);   // last use
      v.x *= a.scale;
      v.y *= a.scale;
      return v;
    };
    if constexpr (RA > 0) fft::fwd_a_global<RA, true>(s, C, lgC, LS, stw, tid, nt, ld);
    else fft::fwd_a_global_plan<true>(s, C, lgC, LS, N, stw, tid, nt, ld);
  } else if ((MODE == COL_INV_MULCONJ || MODE == COL_INV_SUM) && C >= 2) {
    // two adjacent columns per thread: one 16-byte load per operand (Nw even, spectra
    // 16-byte aligned)
    const int lgH = lgC - 1;
#pragma unroll 4
    for (int idx = tid; idx < N * (C >> 1); idx += nt) {
      const int r = idx >> lgH, cc = (idx & ((C >> 1) - 1)) * 2;
      const size_t off = (size_t)r * a.Nw + c0 + cc;
      float4 v;
      if (MODE == COL_INV_MULCONJ) {
        const int p = u / a.M, m = u - p * a.M;
        const float4 x = *reinterpret_cast<const float4*>(a.src + (size_t)p * NN + off);
        const float4 h = *reinterpret_cast<const float4*>(a.spec + (size_t)m * NN + off);
        const float2 lo = cmulc(make_float2(x.x, x.y), make_float2(h.x, h.y));
        const float2 hi = cmulc(make_float2(x.z, x.w), make_float2(h.z, h.w));
        v = make_float4(lo.x, lo.y, hi.x, hi.y);
      } else {
        float2 lo = make_float2(0.f, 0.f), hi = make_float2(0.f, 0.f);
        const float2* q = a.src + (size_t)u * a.M * NN + off;
#pragma unroll 2
        for (int m = 0; m < a.M; ++m) {
          const float4 x = *reinterpret_cast<const float4*>(q + (size_t)m * NN);
          const float4 h = *reinterpret_cast<const float4*>(a.spec + (size_t)m * NN + off);
          lo = cadd(lo, cmul(make_float2(x.x, x.y), make_float2(h.x, h.y)));
          hi = cadd(hi, cmul(make_float2(x.z, x.w), make_float2(h.z, h.w)));
        }
        v = make_float4(lo.x, lo.y, hi.x, hi.y);
      }
      s[cc * LS + pidx(r)] = make_float2(v.x, v.y);
      s[(cc + 1) * LS + pidx(r)] = make_float2(v.z, v.w);
    }
    if (RA > 0 || (RA < 0 && fft::a_global(N))) {
      __syncthreads();
      auto st = [&](int l, int r, float2 v) {
        if (r < a.rows_out) __stcs(&a.dst[((size_t)u * a.rows_out + r) * a.Nw + c0 + l], v);   // read once
      };
      if constexpr (RA > 0) fft::inv_a_global<RA, true>(s, C, lgC, LS, stw, tid, nt, st);
      else fft::inv_a_global_plan<true>(s, C, lgC, LS, N, stw, tid, nt, st);
      return;
    } else {
      fft::transform_lines_plan<true>(s, C, N, stw, tid, nt);
    }
  } else {
#pragma unroll 4
    for (int idx = tid; idx < N * C; idx += nt) {
      const int r = idx >> lgC, cc = idx & (C - 1);
      const int c = c0 + cc;
      float2 v = make_float2(0.f, 0.f);
      if (MODE == COL_FWD || MODE == COL_INV_PLAIN) {
        if (r < a.rows_in) {
          v = __ldcs(&a.src[((size_t)u * a.rows_in + r) * a.Nw + c]);   // last use
          if (MODE == COL_FWD) { v.x *= a.scale; v.y *= a.scale; }
        }
      } else if (MODE == COL_INV_MULCONJ) {
        const int p = u / a.M, m = u - p * a.M;
        const size_t off = (size_t)r * a.Nw + c;
        v = cmulc(a.src[(size_t)p * NN + off], a.spec[(size_t)m * NN + off]);
      } else {
        const size_t off = (size_t)r * a.Nw + c;
        const float2* q = a.src + (size_t)u * a.M * NN + off;
        for (int m = 0; m < a.M; ++m) v = cadd(v, cmul(q[(size_t)m * NN], a.spec[(size_t)m * NN + off]));
      }
      s[cc * LS + pidx(r)] = v;
    }
    if (MODE != COL_FWD && (RA > 0 || (RA < 0 && fft::a_global(N)))) {
      __syncthreads();
      auto st = [&](int l, int r, float2 v) {
        if (r < a.rows_out) __stcs(&a.dst[((size_t)u * a.rows_out + r) * a.Nw + c0 + l], v);   // read once
      };
      if constexpr (RA > 0) fft::inv_a_global<RA, true>(s, C, lgC, LS, stw, tid, nt, st);
      else fft::inv_a_global_plan<true>(s, C, lgC, LS, N, stw, tid, nt, st);
      return;
    } else {
      fft::transform_lines_plan<MODE != COL_FWD>(s, C, N, stw, tid, nt);
    }
  }
  const int rows_st = (MODE == COL_FWD) ? N : a.rows_out;
#pragma unroll 4
  for (int idx = tid; idx < rows_st * C; idx += nt) {
    const int r = idx >> lgC, cc = idx & (C - 1);
    float2* o = &a.dst[((size_t)u * rows_st + r) * a.Nw + c0 + cc];
    if (MODE == COL_FWD) *o = s[cc * LS + pidx(r)];     // spectra: reused
    else __stcs(o, s[cc * LS + pidx(r)]);              // read once by the row pass
  }
}

// acc[m][f] (+)= sum over pairs of x^[p][f] * conj(q^[p][m][f])  (fixed pair order).  A
// thread takes two adjacent frequencies (16-byte accesses) of kDgM directions
// (blockIdx.y), so x^ is read once per kDgM directions and the kDgM q^ loads of a pair are
// independent.  NN is even (the planner's FFT sides are even: powers of two or multiples of
// 64) and the spectra are 16-byte aligned.
// dg_accum picks kDgM per grid size so that small grids still fill the GPU.
template <int kDgM>
__global__ void dg_accum_kernel(const float2* __restrict__ xhat, const float2* __restrict__ q,
                                float2* __restrict__ acc, int pairs, int M, size_t NN, int init) {
  const size_t h = (size_t)blockIdx.x * blockDim.x + threadIdx.x;   // frequencies 2h, 2h+1
  const size_t NN2 = NN / 2;
  if (h >= NN2) return;
  const int m0 = blockIdx.y * kDgM;
  const int mc = min(kDgM, M - m0);
  const float4* x4 = reinterpret_cast<const float4*>(xhat);
  const float4* q4 = reinterpret_cast<const float4*>(q);
  float4* a4 = reinterpret_cast<float4*>(acc);
  float4 s[kDgM];
#pragma unroll
  for (int j = 0; j < kDgM; ++j)
    s[j] = (j < mc && !init) ? a4[(size_t)(m0 + j) * NN2 + h] : make_float4(0.f, 0.f, 0.f, 0.f);
  for (int p = 0; p < pairs; ++p) {
    const float4 x = __ldg(&x4[(size_t)p * NN2 + h]);
    const float4* qp = q4 + ((size_t)p * M + m0) * NN2 + h;
#pragma unroll
    for (int j = 0; j < kDgM; ++j) {
      if (j < mc) {
        const float4 v = qp[(size_t)j * NN2];
        const float2 lo = cmulc(make_float2(x.x, x.y), make_float2(v.x, v.y));
        const float2 hi = cmulc(make_float2(x.z, x.w), make_float2(v.z, v.w));
        s[j].x += lo.x;
        s[j].y += lo.y;
        s[j].z += hi.x;
        s[j].w += hi.y;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kDgM; ++j)
    if (j < mc) a4[(size_t)(m0 + j) * NN2 + h] = s[j];
}

__device__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    float r = lane < nw ? red[lane] : 0.f;
    r = warp_sum(r);
    if (lane == 0) red[32] = r;
  }
  __syncthreads();
  return red[32];
}

// ---------------------------------------------------------------------------------------
// fields
// ---------------------------------------------------------------------------------------

// Step-0 inputs scattered into a zeroed field (propagator.py:103-191).
__global__ void field_inject_kernel(Geo g, float* __restrict__ field, const int32_t* __restrict__ in_index,
                                    const float* __restrict__ inputs, int B) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)B * g.n_in) return;
  const int b = (int)(i / g.n_in), j = (int)(i - (size_t)b * g.n_in);
  const int idx = in_index[j];
  if (idx < 0) return;
  const int r = idx / g.W, c = idx - (idx / g.W) * g.W;
  field[(size_t)b * g.Fh * g.Fw + (size_t)(r + g.gr) * g.Fw + c + g.gc] = inputs[i];
}

// Field ring for the next convolution: VALID -> border template, CIRCULAR -> wrapped
// interior (SAME keeps its zero halo and never calls this).
__global__ void field_ring_kernel(Geo g, float* __restrict__ field, const float* __restrict__ border, int B) {
  const int FF = g.Fh * g.Fw;
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (size_t)B * FF) return;
  const int b = (int)(i / FF), k = (int)(i - (size_t)b * FF);
  const int fr = k / g.Fw, fc = k - (k / g.Fw) * g.Fw;
  const int r = fr - g.oh, c = fc - g.ow;
  if (r >= 0 && r < g.roi_h && c >= 0 && c < g.roi_w) return;
  float* F = field + (size_t)b * FF;
  if (g.padding == NC_PAD_VALID) {
    F[k] = border[k];   // VALID: the field is the grid
  } else {
    int sr = r % g.roi_h; if (sr < 0) sr += g.roi_h;
    int sc = c % g.roi_w; if (sc < 0) sc += g.roi_w;
    F[k] = F[(sr + g.oh) * g.Fw + sc + g.ow];
  }
}

// ---------------------------------------------------------------------------------------
// forward epilogues (planes z at z + b*zs + m*P)
// ---------------------------------------------------------------------------------------

// Per-(b, m) mean and 1/sqrt(var + eps) from the rows' centred statistics (equal-sized
// rows: the plane mean is the mean of the row means, M2 = sum_r M2_r + n (mean_r - mean)^2),
// the two-stage variance the reference uses for tiled planes (kernels_pallas.py:740-837).
__global__ void __launch_bounds__(kEpiThreads) plane_stats_rows_kernel(Geo g, const float2* __restrict__ rowstats,
                                                                       float* mean, float* rstd,
                                                                       float* rstd_save, float* mean_save,
                                                                       int t) {
  __shared__ float red[33];
  const int bm = blockIdx.x, b = bm / g.M, m = bm - b * g.M;
  const int rows = g.roi_h;
  const float2* rs_ = rowstats + (size_t)bm * rows;
  float mu = 0.f, rs = 1.f;
  if (g.norm) {
    float s = 0.f;
    for (int r = threadIdx.x; r < rows; r += blockDim.x) s += rs_[r].x;
    mu = block_sum(s, red) / (float)rows;
    float q = 0.f;
    for (int r = threadIdx.x; r < rows; r += blockDim.x) {
      const float d = rs_[r].x - mu;
      q += rs_[r].y + (float)g.roi_w * d * d;
    }
    const float var = block_sum(q, red) / (float)g.P;
    rs = 1.0f / sqrtf(var + kNormEps);
  }
  if (threadIdx.x == 0) {
    mean[bm] = mu;
    rstd[bm] = rs;
    if (rstd_save) rstd_save[((size_t)b * g.d + t) * g.M + m] = rs;
    if (mean_save) mean_save[((size_t)b * g.d + t) * g.M + m] = mu;
  }
}

// V consecutive floats (V = 4: one 16-byte access; callers guarantee the alignment).
template <int V>
__device__ __forceinline__ void ldv(const float* __restrict__ p, float* v) {
  if constexpr (V == 4) {
    const float4 t = *reinterpret_cast<const float4*>(p);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) v[i] = p[i];
  }
}
template <int V>
__device__ __forceinline__ void stv(float* __restrict__ p, const float* v) {
  if constexpr (V == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) p[i] = v[i];
  }
}

// ROI epilogue (epilogue.py:28-56): standardise, gate, write the next field's interior and
// the training residual -- or, in universe mode (uroi != null), the last step's ROI cells.
// The planes z are only read: a training call keeps them raw and the backward standardises
// them again from the saved statistics.  One thread per V consecutive pixels of one sample
// (V = 4 when P % 4 == 0).  ACT >= 0 compiles the activation in (tanh, the hidden default);
// ACT = -1 reads it from act_rt.
template <int V, int ACT>
__global__ void hidden_epi_kernel(Geo g, StepParams sp, const float* __restrict__ z, size_t zs,
                                  const float* __restrict__ mean, const float* __restrict__ rstd,
                                  float* __restrict__ field, float* __restrict__ xsave, int t, int B,
                                  int act_rt, float slope, float* __restrict__ uroi) {
  const int act_id = ACT >= 0 ? ACT : act_rt;
  const size_t gidx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gidx * V >= (size_t)B * g.P) return;
  const size_t e0 = gidx * V;
  const int b = (int)(e0 / g.P), p0 = (int)(e0 - (size_t)b * g.P);
  float bb[V], lin[V], act[V];
  ldv<V>(sp.broi + p0, bb);
#pragma unroll
  for (int v = 0; v < V; ++v) { lin[v] = 0.f; act[v] = 0.f; }
  const float* zb = z + (size_t)b * zs + p0;
#pragma unroll 4
  for (int m = 0; m < g.M; ++m) {
    const float mu = mean[b * g.M + m], rs = rstd[b * g.M + m];
    float zv[V];
    ldv<V>(zb + (size_t)m * g.P, zv);
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const float zh = (zv[v] - mu) * rs;
      lin[v] += zh;
      if (act_id != NC_ACT_NONE) act[v] += act_fwd(act_id, zh + bb[v], slope);
    }
  }
  float we[V], se[V], xn[V];
  ldv<V>(sp.weff + p0, we);
  ldv<V>(sp.seff + p0, se);
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const float a = (act_id == NC_ACT_NONE) ? lin[v] + (float)g.M * bb[v] : act[v];
    xn[v] = we[v] * lin[v] + se[v] * a;
  }
  if (uroi) {
    stv<V>(uroi + e0, xn);
    return;
  }
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int p = p0 + v, r = p / g.roi_w, c = p - (p / g.roi_w) * g.roi_w;
    field[(size_t)b * g.Fh * g.Fw + (size_t)(r + g.oh) * g.Fw + c + g.ow] = xn[v];
  }
  if (xsave) stv<V>(xsave + ((size_t)b * (g.d - 1) + t) * g.P + p0, xn);
}

// Output-port epilogue (epilogue.py:82-128) from the raw planes and their statistics.
__global__ void port_out_kernel(Geo g, StepParams sp, const int32_t* __restrict__ out_index,
                                const float* __restrict__ z, size_t zs, const float* __restrict__ mean,
                                const float* __restrict__ rstd, float* __restrict__ out, int B) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * g.n_out) return;
  const int b = i / g.n_out, j = i - b * g.n_out;
  const int idx = out_index[j];
  const int gr_ = idx / g.W, gc_ = idx - (idx / g.W) * g.W;
  const int p = (gr_ - g.pad_h) * g.roi_w + (gc_ - g.pad_w);
  if (gr_ < g.pad_h || gr_ >= g.pad_h + g.roi_h || gc_ < g.pad_w || gc_ >= g.pad_w + g.roi_w) {
    out[i] = __int_as_float(0x7fc00000);   // border outputs run in universe mode only
    return;
  }
  const float wo = sp.weff[p], so = sp.seff[p], bo = sp.broi[p];
  const float* zb = z + (size_t)b * zs + p;
  float lin = 0.f, act = 0.f;
  for (int m = 0; m < g.M; ++m) {
    const float zh = (zb[(size_t)m * g.P] - mean[b * g.M + m]) * rstd[b * g.M + m];
    lin += zh;
    if (g.fact != NC_ACT_NONE) act += act_fwd(g.fact, zh + bo, g.fslope);
  }
  out[i] = (g.fact == NC_ACT_NONE) ? (wo + so) * lin + ((float)g.M * so * bo)
                                   : act_fwd(g.fact, wo * lin + so * act, g.fslope);
}

// ---------------------------------------------------------------------------------------
// backward epilogues
// ---------------------------------------------------------------------------------------

// Plane pixel of output port j, or -1 for a border output (universe mode only).
__device__ __forceinline__ int port_pixel(const Geo& g, const int32_t* __restrict__ out_index, int j) {
  const int idx = out_index[j];
  const int gr_ = idx / g.W, gc_ = idx - (idx / g.W) * g.W;
  if (gr_ < g.pad_h || gr_ >= g.pad_h + g.roi_h || gc_ < g.pad_w || gc_ >= g.pad_w + g.roi_w) return -1;
  return (gr_ - g.pad_h) * g.roi_w + (gc_ - g.pad_w);
}

// Output-step adjoint at the port cells (kernels_pallas.py:1378-1504): sparse plane
// gradients (gz must be zero elsewhere) and the port cells' parameter gradients summed
// over the batch.  One warp per port, lanes over the samples, then a fixed-order warp sum.
// z_t: the raw planes of step t, standardised here with the saved statistics.
__global__ void port_gz_kernel(Geo g, StepParams sp, const int32_t* __restrict__ out_index,
                               const float* __restrict__ gout, const float* __restrict__ z_t,
                               size_t zs, const float* __restrict__ mean_save,
                               const float* __restrict__ rstd_save, int t, float* __restrict__ gz,
                               float* __restrict__ gsum, int B) {
  const int j = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (j >= g.n_out) return;                  // whole warps leave together
  const int p = port_pixel(g, out_index, j);
  if (p < 0) return;
  const size_t P = (size_t)g.P;
  const float wo = sp.weff[p], so = sp.seff[p], bo = sp.broi[p];
  float gp0 = 0.f, gp1 = 0.f, gp2 = 0.f;
  for (int b = lane; b < B; b += 32) {
    const float go = gout[(size_t)b * g.n_out + j];
    const float* Z = z_t + (size_t)b * zs + p;
    const float* mu = mean_save + ((size_t)b * g.d + t) * g.M;
    const float* rs = rstd_save + ((size_t)b * g.d + t) * g.M;
    auto zh = [&](int m) { return (Z[m * P] - mu[m]) * rs[m]; };
    float* GZ = gz + (size_t)b * g.M * P + p;
    float lin = 0.f;
    for (int m = 0; m < g.M; ++m) lin += zh(m);
    if (g.fact == NC_ACT_NONE) {
      gp0 += go * lin;
      gp1 += go * (lin + (float)g.M * bo);
      gp2 += go * (float)g.M * so;
      const float gzh = (wo + so) * go;
      for (int m = 0; m < g.M; ++m) GZ[m * P] = gzh;
    } else {
      float act = 0.f;
      for (int m = 0; m < g.M; ++m) act += act_fwd(g.fact, zh(m) + bo, g.fslope);
      float dpre;
      act_fwd_deriv(g.fact, wo * lin + so * act, g.fslope, &dpre);
      const float gpre = go * dpre;
      gp0 += gpre * lin;
      gp1 += gpre * act;
      float db = 0.f;
      for (int m = 0; m < g.M; ++m) {
        float dd;
        act_fwd_deriv(g.fact, zh(m) + bo, g.fslope, &dd);
        GZ[m * P] = gpre * (wo + so * dd);
        db += gpre * so * dd;
      }
      gp2 += db;
    }
  }
  gp0 = warp_sum(gp0);
  gp1 = warp_sum(gp1);
  gp2 = warp_sum(gp2);
  if (lane == 0) {
    gsum[p] += gp0;
    gsum[P + p] += gp1;
    gsum[2 * P + p] += gp2;
  }
}

// Coefficients of the standardisation adjoint of the output step (see norm_coef_kernel)
// from the port cells alone: the plane gradients are zero elsewhere.  One warp per (b, m)
// plane; each port cell counts once (a cell listed twice holds one gradient), lanes over
// the ports, then a fixed-order warp sum.
__global__ void port_coef_kernel(Geo g, const int32_t* __restrict__ out_index, const float* __restrict__ gz,
                                 const float* __restrict__ z_t, size_t zs,
                                 const float* __restrict__ mean_save, const float* __restrict__ rstd_save,
                                 int t, int nplanes, float4* __restrict__ coef) {
  const int bm = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (bm >= nplanes) return;                 // whole warps leave together
  const int b = bm / g.M, m = bm - b * g.M;
  const size_t st = ((size_t)b * g.d + t) * g.M + m;
  const float mu = mean_save[st], rs = rstd_save[st];
  const float* GZ = gz + (size_t)bm * g.P;
  const float* Z = z_t + (size_t)b * zs + (size_t)m * g.P;
  float s1 = 0.f, s2 = 0.f;
  for (int j = lane; j < g.n_out; j += 32) {
    const int p = port_pixel(g, out_index, j);
    if (p < 0) continue;
    bool first = true;
    for (int i = 0; i < j && first; ++i) first = out_index[i] != out_index[j];
    if (!first) continue;
    const float v = GZ[p];
    s1 += v;
    s2 = fmaf(v, (Z[p] - mu) * rs, s2);
  }
  s1 = warp_sum(s1);
  s2 = warp_sum(s2);
  if (lane == 0) {
    const float inv_n = 1.0f / (float)g.P;
    const float c1 = s1 * inv_n, c2 = s2 * inv_n;
    coef[bm] = make_float4(rs, c1 - mu * rs * c2, rs * c2, 0.f);
  }
}

// Standardisation adjoint per (b, m): gz <- rstd (gz - mean(gz) - zh mean(gz zh)), zh the
// raw planes z_t of step t standardised with the saved statistics.  gzpart (not null): the
// sums come from hidden_gz_kernel's per-CTA partials (ncta of them, added in CTA order) and
// the planes are read once.
__global__ void __launch_bounds__(kStatThreads) norm_bwd_kernel(Geo g, float* __restrict__ gz,
                                                                 const float* __restrict__ z_t, size_t zs,
                                                                 const float* __restrict__ mean_save,
                                                                 const float* __restrict__ rstd_save, int t,
                                                                 int nplanes, int vec,
                                                                 const float* __restrict__ gzpart, int ncta) {
  __shared__ float red[33];
  const float inv_n = 1.0f / (float)g.P;
  for (int bm = blockIdx.x; bm < nplanes; bm += gridDim.x) {
    const int b = bm / g.M, m = bm - b * g.M;
    float* gp = gz + (size_t)bm * g.P;
    const float* zp = z_t + (size_t)b * zs + (size_t)m * g.P;
    const float mu = mean_save[((size_t)b * g.d + t) * g.M + m];
    const float rs = rstd_save[((size_t)b * g.d + t) * g.M + m];
    auto zh = [&](float z) { return (z - mu) * rs; };
    float s1 = 0.f, s2 = 0.f, u1 = 0.f, u2 = 0.f;
    if (gzpart) {
      for (int k = threadIdx.x; k < ncta; k += blockDim.x) {
        s1 += gzpart[((size_t)k * nplanes + bm) * 2 + 0];
        s2 += gzpart[((size_t)k * nplanes + bm) * 2 + 1];
      }
    } else if (vec) {
      const float4* g4 = reinterpret_cast<const float4*>(gp);
      const float4* z4 = reinterpret_cast<const float4*>(zp);
      for (int i = threadIdx.x; i < g.P / 4; i += blockDim.x) {
        const float4 v = g4[i], w = z4[i];
        s1 += v.x + v.y;
        u1 += v.z + v.w;
        s2 = fmaf(v.x, zh(w.x), fmaf(v.y, zh(w.y), s2));
        u2 = fmaf(v.z, zh(w.z), fmaf(v.w, zh(w.w), u2));
      }
    } else {
      for (int p = threadIdx.x; p < g.P; p += blockDim.x) {
        const float v = gp[p];
        s1 += v;
        s2 = fmaf(v, zh(zp[p]), s2);
      }
    }
    const float c1 = block_sum(s1 + u1, red) * inv_n;
    const float c2 = block_sum(s2 + u2, red) * inv_n;
    if (vec) {
      float4* g4 = reinterpret_cast<float4*>(gp);
      const float4* z4 = reinterpret_cast<const float4*>(zp);
      for (int i = threadIdx.x; i < g.P / 4; i += blockDim.x) {
        float4 v = g4[i];
        const float4 w = z4[i];
        v.x = rs * (v.x - c1 - zh(w.x) * c2);
        v.y = rs * (v.y - c1 - zh(w.y) * c2);
        v.z = rs * (v.z - c1 - zh(w.z) * c2);
        v.w = rs * (v.w - c1 - zh(w.w) * c2);
        g4[i] = v;
      }
    } else {
      for (int p = threadIdx.x; p < g.P; p += blockDim.x) gp[p] = rs * (gp[p] - c1 - zh(zp[p]) * c2);
    }
  }
}

// Coefficients of the standardisation adjoint gz <- rstd (gz - mean(gz) - zhat mean(gz zhat))
// from hidden_gz_kernel's per-CTA sums (ncta of them, one warp per plane, lanes over the
// CTAs in a fixed order); the next row pass applies them while it reads the planes.  With
// zhat = (z - mu) rstd of the raw planes z the row pass reads, the adjoint is
// k.x (gz - k.y - z k.z) with k = (rstd, c1 - mu rstd c2, rstd c2), c1 = mean(gz),
// c2 = mean(gz zhat).
__global__ void norm_coef_kernel(Geo g, const float* __restrict__ gzpart, int ncta,
                                 const float* __restrict__ mean_save, const float* __restrict__ rstd_save,
                                 int t, int nplanes, float4* __restrict__ coef) {
  const int bm = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (bm >= nplanes) return;                 // whole warps leave together
  float s1 = 0.f, s2 = 0.f;
  for (int k = lane; k < ncta; k += 32) {
    s1 += gzpart[((size_t)k * nplanes + bm) * 2 + 0];
    s2 += gzpart[((size_t)k * nplanes + bm) * 2 + 1];
  }
  s1 = warp_sum(s1);
  s2 = warp_sum(s2);
  if (lane == 0) {
    const float inv_n = 1.0f / (float)g.P;
    const int b = bm / g.M, m = bm - b * g.M;
    const size_t st = ((size_t)b * g.d + t) * g.M + m;
    const float mu = mean_save[st], rs = rstd_save[st];
    const float c1 = s1 * inv_n, c2 = s2 * inv_n;
    coef[bm] = make_float4(rs, c1 - mu * rs * c2, rs * c2, 0.f);
  }
}

// Field adjoint at interior cell (r, c); CIRCULAR folds the wrapped halo copies back.
__device__ __forceinline__ float field_grad(const Geo& g, const float* dxb, int r, int c) {
  if (g.padding != NC_PAD_CIRCULAR) return dxb[(size_t)(r + g.oh) * g.Fw + c + g.ow];
  float s = 0.f;
  for (int fr = (r + g.oh) % g.roi_h; fr < g.Fh; fr += g.roi_h)
    for (int fc = (c + g.ow) % g.roi_w; fc < g.Fw; fc += g.roi_w) s += dxb[(size_t)fr * g.Fw + fc];
  return s;
}

// ROI-epilogue adjoint (kernels_pallas.py:221-291) for the samples of chunk blockIdx.y:
// the cell gradient comes from the field adjoint dx (hidden step t-1) or, in universe mode,
// from gy_roi (B, P) with the final activation; per-chunk pixel-gradient partials go to gpart.
// Warp sums of four values in six shuffles: the first two butterfly levels split the values
// over the half- and quarter-warps, the last three finish one value per 8-lane group.
// Afterwards lanes 0, 8, 16 and 24 hold the sums of a, b, c and d.
__device__ __forceinline__ float warp_sum4(float a, float b, float c, float d, int lane) {
  const bool h16 = (lane & 16) != 0, h8 = (lane & 8) != 0;
  float x0 = h16 ? c : a, x1 = h16 ? d : b;
  const float y0 = h16 ? a : c, y1 = h16 ? b : d;
  x0 += __shfl_xor_sync(0xffffffffu, y0, 16);
  x1 += __shfl_xor_sync(0xffffffffu, y1, 16);
  float z = h8 ? x1 : x0;
  z += __shfl_xor_sync(0xffffffffu, h8 ? x0 : x1, 8);
  z += __shfl_xor_sync(0xffffffffu, z, 4);
  z += __shfl_xor_sync(0xffffffffu, z, 2);
  z += __shfl_xor_sync(0xffffffffu, z, 1);
  return z;
}

// z_t: the raw planes of step t, standardised here with the saved statistics.
// gzpart (not null): the CTA's sums of gz and gz * zhat over its pixels per (b, m) of its
// chunk, at gzpart[((blockIdx.x * B + b) * M + m) * 2 + {0, 1}] (warp_sum4 over directions
// m, m+1, then the warps in order), so the standardisation adjoint needs one pass.  `red`
// in dynamic shared memory holds bc * M * 2 values per warp.  ACT as hidden_epi_kernel.
template <int V, int ACT>
__global__ void __launch_bounds__(256, ACT >= 0 ? 3 : 4) hidden_gz_kernel(Geo g, StepParams sp, const float* __restrict__ dx,
                                 const float* __restrict__ z_t, size_t zs,
                                 const float* __restrict__ mean_save, const float* __restrict__ rstd_save,
                                 int t, float* __restrict__ gz,
                                 float* __restrict__ gpart, int B, int bc, int act_rt, float slope,
                                 const float* __restrict__ gy_roi, float* __restrict__ gzpart) {
  extern __shared__ float red[];
  const int act_id = ACT >= 0 ? ACT : act_rt;
  const int gi = blockIdx.x * blockDim.x + threadIdx.x;
  const bool on = gi * V < g.P;       // threads past the plane join the warp sums with zeros
  const int p0 = on ? gi * V : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int k = blockIdx.y;
  const int b0 = k * bc, b1 = min(B, b0 + bc);
  const size_t P = (size_t)g.P, FF = (size_t)g.Fh * g.Fw;
  float bb[V], we[V], se[V], gp0[V], gp1[V], gp2[V];
  ldv<V>(sp.broi + p0, bb);
  ldv<V>(sp.weff + p0, we);
  ldv<V>(sp.seff + p0, se);
#pragma unroll
  for (int v = 0; v < V; ++v) { gp0[v] = 0.f; gp1[v] = 0.f; gp2[v] = 0.f; }
  for (int b = b0; b < b1; ++b) {
    float gy[V], lin[V], act[V], dsum[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int p = p0 + v, r = p / g.roi_w, c = p - (p / g.roi_w) * g.roi_w;
      gy[v] = !on ? 0.f : gy_roi ? gy_roi[(size_t)b * P + p] : field_grad(g, dx + (size_t)b * FF, r, c);
      lin[v] = 0.f; act[v] = 0.f; dsum[v] = 0.f;
    }
    const float* Z = z_t + (size_t)b * zs + p0;
    const float* mu = mean_save + ((size_t)b * g.d + t) * g.M;
    const float* rs = rstd_save + ((size_t)b * g.d + t) * g.M;
    float* GZ = gz + (size_t)b * g.M * P + p0;
    for (int m = 0; m < g.M; m += 2) {          // directions m, m+1 (m+1 < M or empty)
      float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        if (m + k >= g.M) break;
        float zv[V], gv[V];
        if (on) {
          ldv<V>(Z + (size_t)(m + k) * P, zv);
          const float mk = mu[m + k], rk = rs[m + k];
#pragma unroll
          for (int v = 0; v < V; ++v) zv[v] = (zv[v] - mk) * rk;
        } else {
#pragma unroll
          for (int v = 0; v < V; ++v) zv[v] = 0.f;
        }
#pragma unroll
        for (int v = 0; v < V; ++v) {
          float dd;
          const float av = act_fwd_deriv(act_id, zv[v] + bb[v], slope, &dd);
          lin[v] += zv[v];
          act[v] += av;
          dsum[v] += dd;
          gv[v] = on ? we[v] * gy[v] + se[v] * gy[v] * dd : 0.f;
          s[2 * k] += gv[v];
          s[2 * k + 1] = fmaf(gv[v], zv[v], s[2 * k + 1]);
        }
        if (on) stv<V>(GZ + (size_t)(m + k) * P, gv);
      }
      if (gzpart) {
        const float r = warp_sum4(s[0], s[1], s[2], s[3], lane);
        const int e = lane >> 3;                  // 0: s1(m), 1: s2(m), 2: s1(m+1), 3: s2(m+1)
        if ((lane & 7) == 0 && m + (e >> 1) < g.M)
          red[((size_t)((b - b0) * g.M + m + (e >> 1)) * nw + warp) * 2 + (e & 1)] = r;
      }
    }
#pragma unroll
    for (int v = 0; v < V; ++v) {
      gp0[v] += gy[v] * lin[v];
      gp1[v] += gy[v] * act[v];
      gp2[v] += se[v] * gy[v] * dsum[v];
    }
  }
  if (on) {
    stv<V>(gpart + ((size_t)k * 3 + 0) * P + p0, gp0);
    stv<V>(gpart + ((size_t)k * 3 + 1) * P + p0, gp1);
    stv<V>(gpart + ((size_t)k * 3 + 2) * P + p0, gp2);
  }
  if (gzpart) {
    __syncthreads();
    const int nv = (b1 - b0) * g.M * 2;
    for (int i = threadIdx.x; i < nv; i += blockDim.x) {
      const int bm = i >> 1, e = i & 1;      // bm = (b - b0) * M + m
      float s = 0.f;
      for (int w = 0; w < nw; ++w) s += red[((size_t)bm * nw + w) * 2 + e];
      gzpart[(((size_t)blockIdx.x * B + b0) * g.M + bm) * 2 + e] = s;
    }
  }
}

// gsum += sum over chunks of gpart (chunk order).
__global__ void gsum_chunks_kernel(const float* __restrict__ gpart, float* __restrict__ gsum, int P,
                                   int nch) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 3 * P) return;
  const int k3 = i / P, p = i - k3 * P;
  float s = 0.f;
  for (int k = 0; k < nch; ++k) s += gpart[((size_t)k * 3 + k3) * P + p];
  gsum[i] += s;
}

// VALID border-template gradient: the ring of the field adjoint summed over the batch.
__global__ void ring_grad_kernel(Geo g, const float* __restrict__ dx, float* __restrict__ gborder, int B) {
  const int FF = g.Fh * g.Fw;
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= FF) return;
  const int fr = k / g.Fw, fc = k - (k / g.Fw) * g.Fw;
  const int r = fr - g.oh, c = fc - g.ow;
  if (r >= 0 && r < g.roi_h && c >= 0 && c < g.roi_w) return;
  float s = 0.f;
  for (int b = 0; b < B; ++b) s += dx[(size_t)b * FF + k];
  gborder[k] += s;   // the VALID field is the grid
}

// ---------------------------------------------------------------------------------------
// host helpers
// ---------------------------------------------------------------------------------------

nc_status launched(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, what);
  note_launch();
  return NC_OK;
}

int rows_per_cta(int N) {
  int L = 40960 / (9 * N);
  if (L < 1) L = 1;
  if (L > 64) L = 64;
  return L;
}

size_t rows_smem(int N, int L) {
  const int TN = fft::plan_twiddle_len(N);
  return sizeof(float2) * ((size_t)kLineRefF2 * L + (size_t)((TN + 1) & ~1) + (size_t)L * line_stride(N));
}

// Columns per CTA: 8 from 512-point columns on (37 KB of lines at N = 512, six CTAs per
// SM; measured faster than 16 at N = 512 and than 4 at N = 1024), 16 below, 16 for the
// 1024-thread CTAs (cols_threads).
int cols_per_cta(int Nh, int Nw, bool big) {
  int C = (big || Nh < 512) ? 16 : 8;
  return C < Nw ? C : Nw;
}

size_t cols_smem(int Nh, int C) {
  const int TN = fft::plan_twiddle_len(Nh);
  return sizeof(float2) * ((size_t)((TN + 1) & ~1) + (size_t)C * col_line_stride(Nh));
}

nc_status smem_attr(const void* fn, size_t bytes) {
  if (bytes > 48 * 1024)
    NC_CUDA_CHECK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  return NC_OK;
}

// RA of the transform kernels for N-point lines (see fft_ctas): a specialisation for
// N = 128 ... 512, the run-time variant for 1024.
int kernel_ra(int N) {
  if (!fft::a_global(N)) return 0;
  const int R = N >> 6;
  return (R == 2 || R == 3 || R == 4 || R == 5 || R == 6 || R == 8) ? R : -1;
}

template <int RA>
nc_status rows_fwd_ra(const Planes& a, float2* dst, int N, const float2* tw, cudaStream_t st) {
  const int L = rows_per_cta(N);
  const size_t smem = rows_smem(N, L);
  NC_CHECK(smem_attr((const void*)rows_fwd_kernel<RA>, smem));
  const int lines = a.units * a.rows;
  rows_fwd_kernel<RA><<<(lines + L - 1) / L, kFftThreads, smem, st>>>(a, dst, N, tw, L);
  return launched("rows_fwd_kernel launch");
}

template <int RA>
nc_status rows_inv_ra(const float2* src, const Planes& a, int N, const float2* tw, cudaStream_t st) {
  const int L = rows_per_cta(N);
  const size_t smem = rows_smem(N, L);
  NC_CHECK(smem_attr((const void*)rows_inv_kernel<RA>, smem));
  const int lines = a.units * a.rows;
  rows_inv_kernel<RA><<<(lines + L - 1) / L, kFftThreads, smem, st>>>(src, a, N, tw, L);
  return launched("rows_inv_kernel launch");
}

nc_status rows_fwd(const Planes& a, float2* dst, int N, const float2* tw, cudaStream_t st) {
  switch (kernel_ra(N)) {
    case 2: return rows_fwd_ra<2>(a, dst, N, tw, st);
    case 3: return rows_fwd_ra<3>(a, dst, N, tw, st);
    case 4: return rows_fwd_ra<4>(a, dst, N, tw, st);
    case 5: return rows_fwd_ra<5>(a, dst, N, tw, st);
    case 6: return rows_fwd_ra<6>(a, dst, N, tw, st);
    case 8: return rows_fwd_ra<8>(a, dst, N, tw, st);
    case -1: return rows_fwd_ra<-1>(a, dst, N, tw, st);
    default: return rows_fwd_ra<0>(a, dst, N, tw, st);
  }
}

nc_status rows_inv(const float2* src, const Planes& a, int N, const float2* tw, cudaStream_t st) {
  switch (kernel_ra(N)) {
    case 2: return rows_inv_ra<2>(src, a, N, tw, st);
    case 3: return rows_inv_ra<3>(src, a, N, tw, st);
    case 4: return rows_inv_ra<4>(src, a, N, tw, st);
    case 5: return rows_inv_ra<5>(src, a, N, tw, st);
    case 6: return rows_inv_ra<6>(src, a, N, tw, st);
    case 8: return rows_inv_ra<8>(src, a, N, tw, st);
    case -1: return rows_inv_ra<-1>(src, a, N, tw, st);
    default: return rows_inv_ra<0>(src, a, N, tw, st);
  }
}

template <int MODE, int RA>
nc_status cols_ra(const ColArgs& a, int units, const float2* tw, cudaStream_t st) {
  const int C = cols_per_cta(a.Nh, a.Nw, cols_big(MODE, RA));
  const size_t smem = cols_smem(a.Nh, C);
  NC_CHECK(smem_attr((const void*)cols_kernel<MODE, RA>, smem));
  cols_kernel<MODE, RA><<<dim3(a.Nw / C, units), cols_threads(MODE, RA), smem, st>>>(a, tw, C);
  return launched("cols_kernel launch");
}

template <int MODE>
nc_status cols(const ColArgs& a, int units, const float2* tw, cudaStream_t st) {
  switch (kernel_ra(a.Nh)) {
    case 2: return cols_ra<MODE, 2>(a, units, tw, st);
    case 3: return cols_ra<MODE, 3>(a, units, tw, st);
    case 4: return cols_ra<MODE, 4>(a, units, tw, st);
    case 5: return cols_ra<MODE, 5>(a, units, tw, st);
    case 6: return cols_ra<MODE, 6>(a, units, tw, st);
    case 8: return cols_ra<MODE, 8>(a, units, tw, st);
    case -1: return cols_ra<MODE, -1>(a, units, tw, st);
    default: return cols_ra<MODE, 0>(a, units, tw, st);
  }
}

inline unsigned blocks_for(size_t n, int threads) { return (unsigned)((n + threads - 1) / threads); }

// SMs of the current device (148 on B200 if the query fails).
int sm_count() {
  static int sms = 0;
  if (sms == 0) {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0)
      sms = n;
    else
      sms = 148;
  }
  return sms;
}

// Grid of the per-plane statistics kernels: two CTAs per SM looping over the planes.
unsigned stat_grid(int nplanes) {
  const int n = 2 * sm_count();
  return (unsigned)(nplanes < n ? nplanes : n);
}

// float4 plane access: P and the sample stride multiples of 4 (the buffers are 256-byte aligned).
int plane_vec(const Geo& g, size_t zs) { return (g.P % 4 == 0 && zs % 4 == 0) ? 1 : 0; }

// ROI epilogue over all samples (train: xsave; universe mode: uroi); 4 pixels per thread
// when the planes allow 16-byte accesses.
nc_status hidden_epi(const Geo& g, const FftCall& c, const float* z, size_t zs, int t, int act_id, float slope,
                     float* uroi, cudaStream_t st) {
  const size_t n = (size_t)c.batch * g.P;
  float* xs = (c.train && !uroi) ? c.xsave : nullptr;
  auto run = [&](auto kernel, int V) {
    kernel<<<blocks_for(n / V, kEpiThreads), kEpiThreads, 0, st>>>(g, c.sp, z, zs, c.mean, c.rstd, c.field, xs,
                                                                   t, c.batch, act_id, slope, uroi);
  };
  const bool tanh_act = act_id == NC_ACT_TANH;
  if (plane_vec(g, zs))
    run(tanh_act ? hidden_epi_kernel<4, NC_ACT_TANH> : hidden_epi_kernel<4, -1>, 4);
  else
    run(tanh_act ? hidden_epi_kernel<1, NC_ACT_TANH> : hidden_epi_kernel<1, -1>, 1);
  return launched("hidden_epi_kernel launch");
}

// ROI-epilogue adjoint (see hidden_gz_kernel); 4 pixels per thread when possible.
// *ncta: the number of per-CTA sum partials written to c.gzpart for the standardisation
// adjoint, or 0 when they did not fit the kernel's shared memory (norm_bwd then takes two
// passes).
nc_status hidden_gz(const Geo& g, const FftCall& c, const float* z, size_t zs, int tz, int nch, int bc,
                    int act_id, float slope, const float* gy_roi, int* ncta, cudaStream_t st) {
  const size_t red = sizeof(float) * (size_t)bc * g.M * (256 / 32) * 2;
  const bool part = c.gzpart != nullptr && red <= 48 * 1024;
  float* gzp = part ? c.gzpart : nullptr;
  const size_t smem = part ? red : 0;
  const int V = plane_vec(g, zs) ? 4 : 1;
  const unsigned grid = blocks_for((size_t)g.P / V, 256);
  auto run = [&](auto kernel) {
    kernel<<<dim3(grid, nch), 256, smem, st>>>(g, c.sp, c.dx, z, zs, c.mean_save, c.rstd_save, tz, c.gz,
                                               c.gpart, c.batch, bc, act_id, slope, gy_roi, gzp);
  };
  const bool tanh_act = act_id == NC_ACT_TANH;
  if (V == 4)
    run(tanh_act ? hidden_gz_kernel<4, NC_ACT_TANH> : hidden_gz_kernel<4, -1>);
  else
    run(tanh_act ? hidden_gz_kernel<1, NC_ACT_TANH> : hidden_gz_kernel<1, -1>);
  *ncta = part ? (int)grid : 0;
  return launched("hidden_gz_kernel launch");
}

// Filter-gradient spectrum accumulation (dg_accum_kernel) against the field spectra xh: the
// largest direction block (8, 4, 2, 1) that still launches two CTAs per SM.
nc_status dg_accum(const FftCall& c, const float2* xh, int pairs, size_t NN, int init, cudaStream_t st) {
  const int M = c.g.M;
  const unsigned bx = blocks_for(NN / 2, 256);
  const unsigned want = 2 * (unsigned)sm_count();
  int mb = 8;
  while (mb > 1 && bx * (unsigned)((M + mb - 1) / mb) < want) mb >>= 1;
  const dim3 grid(bx, (M + mb - 1) / mb);
  switch (mb) {
    case 8: dg_accum_kernel<8><<<grid, 256, 0, st>>>(xh, c.q, c.dgacc, pairs, M, NN, init); break;
    case 4: dg_accum_kernel<4><<<grid, 256, 0, st>>>(xh, c.q, c.dgacc, pairs, M, NN, init); break;
    case 2: dg_accum_kernel<2><<<grid, 256, 0, st>>>(xh, c.q, c.dgacc, pairs, M, NN, init); break;
    default: dg_accum_kernel<1><<<grid, 256, 0, st>>>(xh, c.q, c.dgacc, pairs, M, NN, init); break;
  }
  return launched("dg_accum_kernel launch");
}

// x^ (pairs) of the field currently in c.field, into xh.
nc_status field_spectra(const FftCall& c, float2* xh, cudaStream_t st) {
  const Geo& g = c.g;
  const int pairs = (c.batch + 1) / 2;
  Planes f{c.field, (size_t)g.Fh * g.Fw, c.batch, 1, g.Fh, g.Fw, 0, g.Fw, 1, pairs, 1.0f};
  NC_CHECK(rows_fwd(f, c.tmp, g.Nw, c.tw_w, st));
  ColArgs ca{c.tmp, nullptr, xh, g.Nh, g.Nw, g.Fh, g.Nh, g.M, 1.0f};
  return cols<COL_FWD>(ca, pairs, c.tw_h, st);
}

// Field of step 0: zeros + injected inputs (+ wrapped halo).
nc_status build_field0(const FftCall& c, cudaStream_t st) {
  const Geo& g = c.g;
  const size_t FF = (size_t)g.Fh * g.Fw;
  NC_CUDA_CHECK(cudaMemsetAsync(c.field, 0, sizeof(float) * FF * c.batch, st));
  if (g.n_in > 0) {
    field_inject_kernel<<<blocks_for((size_t)c.batch * g.n_in, 256), 256, 0, st>>>(g, c.field, c.in_index,
                                                                                c.inputs, c.batch);
    NC_CHECK(launched("field_inject_kernel launch"));
  }
  if (g.padding == NC_PAD_CIRCULAR) {
    field_ring_kernel<<<blocks_for(FF * c.batch, 256), 256, 0, st>>>(g, c.field, c.sp.border, c.batch);
    NC_CHECK(launched("field_ring_kernel launch"));
  }
  return NC_OK;
}

nc_status field_ring(const FftCall& c, cudaStream_t st) {
  const Geo& g = c.g;
  if (g.padding == NC_PAD_SAME) return NC_OK;
  const size_t FF = (size_t)g.Fh * g.Fw;
  field_ring_kernel<<<blocks_for(FF * c.batch, 256), 256, 0, st>>>(g, c.field, c.sp.border, c.batch);
  return launched("field_ring_kernel launch");
}

}  // namespace

// ---------------------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------------------

// Filter spectra G^_m / (Nh Nw), one per direction (the reference hoists them once per
// batch, kernels_greens.py:240-259).
nc_status fft_filter_spectra(const FftCall& c, cudaStream_t st) {
  const Geo& g = c.g;
  Planes gf{c.sp.geff, (size_t)g.K, g.M, 1, g.kh, g.kw, 0, g.kw, 0, g.M, 1.0f};
  NC_CHECK(rows_fwd(gf, c.tmp, g.Nw, c.tw_w, st));
  ColArgs ca{c.tmp, nullptr, c.gspec, g.Nh, g.Nw, g.kh, g.Nh, g.M, 1.0f / ((float)g.Nh * (float)g.Nw)};
  return cols<COL_FWD>(ca, g.M, c.tw_h, st);
}

nc_status fft_forward(const FftCall& c, cudaStream_t st) {
  const Geo& g = c.g;
  const int B = c.batch, pairs = (B + 1) / 2;
  const size_t P = (size_t)g.P, M = (size_t)g.M;
  NC_CHECK(fft_filter_spectra(c, st));

  for (int t = 0; t < g.d; ++t) {
    if (t == 0) {
      NC_CHECK(build_field0(c, st));
    } else {
      NC_CHECK(field_ring(c, st));
    }
    // the field spectra; training keeps one slot per step for the backward
    float2* xh = c.xhat + (c.train ? (size_t)t * pairs * ((size_t)g.Nh * g.Nw) : 0);
    NC_CHECK(field_spectra(c, xh, st));
    // z = IFFT(x^ . conj(G^_m)) on the ROI rows, then columns
    {
      ColArgs ca{xh, c.gspec, c.tmp, g.Nh, g.Nw, 0, g.roi_h, g.M, 1.0f};
      NC_CHECK(cols<COL_INV_MULCONJ>(ca, pairs * g.M, c.tw_h, st));
    }
    float* z = c.train ? c.zhat + (size_t)t * M * P : c.zscr;
    const size_t zs = c.train ? (size_t)g.d * M * P : M * P;
    {
      Planes zp{z, zs, B, g.M, g.roi_h, g.roi_w, g.P, g.roi_w, 1, pairs * g.M, 1.0f, c.rowstats};
      NC_CHECK(rows_inv(c.tmp, zp, g.Nw, c.tw_w, st));
    }
    // plane statistics from the row statistics the row pass wrote
    plane_stats_rows_kernel<<<B * g.M, kEpiThreads, 0, st>>>(g, c.rowstats, c.mean, c.rstd,
                                                             c.train ? c.rstd_save : nullptr,
                                                             c.train ? c.mean_save : nullptr, t);
    NC_CHECK(launched("plane_stats_rows_kernel launch"));
    if (t < g.d - 1) {
      NC_CHECK(hidden_epi(g, c, z, zs, t, g.act, g.slope, nullptr, st));
    } else if (c.uroi) {
      // universe mode: the ROI epilogue with the final activation (propagator.py:657-682)
      NC_CHECK(hidden_epi(g, c, z, zs, t, g.fact, g.fslope, c.uroi, st));
    } else {
      port_out_kernel<<<blocks_for((size_t)B * g.n_out, 128), 128, 0, st>>>(g, c.sp, c.out_index, z, zs,
                                                                             c.mean, c.rstd, c.out, B);
      NC_CHECK(launched("port_out_kernel launch"));
    }
  }
  return NC_OK;
}

// ---------------------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------------------
// Standardisation adjoint of step t's plane gradients in c.gz: deferred to the next row pass
// (*pending = true, coefficients in c.ncoef) when hidden_gz_kernel wrote the per-CTA sums
// (ncta > 0), else applied in place by norm_bwd_kernel (two passes over the planes).
nc_status norm_adjoint(const FftCall& c, const float* z, size_t zs, int t, int ncta, bool* pending,
                       cudaStream_t st) {
  const Geo& g = c.g;
  const int nplanes = c.batch * g.M;
  if (ncta > 0 && c.ncoef) {
    norm_coef_kernel<<<blocks_for((size_t)nplanes * 32, 256), 256, 0, st>>>(g, c.gzpart, ncta, c.mean_save,
                                                                           c.rstd_save, t, nplanes, c.ncoef);
    *pending = true;
    return launched("norm_coef_kernel launch");
  }
  norm_bwd_kernel<<<stat_grid(nplanes), kStatThreads, 0, st>>>(g, c.gz, z, zs, c.mean_save, c.rstd_save, t,
                                                               nplanes, plane_vec(g, zs),
                                                               ncta ? c.gzpart : nullptr, ncta);
  *pending = false;
  return launched("norm_bwd_kernel launch");
}

nc_status fft_backward(const FftCall& c, cudaStream_t st) {
  const Geo& g = c.g;
  const int B = c.batch, pairs = (B + 1) / 2;
  const size_t P = (size_t)g.P, M = (size_t)g.M;
  const size_t NN = (size_t)g.Nh * g.Nw;
  const size_t zs = (size_t)g.d * M * P;
  const int nch = B < kRedChunks ? B : kRedChunks;
  const int bc = (B + nch - 1) / nch;

  NC_CUDA_CHECK(cudaMemsetAsync(c.gsum, 0, sizeof(float) * 3 * P, st));
  if (c.gborder) NC_CUDA_CHECK(cudaMemsetAsync(c.gborder, 0, sizeof(float) * g.H * g.W, st));
  NC_CUDA_CHECK(cudaMemsetAsync(c.gz, 0, sizeof(float) * B * M * P, st));

  // The standardisation adjoint of the planes in c.gz is either applied in place
  // (norm_bwd_kernel) or left `pending`: its coefficients, folded for the raw planes, are in
  // c.ncoef and the row pass that reads c.gz next applies it (the corrected planes have no
  // other reader).
  bool pending = false;
  int pending_t = 0;

  // output step: sparse port adjoint (or the universe ROI adjoint), then the
  // standardisation adjoint (the saved planes are raw; every reader standardises them)
  {
    const int tl = g.d - 1;
    const float* z = c.zhat + (size_t)tl * M * P;
    if (c.guroi) {
      int ncta_out = 0;
      NC_CHECK(hidden_gz(g, c, z, zs, tl, nch, bc, g.fact, g.fslope, c.guroi, &ncta_out, st));
      gsum_chunks_kernel<<<blocks_for(3 * P, 256), 256, 0, st>>>(c.gpart, c.gsum, g.P, nch);
      NC_CHECK(launched("gsum_chunks_kernel launch"));
      if (g.norm) NC_CHECK(norm_adjoint(c, z, zs, tl, ncta_out, &pending, st));
    } else {
      port_gz_kernel<<<blocks_for((size_t)g.n_out * 32, 128), 128, 0, st>>>(g, c.sp, c.out_index, c.gout, z, zs,
                                                                c.mean_save, c.rstd_save, tl, c.gz, c.gsum, B);
      NC_CHECK(launched("port_gz_kernel launch"));
      if (g.norm) {
        // the plane gradients are zero off the ports: their sums come from the port cells
        const int nplanes = B * g.M;
        port_coef_kernel<<<blocks_for((size_t)nplanes * 32, 256), 256, 0, st>>>(
            g, c.out_index, c.gz, z, zs, c.mean_save, c.rstd_save, tl, nplanes, c.ncoef);
        NC_CHECK(launched("port_coef_kernel launch"));
        pending = true;
      }
    }
    pending_t = tl;
  }

  for (int t = g.d - 1; t >= 0; --t) {
    // spectra of the field that entered step t, kept by the training forward
    const float2* xh = c.xhat + (size_t)t * pairs * NN;
    // plane-gradient spectra q^ (pairs, M)
    {
      Planes gp{c.gz, M * P, B, g.M, g.roi_h, g.roi_w, g.P, g.roi_w, 1, pairs * g.M, 1.0f};
      if (pending) {
        gp.zh = c.zhat + (size_t)pending_t * M * P;
        gp.zstride = zs;
        gp.coef = c.ncoef;
      }
      NC_CHECK(rows_fwd(gp, c.tmp, g.Nw, c.tw_w, st));
      ColArgs ca{c.tmp, nullptr, c.q, g.Nh, g.Nw, g.roi_h, g.Nh, g.M, 1.0f};
      NC_CHECK(cols<COL_FWD>(ca, pairs * g.M, c.tw_h, st));
    }
    NC_CHECK(dg_accum(c, xh, pairs, NN, t == g.d - 1 ? 1 : 0, st));
    if (t == 0) break;

    // field adjoint dX = IFFT(sum_m q^_m . G^_m) on the field rows, then columns
    {
      ColArgs ca{c.q, c.gspec, c.tmp, g.Nh, g.Nw, 0, g.Fh, g.M, 1.0f};
      NC_CHECK(cols<COL_INV_SUM>(ca, pairs, c.tw_h, st));
      Planes dp{c.dx, (size_t)g.Fh * g.Fw, B, 1, g.Fh, g.Fw, 0, g.Fw, 1, pairs, 1.0f};
      NC_CHECK(rows_inv(c.tmp, dp, g.Nw, c.tw_w, st));
    }
    if (c.gborder) {
      ring_grad_kernel<<<blocks_for((size_t)g.Fh * g.Fw, 256), 256, 0, st>>>(g, c.dx, c.gborder, B);
      NC_CHECK(launched("ring_grad_kernel launch"));
    }
    // hidden-step adjoint of step t-1
    const float* z = c.zhat + (size_t)(t - 1) * M * P;
    int ncta = 0;
    NC_CHECK(hidden_gz(g, c, z, zs, t - 1, nch, bc, g.act, g.slope, nullptr, &ncta, st));
    gsum_chunks_kernel<<<blocks_for(3 * P, 256), 256, 0, st>>>(c.gpart, c.gsum, g.P, nch);
    NC_CHECK(launched("gsum_chunks_kernel launch"));
    pending = false;
    pending_t = t - 1;
    if (g.norm) NC_CHECK(norm_adjoint(c, z, zs, t - 1, ncta, &pending, st));
  }

  // filter gradient: Re IFFT(acc_m) / (Nh Nw) at lags [0, kh) x [0, kw)
  {
    ColArgs ca{c.dgacc, nullptr, c.tmp, g.Nh, g.Nw, g.Nh, g.kh, g.M, 1.0f};
    NC_CHECK(cols<COL_INV_PLAIN>(ca, g.M, c.tw_h, st));
    Planes dg{c.gdsum, (size_t)g.K, g.M, 1, g.kh, g.kw, 0, g.kw, 0, g.M,
              1.0f / ((float)g.Nh * (float)g.Nw)};
    NC_CHECK(rows_inv(c.tmp, dg, g.Nw, c.tw_w, st));
  }
  return NC_OK;
}

}  // namespace nc
