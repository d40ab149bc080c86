// nc_fft.cuh -- on-chip power-of-two complex FFTs over lines held in shared memory.
//
// A CTA transforms L lines of length N (2 <= N <= 1024) at once.  The forward transform is
// a decimation-in-frequency Cooley-Tukey in place (radix-4 stages, one radix-2 stage when
// log2 N is odd) and leaves the spectrum in digit-reversed order; the inverse is the exact
// adjoint (decimation in time, conjugate twiddles, stages in reverse order), which takes a
// digit-reversed spectrum back to natural order.  Every spectrum of the convolution path
// is produced by the same forward plan, so pointwise products never need the reordering.
// Neither direction scales; callers fold 1/(Nh*Nw) into the filter spectra.
//
// Shared-memory line layout: element e of line l sits at l*line_stride(N) + e + e/8.  The
// pad word every 8 elements keeps the short-span stages and the odd line stride keeps
// column-tile stores free of bank conflicts.
//
// Twiddles: per stage of sub-length S and radix R the table holds (R-1) rows of S/R
// entries, row q-1 = exp(-2 pi i q j / S) for j < S/R, stages in forward order; built on
// the host in double precision (twiddle_table_len / nc_plan_build).
#pragma once

#include <cuda_runtime.h>

namespace nc {
namespace fft {

__host__ __device__ inline int line_stride(int N) { return N + (N >> 3) + 1; }
__device__ __forceinline__ int pidx(int e) { return e + (e >> 3); }

__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(fmaf(a.x, b.x, -a.y * b.y), fmaf(a.x, b.y, a.y * b.x));
}
// a * conj(b)
__device__ __forceinline__ float2 cmulc(float2 a, float2 b) {
  return make_float2(fmaf(a.x, b.x, a.y * b.y), fmaf(a.y, b.x, -a.x * b.y));
}

__host__ __device__ inline int stage_radix(int S) { return (S % 4 == 0) ? 4 : 2; }

// Number of twiddle entries of the N-point plan.
__host__ __device__ inline int twiddle_table_len(int N) {
  int n = 0;
  for (int S = N; S > 1;) {
    const int R = stage_radix(S);
    n += (R - 1) * (S / R);
    S /= R;
  }
  return n;
}

__device__ __forceinline__ int ilog2(int x) { return 31 - __clz(x); }

// One forward (DIF) stage of sub-length S over all lines.
__device__ __forceinline__ void stage_dif(float2* s, int L, int N, int LS, int S, const float2* tw,
                                          int tid, int nt) {
  const int R = stage_radix(S);
  const int h = S / R, lh = ilog2(h);
  const int nbl = N / R, lnb = ilog2(nbl);
  const int total = L * nbl;
  if (R == 4) {
    for (int bf = tid; bf < total; bf += nt) {
      const int l = bf >> lnb, i = bf & (nbl - 1);
      const int j = i & (h - 1), base = ((i >> lh) * S) + j;
      float2* sl = s + l * LS;
      const float2 a0 = sl[pidx(base)], a1 = sl[pidx(base + h)];
      const float2 a2 = sl[pidx(base + 2 * h)], a3 = sl[pidx(base + 3 * h)];
      const float2 t0 = cadd(a0, a2), t1 = csub(a0, a2), t2 = cadd(a1, a3), t3 = csub(a1, a3);
      const float2 y0 = cadd(t0, t2), y2 = csub(t0, t2);
      const float2 y1 = make_float2(t1.x + t3.y, t1.y - t3.x);   // t1 - i t3
      const float2 y3 = make_float2(t1.x - t3.y, t1.y + t3.x);   // t1 + i t3
      sl[pidx(base)] = y0;
      sl[pidx(base + h)] = cmul(y1, tw[j]);
      sl[pidx(base + 2 * h)] = cmul(y2, tw[h + j]);
      sl[pidx(base + 3 * h)] = cmul(y3, tw[2 * h + j]);
    }
  } else {
    for (int bf = tid; bf < total; bf += nt) {
      const int l = bf >> lnb, i = bf & (nbl - 1);
      const int j = i & (h - 1), base = ((i >> lh) * S) + j;
      float2* sl = s + l * LS;
      const float2 a0 = sl[pidx(base)], a1 = sl[pidx(base + h)];
      sl[pidx(base)] = cadd(a0, a1);
      sl[pidx(base + h)] = cmul(csub(a0, a1), tw[j]);
    }
  }
}

// The adjoint of stage_dif (inverse direction).
__device__ __forceinline__ void stage_dit(float2* s, int L, int N, int LS, int S, const float2* tw,
                                          int tid, int nt) {
  const int R = stage_radix(S);
  const int h = S / R, lh = ilog2(h);
  const int nbl = N / R, lnb = ilog2(nbl);
  const int total = L * nbl;
  if (R == 4) {
    for (int bf = tid; bf < total; bf += nt) {
      const int l = bf >> lnb, i = bf & (nbl - 1);
      const int j = i & (h - 1), base = ((i >> lh) * S) + j;
      float2* sl = s + l * LS;
      const float2 a0 = sl[pidx(base)];
      const float2 a1 = cmulc(sl[pidx(base + h)], tw[j]);
      const float2 a2 = cmulc(sl[pidx(base + 2 * h)], tw[h + j]);
      const float2 a3 = cmulc(sl[pidx(base + 3 * h)], tw[2 * h + j]);
      const float2 t0 = cadd(a0, a2), t1 = csub(a0, a2), t2 = cadd(a1, a3), t3 = csub(a1, a3);
      sl[pidx(base)] = cadd(t0, t2);
      sl[pidx(base + 2 * h)] = csub(t0, t2);
      sl[pidx(base + h)] = make_float2(t1.x - t3.y, t1.y + t3.x);       // t1 + i t3
      sl[pidx(base + 3 * h)] = make_float2(t1.x + t3.y, t1.y - t3.x);   // t1 - i t3
    }
  } else {
    for (int bf = tid; bf < total; bf += nt) {
      const int l = bf >> lnb, i = bf & (nbl - 1);
      const int j = i & (h - 1), base = ((i >> lh) * S) + j;
      float2* sl = s + l * LS;
      const float2 a0 = sl[pidx(base)];
      const float2 a1 = cmulc(sl[pidx(base + h)], tw[j]);
      sl[pidx(base)] = cadd(a0, a1);
      sl[pidx(base + h)] = csub(a0, a1);
    }
  }
}

// Transforms L lines in place.  `tw` is the plan's table (shared or global memory).
// Starts after and ends with a __syncthreads(): callers fill / read the lines around it.
template <bool INVERSE>
__device__ void transform_lines(float2* s, int L, int N, const float2* tw, int tid, int nt) {
  const int LS = line_stride(N);
  // stage sub-lengths and table offsets in forward order
  int Ss[12], offs[12], ns = 0, off = 0;
  for (int S = N; S > 1;) {
    const int R = stage_radix(S);
    Ss[ns] = S;
    offs[ns] = off;
    ++ns;
    off += (R - 1) * (S / R);
    S /= R;
  }
  __syncthreads();
  if (!INVERSE) {
    for (int k = 0; k < ns; ++k) {
      stage_dif(s, L, N, LS, Ss[k], tw + offs[k], tid, nt);
      __syncthreads();
    }
  } else {
    for (int k = ns - 1; k >= 0; --k) {
      stage_dit(s, L, N, LS, Ss[k], tw + offs[k], tid, nt);
      __syncthreads();
    }
  }
}

}  // namespace fft

// ---------------------------------------------------------------------------------------
// 64 x 64 planes in natural order, radix-8 in registers (the fused small-grid kernels).
//
// A 64-point transform runs on 8 lanes: lane j loads x[j + 8n] (n < 8), does an 8-point
// DFT, multiplies output q by w64^(j q), the 8 lanes transpose their values with three
// xor-shuffle rounds, and lane q does a second 8-point DFT whose output n' is
// X[q + 8 n'] -- stored back at that position, so spectra stay in natural order.  A CTA
// of 512 threads runs 64 such groups: one pass transforms every row (or every column) of a
// plane.  Plane layout: element (r, c) at r * 66 + c; with this stride the 8-lane groups
// of a half-warp (rows r and r+4, or columns c and c+1) hit 16 distinct bank pairs.
// ---------------------------------------------------------------------------------------
namespace fft64 {

constexpr int kN = 64;
constexpr int kLS = 66;
constexpr int kPlane = kN * kLS;

__device__ __forceinline__ int at(int r, int c) { return r * kLS + c; }

// y[q] = sum_n a[n] w8^(n q) (INVERSE: conjugate roots); radix-2 network, natural order.
template <bool INVERSE>
__device__ __forceinline__ void dft8(float2 a[8]) {
  constexpr float h = 0.70710678118654752f;
  // w8 = (h, -h) forward, (h, +h) inverse; w8^2 = -i (forward) / +i (inverse)
  auto mw1 = [](float2 v) {   // v * w8
    return INVERSE ? make_float2(h * (v.x - v.y), h * (v.x + v.y))
                   : make_float2(h * (v.x + v.y), h * (v.y - v.x));
  };
  auto mw2 = [](float2 v) {   // v * w8^2
    return INVERSE ? make_float2(-v.y, v.x) : make_float2(v.y, -v.x);
  };
  auto mw3 = [](float2 v) {   // v * w8^3
    return INVERSE ? make_float2(-h * (v.x + v.y), h * (v.x - v.y))
                   : make_float2(h * (v.y - v.x), -h * (v.x + v.y));
  };
  const float2 b0 = fft::cadd(a[0], a[4]), b1 = fft::cadd(a[1], a[5]);
  const float2 b2 = fft::cadd(a[2], a[6]), b3 = fft::cadd(a[3], a[7]);
  const float2 b4 = fft::csub(a[0], a[4]), b5 = mw1(fft::csub(a[1], a[5]));
  const float2 b6 = mw2(fft::csub(a[2], a[6])), b7 = mw3(fft::csub(a[3], a[7]));
  const float2 c0 = fft::cadd(b0, b2), c1 = fft::cadd(b1, b3);
  const float2 c2 = fft::csub(b0, b2), c3 = mw2(fft::csub(b1, b3));
  const float2 c4 = fft::cadd(b4, b6), c5 = fft::cadd(b5, b7);
  const float2 c6 = fft::csub(b4, b6), c7 = mw2(fft::csub(b5, b7));
  a[0] = fft::cadd(c0, c1);
  a[4] = fft::csub(c0, c1);
  a[2] = fft::cadd(c2, c3);
  a[6] = fft::csub(c2, c3);
  a[1] = fft::cadd(c4, c5);
  a[5] = fft::csub(c4, c5);
  a[3] = fft::cadd(c6, c7);
  a[7] = fft::csub(c6, c7);
}

// 8 x 8 transpose across the 8 lanes of a group: afterwards lane l holds, in v[e], what
// lane e held in v[l].
__device__ __forceinline__ void transpose8(float2 v[8], int lane8) {
#pragma unroll
  for (int s = 4; s >= 1; s >>= 1) {
    const bool up = (lane8 & s) != 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (e & s) continue;
      const float2 send = up ? v[e] : v[e | s];
      float2 recv;
      recv.x = __shfl_xor_sync(0xffffffffu, send.x, s);
      recv.y = __shfl_xor_sync(0xffffffffu, send.y, s);
      if (up) v[e] = recv; else v[e | s] = recv;
    }
  }
}

// Lane roles of a 512-thread CTA: group g = one line, j = lane within the group.
struct Lane {
  int j;      // 0..7
  int row;    // line index of a row pass
  int col;    // line index of a column pass
};

__device__ __forceinline__ Lane lane_of(int tid) {
  const int w = tid >> 5, lane = tid & 31;
  Lane L;
  L.j = lane & 7;
  L.row = 8 * (w >> 1) + 2 * (w & 1) + (lane >> 4) + 4 * ((lane >> 3) & 1);
  L.col = 4 * w + (lane >> 3);
  return L;
}

// The middle of a 64-point transform: first DFT8 done on v (v[n] = x[j + 8n]), then
// twiddle, transpose, second DFT8: afterwards v[n'] = X[j + 8 n'].
template <bool INVERSE>
__device__ __forceinline__ void fft64_lanes(float2 v[8], int j, const float2* tw64) {
  dft8<INVERSE>(v);
#pragma unroll
  for (int q = 1; q < 8; ++q) {
    const float2 w = tw64[(j * q) & 63];
    v[q] = INVERSE ? fft::cmulc(v[q], w) : fft::cmul(v[q], w);
  }
  transpose8(v, j);
  dft8<INVERSE>(v);
}

// Transforms rows [0, nrows) (COLS = false) or all 64 columns (COLS = true) of a plane in
// place.  All 512 threads must call it (the shuffles need whole warps); lines beyond
// nrows are computed on zeros and not stored.  No barrier inside: callers separate
// passes that read each other's data with __syncthreads().
template <bool COLS, bool INVERSE>
__device__ __forceinline__ void pass64(float2* s, int nrows, const float2* tw64, const Lane& L) {
  const int line = COLS ? L.col : L.row;
  const bool active = COLS || line < nrows;
  if (!COLS && !__any_sync(0xffffffffu, active)) return;   // whole warp beyond nrows
  float2 v[8];
#pragma unroll
  for (int n = 0; n < 8; ++n)
    v[n] = active ? s[COLS ? at(L.j + 8 * n, line) : at(line, L.j + 8 * n)] : make_float2(0.f, 0.f);
  fft64_lanes<INVERSE>(v, L.j, tw64);
  if (active) {
#pragma unroll
    for (int n = 0; n < 8; ++n) s[COLS ? at(L.j + 8 * n, line) : at(line, L.j + 8 * n)] = v[n];
  }
}

// pass64 over two planes at once (independent transforms interleave).
template <bool COLS, bool INVERSE>
__device__ __forceinline__ void pass64x2(float2* s1, float2* s2, int nrows, const float2* tw64,
                                         const Lane& L) {
  const int line = COLS ? L.col : L.row;
  const bool active = COLS || line < nrows;
  if (!COLS && !__any_sync(0xffffffffu, active)) return;
  float2 v[8], u[8];
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    const int o = COLS ? at(L.j + 8 * n, line) : at(line, L.j + 8 * n);
    v[n] = active ? s1[o] : make_float2(0.f, 0.f);
    u[n] = active ? s2[o] : make_float2(0.f, 0.f);
  }
  fft64_lanes<INVERSE>(v, L.j, tw64);
  fft64_lanes<INVERSE>(u, L.j, tw64);
  if (active) {
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int o = COLS ? at(L.j + 8 * n, line) : at(line, L.j + 8 * n);
      s1[o] = v[n];
      s2[o] = u[n];
    }
  }
}

// tw64[e] = exp(-2 pi i e / 64) (sincospif: CUDA's own single-precision routine).
__device__ __forceinline__ void init_tw64(float2* tw64, int tid) {
  if (tid < kN) {
    float sn, cs;
    sincospif(-2.0f * (float)tid / (float)kN, &sn, &cs);
    tw64[tid] = make_float2(cs, sn);
  }
}

}  // namespace fft64

// ---------------------------------------------------------------------------------------
// Two-stage line transforms for N = 64 * R, R in {1, 2, 3, 4, 5, 6, 8, 16} (64 <= N <=
// 1024): the lines of the per-step FFT regime (nc_fftconv.cu) in two passes through shared
// memory instead of log4(N) radix-4 passes.  The radices 3, 5 and 6 let the planner pick a
// line length close to the field (286 -> 320 instead of 512).
//
// With n = n2 + 64 n1 and f = k1 + R k2 (n2, k2 < 64; n1, k1 < R):
//   X[k1 + R k2] = sum_n2 w64^(n2 k2) * ( wN^(n2 k1) * sum_n1 x[n2 + 64 n1] wR^(n1 k1) ).
// Stage A: one thread per (line, n2) does the radix-R DFT over n1 in registers, multiplies
// by wN^(n2 k1) and stores y[k1][n2] at position 64 k1 + n2.  Stage B: the 64-point DFT of
// each block k1 over n2 on 8 lanes (fft64::fft64_lanes), stored at 64 k1 + k2.  Position
// 64 k1 + k2 of a line therefore holds frequency k1 + R k2: a fixed permutation shared by
// every spectrum of the plan (products are pointwise), which the inverse -- the exact
// adjoint, stage B then stage A with conjugate roots -- takes back to natural order.
//
// Twiddles (plan table, built on the host in double precision): [k1 * 64 + n2] =
// exp(-2 pi i n2 k1 / N) for k1 < R, n2 < 64, then exp(-2 pi i e / 64) for e < 64.
// ---------------------------------------------------------------------------------------
namespace fft {

// Radices of the first stage (a DFT below for each).  Radices 10 and 12 would need more
// registers than the run-time-radix kernels of N = 1024 can give without spilling, so
// lines of 513 ... 1023 points keep N = 1024.
__host__ __device__ inline bool stage_a_radix(int R) {
  return R == 1 || R == 2 || R == 3 || R == 4 || R == 5 || R == 6 || R == 8 || R == 16;
}
__host__ __device__ inline bool two_stage(int N) {
  return N >= 64 && N <= 1024 && N % 64 == 0 && stage_a_radix(N / 64);
}

// Plan twiddle entries for an N-point line transform.
__host__ __device__ inline int plan_twiddle_len(int N) {
  return two_stage(N) ? N + 64 : twiddle_table_len(N);
}

// y[k] = sum_n a[n] wR^(n k), wR = exp(-+2 pi i / R); natural order in and out.
template <int R, bool INV>
__device__ __forceinline__ void dft_r(float2* a);

// cos and sin of 2 pi e / R for the composite radix 6 (exact values; e < R).
template <int R>
__device__ __forceinline__ float2 root_cs(int e) {
  static_assert(R == 6, "composite radix 6");
  constexpr float h3 = 0.86602540378443865f;                 // sqrt(3) / 2
  constexpr float c[6] = {1.f, 0.5f, -0.5f, -1.f, -0.5f, 0.5f};
  constexpr float s[6] = {0.f, h3, h3, 0.f, -h3, -h3};
  return make_float2(c[e], s[e]);
}

// R = P * Q from a DFT-Q and a DFT-P (Cooley-Tukey): with n = n1 + P n2, k = k1 + Q k2,
//   X[k1 + Q k2] = sum_n1 wP^(n1 k2) * ( wR^(n1 k1) * sum_n2 x[n1 + P n2] wQ^(n2 k1) ).
template <int P, int Q, bool INV>
__device__ __forceinline__ void dft_pq(float2* a) {
  constexpr int R = P * Q;
  float2 b[R];
#pragma unroll
  for (int n1 = 0; n1 < P; ++n1) {
    float2 q[Q];
#pragma unroll
    for (int n2 = 0; n2 < Q; ++n2) q[n2] = a[n1 + P * n2];
    dft_r<Q, INV>(q);
#pragma unroll
    for (int k1 = 0; k1 < Q; ++k1) {
      float2 v = q[k1];
      const int e = n1 * k1;
      if (e != 0) {
        const float2 cs = root_cs<R>(e);
        v = cmul(v, make_float2(cs.x, INV ? cs.y : -cs.y));   // wR^e (conjugate inverse)
      }
      b[n1 * Q + k1] = v;
    }
  }
#pragma unroll
  for (int k1 = 0; k1 < Q; ++k1) {
    float2 q[P];
#pragma unroll
    for (int n1 = 0; n1 < P; ++n1) q[n1] = b[n1 * Q + k1];
    dft_r<P, INV>(q);
#pragma unroll
    for (int k2 = 0; k2 < P; ++k2) a[k1 + Q * k2] = q[k2];
  }
}

template <int R, bool INV>
__device__ __forceinline__ void dft_r(float2* a) {
  if constexpr (R == 3) {
    // y1 = x0 + c t1 -/+ i s t2, y2 = x0 + c t1 +/- i s t2 with t1 = x1 + x2, t2 = x1 - x2,
    // c = cos(2 pi / 3) = -1/2, s = sin(2 pi / 3) (upper signs forward)
    constexpr float s3 = 0.86602540378443865f;
    const float2 t1 = cadd(a[1], a[2]), t2 = csub(a[1], a[2]);
    const float2 m = make_float2(fmaf(-0.5f, t1.x, a[0].x), fmaf(-0.5f, t1.y, a[0].y));
    const float2 is = make_float2(-s3 * t2.y, s3 * t2.x);   // i s t2
    a[0] = cadd(a[0], t1);
    a[1] = INV ? cadd(m, is) : csub(m, is);
    a[2] = INV ? csub(m, is) : cadd(m, is);
  } else if constexpr (R == 5) {
    // t1 = x1 + x4, t2 = x2 + x3, t3 = x1 - x4, t4 = x2 - x3; with c1, c2 = cos(2 pi / 5),
    // cos(4 pi / 5) and s1, s2 = sin(2 pi / 5), sin(4 pi / 5):
    //   y1, y4 = x0 + c1 t1 + c2 t2 -/+ i (s1 t3 + s2 t4)
    //   y2, y3 = x0 + c2 t1 + c1 t2 -/+ i (s2 t3 - s1 t4)      (upper signs forward)
    constexpr float c1 = 0.30901699437494742f, c2 = -0.80901699437494742f;
    constexpr float s1 = 0.95105651629515357f, s2 = 0.58778525229247314f;
    const float2 t1 = cadd(a[1], a[4]), t2 = cadd(a[2], a[3]);
    const float2 t3 = csub(a[1], a[4]), t4 = csub(a[2], a[3]);
    const float2 r1 = make_float2(fmaf(c2, t2.x, fmaf(c1, t1.x, a[0].x)), fmaf(c2, t2.y, fmaf(c1, t1.y, a[0].y)));
    const float2 r2 = make_float2(fmaf(c1, t2.x, fmaf(c2, t1.x, a[0].x)), fmaf(c1, t2.y, fmaf(c2, t1.y, a[0].y)));
    const float2 u1 = make_float2(fmaf(s2, t4.x, s1 * t3.x), fmaf(s2, t4.y, s1 * t3.y));
    const float2 u2 = make_float2(fmaf(-s1, t4.x, s2 * t3.x), fmaf(-s1, t4.y, s2 * t3.y));
    const float2 iu1 = make_float2(-u1.y, u1.x), iu2 = make_float2(-u2.y, u2.x);   // i u
    a[0] = cadd(a[0], cadd(t1, t2));
    a[1] = INV ? cadd(r1, iu1) : csub(r1, iu1);
    a[4] = INV ? csub(r1, iu1) : cadd(r1, iu1);
    a[2] = INV ? cadd(r2, iu2) : csub(r2, iu2);
    a[3] = INV ? csub(r2, iu2) : cadd(r2, iu2);
  } else if constexpr (R == 6) {
    dft_pq<2, 3, INV>(a);
  } else if constexpr (R == 2) {
    const float2 t = a[1];
    a[1] = csub(a[0], t);
    a[0] = cadd(a[0], t);
  } else if constexpr (R == 4) {
    // w4 = -i (forward) / +i (inverse)
    const float2 t0 = cadd(a[0], a[2]), t1 = csub(a[0], a[2]);
    const float2 t2 = cadd(a[1], a[3]), t3 = csub(a[1], a[3]);
    const float2 jt3 = INV ? make_float2(-t3.y, t3.x) : make_float2(t3.y, -t3.x);   // t3 * w4
    a[0] = cadd(t0, t2);
    a[2] = csub(t0, t2);
    a[1] = cadd(t1, jt3);
    a[3] = csub(t1, jt3);
  } else if constexpr (R == 8) {
    fft64::dft8<INV>(a);
  } else if constexpr (R == 16) {
    // n = n1 + 4 n2, k = k1 + 4 k2:  X[k1 + 4 k2] = sum_n1 w4^(n1 k2) w16^(n1 k1)
    //                                 * sum_n2 x[n1 + 4 n2] w4^(n2 k1)
    float2 b[16];
#pragma unroll
    for (int n1 = 0; n1 < 4; ++n1) {
      float2 q[4] = {a[n1], a[n1 + 4], a[n1 + 8], a[n1 + 12]};
      dft_r<4, INV>(q);
#pragma unroll
      for (int k1 = 0; k1 < 4; ++k1) {
        float2 v = q[k1];
        const int e = n1 * k1;                        // w16^e, e < 10
        if (e != 0) {
          // cos(2 pi e / 16), sin(2 pi e / 16)
          constexpr float c1 = 0.92387953251128674f, s1 = 0.38268343236508978f;
          constexpr float h = 0.70710678118654752f;
          constexpr float kc[10] = {1.f, c1, h, s1, 0.f, -s1, -h, -c1, -1.f, -c1};
          constexpr float ks[10] = {0.f, s1, h, c1, 1.f, c1, h, s1, 0.f, -s1};
          v = cmul(v, make_float2(kc[e], INV ? ks[e] : -ks[e]));
        }
        b[n1 * 4 + k1] = v;
      }
    }
#pragma unroll
    for (int k1 = 0; k1 < 4; ++k1) {
      float2 q[4] = {b[k1], b[4 + k1], b[8 + k1], b[12 + k1]};
      dft_r<4, INV>(q);
#pragma unroll
      for (int k2 = 0; k2 < 4; ++k2) a[k1 + 4 * k2] = q[k2];
    }
  }
}

// Stage A over all lines (see above); R == 1 is the identity.
template <int R, bool INV>
__device__ __forceinline__ void stage_a(float2* s, int L, int LS, const float2* twA, int tid, int nt) {
  for (int task = tid; task < L * 64; task += nt) {
    const int l = task >> 6, n2 = task & 63;
    float2* sl = s + l * LS;
    float2 v[R];
    if (!INV) {
#pragma unroll
      for (int n1 = 0; n1 < R; ++n1) v[n1] = sl[pidx(n2 + 64 * n1)];
      dft_r<R, false>(v);
#pragma unroll
      for (int k1 = 1; k1 < R; ++k1) v[k1] = cmul(v[k1], twA[k1 * 64 + n2]);
#pragma unroll
      for (int k1 = 0; k1 < R; ++k1) sl[pidx(64 * k1 + n2)] = v[k1];
    } else {
#pragma unroll
      for (int k1 = 0; k1 < R; ++k1) v[k1] = sl[pidx(64 * k1 + n2)];
#pragma unroll
      for (int k1 = 1; k1 < R; ++k1) v[k1] = cmulc(v[k1], twA[k1 * 64 + n2]);
      dft_r<R, true>(v);
#pragma unroll
      for (int n1 = 0; n1 < R; ++n1) sl[pidx(n2 + 64 * n1)] = v[n1];
    }
  }
}

// Stage B: 64-point transforms of the L * R blocks, 8 lanes per block, four per warp.
// The loop bound is warp-uniform (the shuffles need whole warps).
template <bool INV>
__device__ __forceinline__ void stage_b(float2* s, int L, int R, int LS, const float2* tw64, int tid,
                                        int nt) {
  const int lane = tid & 31, j = lane & 7;
  const int nblk = L * R, quads = (nblk + 3) >> 2;
  for (int q = tid >> 5; q < quads; q += nt >> 5) {
    const int blk = 4 * q + (lane >> 3);
    const bool active = blk < nblk;
    const int l = active ? blk / R : 0, k1 = active ? blk - (blk / R) * R : 0;
    float2* sb = s + l * LS;
    float2 v[8];
#pragma unroll
    for (int n = 0; n < 8; ++n) v[n] = active ? sb[pidx(64 * k1 + j + 8 * n)] : make_float2(0.f, 0.f);
    fft64::fft64_lanes<INV>(v, j, tw64);
    if (active) {
#pragma unroll
      for (int n = 0; n < 8; ++n) sb[pidx(64 * k1 + j + 8 * n)] = v[n];
    }
  }
}

// Shared-memory two-stage plan for R in {1, 2, 4, 8, 16}.  The kernels run it only for
// N = 64 (R = 1); longer lines take the global-stage variants below (fwd_a_global /
// inv_a_global), which also serve R = 3, 5 and 6.
template <bool INV>
__device__ void transform_lines_2s(float2* s, int L, int N, const float2* tw, int tid, int nt) {
  const int R = N >> 6, LS = line_stride(N);
  const float2* tw64 = tw + N;
  __syncthreads();
  if (!INV) {
    switch (R) {
      case 2: stage_a<2, false>(s, L, LS, tw, tid, nt); break;
      case 4: stage_a<4, false>(s, L, LS, tw, tid, nt); break;
      case 8: stage_a<8, false>(s, L, LS, tw, tid, nt); break;
      case 16: stage_a<16, false>(s, L, LS, tw, tid, nt); break;
      default: break;
    }
    if (R > 1) __syncthreads();
    stage_b<false>(s, L, R, LS, tw64, tid, nt);
  } else {
    stage_b<true>(s, L, R, LS, tw64, tid, nt);
    if (R > 1) __syncthreads();
    switch (R) {
      case 2: stage_a<2, true>(s, L, LS, tw, tid, nt); break;
      case 4: stage_a<4, true>(s, L, LS, tw, tid, nt); break;
      case 8: stage_a<8, true>(s, L, LS, tw, tid, nt); break;
      case 16: stage_a<16, true>(s, L, LS, tw, tid, nt); break;
      default: break;
    }
  }
  __syncthreads();
}

// The line transform of the plan for N: two-stage for 64 <= N <= 1024, radix-4 otherwise.
// Starts after and ends with a __syncthreads().
template <bool INV>
__device__ void transform_lines_plan(float2* s, int L, int N, const float2* tw, int tid, int nt) {
  if (two_stage(N))
    transform_lines_2s<INV>(s, L, N, tw, tid, nt);
  else
    transform_lines<INV>(s, L, N, tw, tid, nt);
}

// ---------------------------------------------------------------------------------------
// Two-stage transforms with the radix-R stage on global memory: the same arithmetic as
// transform_lines_2s (same stage order, twiddles and output permutation), but stage A
// takes its operands from global memory through ld(l, e) (forward) or hands its results
// to st(l, e, v) (inverse) instead of going through shared memory, so each element costs
// four shared-memory accesses instead of six.  Stage B and the copy on its side stay in
// shared memory, where their 8-lane blocks are free of bank conflicts and the global side
// stays fully coalesced.  For R = 1 (N = 64) callers use transform_lines_2s.
//
// LFAST = true (column tiles, L a power of two): consecutive lanes take consecutive lines,
// so the global accesses of a warp coalesce across the tile's columns; the line stride is
// then line_stride_cols(N), which keeps this mapping, stage B and the column-tile copy
// loops free of bank conflicts.  LFAST = false (rows): consecutive lanes take consecutive
// elements of a line, stride line_stride.
// ---------------------------------------------------------------------------------------
__host__ __device__ inline int line_stride_cols(int N) {
  const int b = N + (N >> 3);
  return b + ((4 - b) & 15);   // b rounded up to 4 (mod 16) float2 words
}

template <bool LFAST>
__device__ __forceinline__ void task_of(int task, int L, int lgL, int& l, int& n2) {
  if (LFAST) { l = task & (L - 1); n2 = task >> lgL; }
  else { l = task >> 6; n2 = task & 63; }
}

// Forward, R > 1: stage A from ld(l, e) (natural order, e < N) into the lines, then stage B
// in place; afterwards position 64 k1 + k2 of line l holds frequency k1 + R k2.  Starts
// after a barrier that published the twiddles, ends with a barrier.
template <int R, bool LFAST, class Ld>
__device__ __forceinline__ void fwd_a_global(float2* s, int L, int lgL, int LS, const float2* tw, int tid,
                                             int nt, Ld ld) {
  for (int task = tid; task < L * 64; task += nt) {
    int l, n2;
    task_of<LFAST>(task, L, lgL, l, n2);
    float2 v[R];
#pragma unroll
    for (int n1 = 0; n1 < R; ++n1) v[n1] = ld(l, n2 + 64 * n1);
    dft_r<R, false>(v);
#pragma unroll
    for (int k1 = 1; k1 < R; ++k1) v[k1] = cmul(v[k1], tw[k1 * 64 + n2]);
    float2* sl = s + l * LS;
#pragma unroll
    for (int k1 = 0; k1 < R; ++k1) sl[pidx(64 * k1 + n2)] = v[k1];
  }
  __syncthreads();
  stage_b<false>(s, L, R, LS, tw + 64 * R, tid, nt);
  __syncthreads();
}

// Inverse, R > 1: stage B in place on the lines (spectrum order), then stage A hands
// element e (natural order, every e < N) of line l to st(l, e, v).  Starts after a barrier
// that published the lines and the twiddles; returns without a barrier.
template <int R, bool LFAST, class St>
__device__ __forceinline__ void inv_a_global(float2* s, int L, int lgL, int LS, const float2* tw, int tid,
                                             int nt, St st) {
  stage_b<true>(s, L, R, LS, tw + 64 * R, tid, nt);
  __syncthreads();
  for (int task = tid; task < L * 64; task += nt) {
    int l, n2;
    task_of<LFAST>(task, L, lgL, l, n2);
    const float2* sl = s + l * LS;
    float2 v[R];
#pragma unroll
    for (int k1 = 0; k1 < R; ++k1) v[k1] = sl[pidx(64 * k1 + n2)];
#pragma unroll
    for (int k1 = 1; k1 < R; ++k1) v[k1] = cmulc(v[k1], tw[k1 * 64 + n2]);
    dft_r<R, true>(v);
#pragma unroll
    for (int n1 = 0; n1 < R; ++n1) st(l, n2 + 64 * n1, v[n1]);
  }
}

// Whether the global-stage variants apply: two-stage plans with a radix-R stage.
__host__ __device__ inline bool a_global(int N) { return two_stage(N) && N > 64; }

// Runtime R = N / 64 dispatch for the run-time-radix kernels (N = 1024 in practice; radices
// 3, 5 and 6 have specialised kernels, and leaving them out here keeps the register use of
// these kernels down).
template <bool LFAST, class Ld>
__device__ __forceinline__ void fwd_a_global_plan(float2* s, int L, int lgL, int LS, int N, const float2* tw,
                                                  int tid, int nt, Ld ld) {
  switch (N >> 6) {
    case 2: fwd_a_global<2, LFAST>(s, L, lgL, LS, tw, tid, nt, ld); break;
    case 4: fwd_a_global<4, LFAST>(s, L, lgL, LS, tw, tid, nt, ld); break;
    case 8: fwd_a_global<8, LFAST>(s, L, lgL, LS, tw, tid, nt, ld); break;
    case 16: fwd_a_global<16, LFAST>(s, L, lgL, LS, tw, tid, nt, ld); break;
    default: break;
  }
}

template <bool LFAST, class St>
__device__ __forceinline__ void inv_a_global_plan(float2* s, int L, int lgL, int LS, int N, const float2* tw,
                                                  int tid, int nt, St st) {
  switch (N >> 6) {
    case 2: inv_a_global<2, LFAST>(s, L, lgL, LS, tw, tid, nt, st); break;
    case 4: inv_a_global<4, LFAST>(s, L, lgL, LS, tw, tid, nt, st); break;
    case 8: inv_a_global<8, LFAST>(s, L, lgL, LS, tw, tid, nt, st); break;
    case 16: inv_a_global<16, LFAST>(s, L, lgL, LS, tw, tid, nt, st); break;
    default: break;
  }
}

}  // namespace fft
}  // namespace nc
