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
}  // namespace nc
