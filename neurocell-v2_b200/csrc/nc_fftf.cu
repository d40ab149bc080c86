// nc_fftf.cu -- per-sample fused FFT propagation for small grids (FFT side 64), sm_100a.
//
// One CTA owns one sample for all d steps, as in the direct kernels, but convolves in the
// frequency domain: the field spectrum X^ (64 x 64 complex) and a working spectrum stay in
// shared memory, and two directions share one complex inverse transform.  With the
// per-launch tables H_j = conj(G^_{2j}) + i conj(G^_{2j+1}) (spectra / 64^2, natural order;
// H_j(w) = F_j(-w) with F_j = FFT(g_{2j} + i g_{2j+1})):
//   forward      IFFT(X^ . H_j)               = z_{2j} + i z_{2j+1}        (X^ is Hermitian)
//   field adjoint Re IFFT(sum_j Q^_j . conj(H_j)) = sum_m gz_m (*) G_m, with
//                Q^_j = FFT(gz_{2j} + i gz_{2j+1}) (the imaginary part holds cross terms only)
//   filter adjoint IFFT(X^ . conj(Q^_j)) / 64^2 = corr(X, gz_{2j}) - i corr(X, gz_{2j+1}).
// So a step costs one field transform plus M/2 inverse transforms forward, and M/2 forward
// plus M/2 pruned inverse transforms plus one inverse backward, instead of 2*M*P*K FMAs per
// pass.  The 64-point transforms are radix-8 in registers with shuffle transposes
// (nc_fft.cuh, fft64).  The epilogues (neurocell/epilogue.py:28-56, :82-128; centred two-pass variance of
// neurocell/kernels_pallas.py:202-205) run plane pair by plane pair, accumulating the
// per-pixel sums over directions, so no more than two planes are ever on chip.
#include <cuda_runtime.h>

#include "nc_common.cuh"
#include "nc_errors.h"
#include "nc_fft.cuh"
#include "nc_fftf.h"
#include "nc_prestep.cuh"

namespace nc {

using fft::cadd;
using fft::cmul;
using fft::cmulc;

namespace {

constexpr int kN = kFftfN;                    // FFT side
constexpr int kPlane = fft64::kPlane;         // float2 per on-chip plane
constexpr int kThreads = 512;
constexpr float kInvNN = 1.0f / (float)(kN * kN);
static_assert(kN == fft64::kN, "fused kernels are built on the 64-point transforms");
static_assert(kPlane == kFftfPlane, "stored spectra use the on-chip plane layout");
constexpr unsigned kPlaneBytes = kPlane * sizeof(float2);        // 33,792
constexpr unsigned kPlaneChunk = kPlaneBytes / 4;                // 8,448: bulk copy size

__device__ __forceinline__ int at2(int r, int c) { return fft64::at(r, c); }

// ---- bulk copies global -> shared (cp.async.bulk, completion on an mbarrier) ------------
// Used to stage the next direction pair's spectra and saved planes while the current pair
// computes.  Every wait is bounded.  A wait that gives up sets the call's status word in the
// workspace (StepParams::status, read by nc_workspace_status) and the CTA's abort flag in
// shared memory, then waits once more (bounded) for the copy in flight.  The kernels read
// the abort flag after the next barrier, wait (bounded) for every copy they still have in
// flight, and return together; every output of that launch is then invalid.
constexpr int kWaitLimit = 1 << 20;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// Orders this thread's earlier generic-proxy accesses of shared memory before its bulk copies.
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// `bytes` and both addresses are multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Waits for the completion of phase `parity` of `bar` (bounded, see above).
__device__ __forceinline__ void mbar_wait(uint64_t* bar, unsigned parity, int* status, volatile int* abort_flag) {
  for (int it = 0; it < kWaitLimit; ++it)
    if (mbar_try_wait(bar, parity)) return;
  if (status) atomicExch(status, 1);
  *abort_flag = 1;
  for (int it = 0; it < kWaitLimit; ++it)
    if (mbar_try_wait(bar, parity)) return;
}
// Before an early return: bounded waits for the copies issued on `bar` and not yet waited.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, unsigned used, unsigned issued) {
  for (; used < issued; ++used)
    for (int it = 0; it < kWaitLimit; ++it)
      if (mbar_try_wait(bar, used & 1u)) break;
}

#if NC_PHASE_TIMING
// Debug builds only: clock64 cycles of CTA 0's thread 0 between phase marks, summed over
// launches ([0] forward, [1] backward; see the FFTF_MARK slots in each kernel).
__device__ long long g_fftf_phase[2][16];
#define FFTF_T0() long long fftf_t_last = clock64()
#define FFTF_MARK(kern, slot)                                          \
  do {                                                                 \
    if (blockIdx.x == 0 && threadIdx.x == 0) {                         \
      const long long now = clock64();                                 \
      g_fftf_phase[kern][slot] += now - fftf_t_last;                   \
      fftf_t_last = now;                                               \
    }                                                                  \
  } while (0)
#else
#define FFTF_T0() \
  do {            \
  } while (0)
#define FFTF_MARK(kern, slot) \
  do {                        \
  } while (0)
#endif

// Forward 2-D transform of rows [0, nrows) then all columns; barriers on both sides.
__device__ __forceinline__ void fwd2d(float2* s, int nrows, const float2* tw, const fft64::Lane& L) {
  __syncthreads();
  fft64::pass64<false, false>(s, nrows, tw, L);
  __syncthreads();
  fft64::pass64<true, false>(s, kN, tw, L);
  __syncthreads();
}

// Inverse 2-D transform: all columns, then rows [0, nrows) (the rows that are kept).
__device__ __forceinline__ void inv2d(float2* s, int nrows, const float2* tw, const fft64::Lane& L) {
  __syncthreads();
  fft64::pass64<true, true>(s, kN, tw, L);
  __syncthreads();
  fft64::pass64<false, true>(s, nrows, tw, L);
  __syncthreads();
}

// The fused kernels run 1024 threads: two halves of 512, each laid out as 64 groups of
// 8 lanes (fft64::lane_of), so one half transforms every row or column of one plane.  A
// round of the d-step loop holds two direction pairs in two working planes; half h works on
// plane h wherever a phase has one transform per line and plane.
constexpr int kThreadsF = 1024;
constexpr int kPosPerThread = kN * kN / kThreadsF;   // plane positions per thread (4)

// ROI pixels p = tid + 1024 k of this thread: their plane offsets (r, c) -> at2(r, c), or -1.
__device__ __forceinline__ void pixel_offsets(const Geo& g, int tid, int poff[kPosPerThread]) {
#pragma unroll
  for (int k = 0; k < kPosPerThread; ++k) {
    const int p = tid + k * kThreadsF;
    const int r = p / g.roi_w, c = p - (p / g.roi_w) * g.roi_w;
    poff[k] = p < g.P ? at2(r, c) : -1;
  }
}

// Warp sums of eight values by a reduce-scatter butterfly: exchanging half of the values
// with lane ^ 16, then half of the rest with lane ^ 8, then one with lane ^ 4, leaves each
// lane the sum over 8 lanes of value k = 4 b4 + 2 b3 + b2 (b_i = bit i of the lane); two
// more xor steps (2, 1) complete it over the warp.  9 shuffles instead of 40, fixed order;
// on return every lane of quad k (lanes 4k' .. 4k'+3 with those bits) holds warp sum k.
__device__ __forceinline__ float warp_reduce8(const float v[8], int lane) {
  const bool b4 = (lane & 16) != 0, b3 = (lane & 8) != 0, b2 = (lane & 4) != 0;
  float a[4], c[2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float keep = b4 ? v[i + 4] : v[i], send = b4 ? v[i] : v[i + 4];
    a[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float keep = b3 ? a[i + 2] : a[i], send = b3 ? a[i] : a[i + 2];
    c[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  float r = (b2 ? c[1] : c[0]) + __shfl_xor_sync(0xffffffffu, b2 ? c[0] : c[1], 4);
  r += __shfl_xor_sync(0xffffffffu, r, 2);
  r += __shfl_xor_sync(0xffffffffu, r, 1);
  return r;
}

// Sum of eight per-thread values over the 1024-thread CTA, broadcast to every thread, in a
// fixed order: each warp's sums (warp_reduce8) go to half `par` of `red` (2 x (8 x 32 + 8)
// floats); after a barrier warp k < 8 adds value k over the 32 warps; after a second barrier
// every thread reads the eight sums.  Alternating halves make a barrier before the writes
// unnecessary: a thread writes half `par` again only after the barriers of the next call,
// which every thread reaches after its reads of this call.  Callers flip `par` after each
// call.
constexpr int kRedHalf = 8 * 32 + 8;
__device__ __forceinline__ void block_sum8(float v[8], float* red, int& par) {
  static_assert(kThreadsF / 32 == 32, "32 warp partials");
  float* h = red + par * kRedHalf;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float r = warp_reduce8(v, lane);
  if ((lane & 3) == 0) h[(lane >> 2) * 32 + w] = r;   // lane 4k holds value k
  __syncthreads();
  if (w < 8) {
    const float t = warp_sum(h[w * 32 + lane]);
    if (lane == 0) h[256 + w] = t;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 8; ++k) v[k] = h[256 + k];
  par ^= 1;
}

// Forward 2-D transform of rows [0, nrows) then all columns by the first half (one plane
// has one transform per line); barriers on both sides for the whole CTA.
__device__ __forceinline__ void fwd2d_h0(float2* s, int nrows, const float2* tw, const fft64::Lane& L,
                                         int half) {
  __syncthreads();
  if (half == 0) fft64::pass64<false, false>(s, nrows, tw, L);
  __syncthreads();
  if (half == 0) fft64::pass64<true, false>(s, kN, tw, L);
  __syncthreads();
}

// Inverse 2-D transform (all columns, then rows [0, nrows)) by the first half.
__device__ __forceinline__ void inv2d_h0(float2* s, int nrows, const float2* tw, const fft64::Lane& L,
                                         int half) {
  __syncthreads();
  if (half == 0) fft64::pass64<true, true>(s, kN, tw, L);
  __syncthreads();
  if (half == 0) fft64::pass64<false, true>(s, nrows, tw, L);
  __syncthreads();
}

// Inverse row pass of the ROI rows of one plane that also leaves each row's centred
// statistics (mean, M2 over its `roi_w` columns) of the re and im parts in
// rowst[row * 4 + k0] and rowst[row * 4 + k0 + 1].  The 8 lanes of a row sum their values
// with three xor shuffles, then sum the squared deviations from the row mean the same way;
// the row values never leave registers for it.
__device__ __forceinline__ void rows_inv_stats(float2* s, int nrows, int roi_w, const float2* tw64,
                                               const fft64::Lane& L, float2* rowst, int k0) {
  const int line = L.row;
  const bool active = line < nrows;
  if (!__any_sync(0xffffffffu, active)) return;
  float2 v[8];
#pragma unroll
  for (int n = 0; n < 8; ++n) v[n] = active ? s[at2(line, L.j + 8 * n)] : make_float2(0.f, 0.f);
  fft64::fft64_lanes<true>(v, L.j, tw64);
  float sx = 0.f, sy = 0.f;
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    if (L.j + 8 * n < roi_w) {
      sx += v[n].x;
      sy += v[n].y;
    }
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    sx += __shfl_xor_sync(0xffffffffu, sx, o);
    sy += __shfl_xor_sync(0xffffffffu, sy, o);
  }
  const float inv_w = 1.0f / (float)roi_w;
  const float mx = sx * inv_w, my = sy * inv_w;
  float qx = 0.f, qy = 0.f;
#pragma unroll
  for (int n = 0; n < 8; ++n) {
    if (L.j + 8 * n < roi_w) {
      const float dx = v[n].x - mx, dy = v[n].y - my;
      qx = fmaf(dx, dx, qx);
      qy = fmaf(dy, dy, qy);
    }
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    qx += __shfl_xor_sync(0xffffffffu, qx, o);
    qy += __shfl_xor_sync(0xffffffffu, qy, o);
  }
  if (active) {
#pragma unroll
    for (int n = 0; n < 8; ++n) s[at2(line, L.j + 8 * n)] = v[n];
    if (L.j == 0) rowst[line * 4 + k0] = make_float2(mx, qx);
    if (L.j == 1) rowst[line * 4 + k0 + 1] = make_float2(my, qy);
  }
}

// Plane statistics of the four real planes from the row statistics (after a barrier):
// warp k < 4 takes plane k, lane l rows l and l + 32.  Every row holds roi_w cells, so the
// plane mean is the mean of the row means and M2 = sum_r M2_r + roi_w sum_r (mean_r -
// mean)^2 -- the reference's two-stage variance for tiled planes
// (neurocell/kernels_pallas.py:740-837) -- in two fixed-order warp sums; lane 0 writes
// (mean, 1 / sqrt(var + eps)) to st[k].  inv_h = 1 / roi_h, inv_n = 1 / (roi_h roi_w) come
// from the caller (no division on this path, which every warp of the CTA waits for).
__device__ __forceinline__ void merge_row_stats(const float2* rowst, int roi_h, int roi_w, float inv_h,
                                                float inv_n, float2* st) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (w >= 4) return;
  const bool h0 = lane < roi_h, h1 = lane + 32 < roi_h;
  const float2 r0 = h0 ? rowst[lane * 4 + w] : make_float2(0.f, 0.f);
  const float2 r1 = h1 ? rowst[(lane + 32) * 4 + w] : make_float2(0.f, 0.f);
  const float mean = warp_sum(r0.x + r1.x) * inv_h;
  const float d0 = h0 ? r0.x - mean : 0.f, d1 = h1 ? r1.x - mean : 0.f;
  float dev = fmaf(d0, d0, d1 * d1), m2 = r0.y + r1.y;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    dev += __shfl_xor_sync(0xffffffffu, dev, o);
    m2 += __shfl_xor_sync(0xffffffffu, m2, o);
  }
  m2 = fmaf((float)roi_w, dev, m2);
  if (lane == 0) st[w] = make_float2(mean, rsqrtf(fmaf(m2, inv_n, kNormEps)));
}

// Field of step t into X (real part; zero imaginary, zero beyond Fh x Fw).
//   src_interior(p): the ROI value; ring: VALID border template, SAME zero, CIRCULAR wrap.
// Step 0 (src == nullptr): zeros, injected inputs, wrapped halo.
__device__ void load_field(const FftfArgs& a, float2* X, const float* roi_src, const float* inp,
                           int tid, int nt) {
  const Geo& g = a.g;
  if (!roi_src) {
    for (int i = tid; i < kPlane; i += nt) X[i] = make_float2(0.f, 0.f);
    __syncthreads();
    for (int j = tid; j < g.n_in; j += nt) {
      const int idx = a.in_index[j];
      if (idx < 0) continue;
      const int r = idx / g.W, c = idx - (idx / g.W) * g.W;
      X[at2(r + g.gr, c + g.gc)].x = inp[j];
    }
    __syncthreads();
    if (g.padding == NC_PAD_CIRCULAR) {
      for (int i = tid; i < g.Fh * g.Fw; i += nt) {
        const int fr = i / g.Fw, fc = i - (i / g.Fw) * g.Fw;
        const int r = fr - g.oh, c = fc - g.ow;
        if (r >= 0 && r < g.roi_h && c >= 0 && c < g.roi_w) continue;
        int sr = r % g.roi_h; if (sr < 0) sr += g.roi_h;
        int sc = c % g.roi_w; if (sc < 0) sc += g.roi_w;
        X[at2(fr, fc)].x = X[at2(sr + g.oh, sc + g.ow)].x;
      }
      __syncthreads();
    }
    return;
  }
  for (int i = tid; i < kN * kN; i += nt) {
    const int fr = i / kN, fc = i - (i / kN) * kN;
    float v = 0.f;
    if (fr < g.Fh && fc < g.Fw) {
      int r = fr - g.oh, c = fc - g.ow;
      const bool inside = r >= 0 && r < g.roi_h && c >= 0 && c < g.roi_w;
      if (inside) {
        v = roi_src[r * g.roi_w + c];
      } else if (g.padding == NC_PAD_VALID) {
        v = a.sp.border[fr * g.W + fc];
      } else if (g.padding == NC_PAD_CIRCULAR) {
        r %= g.roi_h; if (r < 0) r += g.roi_h;
        c %= g.roi_w; if (c < 0) c += g.roi_w;
        v = roi_src[r * g.roi_w + c];
      }
    }
    X[at2(fr, fc)] = make_float2(v, 0.f);
  }
}


// ---------------------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------------------
// ACT / FACT: the hidden and final activations as compile-time constants (the common
// tanh / identity chip), or kActRuntime to read them from the geometry.  Fixing them lets
// the compiler specialise the per-pixel epilogue loops.
constexpr int kActRuntime = -1;

template <int ACT, int FACT>
__global__ void __launch_bounds__(kThreadsF, 1) fftf_fwd_kernel(FftfArgs a) {
  pdl_enter();   // see pdl_wait
  extern __shared__ float4 smem4[];
  uint64_t* hbar = reinterpret_cast<uint64_t*>(smem4);   // staging barrier (16 B slot)
  volatile int* abort_flag = reinterpret_cast<int*>(smem4) + 2;   // in the same slot
  float2* stw = reinterpret_cast<float2*>(smem4 + 1);
  float2* X = stw + kN;
  float2* W = X + kPlane;                                 // the round's two working planes
  float2* Hs = W + 2 * kPlane;                            // staged spectra of one round
  const bool stage = a.stage != 0;
  float2* rowst = Hs + (stage ? 2 * kPlane : 0);          // (64 rows, 4 planes) row statistics
  float2* pst = rowst + 4 * kN;                           // 4 plane statistics (8 slots)
  float* lin = reinterpret_cast<float*>(pst + 8);
  float* acc = lin + a.g.P;
  float* bsm = acc + a.g.P;                               // b on the ROI, read every round
  const Geo& g = a.g;
  const int tid = threadIdx.x, nt = blockDim.x, b = blockIdx.x;
  const int half = tid >> 9;                              // working plane of this thread
  const size_t P = (size_t)g.P, M = (size_t)g.M;
  const int pairs = g.M / 2;
  const float inv_h = 1.0f / (float)g.roi_h, inv_n = 1.0f / (float)g.P;   // plane statistics
  fft64::init_tw64(stw, tid);
  const fft64::Lane Ln = fft64::lane_of(tid & 511);
  int poff[kPosPerThread];
  pixel_offsets(g, tid, poff);
  for (int p = tid; p < g.P; p += nt) bsm[p] = a.sp.broi[p];   // published by the first barriers
  // Spectra of round j0 (pairs j0, j0+1) -> Hs: the stored planes already have the on-chip
  // layout (row stride 66: the column pass reads them without bank conflicts), so they
  // move as four bulk copies each.  Warp 0, after a barrier that ends the previous readers
  // of Hs.
  unsigned huse = 0, hiss = 0;
  auto issue_h = [&](int j0) {
    ++hiss;
    if (tid < 32) {
      const int np = (j0 + 1 < pairs) ? 2 : 1;
      if (tid == 0) mbar_expect_tx(hbar, np * kPlaneBytes);
      __syncwarp();
      fence_proxy_async();
      if (tid < 4 * np)
        bulk_g2s(reinterpret_cast<char*>(Hs) + tid * kPlaneChunk,
                 reinterpret_cast<const char*>(a.H + (size_t)j0 * kPlane) + tid * kPlaneChunk,
                 kPlaneChunk, hbar);
    }
  };
  if (tid == 0) *abort_flag = 0;
  if (stage) {
    if (tid == 0) mbar_init(hbar, 1);
    __syncthreads();
    issue_h(0);
  }
  FFTF_T0();

  for (int t = 0; t < g.d; ++t) {
    const bool last = (t == g.d - 1);
    load_field(a, X, t == 0 ? nullptr : lin, a.inputs + (size_t)b * g.n_in, tid, nt);
    FFTF_MARK(0, 0);
    fwd2d_h0(X, g.Fh, stw, Ln, half);
    if (a.train && a.xspec) {          // the backward reuses this step's field spectrum
      float2* xo = a.xspec + ((size_t)b * g.d + t) * kPlane;
      for (int i = tid; i < kPlane; i += nt) xo[i] = X[i];
    }
    FFTF_MARK(0, 1);
    const int act_id = last ? (FACT != kActRuntime ? FACT : g.fact) : (ACT != kActRuntime ? ACT : g.act);
    const float slope = last ? g.fslope : g.slope;
    for (int p = tid; p < g.P; p += nt) { lin[p] = 0.f; acc[p] = 0.f; }

    // two direction pairs (four planes) per round: half h transforms plane h
    for (int j = 0; j < pairs; j += 2) {
      const bool two = j + 1 < pairs;
      const bool mine = half == 0 || two;                 // uniform over each half
      float2* Wh = W + half * kPlane;
      if (stage) {
        mbar_wait(hbar, huse & 1u, a.sp.status, abort_flag);
        ++huse;
      }
      FFTF_MARK(0, 7);
      // inverse column pass of X^ . H_{j+h} (product taken at load time)
      if (mine) {
        const float2* Hh = stage ? Hs + half * kPlane : a.H + (size_t)(j + half) * kPlane;
        float2 v[8];
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const int o = at2(Ln.j + 8 * n, Ln.col);
          v[n] = cmul(X[o], stage ? Hh[o] : __ldg(&Hh[o]));
        }
        fft64::fft64_lanes<true>(v, Ln.j, stw);
#pragma unroll
        for (int n = 0; n < 8; ++n) Wh[at2(Ln.j + 8 * n, Ln.col)] = v[n];
      }
      __syncthreads();
      if (stage && *abort_flag) {        // uniform: set before the barrier above
        mbar_drain(hbar, huse, hiss);
        return;
      }
      if (stage) {                       // the next round's spectra land during this round
        const int nj = (j + 2 < pairs) ? j + 2 : (t + 1 < g.d ? 0 : -1);
        if (nj >= 0) issue_h(nj);
      }
      FFTF_MARK(0, 2);
      // inverse row pass of the ROI rows (warps beyond them skip); with the spatial norm the
      // pass also leaves every row's centred statistics, merged per plane below
      if (mine) {
        if (g.norm) rows_inv_stats(Wh, g.roi_h, g.roi_w, stw, Ln, rowst, 2 * half);
        else fft64::pass64<false, true>(Wh, g.roi_h, stw, Ln);
      }
      __syncthreads();
      FFTF_MARK(0, 3);
      // plane statistics of 2j, 2j+1 (plane 0 re, im) and 2j+2, 2j+3 (plane 1): centred per
      // row, merged over the rows with Chan's formula
      float mu[4] = {0.f, 0.f, 0.f, 0.f}, rs[4] = {1.f, 1.f, 1.f, 1.f};
      if (g.norm) {
        merge_row_stats(rowst, g.roi_h, g.roi_w, inv_h, inv_n, pst);
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 q = pst[k];
          mu[k] = q.x;
          rs[k] = q.y;
        }
      }
      FFTF_MARK(0, 4);
      const int np = two ? 4 : 2;
      if (a.train && tid < np)           // pst holds them when norm is on (no indexed registers)
        a.rstd[((size_t)b * g.d + t) * M + 2 * j + tid] = g.norm ? pst[tid].y : 1.0f;
      float* zh = a.train ? a.zhat + (((size_t)b * g.d + t) * M + 2 * j) * P : nullptr;
      const float2* W0 = W;
      const float2* W1 = W + kPlane;
#pragma unroll
      for (int k = 0; k < kPosPerThread; ++k) {
        if (poff[k] < 0) continue;
        const int p = tid + k * kThreadsF;
        const float2 w = W0[poff[k]], u = W1[poff[k]];
        const float h0 = (w.x - mu[0]) * rs[0], h1 = (w.y - mu[1]) * rs[1];
        const float h2 = (u.x - mu[2]) * rs[2], h3 = (u.y - mu[3]) * rs[3];
        const float bb = bsm[p];
        if (zh) { zh[p] = h0; zh[P + p] = h1; }
        float l = h0 + h1;
        float ac = (act_id != NC_ACT_NONE) ? act_fwd(act_id, h0 + bb, slope) + act_fwd(act_id, h1 + bb, slope) : 0.f;
        if (two) {
          if (zh) { zh[2 * P + p] = h2; zh[3 * P + p] = h3; }
          l += h2 + h3;
          if (act_id != NC_ACT_NONE) ac += act_fwd(act_id, h2 + bb, slope) + act_fwd(act_id, h3 + bb, slope);
        }
        lin[p] += l;
        acc[p] += ac;
      }
      __syncthreads();
      FFTF_MARK(0, 5);
    }
    __syncthreads();
    if (last && a.uroi) {
      // universe mode: the last step's ROI cells (ROI epilogue with the final activation)
      for (int p = tid; p < g.P; p += nt) {
        const float bb = a.sp.broi[p];
        const float act = (g.fact == NC_ACT_NONE) ? lin[p] + (float)g.M * bb : acc[p];
        a.uroi[(size_t)b * P + p] = a.sp.weff[p] * lin[p] + a.sp.seff[p] * act;
      }
    } else if (!last) {
      float* xs = a.train ? a.xsave + ((size_t)b * (g.d - 1) + t) * P : nullptr;
      for (int p = tid; p < g.P; p += nt) {
        const float bb = a.sp.broi[p];
        const float act = (g.act == NC_ACT_NONE) ? lin[p] + (float)g.M * bb : acc[p];
        const float xn = a.sp.weff[p] * lin[p] + a.sp.seff[p] * act;
        lin[p] = xn;                      // the next step's ROI field
        if (xs) xs[p] = xn;
      }
      __syncthreads();
    } else {
      for (int jo = tid; jo < g.n_out; jo += nt) {
        const int idx = a.out_index[jo];
        const int gr_ = idx / g.W, gc_ = idx - (idx / g.W) * g.W;
        const int p = (gr_ - g.pad_h) * g.roi_w + (gc_ - g.pad_w);
        if (gr_ < g.pad_h || gr_ >= g.pad_h + g.roi_h || gc_ < g.pad_w || gc_ >= g.pad_w + g.roi_w) {
          a.out[(size_t)b * g.n_out + jo] = __int_as_float(0x7fc00000);   // universe mode only
          continue;
        }
        const float wo = a.sp.weff[p], so = a.sp.seff[p], bo = a.sp.broi[p];
        a.out[(size_t)b * g.n_out + jo] = (g.fact == NC_ACT_NONE)
                                              ? (wo + so) * lin[p] + ((float)g.M * so * bo)
                                              : act_fwd(g.fact, wo * lin[p] + so * acc[p], g.fslope);
      }
    }
    FFTF_MARK(0, 6);
  }
}

// ---------------------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------------------
// Two direction pairs per round, as in the forward.  The field spectra X^ and the pair
// spectra H come from global memory (L2) in the column pass, the standardised planes are
// staged into shared memory four planes at a time; the field adjoint D = sum_j Q^_j .
// conj(H_j) and the per-pixel parameter gradients stay on chip for the whole launch.
template <int ACT, int FACT>
__global__ void __launch_bounds__(kThreadsF, 1) fftf_bwd_kernel(FftfArgs a) {
  pdl_enter();   // see pdl_wait
  extern __shared__ float4 smem4[];
  const Geo& g = a.g;
  const int tid = threadIdx.x, nt = blockDim.x, b = blockIdx.x;
  const int half = tid >> 9, warp = tid >> 5, lane = tid & 31;
  const size_t P = (size_t)g.P, M = (size_t)g.M;
  const int pairs = g.M / 2;
  const int FF = g.Fh * g.Fw;
  uint64_t* zbar = reinterpret_cast<uint64_t*>(smem4);   // staging barrier of the planes
  volatile int* abort_flag = reinterpret_cast<int*>(smem4) + 2;
  float2* stw = reinterpret_cast<float2*>(smem4 + 1);
  float2* W = stw + kN;                                   // the round's two working planes
  float2* D = W + 2 * kPlane;                             // field-adjoint spectrum of the step
  float* red = reinterpret_cast<float*>(D + kPlane);      // block_sum8 halves
  const bool stage = a.stage != 0;
  float* zs = red + 2 * kRedHalf;                         // staged planes 2j .. 2j+3
  float* gy = zs + (stage ? 4 * g.P : 0);
  float* gp0 = gy + g.P;
  float* gp1 = gp0 + g.P;
  float* gp2 = gp1 + g.P;
  float* wsm = gp2 + g.P;                      // w_eff, s_eff, b on the ROI, read every round
  float* ssm = wsm + g.P;
  float* bsm = ssm + g.P;
  float* dg = bsm + g.P;                       // M*K
  float* gport = dg + M * g.K;                 // n_out * M
  int16_t* pmap = reinterpret_cast<int16_t*>(gport + (size_t)g.n_out * M);   // P
  float* ring = a.gring ? a.gring + (size_t)b * FF : nullptr;                 // global, this sample
  fft64::init_tw64(stw, tid);
  const fft64::Lane Ln = fft64::lane_of(tid & 511);
  for (int p = tid; p < g.P; p += nt) {
    gp0[p] = 0.f; gp1[p] = 0.f; gp2[p] = 0.f; pmap[p] = -1;
    wsm[p] = a.sp.weff[p]; ssm[p] = a.sp.seff[p]; bsm[p] = a.sp.broi[p];
  }
  for (int i = tid; i < (int)(M * g.K); i += nt) dg[i] = 0.f;
  if (ring)
    for (int i = tid; i < FF; i += nt) ring[i] = 0.f;
  if (tid == 0) *abort_flag = 0;
  if (stage && tid == 0) mbar_init(zbar, 1);
  __syncthreads();
  // Saved planes 2j .. 2j+3 of step t_ (4P contiguous floats, P % 4 == 0) -> zs.  Warp 0,
  // after a barrier that ends the previous readers of zs.
  unsigned zuse = 0, ziss = 0;
  auto issue_z = [&](int t_, int j_) {
    ++ziss;
    if (tid < 32) {
      const int np = (j_ + 1 < pairs) ? 2 : 1;
      const unsigned bytes = (unsigned)(2 * np * P * sizeof(float));
      if (tid == 0) mbar_expect_tx(zbar, bytes);
      __syncwarp();
      fence_proxy_async();
      const char* src = reinterpret_cast<const char*>(a.zhat + (((size_t)b * g.d + t_) * M + 2 * j_) * P);
      constexpr unsigned kChunk = 4096;
      for (unsigned o = tid * kChunk; o < bytes; o += 32 * kChunk)
        bulk_g2s(reinterpret_cast<char*>(zs) + o, src + o, min(kChunk, bytes - o), zbar);
    }
  };
  if (stage) issue_z(g.d - 1, 0);
  int rpar = 0;                  // block_sum8 half
  FFTF_T0();

  // output step (t = d-1): the port cells' plane gradients and parameter gradients
  // (kernels_pallas.py:1378-1504); universe mode: the last step's cell gradient instead
  if (a.guroi) {
    for (int p = tid; p < g.P; p += nt) gy[p] = a.guroi[(size_t)b * P + p];
  } else {
    const float* ZH = a.zhat + ((size_t)b * g.d + (g.d - 1)) * M * P;
    for (int jo = tid; jo < g.n_out; jo += nt) {
      const int idx = a.out_index[jo];
      const int gr_ = idx / g.W, gc_ = idx - (idx / g.W) * g.W;
      const int p = (gr_ - g.pad_h) * g.roi_w + (gc_ - g.pad_w);
      if (gr_ < g.pad_h || gr_ >= g.pad_h + g.roi_h || gc_ < g.pad_w || gc_ >= g.pad_w + g.roi_w) continue;
      pmap[p] = (int16_t)jo;
      const float go = a.gout[(size_t)b * g.n_out + jo];
      const float wo = a.sp.weff[p], so = a.sp.seff[p], bo = a.sp.broi[p];
      float lin = 0.f;
      for (int m = 0; m < g.M; ++m) lin += ZH[m * P + p];
      if (g.fact == NC_ACT_NONE) {
        gp0[p] += go * lin;
        gp1[p] += go * (lin + (float)g.M * bo);
        gp2[p] += go * (float)g.M * so;
        for (int m = 0; m < g.M; ++m) gport[jo * g.M + m] = (wo + so) * go;
      } else {
        float act = 0.f;
        for (int m = 0; m < g.M; ++m) act += act_fwd(g.fact, ZH[m * P + p] + bo, g.fslope);
        float dpre;
        act_fwd_deriv(g.fact, wo * lin + so * act, g.fslope, &dpre);
        const float gpre = go * dpre;
        gp0[p] += gpre * lin;
        gp1[p] += gpre * act;
        float db = 0.f;
        for (int m = 0; m < g.M; ++m) {
          float dd;
          act_fwd_deriv(g.fact, ZH[m * P + p] + bo, g.fslope, &dd);
          gport[jo * g.M + m] = gpre * (wo + so * dd);
          db += gpre * so * dd;
        }
        gp2[p] += db;
      }
    }
  }
  __syncthreads();
  FFTF_MARK(1, 0);

  // column-pass lanes: warp w takes columns 2w, 2w+1 of both planes; lanes 0-15 plane 0,
  // lanes 16-31 plane 1 (lane ^ 16 holds the same positions of the other plane)
  const int cj = lane & 7, ccol = 2 * warp + ((lane >> 3) & 1), cpl = lane >> 4;

  for (int t = g.d - 1; t >= 0; --t) {
    const bool last = (t == g.d - 1);
    if (t > 0)
      for (int i = tid; i < kPlane; i += nt) D[i] = make_float2(0.f, 0.f);
    FFTF_MARK(1, 1);
    const float* ZH = a.zhat + ((size_t)b * g.d + t) * M * P;
    const float2* Xs = a.xspec + ((size_t)b * g.d + t) * kPlane;
    // universe mode runs the last step's ROI epilogue with the final activation
    const int act_id = last ? (FACT != kActRuntime ? FACT : g.fact) : (ACT != kActRuntime ? ACT : g.act);
    const float slope = last ? g.fslope : g.slope;

    for (int j = 0; j < pairs; j += 2) {
      const bool two = j + 1 < pairs;
      const bool mine = half == 0 || two;
      const float* zp = stage ? zs : ZH + (size_t)(2 * j) * P;   // planes 2j .. 2j+3
      if (stage) {
        mbar_wait(zbar, zuse & 1u, a.sp.status, abort_flag);
        ++zuse;
      }
      FFTF_MARK(1, 9);
      // plane gradients before the standardisation adjoint at plane positions
      // i = tid + 1024 k (row i / 64, column i % 64; zero outside the ROI) of both pairs,
      // stored raw, and their moments
      float mo[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k = 0; k < kPosPerThread; ++k) {
        const int i = tid + k * kThreadsF, r = i >> 6, c = i & (kN - 1);
        float2 v0 = make_float2(0.f, 0.f), v1 = v0;
        if (r < g.roi_h && c < g.roi_w) {
          const int p = r * g.roi_w + c;
          const float h0 = zp[p], h1 = zp[P + p];
          const float h2 = two ? zp[2 * P + p] : 0.f, h3 = two ? zp[3 * P + p] : 0.f;
          if (last && !a.guroi) {
            const int jo = pmap[p];
            if (jo >= 0) {
              const float* gq = gport + jo * g.M + 2 * j;
              v0 = make_float2(gq[0], gq[1]);
              if (two) v1 = make_float2(gq[2], gq[3]);
            }
          } else {
            const float y = gy[p], bb = bsm[p], wy = wsm[p] * y, sy = ssm[p] * y;
            float d0, d1, d2 = 0.f, d3 = 0.f;
            float as = act_fwd_deriv(act_id, h0 + bb, slope, &d0) + act_fwd_deriv(act_id, h1 + bb, slope, &d1);
            float hs = h0 + h1;
            if (two) {
              as += act_fwd_deriv(act_id, h2 + bb, slope, &d2) + act_fwd_deriv(act_id, h3 + bb, slope, &d3);
              hs += h2 + h3;
            }
            v0 = make_float2(fmaf(sy, d0, wy), fmaf(sy, d1, wy));
            v1 = make_float2(fmaf(sy, d2, wy), fmaf(sy, d3, wy));
            // pixel-parameter gradients, summed over the round's directions
            gp0[p] = fmaf(y, hs, gp0[p]);
            gp1[p] = fmaf(y, as, gp1[p]);
            gp2[p] = fmaf(sy, (d0 + d1) + (d2 + d3), gp2[p]);
          }
          mo[0] += v0.x; mo[1] = fmaf(v0.x, h0, mo[1]);
          mo[2] += v0.y; mo[3] = fmaf(v0.y, h1, mo[3]);
          mo[4] += v1.x; mo[5] = fmaf(v1.x, h2, mo[5]);
          mo[6] += v1.y; mo[7] = fmaf(v1.y, h3, mo[7]);
        }
        W[at2(r, c)] = v0;
        W[kPlane + at2(r, c)] = v1;
      }
      FFTF_MARK(1, 2);
      if (g.norm) {
        block_sum8(mo, red, rpar);       // its barriers also publish the raw stores
        if (stage && *abort_flag) {      // uniform: set before the barriers above
          mbar_drain(zbar, zuse, ziss);
          return;
        }
        // the standardisation adjoint gz = rs (v - mean(v) - z^ mean(v z^)) per plane
        const float inv_n = 1.0f / (float)g.P;
        const size_t rb = ((size_t)b * g.d + t) * M + 2 * j;
        const float r0 = a.rstd[rb], r1 = a.rstd[rb + 1];
        const float r2 = two ? a.rstd[rb + 2] : 0.f, r3 = two ? a.rstd[rb + 3] : 0.f;
#pragma unroll
        for (int k = 0; k < kPosPerThread; ++k) {
          const int i = tid + k * kThreadsF, r = i >> 6, c = i & (kN - 1);
          if (r >= g.roi_h || c >= g.roi_w) continue;
          const int p = r * g.roi_w + c, o = at2(r, c);
          const float2 v0 = W[o], v1 = W[kPlane + o];
          W[o] = make_float2(r0 * (v0.x - mo[0] * inv_n - zp[p] * (mo[1] * inv_n)),
                             r1 * (v0.y - mo[2] * inv_n - zp[P + p] * (mo[3] * inv_n)));
          if (two)
            W[kPlane + o] = make_float2(r2 * (v1.x - mo[4] * inv_n - zp[2 * P + p] * (mo[5] * inv_n)),
                                        r3 * (v1.y - mo[6] * inv_n - zp[3 * P + p] * (mo[7] * inv_n)));
        }
      }
      __syncthreads();
      if (stage && *abort_flag) {
        mbar_drain(zbar, zuse, ziss);
        return;
      }
      if (stage) {                       // the next round's planes land during this round
        if (j + 2 < pairs) issue_z(t, j + 2);
        else if (t > 0) issue_z(t - 1, 0);
      }
      FFTF_MARK(1, 3);
      // Q^ = FFT(gz_{2(j+h)} + i gz_{2(j+h)+1}): rows of the ROI, then the columns
      if (mine) fft64::pass64<false, false>(W + half * kPlane, g.roi_h, stw, Ln);
      __syncthreads();
      FFTF_MARK(1, 4);
      {
        const bool cact = cpl == 0 || two;
        float2* Wc = W + cpl * kPlane;
        float2 q[8];
#pragma unroll
        for (int n = 0; n < 8; ++n) q[n] = cact ? Wc[at2(cj + 8 * n, ccol)] : make_float2(0.f, 0.f);
        fft64::fft64_lanes<false>(q, cj, stw);
        if (t > 0) {
          // D += Q^_j . conj(H_j) + Q^_{j+1} . conj(H_{j+1}): plane-0 lanes add the partner's
          // term (lane ^ 16) to their own and update D
          const float2* Hc = a.H + (size_t)(j + cpl) * kPlane;
#pragma unroll
          for (int n = 0; n < 8; ++n) {
            const int o = at2(cj + 8 * n, ccol);
            const float2 dv = cact ? cmulc(q[n], __ldg(&Hc[o])) : make_float2(0.f, 0.f);
            const float ox = __shfl_xor_sync(0xffffffffu, dv.x, 16);
            const float oy = __shfl_xor_sync(0xffffffffu, dv.y, 16);
            if (cpl == 0) D[o] = cadd(D[o], make_float2(dv.x + ox, dv.y + oy));
          }
        }
        // X^ . conj(Q^) (filter adjoint), then the inverse column pass in registers
#pragma unroll
        for (int n = 0; n < 8; ++n) q[n] = cmulc(__ldg(&Xs[at2(cj + 8 * n, ccol)]), q[n]);
        fft64::fft64_lanes<true>(q, cj, stw);
        if (cact) {
#pragma unroll
          for (int n = 0; n < 8; ++n) Wc[at2(cj + 8 * n, ccol)] = q[n];
        }
      }
      __syncthreads();
      FFTF_MARK(1, 5);
      // corr(X, gz_{2m}) - i corr(X, gz_{2m+1}) at lags [0, kh) x [0, kw) for pair m = j + h:
      // inverse row pass of the first kh rows (warps beyond them skip), kept in registers
      if (mine) {
        const bool lagok = Ln.row < g.kh;
        if (__any_sync(0xffffffffu, lagok)) {
          const float2* Wh = W + half * kPlane;
          float2 w[8];
#pragma unroll
          for (int n = 0; n < 8; ++n) w[n] = lagok ? Wh[at2(Ln.row, Ln.j + 8 * n)] : make_float2(0.f, 0.f);
          fft64::fft64_lanes<true>(w, Ln.j, stw);
          if (lagok) {
            const int m1 = 2 * (j + half), m2 = m1 + 1;
#pragma unroll
            for (int n = 0; n < 8; ++n) {
              const int vv = Ln.j + 8 * n;
              if (vv >= g.kw) continue;
              const int k = Ln.row * g.kw + vv;
              dg[(size_t)m1 * g.K + k] += w[n].x * kInvNN;
              dg[(size_t)m2 * g.K + k] -= w[n].y * kInvNN;
            }
          }
        }
      }
      __syncthreads();
      FFTF_MARK(1, 6);
    }
    if (t == 0) break;

    // field adjoint of step t: Re IFFT(D) on the field rows
    inv2d_h0(D, g.Fh, stw, Ln, half);
    for (int p = tid; p < g.P; p += nt) {
      const int r = p / g.roi_w, c = p - (p / g.roi_w) * g.roi_w;
      float s;
      if (g.padding != NC_PAD_CIRCULAR) {
        s = D[at2(r + g.oh, c + g.ow)].x;
      } else {
        s = 0.f;
        for (int fr = (r + g.oh) % g.roi_h; fr < g.Fh; fr += g.roi_h)
          for (int fc = (c + g.ow) % g.roi_w; fc < g.Fw; fc += g.roi_w) s += D[at2(fr, fc)].x;
      }
      gy[p] = s;
    }
    if (ring) {
      for (int i = tid; i < FF; i += nt) {
        const int fr = i / g.Fw, fc = i - (i / g.Fw) * g.Fw;
        const int r = fr - g.oh, c = fc - g.ow;
        if (r >= 0 && r < g.roi_h && c >= 0 && c < g.roi_w) continue;
        ring[i] += D[at2(fr, fc)].x;
      }
    }
    __syncthreads();
    FFTF_MARK(1, 7);
  }

  // per-sample partials; the batch sums run in fixed order afterwards
  float* gpx = a.gpix + (size_t)b * 3 * P;
  for (int p = tid; p < g.P; p += nt) { gpx[p] = gp0[p]; gpx[P + p] = gp1[p]; gpx[2 * P + p] = gp2[p]; }
  float* gd = a.gdpart + (size_t)b * M * g.K;
  for (int i = tid; i < (int)(M * g.K); i += nt) gd[i] = dg[i];
  FFTF_MARK(1, 8);
}

// H_j(w) = conj(G^_{2j}(w)) + i conj(G^_{2j+1}(w)) = F_j(-w) / 64^2 with
// F_j = FFT(g_{2j} + i g_{2j+1}) (both filters real); one CTA per direction pair.  The taps
// are gated here (geff_tap), so the spectra do not wait for the pre-step kernel.
__device__ __forceinline__ void pair_spectra_cta(const Geo& g, const float* __restrict__ filters,
                                                 float2* __restrict__ H, int j, float2* plane, float2* stw) {
  const int tid = threadIdx.x, nt = blockDim.x;
  fft64::init_tw64(stw, tid);
  const fft64::Lane Ln = fft64::lane_of(tid);
  const int k1 = 2 * j * g.K, k2 = k1 + g.K;
  for (int i = tid; i < kN * kN; i += nt) {
    const int r = i / kN, c = i - (i / kN) * kN;
    plane[at2(r, c)] = (r < g.kh && c < g.kw)
                           ? make_float2(geff_tap(g, filters, k1 + r * g.kw + c), geff_tap(g, filters, k2 + r * g.kw + c))
                           : make_float2(0.f, 0.f);
  }
  fwd2d(plane, g.kh, stw, Ln);
  float2* Hj = H + (size_t)j * kPlane;             // stored in the on-chip plane layout
  for (int i = tid; i < kPlane; i += nt) {
    const int r = i / fft64::kLS, c = i - (i / fft64::kLS) * fft64::kLS;
    float2 v = make_float2(0.f, 0.f);
    if (c < kN) {
      v = plane[at2((kN - r) & (kN - 1), (kN - c) & (kN - 1))];
      v = make_float2(v.x * kInvNN, v.y * kInvNN);
    }
    Hj[i] = v;
  }
}

// The pre-step fusion and the pair spectra in one launch: CTAs [0, M/2) build H_j, the
// others run the per-cell pre-step (nc_prestep.cuh) and write the gated filters.
__global__ void __launch_bounds__(kThreads, 1) fftf_prestep_spectra_kernel(
    Geo g, StepParams sp, const float* __restrict__ cell, const float* __restrict__ filters,
    const uint8_t* __restrict__ io, const uint8_t* __restrict__ owm, const uint8_t* __restrict__ bmask,
    nc_codd codd, float2* __restrict__ H) {
  __shared__ float2 plane[kPlane];
  __shared__ float2 stw[kN];
  const int pairs = g.M / 2;
  if (blockIdx.x == 0 && threadIdx.x == 0 && sp.status) *sp.status = 0;   // a new forward call starts
  if ((int)blockIdx.x < pairs) {
    pair_spectra_cta(g, filters, H, blockIdx.x, plane, stw);
    return;
  }
  const int i = ((int)blockIdx.x - pairs) * blockDim.x + threadIdx.x;
  if (i < g.H * g.W) prestep_cell(g, sp, cell, io, owm, bmask, codd, i);
  const int stride = ((int)gridDim.x - pairs) * blockDim.x;
  for (int j = i; j < g.M * g.K; j += stride) sp.geff[j] = geff_tap(g, filters, j);
}

nc_status launched(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, what);
  note_launch();
  return NC_OK;
}

}  // namespace

size_t fftf_fwd_smem(const Geo& g, bool stage) {
  return 16 + sizeof(float2) * (kN + (3 + (stage ? 2 : 0)) * (size_t)kPlane + 4 * kN + 8) +
         sizeof(float) * 3 * (size_t)g.P;
}

// The ring gradient accumulates in global memory, so `ring` does not change the size.
size_t fftf_bwd_smem(const Geo& g, bool ring, bool stage) {
  (void)ring;
  const size_t f = (size_t)2 * kRedHalf + (stage ? 4 * (size_t)g.P : 0) + 7 * (size_t)g.P +
                   (size_t)g.M * g.K + (size_t)g.n_out * g.M;
  return 16 + sizeof(float2) * (kN + 3 * (size_t)kPlane) + sizeof(float) * f + sizeof(int16_t) * (size_t)g.P + 16;
}

bool fftf_fits(const Geo& g) {
  if (g.Nh != kN || g.Nw != kN || g.M % 2 != 0 || g.P > 32767) return false;
  return fftf_fwd_smem(g, false) <= kFftfSmemMax && fftf_bwd_smem(g, false, false) <= kFftfSmemMax;
}

nc_status fftf_prestep_spectra(const Geo& g, const StepParams& sp, const float* cell, const float* filters,
                               const uint8_t* io, const uint8_t* owm, const uint8_t* bmask,
                               const nc_codd& codd, float2* H, cudaStream_t st) {
  const int HW = g.H * g.W;
  const int grid = g.M / 2 + (HW + kThreads - 1) / kThreads;
  fftf_prestep_spectra_kernel<<<grid, kThreads, 0, st>>>(g, sp, cell, filters, io, owm, bmask, codd, H);
  return launched("fftf_prestep_spectra_kernel launch");
}

// The tanh hidden / identity final activation pair runs the specialised kernels.
static bool fixed_acts(const Geo& g) { return g.act == NC_ACT_TANH && g.fact == NC_ACT_NONE; }

nc_status fftf_forward(const FftfArgs& args, cudaStream_t st) {
  FftfArgs a = args;
  a.stage = fftf_fwd_smem(a.g, true) <= kFftfSmemMax ? 1 : 0;
  const size_t smem = fftf_fwd_smem(a.g, a.stage != 0);
  const void* fn = fixed_acts(a.g) ? (const void*)fftf_fwd_kernel<NC_ACT_TANH, NC_ACT_NONE>
                                   : (const void*)fftf_fwd_kernel<kActRuntime, kActRuntime>;
  NC_CUDA_CHECK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  void* kargs[] = {&a};
  PdlLaunch l(dim3(a.batch), dim3(kThreadsF), smem, st);
  NC_CUDA_CHECK(cudaLaunchKernelExC(&l.cfg, fn, kargs));
  return launched("fftf_fwd_kernel launch");
}

nc_status fftf_backward(const FftfArgs& args, cudaStream_t st) {
  FftfArgs a = args;
  const bool ring = a.gring != nullptr;
  a.stage = (a.g.P % 4 == 0 && fftf_bwd_smem(a.g, ring, true) <= kFftfSmemMax) ? 1 : 0;
  if (!a.xspec || !a.zhat) return set_error(NC_ERR_INVALID, "fused FFT backward needs the forward's saved spectra and planes");
  const size_t smem = fftf_bwd_smem(a.g, ring, a.stage != 0);
  const void* fn = fixed_acts(a.g) ? (const void*)fftf_bwd_kernel<NC_ACT_TANH, NC_ACT_NONE>
                                   : (const void*)fftf_bwd_kernel<kActRuntime, kActRuntime>;
  NC_CUDA_CHECK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  void* kargs[] = {&a};
  PdlLaunch l(dim3(a.batch), dim3(kThreadsF), smem, st);
  NC_CUDA_CHECK(cudaLaunchKernelExC(&l.cfg, fn, kargs));
  return launched("fftf_bwd_kernel launch");
}

}  // namespace nc

#if NC_PHASE_TIMING
// Debug builds only: copies (and clears) the fused-FFT phase clocks, 2 x 16 long longs.
extern "C" int nc_debug_fftf_phases(long long* out) {
  if (cudaMemcpyFromSymbol(out, nc::g_fftf_phase, sizeof(long long) * 32) != cudaSuccess) return 1;
  static const long long zero[32] = {};
  if (cudaMemcpyToSymbol(nc::g_fftf_phase, zero, sizeof(zero)) != cudaSuccess) return 1;
  return 0;
}
#endif
