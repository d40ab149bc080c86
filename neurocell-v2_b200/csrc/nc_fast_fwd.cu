// nc_fast_fwd.cu -- register-tiled fused forward for M = 16 directions (sm_100a).
//
// One CTA owns one sample for all d steps.  Thread <-> (8-row vertical strip of the ROI,
// column, group of MT directions): the LP = 16/MT lanes of a pixel strip are adjacent, so
// each holds MT x 8 accumulators.  Each (u, v) tap costs MT/4 broadcast float4 filter loads
// and 1 field load for 8*MT FMAs; the kernel-row loop slides an 8-row window down the
// field column in unrolled chunks of 8 rows.  MT = 4 gives 1024 threads (32 warps) per CTA
// with at most 64 registers each: twice the warps of MT = 8 to hide shared-memory latency.
// The response planes never leave registers: plane statistics are block reductions, the
// direction groups of a pixel are combined with lane shuffles, and the epilogue writes the
// next field straight into shared memory.  Numerics follow neurocell/epilogue.py:28-128
// with the centred two-pass variance of neurocell/kernels_pallas.py:200-205.
#include "nc_fast_dev.cuh"

namespace nc {
namespace fast {

#ifndef NC_FWD_MT
#define NC_FWD_MT 8            // directions per thread (8 -> 512 threads, 4 -> 1024)
#endif

constexpr int FR = 8;          // rows per strip

template <int KH, int KW, int MT>
struct FwdCfg {
  static constexpr int LP = M / MT;              // lanes per pixel strip
  static constexpr int NTF = 256 * LP;           // threads per CTA
  static constexpr int NWF = NTF / 32;
};

template <int KH, int KW, int MT>
__global__ void __launch_bounds__(FwdCfg<KH, KW, MT>::NTF, 1) fwd_kernel_mt(FwdArgs a) {
  using C = FwdCfg<KH, KW, MT>;
  constexpr int K = KH * KW;
  constexpr int LP = C::LP, NTF = C::NTF, NWF = C::NWF;
  extern __shared__ __align__(16) float sm[];
  const Geo& g = a.g;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.x;
  const int P = g.P, RW = g.roi_w, ROWS = g.roi_h;
  const int FS = g.Fw;
  const int FROWS = g.Fh + FR;
  float* Gt = sm;                                   // [k][m]
  float* F = Gt + K * M;                            // FROWS x FS
  int* pmap = reinterpret_cast<int*>(F + FROWS * FS);
  float* red = reinterpret_cast<float*>(pmap + P);  // NWF * M
  float* s_mean = red + NWF * M;
  float* s_rstd = s_mean + M;

  for (int i = tid; i < K * M; i += NTF) {
    const int k = i / M, m = i - k * M;
    Gt[i] = a.sp.geff[m * K + k];
  }
  for (int p = tid; p < P; p += NTF) pmap[p] = -1;
  inject(g, F, FS, FROWS, a.in_index, a.inputs + (size_t)b * g.n_in);
  for (int j = tid; j < g.n_out; j += NTF) {
    const int p = out_pixel(g, a.out_index[j]);
    if (p >= 0) pmap[p] = j;
    else a.out[(size_t)b * g.n_out + j] = __int_as_float(0x7fc00000);   // border output: NaN
  }
  if (g.padding == NC_PAD_CIRCULAR) wrap_ring(g, F, FS);
  __syncthreads();

  const int h = tid % LP;                // direction group: m in [MT*h, MT*h + MT)
  const int item = tid / LP;
  const int nstrip = (ROWS + FR - 1) / FR;
  const bool active = item < nstrip * RW;
  const int s = active ? item / RW : 0;
  const int c = active ? item - s * RW : 0;
  const int r0 = s * FR;
  bool pv[FR];
#pragma unroll
  for (int i = 0; i < FR; ++i) pv[i] = active && (r0 + i < ROWS);
  const float inv_p = 1.0f / (float)P;
  const int m0 = MT * h;

  for (int t = 0; t < g.d; ++t) {
    NC_PHASE_MARK(t, 0);
    float acc[MT][FR];   // acc[k][i] = z[m0+k] at row r0+i
#pragma unroll
    for (int k = 0; k < MT; ++k)
#pragma unroll
      for (int i = 0; i < FR; ++i) acc[k][i] = 0.f;

    if (active) {
      // the window slot of field row r0+u+i is (u+i) % FR; row r0+u+FR replaces r0+u
      auto tap = [&](const float* grow, float (&w)[FR], int du, const float* next) {
        const float4* gp = reinterpret_cast<const float4*>(grow + m0);
#pragma unroll
        for (int q4 = 0; q4 < MT / 4; ++q4) {
          const float4 gg = gp[q4];
#pragma unroll
          for (int i = 0; i < FR; ++i) {
            const float x = w[(du + i) % FR];
            acc[4 * q4 + 0][i] = fmaf(gg.x, x, acc[4 * q4 + 0][i]);
            acc[4 * q4 + 1][i] = fmaf(gg.y, x, acc[4 * q4 + 1][i]);
            acc[4 * q4 + 2][i] = fmaf(gg.z, x, acc[4 * q4 + 2][i]);
            acc[4 * q4 + 3][i] = fmaf(gg.w, x, acc[4 * q4 + 3][i]);
          }
        }
        if (next) w[du % FR] = *next;
      };
      constexpr int KHC = (KH / FR) * FR;
#pragma unroll 1
      for (int v = 0; v < KW; ++v) {
        const float* col = F + r0 * FS + c + v;
        float w[FR];
#pragma unroll
        for (int i = 0; i < FR; ++i) w[i] = col[i * FS];
#pragma unroll 1
        for (int u0 = 0; u0 < KHC; u0 += FR) {
#pragma unroll
          for (int du = 0; du < FR; ++du) {
            const int u = u0 + du;
            tap(Gt + (u * KW + v) * M, w, du, col + (u + FR) * FS);
          }
        }
#pragma unroll
        for (int du = 0; du < KH - KHC; ++du) {
          const int u = KHC + du;
          tap(Gt + (u * KW + v) * M, w, du, (u + 1 < KH) ? col + (u + FR) * FS : nullptr);
        }
      }
    }

    NC_PHASE_MARK(t, 1);
    // plane statistics (centred two-pass); lanes congruent mod LP share a direction group
    auto reduce_group = [&](float (&part)[MT], float* out) {
#pragma unroll
      for (int k = 0; k < MT; ++k) {
        float v = part[k];
#pragma unroll
        for (int o = LP; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        part[k] = v;
      }
      if (lane < LP) {
#pragma unroll
        for (int k = 0; k < MT; ++k) red[warp * M + MT * lane + k] = part[k];
      }
      __syncthreads();
      if (tid < M) {
        float sacc = 0.f;
        for (int w = 0; w < NWF; ++w) sacc += red[w * M + tid];
        out[tid] = sacc * inv_p;
      }
      __syncthreads();
    };
    if (g.norm) {
      float part[MT];
#pragma unroll
      for (int k = 0; k < MT; ++k) {
        float sacc = 0.f;
#pragma unroll
        for (int i = 0; i < FR; ++i) sacc += pv[i] ? acc[k][i] : 0.f;
        part[k] = sacc;
      }
      reduce_group(part, s_mean);
#pragma unroll
      for (int k = 0; k < MT; ++k) {
        const float mu = s_mean[m0 + k];
        float sacc = 0.f;
#pragma unroll
        for (int i = 0; i < FR; ++i) {
          const float d = acc[k][i] - mu;
          sacc += pv[i] ? d * d : 0.f;
        }
        part[k] = sacc;
      }
      reduce_group(part, s_rstd);
      if (tid < M) s_rstd[tid] = 1.0f / sqrtf(s_rstd[tid] + kNormEps);
      __syncthreads();
    } else {
      if (tid < M) { s_mean[tid] = 0.f; s_rstd[tid] = 1.f; }
      __syncthreads();
    }
    if (a.train && tid < M) a.rstd[((size_t)b * g.d + t) * M + tid] = s_rstd[tid];

    NC_PHASE_MARK(t, 2);
    float* ZH = a.train ? a.zhat + ((size_t)b * g.d + t) * (size_t)M * P : nullptr;
    const bool last = (t == g.d - 1);
    const int fact = last ? g.fact : g.act;
    const float fslope = last ? g.fslope : g.slope;
    float* xs = (a.train && !last) ? a.xsave + ((size_t)b * (g.d - 1) + t) * P : nullptr;
#pragma unroll
    for (int i = 0; i < FR; ++i) {
      const int p = (r0 + i) * RW + c;
      const int j = (pv[i] && last) ? pmap[p] : -1;
      const bool need = pv[i] && (!last || ZH || j >= 0);
      const float bb = need ? a.sp.broi[p] : 0.f;
      float lin = 0.f, act = 0.f;
      if (need) {
#pragma unroll
        for (int k = 0; k < MT; ++k) {
          const int m = m0 + k;
          const float zh = (acc[k][i] - s_mean[m]) * s_rstd[m];
          if (ZH) ZH[(size_t)m * P + p] = zh;
          lin += zh;
          if (fact != NC_ACT_NONE) act += act_fwd(fact, zh + bb, fslope);
        }
      }
      // combine the direction groups of this pixel (butterfly: every lane gets the sum)
#pragma unroll
      for (int o = 1; o < LP; o <<= 1) {
        lin += __shfl_xor_sync(0xffffffffu, lin, o);
        act += __shfl_xor_sync(0xffffffffu, act, o);
      }
      if (!pv[i]) continue;
      if (!last) {
        if (g.act == NC_ACT_NONE) act = lin + (float)M * bb;
        const float xn = a.sp.weff[p] * lin + a.sp.seff[p] * act;
        if (i / (FR / LP) == h) {      // lane h writes its share of the strip's rows
          F[(r0 + i + g.oh) * FS + c + g.ow] = xn;
          if (xs) xs[p] = xn;
        }
      } else if (j >= 0 && h == 0) {
        const float wo = a.sp.weff[p], so = a.sp.seff[p];
        const float o = (g.fact == NC_ACT_NONE) ? (wo + so) * lin + ((float)M * so * bb)
                                                : act_fwd(g.fact, wo * lin + so * act, g.fslope);
        a.out[(size_t)b * g.n_out + j] = o;
      }
    }
    if (!last) {
      __syncthreads();
      if (t == 0 && g.padding == NC_PAD_VALID) {
        border_ring(g, F, FS, a.sp.border);
        __syncthreads();
      }
      if (g.padding == NC_PAD_CIRCULAR) {
        wrap_ring(g, F, FS);
        __syncthreads();
      }
    }
    NC_PHASE_MARK(t, 3);
  }
}

}  // namespace fast

FastFwd fast_fwd_select(const Geo& g) {
  using namespace fast;
  FastFwd f{nullptr, 0, 0};
  if (g.M != M) return f;
  const int items = ((g.roi_h + FR - 1) / FR) * g.roi_w;
  const size_t smem = sizeof(float) * ((size_t)g.K * M + (size_t)(g.Fh + FR) * g.Fw + (size_t)g.P +
                                       (size_t)32 * M + 2 * M);
#define NC_FWD_INST(KH_, KW_)                                                        \
  if (g.kh == KH_ && g.kw == KW_) {                                                  \
    using C = FwdCfg<KH_, KW_, NC_FWD_MT>;                                            \
    if (items * C::LP > C::NTF) return f;                                            \
    f.fn = (const void*)fwd_kernel_mt<KH_, KW_, NC_FWD_MT>;                           \
    f.threads = C::NTF;                                                              \
    f.smem = smem;                                                                   \
    return f;                                                                        \
  }
  NC_FWD_INST(23, 13)
#undef NC_FWD_INST
  return f;
}

}  // namespace nc

#if NC_PHASE_TIMING
// Debug builds only: the forward kernel's phase clocks of CTA 0 ([8][8]).
extern "C" int nc_debug_fwd_phase_times(long long* out) {
  return cudaMemcpyFromSymbol(out, nc::fast::g_nc_phase, sizeof(long long) * 64) == cudaSuccess ? 0 : 1;
}
#endif
