// nc_fast.cu -- register-tiled fused forward/backward for M = 16 directions (sm_100a).
//
// Same algorithm and outputs as nc_fused.cu, specialised on the kernel size so that the
// Green's convolution runs at FP32-pipe speed.  One CTA (512 threads) owns one sample for
// all d steps.  Every multiply-add is a packed two-lane FFMA (`__ffma2_rn`, IEEE fma on
// each lane, so results equal scalar fmaf): one issue slot feeds the FP32 pipe for two
// cycles, which keeps the pipe busy while loads and address arithmetic issue in between.
//
//  * forward: thread <-> (4-row vertical strip, column) of the ROI with all 16 directions
//    in registers as 8 direction pairs x 4 rows.  Each (u, v) tap costs 1 field load,
//    1 duplicate move and 4 broadcast float4 filter loads for 32 FFMA2.  The response
//    planes never leave registers: plane statistics are block reductions and the
//    epilogue writes the next field straight into shared memory.
//  * backward: the same mapping computes the plane gradients (output-port or hidden
//    epilogue adjoint, then the standardisation adjoint) into a zero-padded shared buffer
//    that interleaves direction pairs (float2); then
//      dG: thread <-> (direction pair, ROI row group, kernel-row pair) accumulates all kw
//          taps with a kw-deep float2 ring buffer of the two field rows sliding along the
//          columns: 2 field loads, 1 gradient-pair load, 2 moves per 26 FFMA2;
//      dX: thread <-> (ROI row, 10-column strip, direction pair): a 22-wide float2
//          window of plane gradients against 13 filter pairs, 130 FFMA2 per kernel row;
//    partial sums are combined with fixed-order warp shuffles.
// All reductions have a fixed order: results are bitwise reproducible.
#include <cuda_runtime.h>

#include "nc_common.cuh"
#include "nc_fast.cuh"
#include "nc_fast_dev.cuh"
#include "nc_kernels.cuh"

namespace nc {
namespace fast {

using namespace fastc;

// ---------------------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------------------
template <int KH, int KW>
__global__ void __launch_bounds__(NT, 1) bwd_kernel(BwdArgs a, FastBwdLayout L) {
  constexpr int K = KH * KW;
  constexpr int OW = (KW - 1) / 2;
  constexpr int NUP = (KH + 1) / 2;          // kernel-row pairs = dG warps
  constexpr int WIN = CWX + KW - 1;          // dX window width
  extern __shared__ __align__(16) float sm[];
  const Geo& g = a.g;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.x;
  const int P = g.P, RW = g.roi_w, ROWS = g.roi_h;
  float2* Gx = reinterpret_cast<float2*>(sm + L.gx);   // [mp][u][vs]: (G[2mp], G[2mp+1])
  float* F = sm + L.f;                                 // (Fh + 2) x fs
  float2* GZ = reinterpret_cast<float2*>(sm + L.gz);   // [mp] planes of ps, rows of rs (float2)
  float* GY = sm + L.gy;                               // P
  float* red = sm + L.red;                             // NW * 2M
  float* s_rstd = sm + L.stats;
  float* s_c1 = s_rstd + M;
  float* s_c2 = s_c1 + M;
  const int FS = L.fs, RS = L.rs, PS = L.ps, VS = L.vs;

  for (int i = tid; i < MP * KH * VS; i += NT) {
    const int v = i % VS, r = i / VS;           // r = mp * KH + u
    const int mp = r / KH, u = r - mp * KH;
    float2 val = make_float2(0.f, 0.f);
    if (v < KW) {
      val.x = a.sp.geff[(2 * mp) * K + u * KW + v];
      val.y = a.sp.geff[(2 * mp + 1) * K + u * KW + v];
    }
    Gx[i] = val;
  }
  for (int i = tid; i < MP * PS + WIN; i += NT) GZ[i] = make_float2(0.f, 0.f);
  for (int i = tid; i < (g.Fh + 2) * FS; i += NT) F[i] = 0.f;
  __syncthreads();
  if (g.padding == NC_PAD_VALID && g.d > 1) border_ring(g, F, FS, a.sp.border);

  const float inv_p = 1.0f / (float)P;
  float* dg = a.gdpart + (size_t)b * M * K;
  // VALID with d > 1: the plane gradients of steps t >= 1 overwrite the standardised planes
  // they were computed from (store only, no read-modify-write); a batch-and-step reduction
  // sums them afterwards for the border-template adjoint
  const bool keep_gz = a.gdelta != nullptr;

  for (int t = g.d - 1; t >= 0; --t) {
    NC_PHASE_MARK(t, 0);
    // ---- phase A: plane gradients of step t into GZ ---------------------------------------
    // thread <-> pixel, all 16 directions: plane loads and stores are coalesced along the
    // pixel index; per-pixel sums over directions stay in the thread
    float* ZH = a.zhat + ((size_t)b * g.d + t) * (size_t)M * P;
    if (tid < M) s_rstd[tid] = a.rstd[((size_t)b * g.d + t) * M + tid];
    float* gpp = a.gpix + ((size_t)b * g.d + t) * 3 * P;   // this step's pixel partials
    float c1p[M], c2p[M];
#pragma unroll
    for (int m = 0; m < M; ++m) { c1p[m] = 0.f; c2p[m] = 0.f; }
    auto store_gz = [&](int p, const float (&gzh)[M], const float (&z)[M]) {
      const int r = p / RW, cc = p - r * RW;
      float2* gzp = GZ + r * RS + OW + cc;
#pragma unroll
      for (int q = 0; q < MP; ++q) gzp[q * PS] = make_float2(gzh[2 * q], gzh[2 * q + 1]);
#pragma unroll
      for (int m = 0; m < M; ++m) {
        c1p[m] += gzh[m];
        c2p[m] = fmaf(gzh[m], z[m], c2p[m]);
      }
    };
    if (t == g.d - 1) {
      // output step: only port cells carry a gradient (kernels_pallas.py:1107-1179)
      for (int i = tid; i < 3 * P; i += NT) gpp[i] = 0.f;
      __syncthreads();
#pragma unroll 1
      for (int j = tid; j < g.n_out; j += NT) {
        const int p = out_pixel(g, a.out_index[j]);
        if (p < 0) continue;                 // border outputs run in universe mode only
        float z[M], gzh[M];
#pragma unroll
        for (int m = 0; m < M; ++m) z[m] = ZH[(size_t)m * P + p];
        const float go = a.gout[(size_t)b * g.n_out + j];
        const float wo = a.sp.weff[p], so = a.sp.seff[p], bo = a.sp.broi[p];
        float lin = 0.f;
#pragma unroll
        for (int m = 0; m < M; ++m) lin += z[m];
        if (g.fact == NC_ACT_NONE) {
          gpp[p] = go * lin;
          gpp[P + p] = go * (lin + (float)M * bo);
          gpp[2 * P + p] = go * (float)M * so;
#pragma unroll
          for (int m = 0; m < M; ++m) gzh[m] = (wo + so) * go;
        } else {
          float act = 0.f;
#pragma unroll
          for (int m = 0; m < M; ++m) act += act_fwd(g.fact, z[m] + bo, g.fslope);
          float dpre;
          act_fwd_deriv(g.fact, wo * lin + so * act, g.fslope, &dpre);
          const float gpre = go * dpre;
          float db = 0.f;
#pragma unroll
          for (int m = 0; m < M; ++m) {
            float dd;
            act_fwd_deriv(g.fact, z[m] + bo, g.fslope, &dd);
            gzh[m] = gpre * (wo + so * dd);
            db += gpre * so * dd;
          }
          gpp[p] = gpre * lin;
          gpp[P + p] = gpre * act;
          gpp[2 * P + p] = db;
        }
        store_gz(p, gzh, z);
      }
    } else {
      // hidden step t (kernels_pallas.py:221-291); GY holds d loss / d field_{t+1}
#pragma unroll 1
      for (int p = tid; p < P; p += NT) {
        float z[M], gzh[M];
#pragma unroll
        for (int m = 0; m < M; ++m) z[m] = ZH[(size_t)m * P + p];
        const float gy = GY[p];
        const float bb = a.sp.broi[p], we = a.sp.weff[p], se = a.sp.seff[p];
        float lin = 0.f, act = 0.f, dsum = 0.f;
#pragma unroll
        for (int m = 0; m < M; ++m) {
          float dd;
          const float av = act_fwd_deriv(g.act, z[m] + bb, g.slope, &dd);
          lin += z[m];
          act += av;
          dsum += dd;
          gzh[m] = we * gy + se * gy * dd;
        }
        gpp[p] = gy * lin;
        gpp[P + p] = gy * act;
        gpp[2 * P + p] = se * gy * dsum;
        store_gz(p, gzh, z);
      }
    }
    NC_PHASE_MARK(t, 4);
    if (g.norm) {
      // c1 = mean(g zhat), c2 = mean(g zhat * zhat) per plane
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const float s1 = warp_sum(c1p[m]);
        const float s2 = warp_sum(c2p[m]);
        if (lane == 0) {
          red[warp * 2 * M + m] = s1;
          red[warp * 2 * M + M + m] = s2;
        }
      }
      __syncthreads();
      if (tid < 2 * M) {
        float sacc = 0.f;
        for (int w = 0; w < NW; ++w) sacc += red[w * 2 * M + tid];
        if (tid < M) s_c1[tid] = sacc * inv_p;
        else s_c2[tid - M] = sacc * inv_p;
      }
      __syncthreads();
    }
    NC_PHASE_MARK(t, 5);
    // standardisation adjoint GZ <- rstd (GZ - c1 - zhat c2); keep gz for the border adjoint
    if (g.norm || (keep_gz && t >= 1)) {
      if (!g.norm) __syncthreads();
#pragma unroll 1
      for (int p = tid; p < P; p += NT) {
        const int r = p / RW, cc = p - r * RW;
        float2* gzp = GZ + r * RS + OW + cc;
        float z[M];
        if (g.norm) {
#pragma unroll
          for (int m = 0; m < M; ++m) z[m] = ZH[(size_t)m * P + p];
        }
#pragma unroll
        for (int q = 0; q < MP; ++q) {
          float2 v = gzp[q * PS];
          if (g.norm) {
            v.x = s_rstd[2 * q] * (v.x - s_c1[2 * q] - z[2 * q] * s_c2[2 * q]);
            v.y = s_rstd[2 * q + 1] * (v.y - s_c1[2 * q + 1] - z[2 * q + 1] * s_c2[2 * q + 1]);
            gzp[q * PS] = v;
          }
          if (keep_gz && t >= 1) {
            ZH[(size_t)(2 * q) * P + p] = v.x;
            ZH[(size_t)(2 * q + 1) * P + p] = v.y;
          }
        }
      }
    }
    // ---- field entering step t -----------------------------------------------------------
    __syncthreads();
    NC_PHASE_MARK(t, 1);
    if (t == 0) {
      inject(g, F, FS, g.Fh + 2, a.in_index, a.inputs + (size_t)b * g.n_in);
      if (g.padding == NC_PAD_CIRCULAR) wrap_ring(g, F, FS);
    } else {
      const float* xs = a.xsave + ((size_t)b * (g.d - 1) + (t - 1)) * P;
      for (int p = tid; p < P; p += NT) {
        const int r = p / RW, cc = p - (p / RW) * RW;
        F[(r + g.oh) * FS + cc + g.ow] = xs[p];
      }
      if (g.padding == NC_PAD_CIRCULAR) {
        __syncthreads();
        wrap_ring(g, F, FS);
      }
    }
    __syncthreads();
    NC_PHASE_MARK(t, 2);

    // ---- phase B: dG[m,u,v] += sum_{r,c} GZ[m,r,c] F[r+u, c+v]   (warps 0 .. NUP-1) -----
    if (warp < NUP) {
      const int mp = lane >> 2, rg = lane & 3;
      const int u0 = 2 * warp;
      const int rpg = (ROWS + RG - 1) / RG;
      const int rb = rg * rpg, re = min(ROWS, rb + rpg);
      const int ncb = (RW + KW - 1) / KW;
      // acc[x][v] = (dG[2mp+x, u0, v], dG[2mp+x, u0+1, v])
      float2 acc[2][KW];
#pragma unroll
      for (int x = 0; x < 2; ++x)
#pragma unroll
        for (int v = 0; v < KW; ++v) acc[x][v] = make_float2(0.f, 0.f);
#pragma unroll 1
      for (int r = rb; r < re; ++r) {
        const float2* gzr = GZ + mp * PS + r * RS + OW;
        const float* f0 = F + (r + u0) * FS;
        const float* f1 = f0 + FS;
        float2 w[KW];   // w[slot] = (F[r+u0, col], F[r+u0+1, col]), slot = col % KW
#pragma unroll
        for (int v = 0; v < KW - 1; ++v) w[v] = make_float2(f0[v], f1[v]);
#pragma unroll 1
        for (int cb = 0; cb < ncb; ++cb) {
          const int cbase = cb * KW;
#pragma unroll
          for (int j = 0; j < KW; ++j) {
            w[(j + KW - 1) % KW] = make_float2(f0[cbase + j + KW - 1], f1[cbase + j + KW - 1]);
            const float2 gz = gzr[cbase + j];
            const float2 a0 = dup2(gz.x), a1 = dup2(gz.y);
#pragma unroll
            for (int v = 0; v < KW; ++v) {
              const float2 x = w[(j + v) % KW];
              acc[0][v] = ffma2(a0, x, acc[0][v]);
              acc[1][v] = ffma2(a1, x, acc[1][v]);
            }
          }
        }
      }
#pragma unroll
      for (int x = 0; x < 2; ++x)
#pragma unroll
        for (int v = 0; v < KW; ++v) {
          float2 q = acc[x][v];
          q.x += __shfl_xor_sync(0xffffffffu, q.x, 1);
          q.y += __shfl_xor_sync(0xffffffffu, q.y, 1);
          q.x += __shfl_xor_sync(0xffffffffu, q.x, 2);
          q.y += __shfl_xor_sync(0xffffffffu, q.y, 2);
          acc[x][v] = q;
        }
      if (rg == 0) {
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          float* d0 = dg + (2 * mp + x) * K + u0 * KW;
#pragma unroll
          for (int v = 0; v < KW; ++v) d0[v] = (t == g.d - 1) ? acc[x][v].x : d0[v] + acc[x][v].x;
          if (u0 + 1 < KH) {
            float* d1 = d0 + KW;
#pragma unroll
            for (int v = 0; v < KW; ++v) d1[v] = (t == g.d - 1) ? acc[x][v].y : d1[v] + acc[x][v].y;
          }
        }
      }
    }
    NC_WARP_MARK(t, 0);

    // ---- phase C: GY[r,c] = sum_m sum_{u,v} G[m,u,v] GZ[m, r+oh-u, c+ow-v]   (t >= 1) ----
    if (t >= 1) {
      const int nsx = (RW + CWX - 1) / CWX;
      const int nitems = ROWS * nsx * MP;
      // warps NUP.. start first so every SM sub-partition carries the same load
      const int vt = ((warp + NW - NUP) % NW) * 32 + lane;
      for (int it = vt; it < nitems; it += NT) {
        const int mp = it & (MP - 1);
        const int rs_ = it >> 3;
        const int sx = rs_ % nsx, r = rs_ / nsx;
        const int c0 = sx * CWX;
        float2 acc[CWX];
#pragma unroll
        for (int j = 0; j < CWX; ++j) acc[j] = make_float2(0.f, 0.f);
        const float2* plane = GZ + mp * PS;
        const int u_lo = max(0, r + g.oh - ROWS + 1), u_hi = min(KH - 1, r + g.oh);
#pragma unroll 1
        for (int u = u_lo; u <= u_hi; ++u) {
          const float2* row = plane + (r + g.oh - u) * RS + OW + c0 + OW - (KW - 1);
          float2 win[WIN];
#pragma unroll
          for (int q = 0; q < WIN; ++q) win[q] = row[q];
          const float2* gq = Gx + (mp * KH + u) * VS;
#pragma unroll
          for (int v = 0; v < KW; ++v) {
            const float2 wv = gq[v];
#pragma unroll
            for (int j = 0; j < CWX; ++j) acc[j] = ffma2(wv, win[j + KW - 1 - v], acc[j]);
          }
        }
#pragma unroll
        for (int j = 0; j < CWX; ++j) {
          float q = acc[j].x + acc[j].y;
          q += __shfl_xor_sync(0xffffffffu, q, 1);
          q += __shfl_xor_sync(0xffffffffu, q, 2);
          q += __shfl_xor_sync(0xffffffffu, q, 4);
          acc[j].x = q;
        }
        if (mp == 0) {
#pragma unroll
          for (int j = 0; j < CWX; ++j)
            if (c0 + j < RW) GY[r * RW + c0 + j] = acc[j].x;
        }
      }
    }
    NC_WARP_MARK(t, 1);
    __syncthreads();
    NC_PHASE_MARK(t, 3);
  }
}

// ---------------------------------------------------------------------------------------
// dispatch
// ---------------------------------------------------------------------------------------
template <int KH, int KW>
struct Inst {
  static bool fits(const Geo& g) {
    if (g.M != M || g.kh != KH || g.kw != KW) return false;
    if (((g.roi_h + RH - 1) / RH) * g.roi_w > NT) return false;   // backward mapping
    if ((KH + 1) / 2 > NW) return false;
    if (g.P % 4 != 0) return false;   // float4 batch reductions of the per-step partials
    const FastFwd f = fast_fwd_select(g);
    return f.fn && f.smem <= kFastSmemMax && fast_bwd_layout(g, KH, KW).bytes <= kFastSmemMax;
  }
};

}  // namespace fast

// Number of distinct values among {x_i mod m}.
static int distinct_mod(const long* x, int n, long m) {
  int cnt = 0;
  for (int i = 0; i < n; ++i) {
    bool seen = false;
    for (int k = 0; k < i; ++k)
      if (((x[k] % m) + m) % m == ((x[i] % m) + m) % m) seen = true;
    if (!seen) ++cnt;
  }
  return cnt;
}

FastBwdLayout fast_bwd_layout(const Geo& g, int kh, int kw) {
  using namespace fastc;
  FastBwdLayout L;
  const int ow = (kw - 1) / 2;
  const int ncb = (g.roi_w + kw - 1) / kw;
  const int rpg = (g.roi_h + RG - 1) / RG;
  // field stride: the RG row groups of a dG warp read rows rg*rpg apart -> distinct banks
  int fs = ncb * kw + kw - 1;
  if (fs < g.Fw) fs = g.Fw;
  for (int cand = fs; cand < fs + 32; ++cand) {
    long off[RG];
    for (int r = 0; r < RG; ++r) off[r] = (long)r * rpg * cand;
    if (distinct_mod(off, RG, 32) == RG) { fs = cand; break; }
  }
  L.fs = fs;
  // plane-gradient row stride (float2): the 16 lanes of a half-warp (4 pairs x 4 row
  // groups) read pairs (mp * ps + rg * rpg * rs) -> distinct 8-byte bank pairs
  int rs = g.roi_w + 2 * ow;
  int ps = 0;
  bool found = false;
  for (int rc = rs; rc < rs + 16 && !found; ++rc) {
    for (int pc = g.roi_h * rc; pc < g.roi_h * rc + 16; ++pc) {
      long off[16];
      for (int mp = 0; mp < 4; ++mp)
        for (int r = 0; r < RG; ++r) off[mp * RG + r] = (long)mp * pc + (long)r * rpg * rc;
      if (distinct_mod(off, 16, 16) == 16) { rs = rc; ps = pc; found = true; break; }
    }
  }
  if (!found) ps = g.roi_h * rs + 1;
  L.rs = rs;
  L.ps = ps;
  L.vs = (kw + 1) & ~1;
  size_t o = 0;
  auto take = [&](size_t n) { size_t r = o; o += (n + 3) & ~size_t(3); return r; };
  L.gx = take((size_t)MP * kh * L.vs * 2);
  L.f = take((size_t)(g.Fh + 2) * L.fs);
  L.gz = take(((size_t)MP * L.ps + CWX + kw) * 2);
  L.gy = take((size_t)g.P);
  L.red = take((size_t)NW * 2 * M);
  L.stats = take(3 * M + 1);
  L.bytes = o * sizeof(float);
  return L;
}

// Returns the kernels for this geometry, or nullptrs when no specialisation applies.
FastKernels fast_kernels(const Geo& g) {
  FastKernels k{};
#define NC_FAST_INST(KH_, KW_)                                                        \
  if (fast::Inst<KH_, KW_>::fits(g)) {                                                \
    const FastFwd f = fast_fwd_select(g);                                             \
    k.fwd = f.fn;                                                                     \
    k.fwd_smem = f.smem;                                                              \
    k.fwd_threads = f.threads;                                                        \
    k.bwd = (const void*)fast::bwd_kernel<KH_, KW_>;                                  \
    k.bl = fast_bwd_layout(g, KH_, KW_);                                               \
    k.bwd_smem = k.bl.bytes;                                                          \
    return k;                                                                         \
  }
  NC_FAST_INST(23, 13)
#undef NC_FAST_INST
  return k;
}

}  // namespace nc

#if NC_PHASE_TIMING
// Debug builds only: copies the phase clocks of CTA 0 ([8][4] then [8][32][2]) to `out`.
extern "C" int nc_debug_phase_times(long long* out) {
  if (cudaMemcpyFromSymbol(out, nc::fast::g_nc_phase, sizeof(long long) * 64) != cudaSuccess) return 1;
  if (cudaMemcpyFromSymbol(out + 64, nc::fast::g_nc_warp, sizeof(long long) * 512) != cudaSuccess) return 1;
  return 0;
}
#endif
