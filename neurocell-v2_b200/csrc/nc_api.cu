// nc_api.cu -- the extern "C" entry points declared in include/neurocell_b200.h.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <atomic>
#include <cmath>
#include <vector>

#include <cuda_runtime.h>

#include "nc_errors.h"
#include "nc_fast.cuh"
#include "nc_fft.cuh"
#include "nc_fftconv.h"
#include "nc_fftf.h"
#include "nc_internal.h"
#include "nc_kernels.cuh"

namespace nc {

// kernels (nc_fused.cu, nc_aux.cu)
__global__ void vnn_fused_fwd_kernel(FwdArgs a);
__global__ void vnn_fused_bwd_kernel(BwdArgs a);
__global__ void prestep_kernel(Geo g, StepParams sp, const float* cell, const float* filters,
                               const uint8_t* io, const uint8_t* owm, const uint8_t* bmask,
                               nc_codd codd);
__global__ void codd_kernel(int HW, const float* s_raw, const uint8_t* io, int hard_pin,
                            nc_codd codd, float* out);
__global__ void batch_sum_kernel(const float* in, size_t stride, int n, int batch, float* out);
__global__ void batch_step_sum4_kernel(const float* in, int batch, int d, int t0, size_t slot, int n,
                                       int bc, float* part);
__global__ void rows_sum_kernel(const float* part, int rows, int n, float* out);
__global__ void seg_batch_sum1_kernel(SegSum j, int batch, int bc, float* part);

// out[i] = sum_b sum_{t0<=t<d} in[(b*d+t)*slot + i] in two deterministic stages over
// kRedChunks sample chunks (n, slot multiples of 4; `scratch` holds kRedChunks*n floats).
static nc_status batch_step_sum(const float* in, int batch, int d, int t0, size_t slot, int n,
                                float* out, float* scratch, cudaStream_t st) {
  const int chunks = batch < kRedChunks ? batch : kRedChunks;
  const int bc = (batch + chunks - 1) / chunks;
  const int n4 = n / 4;
  dim3 grid((n4 + 255) / 256, chunks);
  batch_step_sum4_kernel<<<grid, 256, 0, st>>>(in, batch, d, t0, slot, n, bc, scratch);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "batch_step_sum4_kernel launch");
  note_launch();
  rows_sum_kernel<<<(n + 255) / 256, 256, 0, st>>>(scratch, chunks, n, out);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "rows_sum_kernel launch");
  note_launch();
  return NC_OK;
}
__global__ void border_grad_kernel(Geo g, const float* G, const float* gdelta, float* gborder);
__global__ void prestep_bwd_kernel(Geo g, StepParams sp, const float* cell, const float* filters,
                                   const uint8_t* owm, const uint8_t* bmask, const float* gsum,
                                   const float* gborder,
                                   const float* gdsum, const float* gring_final, float* gcell,
                                   float* gfilt, int rows, size_t stride);
__global__ void universe_fwd_kernel(Geo g, StepParams sp, const float* cell, const float* uroi,
                                    float* universe, int B);
__global__ void gather_out_kernel(Geo g, const int32_t* out_index, const float* universe, float* out,
                                  int B);
__global__ void universe_bwd_roi_kernel(Geo g, StepParams sp, const float* cell, const float* uroi,
                                        const float* guni, float* guroi, int B);
__global__ void universe_bwd_ring_kernel(Geo g, StepParams sp, const float* cell, const float* guni,
                                         float* gring, int B);
__global__ void universe_bwd_ports_kernel(Geo g, const int32_t* out_index, const float* uroi,
                                          const float* gout, float* guroi, int B);
__global__ void universe_bwd_border_ports_kernel(Geo g, StepParams sp, const float* cell,
                                                 const int32_t* out_index, const float* gout,
                                                 float* gring, int B);
__global__ void universe_embed_fwd_kernel(Geo g, UniWindow wn, const float* cell, const uint8_t* io,
                                          nc_codd codd, const float* uwin, float* universe, int B);
__global__ void universe_embed_bwd_kernel(Geo g, UniWindow wn, const float* cell, const uint8_t* io,
                                          nc_codd codd, const float* guni, float* guwin, float* gcell,
                                          int B);
__global__ void universe_embed_bwd_ports_kernel(Geo g, UniWindow wn, const int32_t* out_index,
                                                const float* cell, const uint8_t* io, nc_codd codd,
                                                const float* gout, float* guwin, float* gcell, int B);
__global__ void mse_kernel(const float* o, const float* y, int n, float* loss, float* g);
__global__ void stage_copy_kernel(StageSegs s);
__global__ void softmax_ce_kernel(const float* x, const int32_t* lab, int batch, int n,
                                  float* loss, float* g);
__global__ void sgd_kernel(float* p, const float* gr, int64_t n, float lr);

static thread_local char g_err[1024];

struct ProfileEvents {
  cudaEvent_t fs = nullptr, fe = nullptr, bs = nullptr, be = nullptr;
};
static thread_local ProfileEvents g_prof;

__global__ void fp32_peak_kernel(int iters, float* sink);

nc_status set_error(nc_status st, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return st;
}

nc_status cuda_error(cudaError_t e, const char* what) {
  return set_error(NC_ERR_CUDA, "%s failed: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

void clear_error() { g_err[0] = 0; }

static std::atomic<uint64_t> g_launches{0};
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

static inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

template <typename T>
static inline T* at(void* base, size_t off) {
  return off == SIZE_MAX ? nullptr : reinterpret_cast<T*>(static_cast<char*>(base) + off);
}
template <typename T>
static inline const T* at(const void* base, size_t off) {
  return off == SIZE_MAX ? nullptr : reinterpret_cast<const T*>(static_cast<const char*>(base) + off);
}

static nc_status check_codd(const nc_codd* c) {
  if (!c) return set_error(NC_ERR_INVALID, "codd options pointer is null");
  if (c->mode < NC_CODD_CONTINUOUS || c->mode > NC_CODD_STE_TERNARY)
    return set_error(NC_ERR_INVALID,
                     "Unsupported codd_mode id %d; choose from (continuous, annealed, ste_binary, ste_ternary)",
                     c->mode);
  if (reinterpret_cast<uintptr_t>(c->temperature_dev) % 4 != 0)
    return set_error(NC_ERR_INVALID, "codd temperature_dev is not 4-byte aligned");
  return NC_OK;
}

// The device address of `p` when the device can access it: device memory, managed memory,
// or page-locked host memory that is mapped into the device's address space (cudaHostAlloc,
// cudaHostRegister with mapping; under unified addressing the same pointer).  Anything else
// (pageable host memory, unknown pointers) is refused on the host, before any launch.
static nc_status device_address(const void* p, const char* name, const void** dev) {
  if (!p) return set_error(NC_ERR_INVALID, "%s is null", name);
  cudaPointerAttributes at;
  cudaError_t e = cudaPointerGetAttributes(&at, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return set_error(NC_ERR_INVALID, "%s: not an address CUDA knows (%s)", name, cudaGetErrorName(e));
  }
  if (at.type == cudaMemoryTypeDevice || at.type == cudaMemoryTypeManaged) {
    *dev = p;
    return NC_OK;
  }
  if (at.type == cudaMemoryTypeHost && at.devicePointer) {
    *dev = at.devicePointer;
    return NC_OK;
  }
  return set_error(NC_ERR_INVALID, "%s is pageable host memory or not mapped for the device; "
                   "pass device memory or page-locked host memory", name);
}

static nc_status check_ptr(const void* p, const char* name) {
  if (!p) return set_error(NC_ERR_INVALID, "%s is null", name);
  if (reinterpret_cast<uintptr_t>(p) % 4 != 0) return set_error(NC_ERR_INVALID, "%s is not 4-byte aligned", name);
  return NC_OK;
}

static StepParams step_params(void* ws, const WsLayout& L) {
  StepParams sp;
  sp.weff = at<float>(ws, L.weff);
  sp.seff = at<float>(ws, L.seff);
  sp.broi = at<float>(ws, L.broi);
  sp.border = at<float>(ws, L.border);
  sp.sprob = at<float>(ws, L.sprob);
  sp.dsprob = at<float>(ws, L.dsprob);
  sp.wpinned = at<float>(ws, L.wpinned);
  sp.geff = at<float>(ws, L.geff);
  sp.status = at<int>(ws, L.status);
  return sp;
}

static size_t fused_smem_bytes(const Geo& g, bool g_smem, bool f_smem, bool big_smem) {
  size_t n = 2 * (size_t)g.M + 32;
  if (g_smem) n += (size_t)g.M * g.K;
  if (f_smem) n += (size_t)g.F_elems;
  if (big_smem) n += (size_t)g.M * g.P;
  return n * sizeof(float);
}

static bool g_fits(const Geo& g) {
  return sizeof(float) * ((size_t)g.M * g.K + 4 * (size_t)g.M + 128) <= kSmemBudget;
}

static nc_status set_smem_attr(const void* fn, size_t bytes) {
  if (bytes <= 48 * 1024) return NC_OK;
  NC_CUDA_CHECK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  return NC_OK;
}

static nc_status launch_check(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, what);
  note_launch();
  return NC_OK;
}

struct Prepared {
  Geo g;
  WsLayout L;
  bool gs, fs, zs, gzs;
  StepParams sp;
  const int32_t* in_index;
  const int32_t* out_index;
  const uint8_t* io;
  const uint8_t* owm;
  const uint8_t* bmask;
  const float2* tw_w;
  const float2* tw_h;
};

static nc_status prepare(const nc_topo* topo, const void* plan, int32_t batch, uint32_t flags,
                         void* ws, size_t ws_bytes, Prepared* pr) {
  NC_CHECK(make_geo(topo, &pr->g));
  if (batch <= 0) return set_error(NC_ERR_INVALID, "batch must be >= 1, got %d", batch);
  if (!plan) return set_error(NC_ERR_INVALID, "plan buffer is null");
  if (!ws) return set_error(NC_ERR_INVALID, "workspace is null");
  if (reinterpret_cast<uintptr_t>(ws) % 256 != 0 || reinterpret_cast<uintptr_t>(plan) % 256 != 0)
    return set_error(NC_ERR_WORKSPACE, "workspace and plan buffers must be 256-byte aligned");
  pr->L = ws_layout(pr->g, batch, flags, &pr->fs, &pr->zs, &pr->gzs);
  pr->gs = g_fits(pr->g);
  if (ws_bytes < pr->L.total)
    return set_error(NC_ERR_WORKSPACE, "workspace too small: %zu bytes given, %zu required", ws_bytes,
                     pr->L.total);
  pr->sp = step_params(ws, pr->L);
  const PlanLayout PL = plan_layout(topo);
  pr->in_index = at<int32_t>(plan, PL.in_index);
  pr->out_index = at<int32_t>(plan, PL.out_index);
  pr->io = at<uint8_t>(plan, PL.io_mask);
  pr->owm = at<uint8_t>(plan, PL.out_w_mask);
  pr->bmask = at<uint8_t>(plan, PL.border_mask);
  pr->tw_w = at<float2>(plan, PL.twid_w);
  pr->tw_h = at<float2>(plan, PL.twid_h);
  return NC_OK;
}

// Arguments of the FFT-regime loop (nc_fftconv.cu) from a prepared call.
static FftCall fft_call(const Prepared& pr, void* ws, const float* inputs, int batch, bool train) {
  FftCall c;
  memset(&c, 0, sizeof(c));
  const WsLayout& L = pr.L;
  c.g = pr.g;
  c.batch = batch;
  c.train = train;
  c.sp = pr.sp;
  c.in_index = pr.in_index;
  c.out_index = pr.out_index;
  c.inputs = inputs;
  c.tw_w = pr.tw_w;
  c.tw_h = pr.tw_h;
  c.field = at<float>(ws, L.f_field);
  c.xhat = at<float2>(ws, L.f_xhat);
  c.tmp = at<float2>(ws, L.f_tmp);
  c.gspec = at<float2>(ws, L.f_gspec);
  c.mean = at<float>(ws, L.f_mean);
  c.rstd = at<float>(ws, L.f_rstd);
  c.rowstats = at<float2>(ws, L.f_rowstats);
  c.gzpart = at<float>(ws, L.f_gzpart);
  c.ncoef = at<float4>(ws, L.f_ncoef);
  c.zscr = at<float>(ws, L.zscr);
  c.zhat = at<float>(ws, L.zhat);
  c.rstd_save = at<float>(ws, L.rstd);
  c.mean_save = at<float>(ws, L.f_mean_save);
  c.xsave = at<float>(ws, L.xsave);
  c.q = at<float2>(ws, L.f_q);
  c.dgacc = at<float2>(ws, L.f_dgacc);
  c.gz = at<float>(ws, L.f_gz);
  c.dx = at<float>(ws, L.f_dx);
  c.gpart = at<float>(ws, L.f_gpart);
  c.gsum = at<float>(ws, L.gsum);
  c.gdsum = at<float>(ws, L.gdsum);
  c.gborder = (pr.g.padding == NC_PAD_VALID && pr.g.d > 1) ? at<float>(ws, L.gborder) : nullptr;
  return c;
}

// Arguments of the fused small-grid FFT kernels (nc_fftf.cu).
static FftfArgs fftf_args(const Prepared& pr, void* ws, const float* inputs, int batch, bool train) {
  FftfArgs a;
  memset(&a, 0, sizeof(a));
  const WsLayout& L = pr.L;
  a.g = pr.g;
  a.sp = pr.sp;
  a.in_index = pr.in_index;
  a.out_index = pr.out_index;
  a.inputs = inputs;
  a.H = at<float2>(ws, L.f_h);
  a.zhat = at<float>(ws, L.zhat);
  a.rstd = at<float>(ws, L.rstd);
  a.xsave = at<float>(ws, L.xsave);
  a.train = train ? 1 : 0;
  a.batch = batch;
  a.gpix = at<float>(ws, L.gpix);
  a.gdpart = at<float>(ws, L.gdpart);
  a.gring = at<float>(ws, L.f_gring);
  a.xspec = at<float2>(ws, L.f_xspec);
  return a;
}

// Universe (B, H, W) from the last step's ROI cells, and the port outputs gathered from it.
static nc_status assemble_universe(const Prepared& pr, const float* cell, const float* uroi,
                                   float* universe, float* out, int batch, cudaStream_t st) {
  const size_t n = (size_t)batch * pr.g.H * pr.g.W;
  universe_fwd_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(pr.g, pr.sp, cell, uroi, universe, batch);
  NC_CHECK(launch_check("universe_fwd_kernel launch"));
  gather_out_kernel<<<(batch * pr.g.n_out + 127) / 128, 128, 0, st>>>(pr.g, pr.out_index, universe, out,
                                                                      batch);
  return launch_check("gather_out_kernel launch");
}

static nc_status launch_prestep(const Prepared& pr, const float* cell, const float* filters,
                                const nc_codd* codd, cudaStream_t st) {
  const int HW = pr.g.H * pr.g.W;
  const int nthreads = 256;
  const int nblocks = (HW + nthreads - 1) / nthreads;
  prestep_kernel<<<nblocks, nthreads, 0, st>>>(pr.g, pr.sp, cell, filters, pr.io, pr.owm, pr.bmask,
                                               *codd);
  return launch_check("prestep_kernel launch");
}

}  // namespace nc

using namespace nc;

extern "C" {

int32_t nc_abi_version(void) { return NC_ABI_VERSION; }

uint64_t nc_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int32_t nc_conv_path(const nc_topo* topo) {
  Geo g;
  if (make_geo(topo, &g) != NC_OK) return 0;
  if (g.algo != NC_CONV_FFT) return 1;
  return fftf_fits(g) ? 3 : 2;
}

const char* nc_last_error(void) { return g_err; }

nc_status nc_workspace_status(const void* d_ws, int32_t* status, void* stream) {
  if (!d_ws || !status) return set_error(NC_ERR_INVALID, "bad nc_workspace_status arguments");
  if (reinterpret_cast<uintptr_t>(d_ws) % 256 != 0)
    return set_error(NC_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  cudaStream_t st = as_stream(stream);
  int v = -1;
  NC_CUDA_CHECK(cudaMemcpyAsync(&v, d_ws, sizeof(int), cudaMemcpyDeviceToHost, st));
  NC_CUDA_CHECK(cudaStreamSynchronize(st));
  *status = v;
  clear_error();
  return NC_OK;
}

size_t nc_plan_bytes(const nc_topo* topo) {
  Geo g;
  if (make_geo(topo, &g) != NC_OK) return 0;
  return plan_layout(topo).total;
}

nc_status nc_plan_build(const nc_topo* topo, const int32_t* in_index, const int32_t* out_index,
                        const uint8_t* io_mask, const uint8_t* out_w_mask,
                        const uint8_t* border_mask, void* d_plan, size_t plan_bytes, void* stream) {
  Geo g;
  NC_CHECK(make_geo(topo, &g));
  const PlanLayout PL = plan_layout(topo);
  if (!d_plan) return set_error(NC_ERR_INVALID, "plan buffer is null");
  if (reinterpret_cast<uintptr_t>(d_plan) % 256 != 0)
    return set_error(NC_ERR_WORKSPACE, "plan buffer must be 256-byte aligned");
  if (plan_bytes < PL.total)
    return set_error(NC_ERR_WORKSPACE, "plan buffer too small: %zu < %zu", plan_bytes, PL.total);
  if ((g.n_in > 0 && !in_index) || !out_index || !io_mask || !out_w_mask)
    return set_error(NC_ERR_INVALID, "null plan table");
  // FFT line twiddles (layouts: nc_fft.cuh): two-stage plans (64 <= N <= 1024) take
  // exp(-2 pi i n2 k1 / N) at [k1 * 64 + n2] then exp(-2 pi i e / 64); radix-4 plans take
  // exp(-2 pi i q j / S) stage by stage
  std::vector<float2> tw[2];
  if (PL.twid_w != SIZE_MAX) {
    for (int side = 0; side < 2; ++side) {
      const int N = side == 0 ? g.Nw : g.Nh;
      if (fft::two_stage(N)) {
        for (int k1 = 0; k1 < N / 64; ++k1)
          for (int n2 = 0; n2 < 64; ++n2) {
            const double a = -2.0 * M_PI * (double)n2 * (double)k1 / (double)N;
            tw[side].push_back(make_float2((float)std::cos(a), (float)std::sin(a)));
          }
        for (int e = 0; e < 64; ++e) {
          const double a = -2.0 * M_PI * (double)e / 64.0;
          tw[side].push_back(make_float2((float)std::cos(a), (float)std::sin(a)));
        }
        continue;
      }
      for (int S = N; S > 1;) {
        const int R = fft::stage_radix(S), h = S / R;
        for (int q = 1; q < R; ++q)
          for (int j = 0; j < h; ++j) {
            const double a = -2.0 * M_PI * (double)q * (double)j / (double)S;
            tw[side].push_back(make_float2((float)std::cos(a), (float)std::sin(a)));
          }
        S /= R;
      }
    }
  }
  const int HW = g.H * g.W;
  for (int j = 0; j < g.n_in; ++j)
    if (in_index[j] >= HW || in_index[j] < -1)
      return set_error(NC_ERR_INVALID, "input index %d out of grid (value %d)", j, in_index[j]);
  for (int j = 0; j < g.n_out; ++j) {
    const int idx = out_index[j];
    if (idx < 0 || idx >= HW) return set_error(NC_ERR_INVALID, "output index %d out of grid", j);
    for (int k = 0; k < j; ++k)
      if (out_index[k] == idx) return set_error(NC_ERR_UNSUPPORTED, "duplicate output cell %d", idx);
  }
  cudaStream_t st = as_stream(stream);
  char* base = static_cast<char*>(d_plan);
  if (g.n_in > 0)
    NC_CUDA_CHECK(cudaMemcpyAsync(base + PL.in_index, in_index, sizeof(int32_t) * g.n_in,
                                  cudaMemcpyHostToDevice, st));
  NC_CUDA_CHECK(cudaMemcpyAsync(base + PL.out_index, out_index, sizeof(int32_t) * g.n_out,
                                cudaMemcpyHostToDevice, st));
  NC_CUDA_CHECK(cudaMemcpyAsync(base + PL.io_mask, io_mask, (size_t)HW, cudaMemcpyHostToDevice, st));
  NC_CUDA_CHECK(cudaMemcpyAsync(base + PL.out_w_mask, out_w_mask, (size_t)HW, cudaMemcpyHostToDevice, st));
  if (border_mask)
    NC_CUDA_CHECK(cudaMemcpyAsync(base + PL.border_mask, border_mask, (size_t)HW, cudaMemcpyHostToDevice, st));
  else
    NC_CUDA_CHECK(cudaMemsetAsync(base + PL.border_mask, 1, (size_t)HW, st));
  if (PL.twid_w != SIZE_MAX) {
    NC_CUDA_CHECK(cudaMemcpyAsync(base + PL.twid_w, tw[0].data(), sizeof(float2) * tw[0].size(),
                                  cudaMemcpyHostToDevice, st));
    NC_CUDA_CHECK(cudaMemcpyAsync(base + PL.twid_h, tw[1].data(), sizeof(float2) * tw[1].size(),
                                  cudaMemcpyHostToDevice, st));
  }
  NC_CUDA_CHECK(cudaStreamSynchronize(st));   // host tables may be freed after return
  return NC_OK;
}

size_t nc_workspace_bytes(const nc_topo* topo, int32_t batch, uint32_t flags) {
  Geo g;
  if (make_geo(topo, &g) != NC_OK || batch <= 0) return 0;
  return ws_layout(g, batch, flags, nullptr, nullptr, nullptr).total;
}

// The forward of both entry points; `universe` (non-null) selects universe mode, in which
// the last step writes its ROI cells to the workspace and the universe is assembled.
static nc_status vnn_forward(const nc_topo* topo, const void* d_plan, const float* cell_params,
                             const float* filters, const float* inputs, int32_t batch,
                             const nc_codd* codd, uint32_t flags, float* out, float* universe,
                             void* d_ws, size_t ws_bytes, void* stream) {
  Prepared pr;
  NC_CHECK(prepare(topo, d_plan, batch, flags, d_ws, ws_bytes, &pr));
  NC_CHECK(check_codd(codd));
  NC_CHECK(check_ptr(cell_params, "cell_params"));
  NC_CHECK(check_ptr(filters, "filters"));
  NC_CHECK(check_ptr(out, "out"));
  if (universe) NC_CHECK(check_ptr(universe, "universe"));
  if (pr.g.n_in > 0) NC_CHECK(check_ptr(inputs, "inputs"));
  cudaStream_t st = as_stream(stream);
  const bool fused_fft = pr.g.algo == NC_CONV_FFT && fftf_fits(pr.g);
  if (fused_fft)   // pre-step and filter-pair spectra in one launch
    NC_CHECK(fftf_prestep_spectra(pr.g, pr.sp, cell_params, filters, pr.io, pr.owm, pr.bmask, *codd,
                                  at<float2>(d_ws, pr.L.f_h), st));
  else
    NC_CHECK(launch_prestep(pr, cell_params, filters, codd, st));
  float* uroi = universe ? at<float>(d_ws, pr.L.uroi) : nullptr;

  const bool train = (flags & NC_FLAG_TRAIN) != 0;
  if (pr.g.algo == NC_CONV_FFT) {
    FftCall c = fft_call(pr, d_ws, inputs, batch, train);
    c.out = out;
    c.uroi = uroi;
    if (fftf_fits(pr.g)) {
      // small grid: direction-pair filter spectra, then one fused kernel per sample
      FftfArgs fa = fftf_args(pr, d_ws, inputs, batch, train);
      fa.out = out;
      fa.uroi = uroi;
      if (g_prof.fs) NC_CUDA_CHECK(cudaEventRecord(g_prof.fs, st));
      NC_CHECK(fftf_forward(fa, st));
      if (g_prof.fe) NC_CUDA_CHECK(cudaEventRecord(g_prof.fe, st));
    } else {
      if (g_prof.fs) NC_CUDA_CHECK(cudaEventRecord(g_prof.fs, st));
      NC_CHECK(fft_forward(c, st));
      if (g_prof.fe) NC_CUDA_CHECK(cudaEventRecord(g_prof.fe, st));
    }
    if (universe) NC_CHECK(assemble_universe(pr, cell_params, uroi, universe, out, batch, st));
    clear_error();
    return NC_OK;
  }
  FwdArgs a;
  memset(&a, 0, sizeof(a));
  a.g = pr.g;
  a.sp = pr.sp;
  a.in_index = pr.in_index;
  a.out_index = pr.out_index;
  a.inputs = inputs;
  a.out = out;
  a.xsave = at<float>(d_ws, pr.L.xsave);
  a.zhat = at<float>(d_ws, pr.L.zhat);
  a.rstd = at<float>(d_ws, pr.L.rstd);
  a.fscr = at<float>(d_ws, pr.L.fscr);
  a.zscr = at<float>(d_ws, pr.L.zscr);
  a.uroi = uroi;
  a.train = train ? 1 : 0;
  a.g_smem = pr.gs ? 1 : 0;
  a.f_smem = (pr.gs && pr.fs) ? 1 : 0;
  a.z_smem = (a.f_smem && pr.zs) ? 1 : 0;
  a.batch = batch;
  if (!a.f_smem && !a.fscr)
    return set_error(NC_ERR_UNSUPPORTED, "field does not fit on chip and no scratch was laid out");
  if (!a.z_smem && !train && !a.zscr)
    return set_error(NC_ERR_UNSUPPORTED, "planes do not fit on chip and no scratch was laid out");
  // universe mode runs the generic kernels (the specialised ones end in the port epilogue)
  const FastKernels fk = universe ? FastKernels{} : fast_kernels(pr.g);
  const void* fn = fk.fwd ? fk.fwd : (const void*)vnn_fused_fwd_kernel;
  const size_t smem = fk.fwd ? fk.fwd_smem : fused_smem_bytes(pr.g, a.g_smem, a.f_smem, a.z_smem);
  NC_CHECK(set_smem_attr(fn, smem));
  if (g_prof.fs) NC_CUDA_CHECK(cudaEventRecord(g_prof.fs, st));
  {
    void* args[] = {&a};
    const int threads = fk.fwd ? fk.fwd_threads : kFusedThreads;
    NC_CUDA_CHECK(cudaLaunchKernel(fn, dim3(batch), dim3(threads), args, smem, st));
  }
  NC_CHECK(launch_check("fused forward kernel launch"));
  if (g_prof.fe) NC_CUDA_CHECK(cudaEventRecord(g_prof.fe, st));
  if (universe) NC_CHECK(assemble_universe(pr, cell_params, uroi, universe, out, batch, st));
  clear_error();
  return NC_OK;
}

nc_status nc_vnn_forward(const nc_topo* topo, const void* d_plan, const float* cell_params,
                         const float* filters, const float* inputs, int32_t batch,
                         const nc_codd* codd, uint32_t flags, float* out, void* d_ws,
                         size_t ws_bytes, void* stream) {
  return vnn_forward(topo, d_plan, cell_params, filters, inputs, batch, codd, flags, out, nullptr, d_ws,
                     ws_bytes, stream);
}

nc_status nc_vnn_forward_universe(const nc_topo* topo, const void* d_plan, const float* cell_params,
                                  const float* filters, const float* inputs, int32_t batch,
                                  const nc_codd* codd, uint32_t flags, float* out, float* universe,
                                  void* d_ws, size_t ws_bytes, void* stream) {
  if (!universe) return set_error(NC_ERR_INVALID, "universe is null");
  return vnn_forward(topo, d_plan, cell_params, filters, inputs, batch, codd, flags, out, universe,
                     d_ws, ws_bytes, stream);
}

// The backward of both entry points; g_universe (non-null) selects universe mode.
static nc_status vnn_backward(const nc_topo* topo, const void* d_plan, const float* cell_params,
                              const float* filters, const float* inputs, int32_t batch,
                              const nc_codd* codd, const float* g_out, const float* g_universe,
                              float* g_cell_params, float* g_filters, void* d_ws, size_t ws_bytes,
                              void* stream) {
  Prepared pr;
  NC_CHECK(prepare(topo, d_plan, batch, NC_FLAG_TRAIN, d_ws, ws_bytes, &pr));
  NC_CHECK(check_codd(codd));
  NC_CHECK(check_ptr(cell_params, "cell_params"));
  NC_CHECK(check_ptr(filters, "filters"));
  NC_CHECK(check_ptr(g_universe ? g_universe : g_out, g_universe ? "g_universe" : "g_out"));
  if (g_universe && g_out) NC_CHECK(check_ptr(g_out, "g_out"));
  NC_CHECK(check_ptr(g_cell_params, "g_cell_params"));
  NC_CHECK(check_ptr(g_filters, "g_filters"));
  if (pr.g.n_in > 0) NC_CHECK(check_ptr(inputs, "inputs"));
  cudaStream_t st = as_stream(stream);
  const Geo& g = pr.g;
  const WsLayout& L = pr.L;
  float* guroi = nullptr;
  float* gringf = nullptr;
  if (g_universe) {
    // universe adjoint: the last step's ROI-cell gradient and the VALID ring gradient
    const float* uroi = at<float>(d_ws, L.uroi);
    guroi = at<float>(d_ws, L.guroi);
    const size_t n = (size_t)batch * g.P;
    universe_bwd_roi_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(g, pr.sp, cell_params, uroi,
                                                                         g_universe, guroi, batch);
    NC_CHECK(launch_check("universe_bwd_roi_kernel launch"));
    if (g_out) {
      universe_bwd_ports_kernel<<<(batch * g.n_out + 127) / 128, 128, 0, st>>>(g, pr.out_index, uroi, g_out,
                                                                               guroi, batch);
      NC_CHECK(launch_check("universe_bwd_ports_kernel launch"));
    }
    if (g.padding == NC_PAD_VALID) {
      gringf = at<float>(d_ws, L.gringf);
      universe_bwd_ring_kernel<<<(g.H * g.W + 255) / 256, 256, 0, st>>>(g, pr.sp, cell_params, g_universe,
                                                                        gringf, batch);
      NC_CHECK(launch_check("universe_bwd_ring_kernel launch"));
      if (g_out) {
        universe_bwd_border_ports_kernel<<<(g.n_out + 127) / 128, 128, 0, st>>>(
            g, pr.sp, cell_params, pr.out_index, g_out, gringf, batch);
        NC_CHECK(launch_check("universe_bwd_border_ports_kernel launch"));
      }
    }
  }
  if (g_universe) g_out = nullptr;   // folded into guroi above
  if (g.algo == NC_CONV_FFT && fftf_fits(g)) {
    FftfArgs fa = fftf_args(pr, d_ws, inputs, batch, true);
    fa.gout = g_out;
    fa.guroi = guroi;
    if (g_prof.bs) NC_CUDA_CHECK(cudaEventRecord(g_prof.bs, st));
    NC_CHECK(fftf_backward(fa, st));
    if (g_prof.be) NC_CUDA_CHECK(cudaEventRecord(g_prof.be, st));
    const int P3 = 3 * g.P, MK = g.M * g.K, FF = g.Fh * g.Fw, HW = g.H * g.W;
    {
      // fixed-order batch sums of the per-sample partials, in two stages: chunk partials
      // here, the chunk sums inside the pre-step adjoint
      SegSum j;
      memset(&j, 0, sizeof(j));
      j.in[0] = fa.gpix; j.n[0] = P3;
      j.in[1] = fa.gdpart; j.n[1] = MK;
      j.nseg = 2;
      if (fa.gring) { j.in[2] = fa.gring; j.n[2] = FF; j.nseg = 3; }
      j.total = j.n[0] + j.n[1] + j.n[2];
      const int chunks = batch < kRedChunks ? batch : kRedChunks;
      const int bc = (batch + chunks - 1) / chunks;
      float* part = at<float>(d_ws, L.redscr);
      {
        PdlLaunch l1(dim3((j.total + 255) / 256, chunks), dim3(256), 0, st);
        NC_CUDA_CHECK(cudaLaunchKernelEx(&l1.cfg, seg_batch_sum1_kernel, j, batch, bc, part));
        NC_CHECK(launch_check("seg_batch_sum1_kernel launch"));
      }
      {
        float* gring_part = fa.gring ? part + P3 + MK : nullptr;
        PdlLaunch l2(dim3((HW + 255) / 256), dim3(256), 0, st);
        NC_CUDA_CHECK(cudaLaunchKernelEx(&l2.cfg, prestep_bwd_kernel, g, pr.sp, cell_params, filters, pr.owm,
                                         pr.bmask, part, gring_part, part + P3, gringf, g_cell_params,
                                         g_filters, chunks, (size_t)j.total));
        NC_CHECK(launch_check("prestep_bwd_kernel launch"));
      }
    }
    clear_error();
    return NC_OK;
  }
  if (g.algo == NC_CONV_FFT) {
    FftCall c = fft_call(pr, d_ws, inputs, batch, true);
    c.gout = g_out;
    c.guroi = guroi;
    if (g_prof.bs) NC_CUDA_CHECK(cudaEventRecord(g_prof.bs, st));
    NC_CHECK(fft_backward(c, st));
    if (g_prof.be) NC_CUDA_CHECK(cudaEventRecord(g_prof.be, st));
    const int HW = g.H * g.W;
    prestep_bwd_kernel<<<(HW + 255) / 256, 256, 0, st>>>(g, pr.sp, cell_params, filters, pr.owm, pr.bmask, c.gsum,
                                                         c.gborder, c.gdsum, gringf, g_cell_params, g_filters, 0, 0);
    NC_CHECK(launch_check("prestep_bwd_kernel launch"));
    clear_error();
    return NC_OK;
  }

  BwdArgs a;
  memset(&a, 0, sizeof(a));
  a.g = g;
  a.sp = pr.sp;
  a.in_index = pr.in_index;
  a.out_index = pr.out_index;
  a.inputs = inputs;
  a.gout = g_out;
  a.xsave = at<float>(d_ws, L.xsave);
  a.zhat = at<float>(d_ws, L.zhat);
  a.rstd = at<float>(d_ws, L.rstd);
  a.fscr = at<float>(d_ws, L.fscr);
  a.gzscr = at<float>(d_ws, L.gzscr);
  a.gpix = at<float>(d_ws, L.gpix);
  a.gdpart = at<float>(d_ws, L.gdpart);
  a.gdelta = at<float>(d_ws, L.gdelta);
  a.guroi = guroi;
  a.g_smem = pr.gs ? 1 : 0;
  a.f_smem = (pr.gs && pr.fs) ? 1 : 0;
  a.gz_smem = (a.f_smem && pr.gzs) ? 1 : 0;
  a.batch = batch;
  if (!a.f_smem && !a.fscr)
    return set_error(NC_ERR_UNSUPPORTED, "field does not fit on chip and no scratch was laid out");
  if (!a.gz_smem && !a.gzscr)
    return set_error(NC_ERR_UNSUPPORTED, "plane gradients do not fit on chip and no scratch was laid out");
  const FastKernels fk = g_universe ? FastKernels{} : fast_kernels(g);
  const void* fn = fk.bwd ? fk.bwd : (const void*)vnn_fused_bwd_kernel;
  const size_t smem = fk.bwd ? fk.bwd_smem : fused_smem_bytes(g, a.g_smem, a.f_smem, a.gz_smem);
  NC_CHECK(set_smem_attr(fn, smem));
  if (g_prof.bs) NC_CUDA_CHECK(cudaEventRecord(g_prof.bs, st));
  {
    FastBwdLayout bl = fk.bl;
    void* args_fast[] = {&a, &bl};
    void* args_v1[] = {&a};
    NC_CUDA_CHECK(cudaLaunchKernel(fn, dim3(batch), dim3(kFusedThreads), fk.bwd ? args_fast : args_v1,
                                   smem, st));
  }
  NC_CHECK(launch_check("fused backward kernel launch"));
  if (g_prof.be) NC_CUDA_CHECK(cudaEventRecord(g_prof.be, st));

  // batch reductions (fixed order -> deterministic)
  float* gsum = at<float>(d_ws, L.gsum);
  float* gdsum = at<float>(d_ws, L.gdsum);
  const int P3 = 3 * g.P, MK = g.M * g.K;
  const int MP = g.M * g.P;
  float* redscr = at<float>(d_ws, L.redscr);
  if (fk.bwd) {
    // specialised kernel: per-step pixel partials (B, d, 3, P)
    NC_CHECK(batch_step_sum(a.gpix, batch, g.d, 0, (size_t)P3, P3, gsum, redscr, st));
  } else {
    batch_sum_kernel<<<(P3 + 255) / 256, 256, 0, st>>>(a.gpix, (size_t)P3, P3, batch, gsum);
    NC_CHECK(launch_check("pixel-partial reduction launch"));
  }
  batch_sum_kernel<<<(MK + 255) / 256, 256, 0, st>>>(a.gdpart, (size_t)MK, MK, batch, gdsum);
  NC_CHECK(launch_check("batch_sum_kernel(filters) launch"));
  float* gborder = nullptr;
  const int HW = g.H * g.W;
  if (a.gdelta) {
    float* gdeltasum = at<float>(d_ws, L.gdeltasum);
    if (fk.bwd) {
      // specialised kernel: gz of steps t >= 1 overwrote the standardised planes (B, d, M, P)
      NC_CHECK(batch_step_sum(a.zhat, batch, g.d, 1, (size_t)MP, MP, gdeltasum, redscr, st));
    } else {
      batch_sum_kernel<<<(MP + 255) / 256, 256, 0, st>>>(a.gdelta, (size_t)MP, MP, batch, gdeltasum);
      NC_CHECK(launch_check("border-gradient reduction launch"));
    }
    gborder = at<float>(d_ws, L.gborder);
    border_grad_kernel<<<(HW + 7) / 8, 256, 0, st>>>(g, pr.sp.geff, gdeltasum, gborder);
    NC_CHECK(launch_check("border_grad_kernel launch"));
  }
  prestep_bwd_kernel<<<(HW + 255) / 256, 256, 0, st>>>(g, pr.sp, cell_params, filters, pr.owm, pr.bmask, gsum,
                                                       gborder, gdsum, gringf, g_cell_params, g_filters, 0, 0);
  NC_CHECK(launch_check("prestep_bwd_kernel launch"));
  clear_error();
  return NC_OK;
}

nc_status nc_vnn_backward(const nc_topo* topo, const void* d_plan, const float* cell_params,
                          const float* filters, const float* inputs, int32_t batch,
                          const nc_codd* codd, const float* g_out, float* g_cell_params,
                          float* g_filters, void* d_ws, size_t ws_bytes, void* stream) {
  return vnn_backward(topo, d_plan, cell_params, filters, inputs, batch, codd, g_out, nullptr,
                      g_cell_params, g_filters, d_ws, ws_bytes, stream);
}

nc_status nc_vnn_backward_universe(const nc_topo* topo, const void* d_plan, const float* cell_params,
                                   const float* filters, const float* inputs, int32_t batch,
                                   const nc_codd* codd, const float* g_out, const float* g_universe,
                                   float* g_cell_params, float* g_filters, void* d_ws,
                                   size_t ws_bytes, void* stream) {
  if (!g_universe) return set_error(NC_ERR_INVALID, "g_universe is null");
  return vnn_backward(topo, d_plan, cell_params, filters, inputs, batch, codd, g_out, g_universe,
                      g_cell_params, g_filters, d_ws, ws_bytes, stream);
}

// Arguments shared by both universe-embedding entry points.
static nc_status check_embed(const nc_topo* topo, const void* d_plan, const float* cell_params,
                             const nc_codd* codd, int32_t win_row, int32_t win_col, int32_t win_h,
                             int32_t win_w, int32_t batch, Geo* g, UniWindow* wn) {
  NC_CHECK(make_geo(topo, g));
  NC_CHECK(check_codd(codd));
  if (!d_plan) return set_error(NC_ERR_INVALID, "plan buffer is null");
  NC_CHECK(check_ptr(cell_params, "cell_params"));
  if (batch <= 0) return set_error(NC_ERR_INVALID, "batch must be >= 1, got %d", batch);
  if (g->padding == NC_PAD_CIRCULAR)
    return set_error(NC_ERR_UNSUPPORTED, "adaptive sub-ROIs are not defined for CIRCULAR chips");
  if (win_h <= 0 || win_w <= 0 || win_row < 0 || win_col < 0 || win_row + win_h > g->H ||
      win_col + win_w > g->W)
    return set_error(NC_ERR_INVALID, "window (%d, %d) + (%d, %d) outside the %dx%d grid", win_row,
                     win_col, win_h, win_w, g->H, g->W);
  *wn = UniWindow{win_row, win_col, win_h, win_w};
  return NC_OK;
}

nc_status nc_universe_embed_forward(const nc_topo* topo, const void* d_plan, const float* cell_params,
                                    const nc_codd* codd, int32_t win_row, int32_t win_col,
                                    int32_t win_h, int32_t win_w, const float* universe_window,
                                    int32_t batch, float* universe, float* out, void* stream) {
  Geo g;
  UniWindow wn;
  NC_CHECK(check_embed(topo, d_plan, cell_params, codd, win_row, win_col, win_h, win_w, batch, &g, &wn));
  NC_CHECK(check_ptr(universe_window, "universe_window"));
  NC_CHECK(check_ptr(universe, "universe"));
  const PlanLayout PL = plan_layout(topo);
  cudaStream_t st = as_stream(stream);
  const size_t n = (size_t)batch * g.H * g.W;
  universe_embed_fwd_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
      g, wn, cell_params, at<uint8_t>(d_plan, PL.io_mask), *codd, universe_window, universe, batch);
  NC_CHECK(launch_check("universe_embed_fwd_kernel launch"));
  if (out) {
    gather_out_kernel<<<(batch * g.n_out + 127) / 128, 128, 0, st>>>(
        g, at<int32_t>(d_plan, PL.out_index), universe, out, batch);
    NC_CHECK(launch_check("gather_out_kernel launch"));
  }
  clear_error();
  return NC_OK;
}

nc_status nc_universe_embed_backward(const nc_topo* topo, const void* d_plan, const float* cell_params,
                                     const nc_codd* codd, int32_t win_row, int32_t win_col,
                                     int32_t win_h, int32_t win_w, const float* g_out,
                                     const float* g_universe, int32_t batch, float* g_universe_window,
                                     float* g_cell_params, void* stream) {
  Geo g;
  UniWindow wn;
  NC_CHECK(check_embed(topo, d_plan, cell_params, codd, win_row, win_col, win_h, win_w, batch, &g, &wn));
  NC_CHECK(check_ptr(g_universe_window, "g_universe_window"));
  NC_CHECK(check_ptr(g_cell_params, "g_cell_params"));
  const PlanLayout PL = plan_layout(topo);
  const uint8_t* io = at<uint8_t>(d_plan, PL.io_mask);
  cudaStream_t st = as_stream(stream);
  universe_embed_bwd_kernel<<<(g.H * g.W + 255) / 256, 256, 0, st>>>(
      g, wn, cell_params, io, *codd, g_universe, g_universe_window, g_cell_params, batch);
  NC_CHECK(launch_check("universe_embed_bwd_kernel launch"));
  if (g_out) {
    universe_embed_bwd_ports_kernel<<<(g.n_out + 127) / 128, 128, 0, st>>>(
        g, wn, at<int32_t>(d_plan, PL.out_index), cell_params, io, *codd, g_out, g_universe_window,
        g_cell_params, batch);
    NC_CHECK(launch_check("universe_embed_bwd_ports_kernel launch"));
  }
  clear_error();
  return NC_OK;
}

nc_status nc_codd_states(const nc_topo* topo, const void* d_plan, const float* states_raw,
                         const nc_codd* codd, float* s_prob, void* stream) {
  Geo g;
  NC_CHECK(make_geo(topo, &g));
  NC_CHECK(check_codd(codd));
  if (!d_plan) return set_error(NC_ERR_INVALID, "plan buffer is null");
  NC_CHECK(check_ptr(states_raw, "states_raw"));
  NC_CHECK(check_ptr(s_prob, "s_prob"));
  const PlanLayout PL = plan_layout(topo);
  const int HW = g.H * g.W;
  codd_kernel<<<(HW + 255) / 256, 256, 0, as_stream(stream)>>>(
      HW, states_raw, at<uint8_t>(d_plan, PL.io_mask), g.hard_pin, *codd, s_prob);
  NC_CHECK(launch_check("codd_kernel launch"));
  clear_error();
  return NC_OK;
}

nc_status nc_mse_loss(const float* out, const float* targets, int32_t batch, int32_t n, float* loss,
                      float* g_out, void* stream) {
  if (batch <= 0 || n <= 0) return set_error(NC_ERR_INVALID, "bad loss shape (%d, %d)", batch, n);
  NC_CHECK(check_ptr(out, "out"));
  NC_CHECK(check_ptr(targets, "targets"));
  const int64_t total = (int64_t)batch * n;
  if (total > 0x7fffffff) return set_error(NC_ERR_INVALID, "loss too large");
  float* lossd = nullptr;
  if (loss) {
    const void* d = nullptr;
    NC_CHECK(device_address(loss, "loss", &d));
    lossd = const_cast<float*>(static_cast<const float*>(d));
  }
  {
    PdlLaunch l(dim3(1), dim3(1024), 0, as_stream(stream));
    NC_CUDA_CHECK(cudaLaunchKernelEx(&l.cfg, mse_kernel, out, targets, (int)total, lossd, g_out));
  }
  NC_CHECK(launch_check("mse_kernel launch"));
  clear_error();
  return NC_OK;
}

nc_status nc_softmax_ce_loss(const float* logits, const int32_t* labels, int32_t batch, int32_t n,
                             float* loss, float* g_logits, void* stream) {
  if (batch <= 0 || n <= 0) return set_error(NC_ERR_INVALID, "bad loss shape (%d, %d)", batch, n);
  NC_CHECK(check_ptr(logits, "logits"));
  NC_CHECK(check_ptr(labels, "labels"));
  float* lossd = nullptr;
  if (loss) {
    const void* d = nullptr;
    NC_CHECK(device_address(loss, "loss", &d));
    lossd = const_cast<float*>(static_cast<const float*>(d));
  }
  {
    PdlLaunch l(dim3(1), dim3(1024), 0, as_stream(stream));
    NC_CUDA_CHECK(cudaLaunchKernelEx(&l.cfg, softmax_ce_kernel, logits, labels, batch, n, lossd, g_logits));
  }
  NC_CHECK(launch_check("softmax_ce_kernel launch"));
  clear_error();
  return NC_OK;
}

nc_status nc_stage_from_host(const nc_stage_seg* segs, int32_t nseg, void* stream) {
  if (!segs || nseg < 1 || nseg > NC_MAX_STAGE_SEGS)
    return set_error(NC_ERR_INVALID, "nc_stage_from_host takes 1..%d segments, got %d", NC_MAX_STAGE_SEGS, nseg);
  StageSegs s;
  memset(&s, 0, sizeof(s));
  size_t most = 0;
  for (int k = 0; k < nseg; ++k) {
    const nc_stage_seg& g = segs[k];
    if (g.bytes % 4 != 0 || reinterpret_cast<uintptr_t>(g.dst) % 4 != 0 ||
        reinterpret_cast<uintptr_t>(g.src) % 4 != 0)
      return set_error(NC_ERR_INVALID, "segment %d: sizes and addresses must be multiples of 4 bytes", k);
    const void* dsrc = nullptr;
    const void* ddst = nullptr;
    NC_CHECK(device_address(g.src, "segment source", &dsrc));
    NC_CHECK(device_address(g.dst, "segment destination", &ddst));
    s.src[k] = dsrc;
    s.dst[k] = const_cast<void*>(ddst);
    s.bytes[k] = g.bytes;
    if (g.bytes > most) most = g.bytes;
  }
  s.n = nseg;
  if (most == 0) return NC_OK;
  const size_t units = (most + 15) / 16;
  unsigned bx = (unsigned)((units + 255) / 256);
  if (bx > 64) bx = 64;
  stage_copy_kernel<<<dim3(bx, nseg), 256, 0, as_stream(stream)>>>(s);
  NC_CHECK(launch_check("stage_copy_kernel launch"));
  clear_error();
  return NC_OK;
}

nc_status nc_sgd_update(float* params, const float* grads, int64_t n, float lr, void* stream) {
  if (n <= 0) return set_error(NC_ERR_INVALID, "bad parameter count %lld", (long long)n);
  NC_CHECK(check_ptr(params, "params"));
  NC_CHECK(check_ptr(grads, "grads"));
  const int64_t blocks64 = (n + 255) / 256;
  const int blocks = (int)(blocks64 < 4096 ? blocks64 : 4096);
  {
    PdlLaunch l(dim3(blocks), dim3(256), 0, as_stream(stream));
    NC_CUDA_CHECK(cudaLaunchKernelEx(&l.cfg, sgd_kernel, params, grads, n, lr));
  }
  NC_CHECK(launch_check("sgd_kernel launch"));
  clear_error();
  return NC_OK;
}

void nc_set_profile_events(void* fwd_start, void* fwd_stop, void* bwd_start, void* bwd_stop) {
  g_prof.fs = reinterpret_cast<cudaEvent_t>(fwd_start);
  g_prof.fe = reinterpret_cast<cudaEvent_t>(fwd_stop);
  g_prof.bs = reinterpret_cast<cudaEvent_t>(bwd_start);
  g_prof.be = reinterpret_cast<cudaEvent_t>(bwd_stop);
}

nc_status nc_fp32_peak_probe(int32_t iters, double* flops, float* sink, void* stream) {
  if (iters <= 0 || !flops || !sink) return set_error(NC_ERR_INVALID, "bad probe arguments");
  int dev = 0, sms = 0;
  NC_CUDA_CHECK(cudaGetDevice(&dev));
  NC_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int blocks = sms * 4, threads = 256;
  fp32_peak_kernel<<<blocks, threads, 0, as_stream(stream)>>>(iters, sink);
  NC_CHECK(launch_check("fp32_peak_kernel launch"));
  *flops = 2.0 * 16.0 * (double)iters * (double)blocks * (double)threads;
  clear_error();
  return NC_OK;
}

}  // extern "C"
