// nc_static.cu -- inference forward whose scratch lives in a static device array.
//
// Who needs this: code that may not call cudaMalloc at all.  Examples are a JAX/XLA FFI
// custom call (XLA preallocates most of the GPU's memory for its own pool, so a cudaMalloc
// from inside a handler can fail, and the handler has no workspace of its own unless the
// framework hands one out), code running while a stream is being captured into a CUDA
// graph (cudaMalloc is not a stream operation and is not allowed there), and hosts with a
// fixed memory budget that forbid allocations after start-up.  Such callers still own the
// plan, parameters, inputs and outputs; only the per-call scratch of nc_vnn_forward comes
// from the array below, which every GPU that loads this library keeps until the process
// exits.
#include <mutex>

#include <cuda.h>
#include <cuda_runtime.h>

#include "nc_errors.h"
#include "nc_internal.h"

namespace nc {
namespace {

// The scratch of every nc_vnn_forward_static call on a device.  Its host-side name is
// only a stand-in: host code must pass the device address from cudaGetSymbolAddress.
constexpr size_t kStaticScratchBytes = NC_STATIC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
// Per device: the context the address was resolved in, and the address.  A context that
// was destroyed and created again (cudaDeviceReset) loads the module again, possibly at
// another address, so a new context resolves again.
CUcontext g_scratch_ctx[kMaxDevices] = {};
void* g_scratch_addr[kMaxDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// The current context through the runtime's driver entry point (no link against libcuda).
nc_status current_context(CUcontext* ctx) {
  static CtxGetCurrentFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetDriverEntryPointByVersion(cuCtxGetCurrent)");
    if (q != cudaDriverEntryPointSuccess || !p)
      return set_error(NC_ERR_CUDA, "cuCtxGetCurrent is not available from the driver");
    fn = reinterpret_cast<CtxGetCurrentFn>(p);
  }
  *ctx = nullptr;
  if (fn(ctx) != CUDA_SUCCESS) return set_error(NC_ERR_CUDA, "cuCtxGetCurrent failed");
  return NC_OK;   // null when the runtime has not made a context current yet
}

// Once per device and context, with that device current: resolve the array's device address.
nc_status static_scratch_address(void** out) {
  int dev = -1;
  NC_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return set_error(NC_ERR_UNSUPPORTED, "device ordinal %d too large", dev);
  CUcontext ctx = nullptr;
  NC_CHECK(current_context(&ctx));
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!ctx || !g_scratch_addr[dev] || g_scratch_ctx[dev] != ctx) {
    void* p = nullptr;
    // also makes the device's primary context current when no call has done so yet
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(static scratch)");
    if (!p) return set_error(NC_ERR_CUDA, "cudaGetSymbolAddress returned a null address");
    NC_CHECK(current_context(&ctx));
    g_scratch_addr[dev] = p;
    g_scratch_ctx[dev] = ctx;
  }
  *out = g_scratch_addr[dev];
  return NC_OK;
}

}  // namespace
}  // namespace nc

using namespace nc;

extern "C" nc_status nc_vnn_forward_static(const nc_topo* topo, const void* d_plan,
                                           const float* cell_params, const float* filters,
                                           const float* inputs, int32_t batch,
                                           const nc_codd* codd, float* out, void* stream) {
  Geo g;
  NC_CHECK(make_geo(topo, &g));
  if (batch <= 0) return set_error(NC_ERR_INVALID, "batch must be >= 1, got %d", batch);
  const size_t need = nc_workspace_bytes(topo, batch, 0u);
  if (need == 0) return set_error(NC_ERR_INVALID, "invalid topology or batch");
  if (need > kStaticScratchBytes)
    return set_error(NC_ERR_WORKSPACE,
                     "nc_vnn_forward_static: this call needs %zu bytes of scratch but the static "
                     "scratch holds %zu bytes; use nc_vnn_forward with a caller workspace or a "
                     "smaller batch",
                     need, (size_t)kStaticScratchBytes);
  void* scratch = nullptr;
  NC_CHECK(static_scratch_address(&scratch));
  // Every scratch byte this forward reads is written earlier in the same call, so nothing
  // has to be cleared between calls.
  return nc_vnn_forward(topo, d_plan, cell_params, filters, inputs, batch, codd, 0u, out, scratch,
                        kStaticScratchBytes, stream);
}
