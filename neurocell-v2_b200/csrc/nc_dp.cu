// nc_dp.cu -- fused cross-GPU gradient sum + SGD over NVLink peer memory (sm_100a).
//
// Push protocol with step-tagged lines.  Each rank owns a receive buffer of 16-byte lines
//   [2 parity][world source ranks][n_lines]   line = {g[2l], step, g[2l+1], step}
// mapped into every peer with CUDA IPC.  Every step each rank stores its gradient, two
// values per line, into slot (parity, own rank) of every PEER's buffer with one 16-byte
// store per line (posted NVLink writes; each 8-byte half {value, step} is written as one
// unit).  A receiver knows a value has arrived when the step tag next to it equals the
// current step, so no fences and no separate flags are needed: block k polls the lines of
// its slice in its OWN buffer (bounded), then sums the slice over ranks 0..world-1 in that
// order (its own contribution straight from `grads`) and applies SGD.  Every rank adds the
// same values in the same order and ends with bitwise identical parameters.  Double
// buffering makes the next step safe: a rank writes slot `parity` again only at step+2,
// after every peer has published step+1, i.e. after every peer finished reading step's
// slot (its step kernel ended before its step+1 kernel began).  Step counters are per block
// and live on the device, so the launch can be captured in a CUDA graph.  No multicast,
// no TMA, no atomics on peer memory: plain stores and volatile loads.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "nc_errors.h"
#include "neurocell_b200.h"

namespace nc {
namespace {

constexpr int kDpBlocks = 32;
constexpr int kDpThreads = 128;

struct Peers {
  uint4* p[NC_DP_MAX_RANKS];
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
__host__ __device__ inline long long n_lines(long long n) { return (n + 1) / 2; }

__device__ __forceinline__ void st_line(uint4* p, uint4 v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint4 ld_line(const uint4* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ float2 load_pair(const float* g, long long n, long long l) {
  const long long i = 2 * l;
  return make_float2(g[i], i + 1 < n ? g[i + 1] : 0.f);
}

// Block k owns lines [k*slice, min(L, (k+1)*slice)) of the L = ceil(n/2) lines.
__global__ void __launch_bounds__(kDpThreads) dp_allreduce_sgd_kernel(
    Peers peers, int world, int rank, long long n, unsigned* counters, int* status, float* grads,
    float* params, float lr_eff, int max_wait) {
  const int k = blockIdx.x;
  const long long L = n_lines(n);
  const long long slice = (L + gridDim.x - 1) / gridDim.x;
  const long long l0 = (long long)k * slice < L ? (long long)k * slice : L;
  const long long l1 = (l0 + slice < L) ? l0 + slice : L;
  __shared__ unsigned s_step;
  __shared__ int s_bad;
  if (threadIdx.x == 0) {
    s_step = counters[k] + 1u;
    s_bad = 0;
  }
  __syncthreads();
  const unsigned step = s_step;
  const int par = (int)(step & 1u);
  auto slot = [&](int owner, int src) {   // slot (par, src) of rank owner's buffer
    return peers.p[owner] + ((size_t)par * world + src) * (size_t)L;
  };
  // 1. push this rank's lines to every peer
  for (long long l = l0 + threadIdx.x; l < l1; l += blockDim.x) {
    const float2 v = load_pair(grads, n, l);
    const uint4 line = make_uint4(__float_as_uint(v.x), step, __float_as_uint(v.y), step);
    for (int r = 0; r < world; ++r)
      if (r != rank) st_line(slot(r, rank) + l, line);
  }
  // 2. wait until every peer's lines of this slice carry this step's tag (bounded)
  int it = 0, bad = 0;
  for (long long l = l0 + threadIdx.x; l < l1 && !bad; l += blockDim.x) {
    for (int r = 0; r < world && !bad; ++r) {
      if (r == rank) continue;
      const uint4* q = slot(rank, r) + l;
      for (;;) {
        const uint4 v = ld_line(q);
        if (v.y == step && v.w == step) break;
        if (++it > max_wait) { bad = 1; break; }
        if (it > 64) __nanosleep(32);
      }
    }
  }
  if (bad) s_bad = 1;
  __syncthreads();
  if (s_bad) {                            // a peer did not arrive: no update, status set
    if (threadIdx.x == 0) atomicExch(status, 1);
    return;
  }
  // 3. sum in rank order, SGD
  for (long long l = l0 + threadIdx.x; l < l1; l += blockDim.x) {
    float2 s = make_float2(0.f, 0.f);
    for (int r = 0; r < world; ++r) {
      float2 v;
      if (r == rank) {
        v = load_pair(grads, n, l);
      } else {
        const uint4 q = ld_line(slot(rank, r) + l);
        v = make_float2(__uint_as_float(q.x), __uint_as_float(q.z));
      }
      if (r == 0) s = v; else { s.x += v.x; s.y += v.y; }
    }
    const long long i = 2 * l;
    grads[i] = s.x;
    params[i] -= lr_eff * s.x;
    if (i + 1 < n) {
      grads[i + 1] = s.y;
      params[i + 1] -= lr_eff * s.y;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) counters[k] = step;
}

}  // namespace
}  // namespace nc

using namespace nc;

extern "C" {

size_t nc_dp_shared_bytes(int64_t n, int32_t world) {
  if (n <= 0 || world < 1 || world > NC_DP_MAX_RANKS) return 0;
  return align256(sizeof(uint4) * 2 * (size_t)world * (size_t)n_lines(n));
}

size_t nc_dp_state_bytes(void) { return align256(sizeof(unsigned) * kDpBlocks + sizeof(int)); }

nc_status nc_dp_alloc(size_t bytes, void** d_ptr) {
  if (!d_ptr || bytes == 0) return set_error(NC_ERR_INVALID, "bad nc_dp_alloc arguments");
  NC_CUDA_CHECK(cudaMalloc(d_ptr, bytes));
  NC_CUDA_CHECK(cudaMemset(*d_ptr, 0, bytes));
  NC_CUDA_CHECK(cudaDeviceSynchronize());
  clear_error();
  return NC_OK;
}

nc_status nc_dp_free(void* d_ptr) {
  if (d_ptr) NC_CUDA_CHECK(cudaFree(d_ptr));
  return NC_OK;
}

nc_status nc_ipc_get(void* d_ptr, void* handle_out) {
  if (!d_ptr || !handle_out) return set_error(NC_ERR_INVALID, "bad nc_ipc_get arguments");
  static_assert(sizeof(cudaIpcMemHandle_t) == NC_IPC_HANDLE_BYTES, "IPC handle size");
  cudaIpcMemHandle_t h;
  NC_CUDA_CHECK(cudaIpcGetMemHandle(&h, d_ptr));
  memcpy(handle_out, &h, sizeof(h));
  return NC_OK;
}

nc_status nc_ipc_open(const void* handle, void** d_peer_ptr) {
  if (!handle || !d_peer_ptr) return set_error(NC_ERR_INVALID, "bad nc_ipc_open arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  NC_CUDA_CHECK(cudaIpcOpenMemHandle(d_peer_ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return NC_OK;
}

nc_status nc_ipc_close(void* d_peer_ptr) {
  if (d_peer_ptr) NC_CUDA_CHECK(cudaIpcCloseMemHandle(d_peer_ptr));
  return NC_OK;
}

nc_status nc_dp_allreduce_sgd(void* const* peers, int32_t world, int32_t rank, void* d_state,
                              float* grads, float* params, int64_t n, float lr,
                              int32_t max_wait_iters, void* stream) {
  if (!peers || world < 1 || world > NC_DP_MAX_RANKS || rank < 0 || rank >= world)
    return set_error(NC_ERR_INVALID, "bad rank layout (world %d, rank %d)", world, rank);
  if (!d_state || !grads || !params || n <= 0 || max_wait_iters <= 0)
    return set_error(NC_ERR_INVALID, "bad nc_dp_allreduce_sgd arguments");
  Peers pp{};
  for (int r = 0; r < world; ++r) {
    if (!peers[r]) return set_error(NC_ERR_INVALID, "peer buffer %d is null", r);
    if (reinterpret_cast<uintptr_t>(peers[r]) % 16 != 0)
      return set_error(NC_ERR_INVALID, "peer buffer %d is not 16-byte aligned", r);
    pp.p[r] = static_cast<uint4*>(peers[r]);
  }
  unsigned* counters = static_cast<unsigned*>(d_state);
  int* status = reinterpret_cast<int*>(counters + kDpBlocks);
  dp_allreduce_sgd_kernel<<<kDpBlocks, kDpThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      pp, world, rank, (long long)n, counters, status, grads, params, lr / (float)world,
      max_wait_iters);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "dp_allreduce_sgd_kernel launch");
  note_launch();
  clear_error();
  return NC_OK;
}

nc_status nc_dp_status(const void* d_state, int32_t* status, void* stream) {
  if (!d_state || !status) return set_error(NC_ERR_INVALID, "bad nc_dp_status arguments");
  const int* s = reinterpret_cast<const int*>(static_cast<const unsigned*>(d_state) + kDpBlocks);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  NC_CUDA_CHECK(cudaMemcpyAsync(status, s, sizeof(int), cudaMemcpyDeviceToHost, st));
  NC_CUDA_CHECK(cudaStreamSynchronize(st));
  return NC_OK;
}

}  // extern "C"
