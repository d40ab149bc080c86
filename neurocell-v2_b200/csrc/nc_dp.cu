// nc_dp.cu -- fused cross-GPU gradient sum + SGD over NVLink peer memory (sm_100a).
//
// Each rank owns a shared buffer  [2 parity slots of n floats][flags: 2 x kDpBlocks u32]
// mapped into every peer with CUDA IPC.  Block k of the kernel owns slice k of the
// gradient: it copies the slice into the slot of this step's parity, publishes it with a
// system-scope release on flag[parity][k] = step, waits (bounded) until every peer's flag
// for the same slice reaches `step`, then sums the slice over ranks 0..world-1 in that
// order with peer loads and applies SGD.  Every rank therefore ends with bitwise identical
// parameters.  Double buffering makes the next step safe: a rank can overwrite slot
// `parity` only at step+2, after every peer has published step+1, i.e. after every peer
// finished reading step's slot.  Step counters are per block and live on the device, so
// the launch can be captured in a CUDA graph.  No multicast and no TMA: plain loads only.
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
  float* p[NC_DP_MAX_RANKS];
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Sum of one element (or one float4) over the ranks, in rank order: all loads are issued
// before the first add so the NVLink round trips overlap.
template <typename T>
__device__ __forceinline__ T rank_sum(const Peers& peers, int world, size_t off);

template <>
__device__ __forceinline__ float rank_sum<float>(const Peers& peers, int world, size_t off) {
  float v[NC_DP_MAX_RANKS];
#pragma unroll
  for (int r = 0; r < NC_DP_MAX_RANKS; ++r) v[r] = (r < world) ? __ldcv(peers.p[r] + off) : 0.f;
  float s = v[0];
#pragma unroll
  for (int r = 1; r < NC_DP_MAX_RANKS; ++r)
    if (r < world) s += v[r];
  return s;
}

template <>
__device__ __forceinline__ float4 rank_sum<float4>(const Peers& peers, int world, size_t off) {
  float4 v[NC_DP_MAX_RANKS];
#pragma unroll
  for (int r = 0; r < NC_DP_MAX_RANKS; ++r)
    v[r] = (r < world) ? __ldcv(reinterpret_cast<const float4*>(peers.p[r] + off))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
  float4 s = v[0];
#pragma unroll
  for (int r = 1; r < NC_DP_MAX_RANKS; ++r)
    if (r < world) { s.x += v[r].x; s.y += v[r].y; s.z += v[r].z; s.w += v[r].w; }
  return s;
}

// Block k owns elements [k*slice, min(n, (k+1)*slice)); `vec` = n % 4 == 0 and the caller's
// buffers are 16-byte aligned, so the slice (a multiple of 4) moves as float4.
__global__ void __launch_bounds__(kDpThreads) dp_allreduce_sgd_kernel(
    Peers peers, int world, int rank, long long n, int vec, size_t flag_off, unsigned* counters,
    int* status, float* grads, float* params, float lr_eff, int max_wait) {
  const int k = blockIdx.x;
  const long long slice = (((n + gridDim.x - 1) / gridDim.x) + 3) & ~3LL;
  const long long i0 = (long long)k * slice < n ? (long long)k * slice : n;
  const long long i1 = (i0 + slice < n) ? i0 + slice : n;
  __shared__ unsigned s_step;
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_step = counters[k] + 1u;
  __syncthreads();
  const unsigned step = s_step;
  const int par = (int)(step & 1u);
  const size_t base = (size_t)par * (size_t)n;
  float* mine = peers.p[rank] + base;
  if (vec) {
    for (long long i = i0 + 4 * threadIdx.x; i < i1; i += 4 * blockDim.x)
      *reinterpret_cast<float4*>(mine + i) = *reinterpret_cast<const float4*>(grads + i);
  } else {
    for (long long i = i0 + threadIdx.x; i < i1; i += blockDim.x) mine[i] = grads[i];
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    unsigned* myflag = reinterpret_cast<unsigned*>(reinterpret_cast<char*>(peers.p[rank]) + flag_off) +
                       par * kDpBlocks + k;
    st_release_sys(myflag, step);
    int ok = 1, it = 0;                   // one poll budget for all peers together
    for (int r = 0; r < world && ok; ++r) {
      const unsigned* f = reinterpret_cast<const unsigned*>(reinterpret_cast<const char*>(peers.p[r]) +
                                                            flag_off) + par * kDpBlocks + k;
      while (ld_acquire_sys(f) != step) {
        if (++it > max_wait) { ok = 0; break; }
        __nanosleep(128);
      }
    }
    if (!ok) atomicExch(status, 1);
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;                      // a peer did not arrive: no update, status set
  __threadfence_system();
  if (vec) {
    for (long long i = i0 + 4 * threadIdx.x; i < i1; i += 4 * blockDim.x) {
      const float4 s = rank_sum<float4>(peers, world, base + (size_t)i);
      *reinterpret_cast<float4*>(grads + i) = s;
      float4 p = *reinterpret_cast<const float4*>(params + i);
      p.x -= lr_eff * s.x; p.y -= lr_eff * s.y; p.z -= lr_eff * s.z; p.w -= lr_eff * s.w;
      *reinterpret_cast<float4*>(params + i) = p;
    }
  } else {
    for (long long i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
      const float s = rank_sum<float>(peers, world, base + (size_t)i);
      grads[i] = s;
      params[i] -= lr_eff * s;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) counters[k] = step;
}

}  // namespace
}  // namespace nc

using namespace nc;

extern "C" {

size_t nc_dp_shared_bytes(int64_t n) {
  if (n <= 0) return 0;
  return align256(sizeof(float) * 2 * (size_t)n) + align256(sizeof(unsigned) * 2 * kDpBlocks);
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
    pp.p[r] = static_cast<float*>(peers[r]);
  }
  unsigned* counters = static_cast<unsigned*>(d_state);
  int* status = reinterpret_cast<int*>(counters + kDpBlocks);
  const size_t flag_off = align256(sizeof(float) * 2 * (size_t)n);
  const int vec = (n % 4 == 0) && (reinterpret_cast<uintptr_t>(grads) % 16 == 0) &&
                  (reinterpret_cast<uintptr_t>(params) % 16 == 0);
  dp_allreduce_sgd_kernel<<<kDpBlocks, kDpThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      pp, world, rank, (long long)n, vec, flag_off, counters, status, grads, params,
      lr / (float)world, max_wait_iters);
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
