// nc_dp.cu -- fused cross-GPU gradient sum + SGD over NVLink peer memory (sm_100a).
//
// Push protocol with step-tagged elements.  Each rank owns a receive buffer of 8-byte
// elements
//   [2 parity][world source ranks][n_elems]   element = (uint64(step) << 32) | float_bits(g)
// mapped into every peer with CUDA IPC.  Every step each rank stores its gradient into slot
// (parity, own rank) of every PEER's buffer, two elements per 16-byte vector store (posted
// NVLink writes).  Each element is one naturally aligned 64-bit access, which the PTX
// memory model makes single-copy atomic even inside a vector access, so a reader sees a
// value together with the tag written with it -- never the current tag beside an older
// value.  A receiver knows a value has arrived when its tag equals the current step, so no
// fences and no separate flags are needed: for each line of its slice, a thread loads that
// line of every peer's slot in its OWN buffer at once (bounded retries) and, once every tag
// is the current step, sums the values that came with the tags over ranks 0..world-1 in
// that order (its own contribution straight from `grads`) and applies SGD.  Every rank adds
// the same values in the same order and ends with bitwise identical parameters.  The grid
// grows with the gradient (one line per thread, at most kDpMaxBlocks blocks: four per SM,
// all resident at once, so no block waits for a peer block that is not running).  Double buffering makes the
// next step safe: a rank writes slot `parity` again only at step+2, after every peer has
// published step+1, i.e. after every peer finished reading step's slot (its step kernel
// ended before its step+1 kernel began).  Step counters are per block and live on the
// device, so the launch can be captured in a CUDA graph.  No multicast, no TMA, no atomics
// on peer memory: plain volatile stores and loads.
//
// Failure: a thread whose peers do not arrive within max_wait polls of one line sets the
// status word; its block stops updating and returns.  The status is terminal: every later
// call on that state returns at once (no stores to peers, no update), so the peers of this
// rank time out at their next step as well and the failure reaches every rank within one
// step.  Lines that arrived before the failure WERE updated, so after a failure the ranks'
// parameters are no longer known to agree: restore them from a consistent copy, then call
// nc_dp_reset on every rank (and a host barrier) before the next exchange.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>

#include "nc_errors.h"
#include "neurocell_b200.h"

namespace nc {
namespace {

constexpr int kDpMaxBlocks = 592;   // 4 per SM of a B200; the state holds one counter each
constexpr int kDpThreads = 128;

struct Peers {
  ulonglong2* p[NC_DP_MAX_RANKS];
};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }
// 16-byte lines of two elements each
__host__ __device__ inline long long n_lines(long long n) { return (n + 1) / 2; }

__device__ __forceinline__ unsigned long long tagged(float v, unsigned step) {
  return ((unsigned long long)step << 32) | (unsigned long long)__float_as_uint(v);
}

__device__ __forceinline__ void st_line(ulonglong2* p, ulonglong2 v) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(v.x), "l"(v.y) : "memory");
}

__device__ __forceinline__ ulonglong2 ld_line(const ulonglong2* p) {
  ulonglong2 v;
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
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
    s_bad = *reinterpret_cast<volatile int*>(status);   // terminal after a failure
  }
  __syncthreads();
  if (s_bad) return;
  const unsigned step = s_step;
  const int par = (int)(step & 1u);
  auto slot = [&](int owner, int src) {   // slot (par, src) of rank owner's buffer
    return peers.p[owner] + ((size_t)par * world + src) * (size_t)L;
  };
  // 1. push this rank's lines to every peer
  for (long long l = l0 + threadIdx.x; l < l1; l += blockDim.x) {
    const float2 v = load_pair(grads, n, l);
    const ulonglong2 line = make_ulonglong2(tagged(v.x, step), tagged(v.y, step));
    for (int r = 0; r < world; ++r)
      if (r != rank) st_line(slot(r, rank) + l, line);
  }
  // 2. per line: every peer's copy with this step's tag (bounded), then the sum in rank
  //    order of the values that came with those tags, and SGD
  int bad = 0;
  for (long long l = l0 + threadIdx.x; l < l1 && !bad; l += blockDim.x) {
    ulonglong2 q[NC_DP_MAX_RANKS];
#pragma unroll
    for (int r = 0; r < NC_DP_MAX_RANKS; ++r) q[r] = make_ulonglong2(0ull, 0ull);
    for (int it = 0;; ++it) {
      bool ready = true;
#pragma unroll
      for (int r = 0; r < NC_DP_MAX_RANKS; ++r) {
        if (r >= world || r == rank) continue;
        q[r] = ld_line(slot(rank, r) + l);
        ready = ready && (unsigned)(q[r].x >> 32) == step && (unsigned)(q[r].y >> 32) == step;
      }
      if (ready) break;
      if (it >= max_wait) { bad = 1; break; }
      if (it > 64) __nanosleep(32);
    }
    if (bad) break;
    const float2 own = load_pair(grads, n, l);
    float2 s = make_float2(0.f, 0.f);
#pragma unroll
    for (int r = 0; r < NC_DP_MAX_RANKS; ++r) {
      if (r < world) {
        const float2 v = r == rank ? own
                                   : make_float2(__uint_as_float((unsigned)q[r].x), __uint_as_float((unsigned)q[r].y));
        if (r == 0) s = v; else { s.x += v.x; s.y += v.y; }
      }
    }
    const long long i = 2 * l;
    grads[i] = s.x;
    params[i] -= lr_eff * s.x;
    if (i + 1 < n) {
      grads[i + 1] = s.y;
      params[i + 1] -= lr_eff * s.y;
    }
  }
  if (bad) s_bad = 1;
  __syncthreads();
  if (s_bad) {                            // a peer did not arrive: status set, no counter
    if (threadIdx.x == 0) atomicExch(status, 1);
    return;
  }
  if (threadIdx.x == 0) counters[k] = step;
}

// Blocks of the exchange for n elements: one 16-byte line per thread, at most kDpMaxBlocks.
inline int dp_blocks(long long n) {
  const long long b = (n_lines(n) + kDpThreads - 1) / kDpThreads;
  return (int)(b < 1 ? 1 : b > kDpMaxBlocks ? kDpMaxBlocks : b);
}

}  // namespace
}  // namespace nc

using namespace nc;

extern "C" {

size_t nc_dp_shared_bytes(int64_t n, int32_t world) {
  if (n <= 0 || world < 1 || world > NC_DP_MAX_RANKS) return 0;
  return align256(sizeof(ulonglong2) * 2 * (size_t)world * (size_t)n_lines(n));
}

size_t nc_dp_state_bytes(void) { return align256(sizeof(unsigned) * kDpMaxBlocks + sizeof(int)); }

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
    pp.p[r] = static_cast<ulonglong2*>(peers[r]);
  }
  unsigned* counters = static_cast<unsigned*>(d_state);
  int* status = reinterpret_cast<int*>(counters + kDpMaxBlocks);
  dp_allreduce_sgd_kernel<<<dp_blocks(n), kDpThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
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
  const int* s = reinterpret_cast<const int*>(static_cast<const unsigned*>(d_state) + kDpMaxBlocks);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  NC_CUDA_CHECK(cudaMemcpyAsync(status, s, sizeof(int), cudaMemcpyDeviceToHost, st));
  NC_CUDA_CHECK(cudaStreamSynchronize(st));
  return NC_OK;
}

nc_status nc_dp_reset(void* d_state, void* d_shared, size_t shared_bytes, void* stream) {
  if (!d_state || !d_shared || shared_bytes == 0 || shared_bytes % 16 != 0)
    return set_error(NC_ERR_INVALID, "bad nc_dp_reset arguments");
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  NC_CUDA_CHECK(cudaMemsetAsync(d_state, 0, nc_dp_state_bytes(), st));
  NC_CUDA_CHECK(cudaMemsetAsync(d_shared, 0, shared_bytes, st));
  clear_error();
  return NC_OK;
}

}  // extern "C"
