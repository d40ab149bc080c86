/*
 * neurocell_b200.h -- C ABI of the B200-native VNN propagation hot path.
 *
 * One shared library, libneurocell_b200.so, built for sm_100a.  Every entry point takes
 * plain pointers, sizes and a cudaStream_t (passed as void*), returns an nc_status, and
 * never allocates device memory: the caller owns the plan buffer, the workspace, the
 * parameters, inputs, outputs and gradients.  All work is stream-ordered; no entry point
 * synchronises the host except nc_plan_build (which copies host tables to the device).
 *
 * Interfaces replaced (paths relative to the shakes76/neurocell-v2 project root):
 *   nc_vnn_forward   -> neurocell/propagator.py:209-734  propagate_vnn_2d(...) forward
 *                       (d-step loop, border hoist, hidden and output-port epilogues) and
 *                       neurocell/params.py:220-322 precompute_step_params (+ Codd 31-80)
 *   nc_vnn_backward  -> the custom_vjp backward rules of the same path:
 *                       neurocell/kernels_pallas.py:1067-1069 (ROI epilogue vjp),
 *                       :1378-1504 (sparse output-port vjp), :1623-1628 and
 *                       neurocell/kernels_greens.py:316-400 (convolution dX / dG vjp),
 *                       plus the XLA autodiff of params.py:220-322
 *   nc_codd_states   -> neurocell/params.py:31-80 compute_codd_state_probs
 *                       (VonNeumannNetwork.effective_states, neurocell/model.py:160-183)
 *   nc_mse_loss      -> neurocell/trainer.py:57-61 default_mse_loss (value and gradient)
 *   nc_softmax_ce_loss -> optax.softmax_cross_entropy_with_integer_labels(...).mean()
 *                       as used by the reference's classification drivers
 *   nc_sgd_update    -> optax.sgd update + apply_updates inside trainer.py:101-106
 */
#ifndef NEUROCELL_B200_H_
#define NEUROCELL_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NC_ABI_VERSION 7

typedef enum nc_status {
  NC_OK = 0,
  NC_ERR_INVALID = 1,      /* bad topology, sizes, pointers or enum values        */
  NC_ERR_WORKSPACE = 2,    /* workspace or plan buffer too small / misaligned     */
  NC_ERR_UNSUPPORTED = 3,  /* valid reference configuration not built here        */
  NC_ERR_CUDA = 4,         /* a CUDA runtime call failed; see nc_last_error()     */
} nc_status;

typedef enum nc_padding { NC_PAD_VALID = 0, NC_PAD_SAME = 1, NC_PAD_CIRCULAR = 2 } nc_padding;

/* Activation ids (neurocell/kernels_pallas.py:76-156). NC_ACT_NONE is `None` (identity). */
typedef enum nc_activation {
  NC_ACT_NONE = 0,
  NC_ACT_TANH = 1,
  NC_ACT_SIGMOID = 2,
  NC_ACT_RELU = 3,
  NC_ACT_LEAKY_RELU = 4,
  NC_ACT_GELU = 5, /* tanh approximation */
} nc_activation;

/*
 * Green's convolution algorithm (the reference's backend choice, propagator.py:58-85):
 * DIRECT = on-chip direct cross-correlation ("nchw_direct" / "pallas_fused"), FFT = 2-D
 * FFT convolution on the next power-of-two grid ("pallas_sram"), AUTO = FFT when
 * kh*kw > 512 (the reference's auto rule), when kh*kw >= 81 and the response planes do
 * not fit on chip, or when the FFT grid is 64 x 64 and kh*kw >= 121 (fused per-sample FFT
 * kernels); else DIRECT.
 */
typedef enum nc_conv_algo { NC_CONV_AUTO = 0, NC_CONV_DIRECT = 1, NC_CONV_FFT = 2 } nc_conv_algo;

/* Codd modes (neurocell/params.py:23-28). */
typedef enum nc_codd_mode {
  NC_CODD_CONTINUOUS = 0,
  NC_CODD_ANNEALED = 1,
  NC_CODD_STE_BINARY = 2,
  NC_CODD_STE_TERNARY = 3,
} nc_codd_mode;

/*
 * Static geometry and options of one network: the POD image of ChipTopology2D
 * (neurocell/topology.py:109-135) plus the model options of VonNeumannNetwork
 * (neurocell/model.py:38-52).  Port tables live in the plan buffer (nc_plan_build).
 */
typedef struct nc_topo {
  int32_t H, W;            /* grid_shape                                             */
  int32_t kh, kw;          /* kernel_size, both odd                                  */
  int32_t M;               /* directions                                             */
  int32_t depth;           /* d >= 1                                                 */
  int32_t padding;         /* nc_padding                                             */
  int32_t n_in;            /* input values per sample (sum over input ports)         */
  int32_t n_out;           /* output cells per sample (out_h * out_w)                */
  int32_t act;             /* nc_activation of hidden steps                          */
  int32_t final_act;       /* nc_activation of the output step (NC_ACT_NONE = None)  */
  float act_slope;         /* leaky_relu negative slope of `act`                     */
  float final_act_slope;   /* leaky_relu negative slope of `final_act`               */
  int32_t norm;            /* spatial standardisation on (1) / off (0)               */
  int32_t hard_pin_io;     /* params.py:55-79                                        */
  int32_t gated_filters;   /* propagator.py:262-264: filters -> sigmoid(filters)     */
  int32_t conv_algo;       /* nc_conv_algo (FFT needs both FFT sides <= 1024)        */
} nc_topo;

/* Per-call Codd options (traced scalars in the reference, trainer.py:285-302). */
typedef struct nc_codd {
  int32_t mode;            /* nc_codd_mode */
  float temperature;       /* tau, clamped to >= 1e-4 as params.py:63 */
  float active_threshold;  /* ste_ternary role-2 threshold (default 0.6) */
  /* Optional device scalar: when not null the kernels read tau from it when they run, so a
     captured CUDA graph replays with the current value (the reference passes tau as a
     traced scalar for the same reason).  Null: `temperature` is used. */
  const float* temperature_dev;
} nc_codd;

/* ---- plan: device copy of the static port tables and masks -------------------------- */

/* Bytes of the device plan buffer for `topo` (256-byte aligned buffer required). */
size_t nc_plan_bytes(const nc_topo* topo);

/*
 * Copies the host tables into the caller's device buffer `d_plan` (stream-ordered).
 *   in_index[n_in]    flat grid index r*W+c of each input value, -1 to drop it
 *                     (neurocell/propagator.py:103-191 injection order)
 *   out_index[n_out]  flat grid index r*W+c of each output cell, pairwise distinct
 *                     (neurocell/epilogue.py:82-128 gather order; a repeated cell, which
 *                     the reference's gather allows, is refused with NC_ERR_UNSUPPORTED);
 *                     cells outside the ROI
 *                     (VALID border) are served by nc_vnn_forward_universe (the reference's
 *                     full-grid output path) -- nc_vnn_forward writes NaN for them
 *   io_mask[H*W]      io_state_mask      (neurocell/topology.py:241-253), 0/1 bytes
 *   out_w_mask[H*W]   out_weight_mask    (neurocell/topology.py:245-253), 0/1 bytes
 *   border_mask[H*W]  1 where the VALID border template border_2d applies, 0 where it is
 *                     forced to zero; null = all ones.  Zeros mark the cells of an adaptive
 *                     sub-ROI window that lie inside the full ROI (the reference zeroes the
 *                     whole ROI of border_2d before cropping, propagator.py:354-366).
 */
nc_status nc_plan_build(const nc_topo* topo, const int32_t* in_index, const int32_t* out_index,
                        const uint8_t* io_mask, const uint8_t* out_w_mask,
                        const uint8_t* border_mask, void* d_plan, size_t plan_bytes, void* stream);

/* ---- forward / backward ---------------------------------------------------------------- */

#define NC_FLAG_TRAIN 1u   /* forward saves what nc_vnn_backward needs */

/* Workspace bytes for `batch` samples (flags: NC_FLAG_TRAIN or 0). */
size_t nc_workspace_bytes(const nc_topo* topo, int32_t batch, uint32_t flags);

/*
 * Forward propagation (propagate_vnn_2d, return_universe=False):
 *   cell_params (3,H,W) = [W, B, S_raw]; filters (M,1,kh,kw) OIHW; inputs (batch, n_in)
 *   out (batch, n_out).  With NC_FLAG_TRAIN the workspace keeps the residuals for one
 *   following nc_vnn_backward call with the same arguments.
 */
nc_status nc_vnn_forward(const nc_topo* topo, const void* d_plan, const float* cell_params,
                         const float* filters, const float* inputs, int32_t batch,
                         const nc_codd* codd, uint32_t flags, float* out, void* d_ws,
                         size_t ws_bytes, void* stream);

/*
 * Vector-Jacobian product of nc_vnn_forward w.r.t. the parameters:
 *   g_out (batch, n_out) -> g_cell_params (3,H,W), g_filters (M,1,kh,kw)  (overwritten).
 * Deterministic: no floating-point atomics; the batch reduction order is fixed.
 */
nc_status nc_vnn_backward(const nc_topo* topo, const void* d_plan, const float* cell_params,
                          const float* filters, const float* inputs, int32_t batch,
                          const nc_codd* codd, const float* g_out, float* g_cell_params,
                          float* g_filters, void* d_ws, size_t ws_bytes, void* stream);

/*
 * propagate_vnn_2d(..., return_universe=True) (neurocell/propagator.py:657-734 and the
 * CIRCULAR branch 330-341): the last step runs the ROI epilogue with the final activation
 * over the whole ROI; universe (batch, H, W) holds those cells, on the VALID ring
 * f(B) * s_prob (B * s_prob without a final activation), with f applied to every cell;
 * out (batch, n_out) are the port cells of the universe (equal to nc_vnn_forward's).
 * Same plan and workspace as nc_vnn_forward.
 */
nc_status nc_vnn_forward_universe(const nc_topo* topo, const void* d_plan, const float* cell_params,
                                  const float* filters, const float* inputs, int32_t batch,
                                  const nc_codd* codd, uint32_t flags, float* out, float* universe,
                                  void* d_ws, size_t ws_bytes, void* stream);

/*
 * Vector-Jacobian product of nc_vnn_forward_universe from the gradients of both results:
 * g_out (batch, n_out, may be null) and g_universe (batch, H, W).
 */
nc_status nc_vnn_backward_universe(const nc_topo* topo, const void* d_plan, const float* cell_params,
                                   const float* filters, const float* inputs, int32_t batch,
                                   const nc_codd* codd, const float* g_out, const float* g_universe,
                                   float* g_cell_params, float* g_filters, void* d_ws,
                                   size_t ws_bytes, void* stream);

/*
 * Full-grid universe of an adaptive sub-ROI call (neurocell/propagator.py:700-718 with
 * roi_bbox, then 726-733).  The sub-ROI runs as its own plan over a grid window of the chip
 * (nc_vnn_forward_universe on the window's cell parameters gives universe_window, shape
 * (batch, win_h, win_w)); this call places it in the full grid.  topo / d_plan describe the
 * FULL chip (VALID or SAME).  The window's top-left grid cell is (win_row, win_col).
 * Writes universe (batch, H, W): the window copied in, every other cell f(f(B) * s_prob)
 * on VALID chips (B * s_prob without a final activation) and f(0) on SAME chips.  When out
 * is not null it also writes out (batch, n_out), gathered from universe at the full plan's
 * output cells.
 */
nc_status nc_universe_embed_forward(const nc_topo* topo, const void* d_plan, const float* cell_params,
                                    const nc_codd* codd, int32_t win_row, int32_t win_col,
                                    int32_t win_h, int32_t win_w, const float* universe_window,
                                    int32_t batch, float* universe, float* out, void* stream);

/*
 * Vector-Jacobian product of nc_universe_embed_forward.  Inputs: g_out (batch, n_out) and
 * g_universe (batch, H, W); either may be null.  Writes g_universe_window
 * (batch, win_h, win_w) and g_cell_params (3, H, W).  g_cell_params is the gradient of the
 * cells outside the window.  Inside the window it is zero, because the window's parameters
 * get their gradient from the sub-ROI call's own backward.
 */
nc_status nc_universe_embed_backward(const nc_topo* topo, const void* d_plan, const float* cell_params,
                                     const nc_codd* codd, int32_t win_row, int32_t win_col,
                                     int32_t win_h, int32_t win_w, const float* g_out,
                                     const float* g_universe, int32_t batch, float* g_universe_window,
                                     float* g_cell_params, void* stream);

/*
 * nc_vnn_forward_static -- no counterpart in the reference.  Inference forward (flags 0)
 * that takes no workspace: its scratch is a static device array of
 * NC_STATIC_SCRATCH_BYTES inside this library, held on every GPU that loads the library
 * until the process exits.  It is for callers that cannot call cudaMalloc: an XLA FFI
 * custom call whose framework already owns nearly all device memory, code running while a
 * stream is being captured, hosts that forbid allocation after start-up.  The caller
 * still allocates the plan, parameters, inputs and outputs.
 *   - Returns NC_ERR_WORKSPACE when nc_workspace_bytes(topo, batch, 0) exceeds the limit.
 *   - The first call on a device resolves the array's device address (with that device
 *     current); make that first call before any stream capture.
 *   - All calls share the one array, which keeps the previous call's contents; nothing in
 *     it has to start at zero.  Calls that overlap on the GPU (other streams, concurrent
 *     graph replays) race on it and must be serialised by the caller.
 *   - Allocates nothing: no cudaMalloc, cudaFree or allocating library routine.
 */
#define NC_STATIC_SCRATCH_BYTES (8u * 1024u * 1024u)
nc_status nc_vnn_forward_static(const nc_topo* topo, const void* d_plan, const float* cell_params,
                                const float* filters, const float* inputs, int32_t batch,
                                const nc_codd* codd, float* out, void* stream);

/* Effective Codd states s_prob (H,W) (params.py:31-80); d_plan supplies io_mask. */
nc_status nc_codd_states(const nc_topo* topo, const void* d_plan, const float* states_raw,
                         const nc_codd* codd, float* s_prob, void* stream);

/* ---- losses and update ----------------------------------------------------------------- */

/* MSE over batch*n values: loss[0] = mean((out-y)^2); g_out = d loss / d out.
   `loss` (both losses) may be device memory or page-locked host memory mapped for the
   device, which the kernel then writes directly (no separate device-to-host copy);
   pageable host memory is refused with NC_ERR_INVALID before any launch. */
nc_status nc_mse_loss(const float* out, const float* targets, int32_t batch, int32_t n,
                      float* loss, float* g_out, void* stream);

/* Mean softmax cross-entropy over `batch` rows of `n` logits with int32 labels. */
nc_status nc_softmax_ce_loss(const float* logits, const int32_t* labels, int32_t batch,
                             int32_t n, float* loss, float* g_logits, void* stream);

/*
 * Batch staging without the copy engine (no counterpart in the reference): copies `nseg`
 * (1..NC_MAX_STAGE_SEGS) byte ranges into device buffers with one kernel that reads the
 * sources directly.  Every source must be page-locked host memory mapped for the device
 * (cudaHostAlloc, or cudaHostRegister with mapping; device memory works too), checked with
 * cudaPointerGetAttributes before the launch: pageable memory is refused with
 * NC_ERR_INVALID.  Sizes and addresses are multiples of 4 bytes.  A training step's batch
 * of a few KB costs about 9 us per cudaMemcpyAsync on the GPU timeline; one such kernel
 * takes the place of the step's input copies.  Stream-ordered: the sources must stay
 * unchanged until the stream has run the kernel.
 */
#define NC_MAX_STAGE_SEGS 4
typedef struct nc_stage_seg {
  void* dst;          /* device buffer                                   */
  const void* src;    /* page-locked, device-mapped host memory (or device) */
  size_t bytes;
} nc_stage_seg;
nc_status nc_stage_from_host(const nc_stage_seg* segs, int32_t nseg, void* stream);

/* In-place SGD: params[i] -= lr * grads[i]  (lr read from host scalar). */
nc_status nc_sgd_update(float* params, const float* grads, int64_t n, float lr, void* stream);

/* ---- data-parallel gradient exchange over NVLink ---------------------------------------- */
/*
 * No counterpart in the reference (it has no multi-GPU code; the north star asks for the
 * ~16k-parameter gradient to be all-reduced across 1/2/4/8 GPUs).  nc_dp_allreduce_sgd
 * fuses the cross-GPU gradient sum with the SGD update in one kernel: every rank stores
 * its packed gradient into its slot of every peer's double-buffered receive buffer over
 * NVLink, each value in one 64-bit element together with the current step number (so a
 * value and its tag always arrive together), waits (bounded) until the elements of all
 * peers in its own buffer carry this step's tag, sums them in rank order from local memory
 * (bitwise identical on every rank) and updates its parameters.
 * Set-up: nc_dp_alloc on every rank, exchange nc_ipc_get handles (e.g. all_gather), open
 * the peers' buffers with nc_ipc_open, zero-initialised state from nc_dp_alloc.
 * Step counters live on the device, so the call can be captured in a CUDA graph.
 */
#define NC_DP_MAX_RANKS 8
#define NC_IPC_HANDLE_BYTES 64

/* Device bytes of the shared receive buffer for n parameters and world ranks (0 when
   world is outside 1..NC_DP_MAX_RANKS). */
size_t nc_dp_shared_bytes(int64_t n, int32_t world);
/* Device bytes of the private per-rank state (step counters, status word). */
size_t nc_dp_state_bytes(void);
/* Set-up time allocations (cudaMalloc + zero fill); not for the hot path. */
nc_status nc_dp_alloc(size_t bytes, void** d_ptr);
nc_status nc_dp_free(void* d_ptr);
/* CUDA IPC of a buffer from nc_dp_alloc: handle_out receives NC_IPC_HANDLE_BYTES bytes. */
nc_status nc_ipc_get(void* d_ptr, void* handle_out);
nc_status nc_ipc_open(const void* handle, void** d_peer_ptr);
nc_status nc_ipc_close(void* d_peer_ptr);

/*
 * grads[n] (this rank's gradient of its mean loss) -> grads[n] = sum over ranks,
 * params[n] -= lr / world * grads[n].  peers[world] are the shared buffers of all ranks
 * (this rank's own at index rank).
 * Failure: a peer that does not arrive within max_wait_iters polls of one line sets the
 * status word (read it with nc_dp_status: 0 = ok, 1 = a peer timed out).  The lines whose
 * peers did not arrive are left untouched; lines whose peers did arrive in that call were
 * updated, so the ranks' parameters no longer agree.  The status is terminal: every later call on
 * this state returns without storing to peers or updating, which makes every peer time out
 * at its next step too.  To go on, restore the parameters from a consistent copy, call
 * nc_dp_reset on every rank and pass a host barrier before the next exchange.
 */
nc_status nc_dp_allreduce_sgd(void* const* peers, int32_t world, int32_t rank, void* d_state,
                              float* grads, float* params, int64_t n, float lr,
                              int32_t max_wait_iters, void* stream);
/* Copies the device status word of d_state to *status (synchronises the stream). */
nc_status nc_dp_status(const void* d_state, int32_t* status, void* stream);
/*
 * Clears this rank's state (step counters, status word) and its own receive buffer
 * (d_shared, shared_bytes from nc_dp_shared_bytes), stream-ordered.  Every rank resets, then
 * the ranks pass a host barrier, with no exchange kernel in flight on any rank.
 */
nc_status nc_dp_reset(void* d_state, void* d_shared, size_t shared_bytes, void* stream);

/* ---- measurement ----------------------------------------------------------------------- */

/*
 * Profiling hook (no reference counterpart): when non-null, nc_vnn_forward records
 * `fwd_start`/`fwd_stop` (cudaEvent_t) on its stream immediately around its fused
 * propagation kernel, and nc_vnn_backward records `bwd_start`/`bwd_stop` around its fused
 * adjoint kernel.  Applies to calls made from the calling host thread; pass nulls to stop.
 */
void nc_set_profile_events(void* fwd_start, void* fwd_stop, void* bwd_start, void* bwd_stop);

/*
 * FP32 FFMA throughput probe (no reference counterpart): launches a dependent-chain FFMA
 * loop on every SM of the current device and writes the FLOPs it performs to *flops.
 * Time it with CUDA events on `stream` to obtain the device's FP32-pipe peak.
 */
nc_status nc_fp32_peak_probe(int32_t iters, double* flops, float* sink, void* stream);

/* ---- misc ------------------------------------------------------------------------------ */

/* Message of the last failing call on this host thread ("" if none). */
const char* nc_last_error(void);

/*
 * Status word of a workspace (the first 4 bytes of every layout): 0 ok; 1 when a kernel of
 * the latest nc_vnn_forward / nc_vnn_forward_universe on d_ws, or of a backward after it,
 * gave up a bounded wait for its own asynchronous copies into shared memory (every result
 * of that call is then invalid).  Each forward clears it when it starts; calls on other
 * workspaces never touch it.  Copies the word to *status and synchronises the stream;
 * not for the hot path.
 */
nc_status nc_workspace_status(const void* d_ws, int32_t* status, void* stream);

/* NC_ABI_VERSION of the loaded library. */
int32_t nc_abi_version(void);

/* Number of kernels this library has launched in the process so far (all host threads;
 * launches recorded into a CUDA graph count once, at capture). */
uint64_t nc_launch_count(void);

/* Which kernels nc_vnn_forward / nc_vnn_backward run for `topo` (no reference counterpart):
 * 1 = direct per-sample kernels, 2 = FFT per-step kernels, 3 = fused per-sample FFT kernels
 * (64 x 64 FFT grids); 0 if the topology is invalid. */
int32_t nc_conv_path(const nc_topo* topo);

#ifdef __cplusplus
}
#endif
#endif /* NEUROCELL_B200_H_ */
