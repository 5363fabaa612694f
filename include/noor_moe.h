/*
 * noor_moe.h -- C ABI of the B200 (sm_100a) sparse-MoE layer forward.
 *
 * This is the drop-in boundary for Noor's noor-core MoE path.  Today the Rust
 * layer code calls a matmul-level FFI (crates/noor-core/src/kernels.rs:141,
 * `matmul_dispatch`, which reaches cblas_sgemm / noor_matmul_f32 / cuBLAS,
 * kernels.rs:6-51, 93-137).  The entry points below replace it at layer level
 * so that `MoELayer::forward` (crates/noor-core/src/layers/moe.rs:145) and
 * `ParallelFFN::forward` (crates/noor-core/src/layers/parallel_ffn.rs:30) keep
 * their signatures and hand the whole layer to the GPU in one call.
 *
 * Conventions (all entry points):
 *  - every function returns an int status, NOOR_MOE_OK (0) on success; the
 *    library never aborts the process.  noor_moe_last_error() gives a
 *    thread-local message for the last failure on the calling thread;
 *  - the caller owns input and output buffers; the library owns device
 *    weights and workspaces;
 *  - pointer mode is chosen by `stream`: stream == NULL means host pointers
 *    and a synchronous call (the reference returns Tensors by value);
 *    stream != NULL means device pointers, enqueued on that cudaStream_t;
 *  - a handle is bound to one (layer, device) and is not re-entrant; distinct
 *    handles may be used from distinct threads.
 */
#ifndef NOOR_MOE_H
#define NOOR_MOE_H

#include <stdint.h>

#if defined(__GNUC__)
#define NOOR_MOE_API __attribute__((visibility("default")))
#else
#define NOOR_MOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define NOOR_MOE_OK 0
#define NOOR_MOE_ERR_INVALID 1     /* bad argument or shape */
#define NOOR_MOE_ERR_CUDA 2        /* a CUDA runtime/driver call failed */
#define NOOR_MOE_ERR_NCCL 3        /* an NCCL call failed or timed out */
#define NOOR_MOE_ERR_OOM 4         /* device allocation failed */
#define NOOR_MOE_ERR_STATE 5       /* call out of order (e.g. forward before weights) */
#define NOOR_MOE_ERR_TIMEOUT 6     /* a device-side bounded wait gave up */
#define NOOR_MOE_ERR_UNSUPPORTED 7 /* shape outside what the kernels implement */

#define NOOR_DTYPE_F32 0   /* f32 storage and f32 CUDA-core math (the reference's dtype) */
#define NOOR_DTYPE_BF16 1  /* BF16 storage, tcgen05 tensor cores, f32 accumulation */

#define NOOR_ACT_GELU_TANH 0 /* GeGLU dense branch, tensor.rs:438-449 (reference default) */
#define NOOR_ACT_SILU 1      /* SwiGLU */

/* Layer descriptor.  Mirrors the `[moe]` config block
 * (crates/noor-core/src/config.rs:32-39) and ParallelFFN::new
 * (parallel_ffn.rs:14-27). */
typedef struct {
  int32_t d_model;
  int32_t n_experts;   /* E */
  int32_t top_k;       /* n_active; clamped to E like moe.rs:99 */
  int32_t expert_ff;   /* SwiGLU expert hidden size */
  int32_t dense_ff;    /* parallel dense branch hidden size */
  int32_t has_shared;  /* unweighted shared SwiGLU expert (moe.rs:168-173) */
  int32_t has_dense;   /* 1: ParallelFFN::forward, (dense + moe)/sqrt(2); 0: MoELayer::forward */
  int32_t dtype;       /* NOOR_DTYPE_* */
  int32_t dense_act;   /* NOOR_ACT_*; the reference's dense branch is GELU_TANH */
  int32_t device;      /* CUDA ordinal this handle lives on */
  int32_t world_size;  /* expert-parallel group size (1 = single GPU) */
  int32_t rank;        /* this process's rank in the group */
  int64_t max_tokens;  /* tokens per call the workspaces are sized for (grown on demand) */
} noor_moe_desc;

typedef struct noor_moe_handle noor_moe_handle;

/* Create a layer handle.  `nccl_comm` is an ncclComm_t spanning world_size
 * ranks (from noor_moe_comm_init_rank), or NULL when world_size == 1.
 * Replaces constructing MoELayer / ParallelFFN (moe.rs:119-143,
 * parallel_ffn.rs:14-27) on the host. */
NOOR_MOE_API int noor_moe_create(const noor_moe_desc* desc, void* nccl_comm, noor_moe_handle** out);

/* Upload weights given in the reference's f32 row-major layouts; the library
 * rounds to BF16 (RNE, tensor.rs:23-28) for BF16 layers and prepacks them
 * K-major for the tensor cores.  Expert arrays hold E pointers (one Tensor per
 * SwiGLUFFN in Vec<SwiGLUFFN>, moe.rs:112); under expert parallelism only the
 * rank's own E/world_size entries are read and the rest may be NULL.
 *   gate   [d, E]   MoERouter::gate (moe.rs:7)
 *   bias   [E]      MoERouter::expert_biases (SMEBU, moe.rs:9)
 *   scales [E]      MoERouter::expert_scales (moe.rs:11)
 *   w_gate[e], w_up[e] [d, ff];  w_down[e] [ff, d]   (ffn.rs:43-50)
 *   shared[3]  nullable {w_gate, w_up, w_down} of the shared expert
 *   dense[3]   {w_gate [d,dff], w_up [d,dff], w_down [dff,d]} (ffn.rs:5-12); NULL if has_dense == 0 */
NOOR_MOE_API int noor_moe_load_weights(noor_moe_handle* h, const float* gate, const float* bias,
                          const float* scales, const float* const* w_gate,
                          const float* const* w_up, const float* const* w_down,
                          const float* const* shared, const float* const* dense);

/* Replace the SMEBU router bias (host f32 [E]); the per-step path of
 * SMEBU::apply_to_router (crates/noor-train/src/optim/smebu.rs:56-61). */
NOOR_MOE_API int noor_moe_set_bias(noor_moe_handle* h, const float* bias);

/* Layer forward over T tokens: MoELayer::forward (moe.rs:145-177) when
 * has_dense == 0, ParallelFFN::forward (parallel_ffn.rs:30-36) otherwise.
 * x [T, d] and out [T, d] are f32 for F32 layers and BF16 bit patterns
 * (uint16) for BF16 layers.  Optional outputs (NULL to skip):
 *   topk_idx [T, k] int32   RouteResult::indices, rank order (moe.rs:17-22)
 *   topk_w   [T, k] f32     RouteResult::weights = sigmoid score * scale
 *   expert_counts [E] int64 this call's ExpertUtilization::record counts
 *                           (moe.rs:40-45), summed over all ranks under EP
 * In device mode (stream != NULL) all pointers are device pointers; for BF16
 * layers x and out must be 16-byte aligned (the tensor cores read x through
 * TMA), else NOOR_MOE_ERR_INVALID.
 * Under expert parallelism every rank calls this collectively with its own
 * T tokens. */
NOOR_MOE_API int noor_moe_forward(noor_moe_handle* h, const void* x, void* out, int64_t T, int32_t* topk_idx,
                     float* topk_w, int64_t* expert_counts, void* stream);

/* The MoE block's FFN sublayer with its sandwich norm (block.rs:87-90,
 * norm.rs:31-60): out = x + rms_norm(F(rms_norm(x, w_pre) * depth_scale),
 * w_post) * depth_scale, F the layer of noor_moe_forward; rms_norm as
 * tensor.rs:462-490 (sum of squares and division in f64).  x is the
 * residual stream h.  Same pointer, dtype, EP and optional-output rules as
 * noor_moe_forward (the routing outputs describe F's input).  Needs
 * noor_moe_set_sandwich first (NOOR_MOE_ERR_STATE otherwise). */
NOOR_MOE_API int noor_moe_ffn_sublayer_forward(noor_moe_handle* h, const void* x, void* out, int64_t T,
                                               int32_t* topk_idx, float* topk_w, int64_t* expert_counts,
                                               void* stream);
/* SandwichNorm's parameters: pre_norm.weight and post_norm.weight [d] (f32,
 * host), eps (RMSNorm eps, f64) and depth_scale (1/sqrt(layer_idx + 1) in
 * f32, norm.rs:44). */
NOOR_MOE_API int noor_moe_set_sandwich(noor_moe_handle* h, const float* pre_w, const float* post_w, double eps,
                                       float depth_scale);

/* Load MoE block `layer` of a Noor GGUF v3 checkpoint (gguf.rs:153-233, the
 * tensor names of collect_model_tensors, gguf.rs:262-280) straight into the
 * handle: blocks.<layer>.moe.router.{gate [d,E], biases [E], scales [E]},
 * .moe.experts.<e>.{w_gate, w_up [d,ff], w_down [ff,d]} for this rank's
 * experts only, .moe.shared.* (has_shared) and .dense.{w_gate, w_up [d,dff],
 * w_down [dff,d]} (has_dense), F32 or F16 on disk, then the same device
 * prepack as noor_moe_load_weights.  With norm_eps >= 0 it also loads
 * .ffn_norm.{pre,post}.weight [d] and calls noor_moe_set_sandwich with that
 * eps and depth_scale = 1/sqrt(layer + 1).  A missing tensor, a wrong shape
 * or a malformed file returns NOOR_MOE_ERR_INVALID naming it. */
NOOR_MOE_API int noor_moe_load_gguf(noor_moe_handle* h, const char* path, int32_t layer, double norm_eps);
/* Host only: dims (up to 8), n_dims and dtype (0 F32, 1 F16) of one tensor
 * of a GGUF file; NOOR_MOE_ERR_INVALID if the file is malformed or has no
 * such tensor. */
NOOR_MOE_API int noor_gguf_tensor_info(const char* path, const char* name, int64_t* dims, int32_t* n_dims,
                                       int32_t* dtype);
/* Host only: one tensor of a GGUF file as f32 (F16 converted exactly), n its
 * element count. */
NOOR_MOE_API int noor_gguf_read_f32(const char* path, const char* name, float* out, int64_t n);

/* Router only: the batched form of MoERouter::route (moe.rs:79-107) plus the
 * utilization histogram.  Same pointer and dtype rules as noor_moe_forward;
 * idx and w are required, counts may be NULL. */
NOOR_MOE_API int noor_moe_route(noor_moe_handle* h, const void* x, int64_t T, int32_t* idx, float* w,
                   int64_t* counts, void* stream);

/* Matmul-level entry point, the live route of kernels.rs:141-163
 * (cblas_sgemm row-major, alpha = 1, beta = 0): C[m,n] = A[m,k] . B[k,n],
 * f32, host pointers, C overwritten.  Runs on the current device. */
NOOR_MOE_API int noor_matmul_f32(const float* a, const float* b, float* c, int64_t m, int64_t k, int64_t n);

/* Thread-local message describing the last failure on this thread ("" if none). */
NOOR_MOE_API const char* noor_moe_last_error(void);

/* Wait for the handle's work on `stream` (NULL = its internal stream) and
 * report any error a kernel flagged on the device (e.g. a bounded wait that
 * timed out, NOOR_MOE_ERR_TIMEOUT).  Clears the flag. */
NOOR_MOE_API int noor_moe_sync(noor_moe_handle* h, void* stream);

NOOR_MOE_API void noor_moe_destroy(noor_moe_handle* h);

/* ---- expert-parallel communicator (NCCL over NVLink / NVSwitch) ---- */

/* Size in bytes of the opaque unique id (NCCL_UNIQUE_ID_BYTES). */
NOOR_MOE_API int noor_moe_comm_id_size(void);
/* Rank 0 creates the id and ships it to the other ranks out of band. */
NOOR_MOE_API int noor_moe_comm_get_id(void* id_out);
/* Collective over world_size ranks; call with the handle's device current. */
NOOR_MOE_API int noor_moe_comm_init_rank(const void* id, int world_size, int rank, int device, void** comm_out);
NOOR_MOE_API int noor_moe_comm_destroy(void* comm);

/* Plan of one expert-parallel exchange, from this rank's per-expert counts
 * counts_local [E] and the counts every rank sent for this rank's experts
 * counts_recv [G][E/G].  Outputs, per peer rank r: send_rows/send_off (rows of
 * the expert-ordered send buffer bound for r) and recv_rows/recv_off (rows
 * arriving from r); and the receive-side grouped-GEMM table of G*E/G groups,
 * group j = (source rank j / (E/G), local expert j % (E/G)): grp_row [G*El+1]
 * (first row), grp_mtile [G*El+1] (first BM-row tile), grp_widx [G*El+1]
 * (local expert).  Pure host arithmetic; the library uses it inside
 * noor_moe_forward and exports it for hosts that run their own transport. */
NOOR_MOE_API int noor_moe_ep_plan(const int64_t* counts_local, const int64_t* counts_recv, int E, int G, int BM,
                                  int64_t* send_rows, int64_t* send_off, int64_t* recv_rows, int64_t* recv_off,
                                  int32_t* grp_row, int32_t* grp_mtile, int32_t* grp_widx);

/* Plan of rank `me` under the peer-memory exchange (the arithmetic the
 * device runs inside noor_moe_forward, here on the host, e.g. to check it
 * for any rank count): from the full count matrix cnt [G][E] (picks of
 * expert e made on rank src), the receive group table of G*E/G = E groups in
 * (local expert, source rank) order -- grp_row [E+1] (first row in the
 * receive buffer), grp_mtile [E+1] (first BM-row tile), grp_widx [E] (local
 * expert), grp_orank [E] (source rank), grp_oshift [E] (output row on the
 * source minus the receive row) -- plus dest_base [E] (first receive row, on
 * expert e's owner, of rank me's picks of e) and counts_glob [E].  Pure host
 * arithmetic. */
NOOR_MOE_API int noor_moe_peer_plan(const int64_t* cnt, int G, int E, int me, int BM, int32_t* grp_row,
                                    int32_t* grp_mtile, int32_t* grp_widx, int32_t* grp_orank, int32_t* grp_oshift,
                                    int32_t* dest_base, int64_t* counts_glob);

/* How a handle's ranks exchange rows (no counterpart in the reference, which
 * runs on one device).  With world_size > 1, noor_moe_create is collective
 * and picks, the same on every rank:
 *   NOOR_MOE_EP_PEER  BF16 layers whose GPUs all reach each other: the rows
 *       move through the ranks' buffers mapped with CUDA IPC (NVLink stores
 *       from the permute and from the expert down projection's epilogue),
 *       synchronised by bounded device-side flag barriers; no host sync
 *       inside a forward.  Each rank's T may not exceed the largest
 *       max_tokens given at creation: a larger batch returns
 *       NOOR_MOE_ERR_INVALID on its rank and every rank skips that step
 *       (the others report it as NOOR_MOE_ERR_INVALID from the device).  A
 *       rank that waits longer than NOOR_MOE_PEER_TIMEOUT_MS (environment,
 *       default 10000) for another returns NOOR_MOE_ERR_TIMEOUT and the
 *       exchange stays closed for the handle.
 *   NOOR_MOE_EP_NCCL  otherwise (or NOOR_MOE_EP_TRANSPORT=nccl): a count
 *       exchange, a host-built plan and NCCL all-to-all-v.
 * Returns NOOR_MOE_EP_NONE for a single-GPU handle, -1 for NULL. */
#define NOOR_MOE_EP_NONE 0
#define NOOR_MOE_EP_NCCL 1
#define NOOR_MOE_EP_PEER 2
NOOR_MOE_API int noor_moe_ep_transport(const noor_moe_handle* h);

/* ---- expert utilization and the SMEBU bias update on the device ---- */

/* The handle accumulates, on the device, the layer's ExpertUtilization
 * (moe.rs:25-65) over every noor_moe_forward since the last reset: counts[E]
 * (picks per expert) and tokens, the global ones under expert parallelism
 * (the same on every rank).  noor_moe_route does not record, as
 * MoERouter::route does not.
 * noor_moe_utilization copies them to the host (counts [E] and tokens, each
 * nullable) after the work queued on `stream` (NULL = the handle's stream),
 * and with reset != 0 clears them (ExpertUtilization::reset). */
NOOR_MOE_API int noor_moe_utilization(noor_moe_handle* h, int64_t* counts, int64_t* tokens, int reset,
                                      void* stream);
/* One training step's bias refresh, on the device: fractions = counts /
 * tokens (ExpertUtilization::fractions, model.rs:180-183), SMEBU::update
 * (smebu.rs:36-48) on the handle's momentum, and apply_to_router
 * (smebu.rs:56-61): the new biases go straight into the router bias the next
 * forward reads; the utilization is reset.  Asynchronous on `stream` (NULL:
 * the handle's stream, synchronous).  Under expert parallelism every rank
 * calls it and all get the same biases. */
NOOR_MOE_API int noor_moe_smebu_update(noor_moe_handle* h, float kappa, float beta, float lambda, void* stream);
/* Read (get, nullable) and/or overwrite (set, nullable) the SMEBU momentum
 * [E] (zeros at creation), e.g. for checkpoints.  Synchronous. */
NOOR_MOE_API int noor_moe_smebu_momentum(noor_moe_handle* h, float* get, const float* set);
/* Copy the router bias [E] the next forward will use to the host. */
NOOR_MOE_API int noor_moe_get_bias(noor_moe_handle* h, float* bias);

/* ---- measurement hooks (CUDA events on the launching stream) ---- */

/* Begin recording a start/stop event pair around every kernel the handle
 * launches, for at most `max_launches` launches. */
NOOR_MOE_API int noor_moe_profile_begin(noor_moe_handle* h, int max_launches);
/* Stop recording, synchronise, and fill per-kernel totals.  names is a buffer
 * of n_slots * 32 chars (NUL-terminated names), total_ms / launches have
 * n_slots entries.  Returns the number of distinct kernels in *n_out. */
NOOR_MOE_API int noor_moe_profile_end(noor_moe_handle* h, char* names, float* total_ms, int32_t* launches,
                         int n_slots, int* n_out);
/* Number of kernels this handle has launched since creation. */
NOOR_MOE_API int64_t noor_moe_launch_count(const noor_moe_handle* h);

/* ---- routing for callers that cannot allocate device memory ---- */

/* Size of the library's fixed routing scratch (one per GPU, held until exit). */
#define NOOR_MOE_STATIC_SCRATCH_BYTES (8 * 1024 * 1024)

/* No counterpart in the reference: an addition of this library.
 * The router plus utilization histogram of noor_moe_route, without a handle
 * and without any device allocation, for callers that cannot call cudaMalloc
 * (code recording a CUDA graph, where allocation is not allowed during
 * capture, or hosts that give all device memory to their own pool up front).
 * All pointers are device pointers; the call is enqueued on `stream`.
 *   x       [T, d]  f32 (dtype F32) or BF16 bits (dtype BF16)
 *   gate    F32: [d, E] f32, the reference layout (moe.rs:7);
 *           BF16: [roundup(E, 8), d] BF16 bits, the gate transposed, rows >= E zero
 *   (BF16: x and gate 16-byte aligned; the tensor cores read them through TMA)
 *   bias, scales [E] f32;  outputs idx [T, k] int32, w [T, k] f32, counts [E] int64.
 * Working memory comes from one fixed array of NOOR_MOE_STATIC_SCRATCH_BYTES
 * per GPU; a call whose T, E, k would need more returns NOOR_MOE_ERR_INVALID
 * (E = 32, k = 4: about 450k tokens for BF16, 57k for F32, which also keeps
 * the f32 scores there).  The first call on each device looks up the array's
 * device address; make that first call before any stream capture.  The
 * address is kept for the life of the process, so do not call this again on a
 * device after cudaDeviceReset.  Every call shares the array and it keeps the
 * last call's contents, so calls that can overlap on the GPU (different
 * streams, different host threads) race: serialise them.
 * Errors found on the host return a status; a bounded wait on the device that
 * gives up (BF16 router) cannot, since the call returns before the work runs:
 * it is reported in the outputs instead, as every counts[e] == -1.  Check
 * counts[0] >= 0 once the stream's work has completed. */
NOOR_MOE_API int noor_moe_route_static(const void* x, const void* gate, const float* bias, const float* scales,
                                       int64_t T, int32_t d, int32_t E, int32_t top_k, int32_t dtype,
                                       int32_t* idx, float* w, int64_t* counts, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NOOR_MOE_H */
