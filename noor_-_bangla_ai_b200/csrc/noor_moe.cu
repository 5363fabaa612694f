// noor_moe.cu -- C ABI, handle, weight prepack and per-call orchestration of
// the B200 sparse-MoE layer forward.
//
// One call of noor_moe_forward runs, on the caller's stream:
//   K1  router            x -> top-k idx / weights, per-block ranks + histogram
//   scan                  histograms -> expert segments, per-block bases, GEMM tile table
//   K2  permute           x rows -> expert-contiguous rows (dst_row per pick)
//   [EP] the rows go to the rank that owns their expert: over NVLink peer
//        memory (BF16: the permute stores into the owner's receive buffer,
//        the down projection's epilogue stores the outputs back), else as a
//        count exchange + all-to-all-v through NCCL send/recv
//   K3  expert GEMM 1     rows . [Wg|Wu]^T  -> silu(g)*u      (tcgen05, SwiGLU epilogue)
//   K3  expert GEMM 2     h . Wd^T          -> y
//   dense branch          x . [Wg|Wu]^T -> gelu(g)*u -> . Wd^T
//   K4  combine           out = (dense + sum_i w_i y_i) / sqrt(2)   (the dense down projection's epilogue)
// which is ParallelFFN::forward (crates/noor-core/src/layers/parallel_ffn.rs:30-36)
// over MoELayer::forward (moe.rs:145-177).
#include <cuda.h>
#include <cuda_runtime.h>
#include <nccl.h>
#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cmath>
#include <cstring>
#include <deque>
#include <string>
#include <mutex>
#include <thread>
#include <vector>

#include <unistd.h>

#include "noor_moe.h"

#include "common.cuh"
#include "gguf.h"
#include "dispatch.cuh"
#include "nccl_dyn.h"
#include "norm.cuh"
#include "peer_ep.cuh"
#include "prepack.cuh"
#include "router.cuh"
#include "router_tc.cuh"
#include "simt_gemm.cuh"
#include "smebu.cuh"
#include "tc_gemm.cuh"

using namespace noor;

// ============================================================== errors

static thread_local std::string g_last_error;

static int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

// A failed runtime call is reported by the call that made it; the runtime's
// last-error state is cleared so that it does not resurface as the launch
// error of a later, unrelated call (faults that poison the context stay).
#define CK(call)                                                                                       \
  do {                                                                                                 \
    cudaError_t e_ = (call);                                                                           \
    if (e_ != cudaSuccess) {                                                                           \
      (void)cudaGetLastError();                                                                        \
      return fail(e_ == cudaErrorMemoryAllocation ? NOOR_MOE_ERR_OOM : NOOR_MOE_ERR_CUDA,              \
                  "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__);                \
    }                                                                                                  \
  } while (0)

#define CKN(call)                                                                                      \
  do {                                                                                                 \
    if (!noor::nccl().ok) return fail(NOOR_MOE_ERR_NCCL, "libnccl.so.2 could not be loaded");          \
    ncclResult_t r_ = (call);                                                                          \
    if (r_ != ncclSuccess)                                                                             \
      return fail(NOOR_MOE_ERR_NCCL, "%s: %s (%s:%d)", #call, noor::nccl().GetErrorString(r_),         \
                  __FILE__, __LINE__);                                                                 \
  } while (0)

#define CKR(call)               \
  do {                          \
    int rc_ = (call);           \
    if (rc_ != NOOR_MOE_OK) return rc_; \
  } while (0)

// ============================================================== device buffers

// A device allocation owned by one object: freed by release() or, at the
// latest, when the object goes out of scope (function-local staging buffers,
// the handle's buffers after destroy() released them).  Not copyable.
struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  DevBuf() = default;
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  ~DevBuf() { release(); }
  int ensure(size_t n) {
    if (n <= bytes) return NOOR_MOE_OK;
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
    if (n == 0) return NOOR_MOE_OK;
    CK(cudaMalloc(&p, n));
    bytes = n;
    return NOOR_MOE_OK;
  }
  void release() {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
  }
  template <typename T>
  T* as() const { return reinterpret_cast<T*>(p); }
};

// ============================================================== tensor maps

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 2-D K-major bf16 operand [rows, K] (row stride K elements), box BK x box_rows,
// 128-byte swizzle (the UMMA K-major SW128 layout).
static int encode_kmajor(CUtensorMap* m, const void* base, int64_t rows, int64_t K, int box_rows) {
  EncodeTiledFn fn = get_encode_fn();
  if (!fn) return fail(NOOR_MOE_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return fail(NOOR_MOE_ERR_INVALID, "tensor-core operand must be 16-byte aligned");
  if ((K * 2) % 16 != 0) return fail(NOOR_MOE_ERR_INVALID, "row stride must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)std::max<int64_t>(rows, 1)};
  cuuint64_t strides[1] = {(cuuint64_t)(K * 2)};
  cuuint32_t box[2] = {(cuuint32_t)tc::BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(NOOR_MOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return NOOR_MOE_OK;
}

// ============================================================== profiling

enum KernelKind : int {
  K_ROUTER = 0, K_ROUTER_SCORES, K_ROUTER_TOPK, K_SCAN, K_PERMUTE, K_EXPERT_GEMM1, K_EXPERT_GEMM2,
  K_DENSE_GEMM1, K_DENSE_GEMM2, K_SHARED_GEMM1, K_SHARED_GEMM2, K_COMBINE, K_PREPACK, K_A2A_DISPATCH,
  K_A2A_COMBINE, K_COUNT_EXCHANGE, K_MATMUL, K_EP_PLAN, K_EP_BARRIER, K_SMEBU, K_NORM_PRE, K_NORM_POST, K_NUM
};
static const char* kKindNames[K_NUM] = {
    "router", "router_scores", "router_topk", "scan", "permute", "expert_gemm1", "expert_gemm2",
    "dense_gemm1", "dense_gemm2", "shared_gemm1", "shared_gemm2", "combine", "prepack",
    "a2a_dispatch", "a2a_combine", "count_exchange", "matmul", "ep_plan", "ep_barrier", "smebu", "norm_pre", "norm_post"};

// ============================================================== handle

struct noor_moe_handle {
  noor_moe_desc desc{};
  int E = 0, k = 0, d = 0, ff = 0, dff = 0, G = 1, rank = 0, El = 0, e0 = 0;
  bool bf16 = true;
  int dev = 0, num_sms = 148;
  ncclComm_t comm = nullptr;
  bool comm_broken = false;
  bool weights = false;

  // router
  DevBuf gate, bias, scales;  // gate: bf16 [Epad][d] (BF16) or f32 [d][E] (F32)
  int Epad = 0;
  // experts (local), dense, shared
  DevBuf w1, w2;                  // BF16 packed
  DevBuf wg32, wu32, wd32;        // F32 reference layout
  DevBuf dw1, dw2, dg32, du32, dd32;
  DevBuf sw1, sw2, sg32, su32, sd32;
  bool has_shared = false, has_dense = false;
  CUtensorMap tm_w1{}, tm_w2{}, tm_dw1{}, tm_dw2{}, tm_sw1{}, tm_sw2{};
  CUtensorMap tm_gate{};  // BF16 router gate [Epad][d], box of roundup(E, 16) rows
  int bn2 = 256;  // n-tile of GEMMs whose N is d
  bool pair2 = false;  // tensor-core GEMMs run on SM pairs (cta_group::2, 256-row tiles)
  int tile_m = 128;    // rows per GEMM tile of the group tables

  // utilization since the last reset (counts [E], then tokens) and the SMEBU
  // momentum [E], on the device
  DevBuf util, smebu_m;

  // sandwich norm of the FFN sublayer (noor_moe_ffn_sublayer_forward)
  bool sandwich = false;
  DevBuf pre_w, post_w;  // f32 [d]
  double norm_eps = 0.0;
  float depth_scale = 1.0f;
  DevBuf xn, ffn;        // normalised input and ParallelFFN output, layer dtype [capT][d]
  CUtensorMap tm_xn{};

  // workspaces
  int64_t capT = 0;
  int64_t cap_recv = 0;  // rows the receive-side buffers (xrecv, h, y) hold
  DevBuf x_in, out_buf, idx, wts, lrank, dst_row, blk_hist, blk_base, counts64, counts_glob, seg_start, mtile_start;
  DevBuf scores;
  DevBuf scan_done;  // zeroed counter for the router's fused scan
  DevBuf seg_acc;    // [E] zeroed running per-expert totals of the router's blocks
  DevBuf xp, h, y, xrecv, ysend;
  DevBuf ymap;  // [picks] token-major output row of each expert-ordered row (BF16, one GPU)
  DevBuf dense_h, dense_out, shared_h, shared_out;
  DevBuf grp_row, grp_mtile, grp_widx, cnt_recv;
  // expert parallelism over peer memory (BF16 layers whose GPUs reach each
  // other): buffers the other ranks store into, sized once for capP tokens
  // per rank and never reallocated, since the other ranks hold mappings.
  bool peer = false;
  int64_t capP = 0;                 // tokens per rank (the largest max_tokens of all ranks)
  DevBuf pxrecv, py, psync;         // receive rows | returned expert outputs | flags + counts
  DevBuf prowmap;                   // [receive rows] sender's token-major output row of each received row
  DevBuf pseq, pstatus, dest_base, grp_orank, grp_oshift;
  noor::peer::Peers peers{};
  void* peer_y[noor::peer::kMaxRanks] = {};
  std::vector<void*> ipc_opened;    // mappings of other processes' buffers, closed on destroy
  CUtensorMap tm_pxrecv{};
  int64_t* h_cnt = nullptr;  // pinned [E + G*El]
  int32_t* h_grp = nullptr;  // pinned [3 * (G*El + 1)]
  CUtensorMap tm_xp{}, tm_xrecv{}, tm_h{}, tm_xin{}, tm_dh{}, tm_sh{};
  CUtensorMap tm_user{};            // map of the caller's x (device mode), reused while x and T repeat
  const void* tm_user_ptr = nullptr;
  int64_t tm_user_T = -1;

  cudaStream_t own = nullptr, aux = nullptr;
  int gemm_pair_cap = 0;  // SM pairs the SM-pair GEMMs may take (0: all); set while a kernel shares the GPU
  int dispatch_sms = 0;   // peer exchange: SMs the permute runs on beside the dense up projection (0: in line),
                          // set by peer_setup
  bool dispatch_bulk = false;  // peer exchange: permute with bulk copies instead of thread loads/stores
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr, ev_done = nullptr;
  int* d_err = nullptr;

  // profiling
  bool prof_on = false;
  int prof_cap = 0, prof_used = 0;
  std::vector<cudaEvent_t> prof_ev;
  std::vector<int> prof_kind;
  int64_t launches = 0;
};

extern "C" int noor_moe_peer_plan(const int64_t* cnt, int G, int E, int me, int BM, int32_t* grp_row,
                                  int32_t* grp_mtile, int32_t* grp_widx, int32_t* grp_orank, int32_t* grp_oshift,
                                  int32_t* dest_base, int64_t* counts_glob) {
  if (!cnt || !grp_row || !grp_mtile || !grp_widx || !grp_orank || !grp_oshift || !dest_base || !counts_glob)
    return fail(NOOR_MOE_ERR_INVALID, "null argument");
  if (G < 1 || G > noor::peer::kMaxRanks || E <= 0 || E % G != 0 || me < 0 || me >= G || BM <= 0)
    return fail(NOOR_MOE_ERR_INVALID, "bad plan arguments");
  std::vector<int32_t> pre((size_t)G * (E + 1));
  for (int src = 0; src < G; ++src) {
    int64_t run = 0;
    for (int e = 0; e < E; ++e) {
      if (cnt[src * E + e] < 0) return fail(NOOR_MOE_ERR_INVALID, "negative count");
      pre[(size_t)src * (E + 1) + e] = (int32_t)run;
      run += cnt[src * E + e];
    }
    if (run > INT32_MAX) return fail(NOOR_MOE_ERR_INVALID, "count overflow");
    pre[(size_t)src * (E + 1) + E] = (int32_t)run;
  }
  const noor::peer::PlanView pv{cnt, pre.data(), E + 1, G, E, E / G, me};
  noor::peer::plan_recv_table(pv, BM, grp_row, grp_mtile, grp_widx, grp_orank, grp_oshift);
  for (int e = 0; e < E; ++e) {
    dest_base[e] = noor::peer::plan_dest_base(pv, e);
    int64_t tot = 0;
    for (int src = 0; src < G; ++src) tot += cnt[src * E + e];
    counts_glob[e] = tot;
  }
  return NOOR_MOE_OK;
}

extern "C" int noor_moe_ep_plan(const int64_t* counts_local, const int64_t* counts_recv, int E, int G, int BM,
                                int64_t* send_rows, int64_t* send_off, int64_t* recv_rows, int64_t* recv_off,
                                int32_t* grp_row, int32_t* grp_mtile, int32_t* grp_widx) {
  if (!counts_local || !counts_recv || E <= 0 || G <= 0 || E % G != 0 || BM <= 0)
    return fail(NOOR_MOE_ERR_INVALID, "bad plan arguments");
  const int El = E / G;
  int64_t so = 0, ro = 0;
  for (int r = 0; r < G; ++r) {
    int64_t sr = 0, rr = 0;
    for (int le = 0; le < El; ++le) {
      if (counts_local[r * El + le] < 0 || counts_recv[r * El + le] < 0)
        return fail(NOOR_MOE_ERR_INVALID, "negative count");
      sr += counts_local[r * El + le];
      rr += counts_recv[r * El + le];
    }
    send_rows[r] = sr;
    send_off[r] = so;
    recv_rows[r] = rr;
    recv_off[r] = ro;
    so += sr;
    ro += rr;
  }
  if (ro > INT32_MAX) return fail(NOOR_MOE_ERR_INVALID, "received rows overflow");
  int64_t r0 = 0, t0 = 0;
  for (int src = 0; src < G; ++src)
    for (int le = 0; le < El; ++le) {
      const int j = src * El + le;
      const int64_t c = counts_recv[j];
      grp_row[j] = (int32_t)r0;
      grp_mtile[j] = (int32_t)t0;
      grp_widx[j] = le;
      r0 += c;
      t0 += (c + BM - 1) / BM;
    }
  grp_row[G * El] = (int32_t)r0;
  grp_mtile[G * El] = (int32_t)t0;
  grp_widx[G * El] = 0;
  return NOOR_MOE_OK;
}

namespace {

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// Launch wrapper: names the launch with an NVTX range (seen by ncu / nsys;
// a no-op without a tool attached), brackets it with profile events when
// enabled and counts it.
template <typename F>
int launch(noor_moe_handle* h, cudaStream_t s, int kind, F&& f) {
  const bool prof = h->prof_on && h->prof_used < h->prof_cap;
  if (prof) CK(cudaEventRecord(h->prof_ev[2 * h->prof_used], s));
  nvtxRangePushA(kKindNames[kind]);
  f();
  nvtxRangePop();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(NOOR_MOE_ERR_CUDA, "launch of %s failed: %s", kKindNames[kind], cudaGetErrorString(e));
  if (prof) {
    CK(cudaEventRecord(h->prof_ev[2 * h->prof_used + 1], s));
    h->prof_kind[h->prof_used] = kind;
    ++h->prof_used;
  }
  ++h->launches;
  return NOOR_MOE_OK;
}

// Like launch() for NCCL phases (not counted as kernels of this library).
template <typename F>
int timed_phase(noor_moe_handle* h, cudaStream_t s, int kind, F&& f) {
  const bool prof = h->prof_on && h->prof_used < h->prof_cap;
  if (prof) CK(cudaEventRecord(h->prof_ev[2 * h->prof_used], s));
  nvtxRangePushA(kKindNames[kind]);
  const int rc = f();
  nvtxRangePop();
  CKR(rc);
  if (prof) {
    CK(cudaEventRecord(h->prof_ev[2 * h->prof_used + 1], s));
    h->prof_kind[h->prof_used] = kind;
    ++h->prof_used;
  }
  return NOOR_MOE_OK;
}

int wait_event_deadline(noor_moe_handle* h, cudaEvent_t ev, double seconds) {
  const auto t0 = std::chrono::steady_clock::now();
  while (true) {
    cudaError_t q = cudaEventQuery(ev);
    if (q == cudaSuccess) return NOOR_MOE_OK;
    if (q != cudaErrorNotReady) return fail(NOOR_MOE_ERR_CUDA, "stream failed: %s", cudaGetErrorString(q));
    const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > seconds) {
      if (h->comm) {
        noor::nccl().CommAbort(h->comm);  // releases NCCL kernels waiting for a lost peer
        h->comm = nullptr;
        h->comm_broken = true;
        return fail(NOOR_MOE_ERR_NCCL, "expert-parallel exchange did not finish within %.0f s; "
                    "communicator aborted", seconds);
      }
      return fail(NOOR_MOE_ERR_TIMEOUT, "device work did not finish within %.0f s", seconds);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

int check_device_error(noor_moe_handle* h) {
  int err = 0;
  CK(cudaMemcpy(&err, h->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (err == 0) return NOOR_MOE_OK;
  cudaMemset(h->d_err, 0, sizeof(int));
  if (err == noor::DEV_PEER_PLAN)
    return fail(NOOR_MOE_ERR_INVALID, "a rank's batch exceeded the expert-parallel capacity; every rank skipped "
                "this step");
  if (err == noor::DEV_TIMEOUT_PEER) {
    // the ranks' barrier counters may now disagree: no further exchange
    h->comm_broken = true;
    return fail(NOOR_MOE_ERR_TIMEOUT, "a wait on another rank gave up; the expert-parallel exchange is closed");
  }
  if (err == noor::DEV_BAD_INDEX)
    return fail(NOOR_MOE_ERR_INVALID, "a bounds check of the debug build failed: a kernel found a row index "
                "outside its buffer and skipped the access");
  return fail(NOOR_MOE_ERR_TIMEOUT, "a kernel's bounded wait gave up (device code %d)", err);
}

int64_t round_up(int64_t a, int64_t b) { return (a + b - 1) / b * b; }

// ============================================================== workspaces

int ensure_workspace(noor_moe_handle* h, int64_t T) {
  if (T <= h->capT) return NOOR_MOE_OK;
  const int64_t capT = round_up(std::max<int64_t>(T, h->desc.max_tokens), 128);
  const int64_t b = h->bf16 ? 2 : 4;
  const int64_t Rl = capT * h->k;           // picks made on this rank
  const int64_t Rr = Rl * h->G;             // worst-case rows received under EP
  const int64_t nblk = (capT + 15) / 16;    // smallest token block: 16 tokens (one router warp)
  const int64_t d = h->d;
  CKR(h->x_in.ensure(capT * d * b));
  CKR(h->out_buf.ensure(capT * d * b));
  CKR(h->idx.ensure(Rl * 4));
  CKR(h->wts.ensure(Rl * 4));
  CKR(h->lrank.ensure(Rl * 4));
  CKR(h->dst_row.ensure(Rl * 4));
  CKR(h->blk_hist.ensure(nblk * h->E * 4));
  CKR(h->blk_base.ensure(nblk * h->E * 4));
  CKR(h->counts64.ensure(h->E * 8));
  CKR(h->counts_glob.ensure(h->E * 8));
  CKR(h->seg_start.ensure((h->E + 1) * 4));
  CKR(h->mtile_start.ensure((h->E + 1) * 4));
  if (!h->bf16) CKR(h->scores.ensure(capT * h->E * 4));
  CKR(h->h.ensure(Rr * h->ff * b));
  h->cap_recv = std::max(h->cap_recv, Rr);
  if (!h->peer) {
    CKR(h->xp.ensure(Rl * d * b));
    CKR(h->y.ensure(Rr * d * b));
  }
  if (h->bf16 && h->G == 1) CKR(h->ymap.ensure(Rl * 4));
  if (h->G > 1 && !h->peer) {
    CKR(h->xrecv.ensure(Rr * d * b));
    CKR(h->ysend.ensure(Rl * d * b));
    const int ng = h->G * h->El;
    CKR(h->grp_row.ensure((ng + 1) * 4));
    CKR(h->grp_mtile.ensure((ng + 1) * 4));
    CKR(h->grp_widx.ensure((ng + 1) * 4));
    CKR(h->cnt_recv.ensure(ng * 8));
  }
  if (h->has_dense) {
    CKR(h->dense_h.ensure(capT * h->dff * b));
    CKR(h->dense_out.ensure(capT * d * 4));
  }
  if (h->has_shared) {
    CKR(h->shared_h.ensure(capT * h->ff * b));
    CKR(h->shared_out.ensure(capT * d * 4));
  }
  if (h->sandwich) {
    CKR(h->xn.ensure(capT * d * b));
    CKR(h->ffn.ensure(capT * d * b));
    if (h->bf16) CKR(encode_kmajor(&h->tm_xn, h->xn.p, capT, d, tc::BM));
  }
  if (h->bf16) {
    if (!h->peer) CKR(encode_kmajor(&h->tm_xp, h->xp.p, Rl, d, tc::BM));
    if (h->G > 1 && !h->peer) CKR(encode_kmajor(&h->tm_xrecv, h->xrecv.p, h->cap_recv, d, tc::BM));
    CKR(encode_kmajor(&h->tm_h, h->h.p, h->cap_recv, h->ff, tc::BM));
    CKR(encode_kmajor(&h->tm_xin, h->x_in.p, capT, d, tc::BM));
    if (h->has_dense) CKR(encode_kmajor(&h->tm_dh, h->dense_h.p, capT, h->dff, tc::BM));
    if (h->has_shared) CKR(encode_kmajor(&h->tm_sh, h->shared_h.p, capT, h->ff, tc::BM));
  }
  h->capT = capT;
  return NOOR_MOE_OK;
}

// Under expert parallelism the rows a rank receives depend on the other
// ranks' batches; grow the receive-side buffers to the planned row count.
int ensure_recv_capacity(noor_moe_handle* h, int64_t rows) {
  if (rows <= h->cap_recv) return NOOR_MOE_OK;
  const int64_t cap = round_up(rows, 128);
  const int64_t b = h->bf16 ? 2 : 4;
  CKR(h->xrecv.ensure(cap * h->d * b));
  CKR(h->h.ensure(cap * h->ff * b));
  CKR(h->y.ensure(cap * h->d * b));
  h->cap_recv = cap;
  if (h->bf16) {
    CKR(encode_kmajor(&h->tm_xrecv, h->xrecv.p, cap, h->d, tc::BM));
    CKR(encode_kmajor(&h->tm_h, h->h.p, cap, h->ff, tc::BM));
  }
  return NOOR_MOE_OK;
}

// ============================================================== GEMM launchers

// Gather-combine arguments of the dense down projection's fused epilogue.
struct CombineArgs {
  const void* y;
  const int32_t* dst_row;
  const float* wts;
  const float* shared;
  int32_t k;
  bool y_token_major;  // y row of pick (t, i) is t*k + i (dst_row unused)
  int64_t y_rows;      // rows y holds (bounds checks of the debug build)
};

// Where the plain-store epilogue puts its rows.  Expert parallelism over
// peer memory: group g's rows go to rank rank[g]'s buffer bases[rank[g]]
// (rank null: the GEMM's own C).  Row r goes to rowmap[r] when rowmap is set
// (token-major y), else to r + shift[g].
struct PeerOut {
  const int32_t* rank;
  const int32_t* shift;
  void* const* bases;
  const int32_t* rowmap;
};

void set_peer_out(tc::Params& p, const PeerOut* po) {
  if (!po) return;
  p.out_rank = po->rank;
  p.out_shift = po->shift;
  if (po->bases)
    for (int r = 0; r < noor::peer::kMaxRanks; ++r) p.out_peer[r] = po->bases[r];
  p.out_rowmap = po->rowmap;
}

// Raise a kernel's dynamic shared-memory limit to at least `bytes`.  Up to
// 48 KB needs no attribute; above it the limit set so far for each
// (kernel, device) is remembered, so the slow host call runs only when a
// launch needs more than before.
template <typename K>
int ensure_smem_limit(K kern, int bytes) {
  if (bytes <= 48 * 1024) return NOOR_MOE_OK;
  static std::mutex mu;
  struct Entry {
    const void* kern;
    int dev;
    int bytes;
  };
  static std::vector<Entry> done;
  int dev = 0;
  CK(cudaGetDevice(&dev));
  const void* key = reinterpret_cast<const void*>(kern);
  std::lock_guard<std::mutex> lock(mu);
  for (auto& e : done)
    if (e.kern == key && e.dev == dev) {
      if (e.bytes >= bytes) return NOOR_MOE_OK;
      CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
      e.bytes = bytes;
      return NOOR_MOE_OK;
    }
  CK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  done.push_back({key, dev, bytes});
  return NOOR_MOE_OK;
}

// c_rows: rows the output buffer(s) hold, for the bounds checks of the
// debug build (0: unchecked).
template <int BN, int EPI>
int launch_tc(noor_moe_handle* h, cudaStream_t s, int kind, const CUtensorMap& tA, const CUtensorMap& tB,
              const GroupTable& gt, int N, int K, void* C, int64_t ldc, int64_t max_mtiles,
              const CombineArgs* comb = nullptr, const PeerOut* po = nullptr, int64_t c_rows = 0) {
  using Cf = tc::Cfg<BN>;
  auto kern = tc::grouped_gemm_kernel<BN, EPI>;
  CKR(ensure_smem_limit(kern, Cf::SMEM_BYTES));
  tc::Params p{};
  p.groups = gt;
  p.N = N;
  p.K = K;
  p.n_tiles = N / BN;
  p.C = C;
  p.ldc = ldc;
  p.err = h->d_err;
  p.out_rows = c_rows;
  if (comb) {
    p.y = static_cast<const bf16*>(comb->y);
    p.dst_row = comb->dst_row;
    p.wts = comb->wts;
    p.shared = comb->shared;
    p.k = comb->k;
    p.y_token_major = comb->y_token_major ? 1 : 0;
    p.y_rows = comb->y_rows;
  }
  set_peer_out(p, po);
  const int64_t tiles = std::max<int64_t>(1, max_mtiles * p.n_tiles);
  const int grid = (int)std::min<int64_t>(h->num_sms, tiles);
  return launch(h, s, kind, [&] { kern<<<grid, tc::NUM_THREADS, Cf::SMEM_BYTES, s>>>(tA, tB, p); });
}

template <int EPI>
int launch_tc2(noor_moe_handle* h, cudaStream_t s, int kind, const CUtensorMap& tA, const CUtensorMap& tB,
               const GroupTable& gt, int N, int K, void* C, int64_t ldc, int64_t max_tiles,
               const CombineArgs* comb = nullptr, const PeerOut* po = nullptr, int64_t c_rows = 0) {
  auto kern = tc::grouped_gemm_2cta_kernel<EPI>;
  CKR(ensure_smem_limit(kern, tc::Cfg2<EPI>::SMEM_BYTES));
  tc::Params p{};
  p.groups = gt;
  p.N = N;
  p.K = K;
  p.n_tiles = N / 256;
  p.C = C;
  p.ldc = ldc;
  p.err = h->d_err;
  p.out_rows = c_rows;
  if (comb) {
    p.y = static_cast<const bf16*>(comb->y);
    p.dst_row = comb->dst_row;
    p.wts = comb->wts;
    p.shared = comb->shared;
    p.k = comb->k;
    p.y_token_major = comb->y_token_major ? 1 : 0;
    p.y_rows = comb->y_rows;
  }
  set_peer_out(p, po);
  const int64_t tiles = std::max<int64_t>(1, max_tiles * p.n_tiles);
  const int pairs = h->gemm_pair_cap > 0 ? std::min(h->gemm_pair_cap, h->num_sms / 2) : h->num_sms / 2;
  const int clusters = (int)std::min<int64_t>(pairs, tiles);
  return launch(h, s, kind,
                [&] { kern<<<2 * clusters, tc::Cfg2<EPI>::THREADS, tc::Cfg2<EPI>::SMEM_BYTES, s>>>(tA, tB, p); });
}

// A tensor-core GEMM with the layer's tile shape: SM pairs with 256-row
// tiles when the layer allows it, else one CTA with 128-row tiles and an
// n-tile of 256 (or 128 when N is not a multiple of 256).  max_tiles counts
// tiles of h->tile_m rows.
template <int EPI>
int launch_gemm(noor_moe_handle* h, cudaStream_t s, int kind, const CUtensorMap& tA, const CUtensorMap& tB,
                const GroupTable& gt, int N, int K, void* C, int64_t ldc, int64_t max_tiles,
                const CombineArgs* comb = nullptr, const PeerOut* po = nullptr, int64_t c_rows = 0) {
  if (h->pair2) return launch_tc2<EPI>(h, s, kind, tA, tB, gt, N, K, C, ldc, max_tiles, comb, po, c_rows);
  if (N % 256 == 0) return launch_tc<256, EPI>(h, s, kind, tA, tB, gt, N, K, C, ldc, max_tiles, comb, po, c_rows);
  if constexpr (tc::epi_gated(EPI)) {
    return fail(NOOR_MOE_ERR_UNSUPPORTED, "gated GEMM needs N a multiple of 256");
  } else {
    return launch_tc<128, EPI>(h, s, kind, tA, tB, gt, N, K, C, ldc, max_tiles, comb, po, c_rows);
  }
}

template <int EPI>
int launch_simt(noor_moe_handle* h, cudaStream_t s, int kind, const GroupTable& gt, const float* A, int64_t lda,
                const float* Bg, const float* Bu, int64_t b_stride, int N, int K, float* C, int64_t ldc,
                int64_t max_mtiles) {
  simt::Params p;
  p.groups = gt;
  p.A = A;
  p.lda = lda;
  p.Bg = Bg;
  p.Bu = Bu;
  p.b_stride = b_stride;
  p.N = N;
  p.K = K;
  p.n_tiles = (N + simt::BN - 1) / simt::BN;
  p.C = C;
  p.ldc = ldc;
  const int64_t tiles = std::max<int64_t>(1, max_mtiles * p.n_tiles);
  const int grid = (int)std::min<int64_t>((int64_t)h->num_sms * 8, tiles);
  return launch(h, s, kind, [&] { simt::grouped_gemm_f32_kernel<EPI><<<grid, simt::THREADS, 0, s>>>(p); });
}

GroupTable dense_group(int64_t rows) {
  GroupTable g;
  g.row_start = g.mtile_start = g.weight_idx = nullptr;
  g.G = 1;
  g.dense_rows = (int32_t)rows;
  return g;
}

// GLU FFN over `rows` rows of A, in two stages: up() writes
// hbuf = act(A.Wg) * (A.Wu); down() writes hbuf . Wd either as f32 `out` or,
// with `comb` (BF16 layers), straight into the layer output through the fused
// gather-combine epilogue.  BF16: tensor cores (tA is A's map); F32: CUDA cores.
struct GluFfn {
  int kind1, kind2;
  const CUtensorMap* tA;
  const void* A;
  int64_t rows;
  int ffn;
  bool silu;
  const CUtensorMap *tW1, *tW2, *tH;
  const float *g32, *u32, *d32;
  void* hbuf;
};

int glu_up(noor_moe_handle* h, cudaStream_t s, const GluFfn& f) {
  const GroupTable gt = dense_group(f.rows);
  const int d = h->d;
  if (h->bf16) {
    const int64_t mt = (f.rows + h->tile_m - 1) / h->tile_m;
    if (f.silu)
      return launch_gemm<tc::EPI_SWIGLU_BF16>(h, s, f.kind1, *f.tA, *f.tW1, gt, 2 * f.ffn, d, f.hbuf, f.ffn, mt,
                                              nullptr, nullptr, h->capT);
    return launch_gemm<tc::EPI_GEGLU_BF16>(h, s, f.kind1, *f.tA, *f.tW1, gt, 2 * f.ffn, d, f.hbuf, f.ffn, mt, nullptr,
                                           nullptr, h->capT);
  }
  const int64_t mt = (f.rows + simt::BM - 1) / simt::BM;
  if (f.silu)
    return launch_simt<simt::EPI_SWIGLU>(h, s, f.kind1, gt, (const float*)f.A, d, f.g32, f.u32, 0, f.ffn, d,
                                         (float*)f.hbuf, f.ffn, mt);
  return launch_simt<simt::EPI_GEGLU>(h, s, f.kind1, gt, (const float*)f.A, d, f.g32, f.u32, 0, f.ffn, d,
                                      (float*)f.hbuf, f.ffn, mt);
}

int glu_down(noor_moe_handle* h, cudaStream_t s, const GluFfn& f, void* out, const CombineArgs* comb) {
  const GroupTable gt = dense_group(f.rows);
  const int d = h->d;
  if (h->bf16) {
    const int64_t mt = (f.rows + h->tile_m - 1) / h->tile_m;
    if (comb)
      return launch_gemm<tc::EPI_COMBINE_BF16>(h, s, f.kind2, *f.tH, *f.tW2, gt, d, f.ffn, out, d, mt, comb, nullptr,
                                               f.rows);
    return launch_gemm<tc::EPI_STORE_F32>(h, s, f.kind2, *f.tH, *f.tW2, gt, d, f.ffn, out, d, mt, nullptr, nullptr,
                                          h->capT);
  }
  const int64_t mt = (f.rows + simt::BM - 1) / simt::BM;
  return launch_simt<simt::EPI_STORE>(h, s, f.kind2, gt, (const float*)f.hbuf, f.ffn, f.d32, nullptr, 0, d, f.ffn,
                                      (float*)out, d, mt);
}

// ============================================================== router

// The BF16 router (router_tc.cuh): one CTA per 128 tokens.  Shared by the
// handle's router and noor_moe_route_static, so both give the same picks.
int launch_route_tc(noor_moe_handle* h, cudaStream_t s, const CUtensorMap& tmx, const CUtensorMap& tmg,
                    const float* bias, const float* scales, int64_t T, int d, int E, int k, const router::RouterOut& ro,
                    const router::FusedScan& fs, int* err) {
  const int npad = router::tc_npad(E);
  const int smem = router::tc_smem_bytes(npad);
  // the epilogue stages the tile's scores in the stage ring
  if (npad > 32 && smem - 1024 < router::tc_scores_bytes(npad))
    return fail(NOOR_MOE_ERR_UNSUPPORTED, "router stage ring too small for %d experts", E);
  const unsigned grid = (unsigned)((T + router::kTcTPB - 1) / router::kTcTPB);
  auto go = [&](auto kern) -> int {
    CKR(ensure_smem_limit(kern, smem));
    auto body = [&] { kern<<<grid, router::kTcThreads, smem, s>>>(tmx, tmg, bias, scales, (int32_t)T, d, E, k, ro, fs, err); };
    if (h) return launch(h, s, K_ROUTER, body);
    body();
    CK(cudaGetLastError());
    return NOOR_MOE_OK;
  };
  switch ((npad + 31) / 32) {
    case 1: return go(router::route_tc_kernel<1>);
    case 2: return go(router::route_tc_kernel<2>);
    case 3: return go(router::route_tc_kernel<3>);
    case 4: return go(router::route_tc_kernel<4>);
    default: return fail(NOOR_MOE_ERR_UNSUPPORTED, "the tensor-core router supports at most 128 experts");
  }
}

// Launch K1 and the scan.  Fills idx, wts, lrank, blk_hist, counts64,
// seg_start, blk_base, mtile_start.  Returns the token-block size in *tpb.
// record: add the batch's counts to the layer's utilization (the forward
// on one GPU; under expert parallelism the global counts are added later).
int run_router(noor_moe_handle* h, cudaStream_t s, const void* x, const CUtensorMap* tmx, int64_t T, int* tpb_out,
               bool record = false) {
  router::RouterOut ro{h->idx.as<int32_t>(), h->wts.as<float>(), h->lrank.as<int32_t>(), h->blk_hist.as<int32_t>()};
  const int E = h->E, k = h->k, d = h->d;
  int tpb = 0;
  router::FusedScan fs{h->scan_done.as<int>(), h->counts64.as<int64_t>(), h->seg_start.as<int32_t>(),
                       h->blk_base.as<int32_t>(), h->mtile_start.as<int32_t>(), h->tile_m,
                       record ? h->util.as<int64_t>() : nullptr, h->seg_acc.as<int32_t>(), h->d_err};
  if (h->bf16) {
    tpb = router::kTcTPB;
    CKR(launch_route_tc(h, s, *tmx, h->tm_gate, h->bias.as<float>(), h->scales.as<float>(), T, d, E, k, ro, fs,
                        h->d_err));
  } else {
    tpb = router::kTopkTPB;
    const int nblk = (int)((T + tpb - 1) / tpb);
    const int64_t n = T * E;
    CKR(launch(h, s, K_ROUTER_SCORES, [&] {
      router::route_f32_scores_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
          (const float*)x, h->gate.as<float>(), h->bias.as<float>(), (int32_t)T, d, E, h->scores.as<float>());
    }));
    const size_t smem = router::topk_smem_bytes(E, k);
    CKR(ensure_smem_limit(router::topk_from_scores_kernel, (int)smem));
    CKR(launch(h, s, K_ROUTER_TOPK, [&] {
      router::topk_from_scores_kernel<<<nblk, router::kTopkTPB, smem, s>>>(h->scores.as<float>(),
                                                                           h->scales.as<float>(), (int32_t)T, E, k, ro,
                                                                           fs);
    }));
  }
  *tpb_out = tpb;
  return NOOR_MOE_OK;
}

// ============================================================== expert parallel exchange

ncclDataType_t act_nccl_type(const noor_moe_handle* h) { return h->bf16 ? ncclBfloat16 : ncclFloat32; }

struct EpPlan {
  std::vector<int64_t> send_rows, send_off, recv_rows, recv_off;
  int64_t recv_total = 0;
  int64_t mtiles = 0;
};

// Exchange per-expert counts, then build the receive-side group table with
// noor_moe_ep_plan (group j = (source rank, local expert), rows contiguous in
// xrecv, weight index = local expert).
int ep_plan(noor_moe_handle* h, cudaStream_t s, EpPlan& plan) {
  const int G = h->G, El = h->El, E = h->E;
  CKR(timed_phase(h, s, K_COUNT_EXCHANGE, [&]() -> int {
    CKN(noor::nccl().GroupStart());
    for (int r = 0; r < G; ++r) {
      CKN(noor::nccl().Send(h->counts64.as<int64_t>() + (int64_t)r * El, El, ncclInt64, r, h->comm, s));
      CKN(noor::nccl().Recv(h->cnt_recv.as<int64_t>() + (int64_t)r * El, El, ncclInt64, r, h->comm, s));
    }
    CKN(noor::nccl().GroupEnd());
    return NOOR_MOE_OK;
  }));
  CK(cudaMemcpyAsync(h->h_cnt, h->counts64.p, E * 8, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(h->h_cnt + E, h->cnt_recv.p, (int64_t)G * El * 8, cudaMemcpyDeviceToHost, s));
  CK(cudaEventRecord(h->ev_done, s));
  CKR(wait_event_deadline(h, h->ev_done, 120.0));
  plan.send_rows.assign(G, 0);
  plan.send_off.assign(G, 0);
  plan.recv_rows.assign(G, 0);
  plan.recv_off.assign(G, 0);
  const int ng = G * El;
  int32_t* row = h->h_grp;
  int32_t* mt = h->h_grp + (ng + 1);
  int32_t* wi = h->h_grp + 2 * (ng + 1);
  CKR(noor_moe_ep_plan(h->h_cnt, h->h_cnt + E, E, G, h->tile_m, plan.send_rows.data(), plan.send_off.data(),
                       plan.recv_rows.data(), plan.recv_off.data(), row, mt, wi));
  plan.recv_total = row[ng];
  plan.mtiles = mt[ng];
  CKR(ensure_recv_capacity(h, plan.recv_total));
  CK(cudaMemcpyAsync(h->grp_row.p, row, (ng + 1) * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(h->grp_mtile.p, mt, (ng + 1) * 4, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(h->grp_widx.p, wi, (ng + 1) * 4, cudaMemcpyHostToDevice, s));
  return NOOR_MOE_OK;
}

int ep_exchange(noor_moe_handle* h, cudaStream_t s, int kind, const EpPlan& plan, const void* sendbuf,
                void* recvbuf, bool reverse) {
  const int64_t row_elems = h->d;
  const int64_t b = h->bf16 ? 2 : 4;
  return timed_phase(h, s, kind, [&]() -> int {
    CKN(noor::nccl().GroupStart());
    for (int r = 0; r < h->G; ++r) {
      const int64_t sr = reverse ? plan.recv_rows[r] : plan.send_rows[r];
      const int64_t so = reverse ? plan.recv_off[r] : plan.send_off[r];
      const int64_t rr = reverse ? plan.send_rows[r] : plan.recv_rows[r];
      const int64_t ro = reverse ? plan.send_off[r] : plan.recv_off[r];
      if (sr > 0)
        CKN(noor::nccl().Send(static_cast<const uint8_t*>(sendbuf) + so * row_elems * b, sr * row_elems, act_nccl_type(h), r,
                     h->comm, s));
      if (rr > 0)
        CKN(noor::nccl().Recv(static_cast<uint8_t*>(recvbuf) + ro * row_elems * b, rr * row_elems, act_nccl_type(h), r,
                     h->comm, s));
    }
    CKN(noor::nccl().GroupEnd());
    return NOOR_MOE_OK;
  });
}

// ============================================================== expert parallel over peer memory

// Whether the side branches (dense up projection, shared expert) run on a
// second stream beside the permute.  Measured on B200 with the Edge layer
// (16384 tokens a GPU), running them in line is faster both on one GPU
// (1.26 ms against 1.40 ms a step) and under expert parallelism over peer
// memory on two GPUs (1.38 ms against 1.43 ms): the permute's copies take
// L2 bandwidth the dense GEMM needs, and the expert GEMM still waits for the
// dense GEMM's SMs, so the overlap costs more than the hidden copy time.
constexpr bool kForkSideSingle = false;
constexpr bool kForkSidePeer = false;
// Under the peer-memory exchange, optionally split the permute: the local
// rows in line, and the rows bound for other ranks (NVLink stores) on a
// second stream beside the dense up projection.  On two B200s this measured
// the same as the single in-line permute (24.2-24.4M tokens/s either way),
// so it is off.
constexpr bool kSplitPermutePeer = false;
// Under the peer-memory exchange with a dense branch, the permute (NVLink
// stores) can run on a second stream on dispatch_sms SMs while the dense up
// projection, which needs only x, runs on the others.  The permute's blocks
// ask for enough shared memory that no GEMM CTA fits beside them (the bulk
// permute: two one-warp blocks per SM, each with a kDispatchSmem row ring;
// the thread permute: one 16-warp block per SM with kDispatchSmemSide,
// unused), and the GEMM is launched with the remaining SM pairs.  (Spreading
// both kernels over every SM was slower.)  On two B200s, Edge-like layer:
// in line 1.301 ms/step; 24 / 32 / 48 SMs beside the GEMM 1.238 / 1.187 /
// 1.209 ms.  Set per process: NOOR_MOE_DISPATCH_SMS (default
// kDispatchSMsDefault; 0 runs the permute in line on every SM) and
// NOOR_MOE_DISPATCH=bulk|threads (default threads).
constexpr int kDispatchSMsDefault = 32;
constexpr int kDispatchSmem = 96 * 1024;
constexpr int kDispatchSmemSide = 160 * 1024;

// Wait, bounded, for the setup collectives queued on the handle's stream.
int setup_sync(noor_moe_handle* h) {
  CK(cudaEventRecord(h->ev_done, h->own));
  return wait_event_deadline(h, h->ev_done, 120.0);
}

// Minimum of v over the ranks (setup only).
int allreduce_min(noor_moe_handle* h, int64_t* v) {
  DevBuf t;
  CKR(t.ensure(16));
  CK(cudaMemcpy(t.p, v, 8, cudaMemcpyHostToDevice));
  CKN(noor::nccl().AllReduce(t.p, t.as<int64_t>() + 1, 1, ncclInt64, ncclMin, h->comm, h->own));
  CKR(setup_sync(h));
  CK(cudaMemcpy(v, t.as<int64_t>() + 1, 8, cudaMemcpyDeviceToHost));
  return NOOR_MOE_OK;
}

// Gather `bytes` bytes from every rank (setup only).
int allgather_bytes(noor_moe_handle* h, const void* mine, void* all, size_t bytes) {
  DevBuf t;
  CKR(t.ensure(bytes * (h->G + 1)));
  CK(cudaMemcpy(t.p, mine, bytes, cudaMemcpyHostToDevice));
  CKN(noor::nccl().AllGather(t.p, t.as<uint8_t>() + bytes, bytes, ncclUint8, h->comm, h->own));
  CKR(setup_sync(h));
  CK(cudaMemcpy(all, t.as<uint8_t>() + bytes, bytes * h->G, cudaMemcpyDeviceToHost));
  return NOOR_MOE_OK;
}

void peer_release(noor_moe_handle* h) {
  for (void* p : h->ipc_opened) cudaIpcCloseMemHandle(p);
  h->ipc_opened.clear();
  DevBuf* bufs[] = {&h->pxrecv, &h->py, &h->psync, &h->prowmap, &h->pseq, &h->pstatus, &h->dest_base,
                    &h->grp_orank, &h->grp_oshift};
  for (DevBuf* b : bufs) b->release();
  h->peer = false;
}

// Choose the exchange and map every rank's buffers.  Collective: every rank
// of the communicator calls it from noor_moe_create, and all take the same
// decision.  Peer memory is used when the layer is BF16, every pair of the
// ranks' GPUs has peer access, every mapping opens and the variable
// NOOR_MOE_EP_TRANSPORT is not "nccl"; otherwise the layer exchanges rows
// through NCCL.  The peer buffers hold capP tokens per rank, capP the
// largest max_tokens over the ranks.
int peer_setup(noor_moe_handle* h) {
  namespace P = noor::peer;
  const int G = h->G, me = h->rank, E = h->E, k = h->k, d = h->d;
  const char* env = std::getenv("NOOR_MOE_EP_TRANSPORT");
  const bool want = h->bf16 && G <= P::kMaxRanks && E <= 128 && !(env && std::strcmp(env, "nccl") == 0);
  struct Info {
    int64_t pid, want, max_tokens;
    char bus[40];
  };
  Info mine{};
  mine.pid = (int64_t)getpid();
  mine.want = want ? 1 : 0;
  mine.max_tokens = std::max<int64_t>(h->desc.max_tokens, 128);
  CK(cudaDeviceGetPCIBusId(mine.bus, sizeof(mine.bus), h->dev));
  std::vector<Info> all(G);
  CKR(allgather_bytes(h, &mine, all.data(), sizeof(Info)));
  int64_t ok = want ? 1 : 0;
  std::vector<int> ord(G, -1);
  int64_t capP = 0;
  for (int r = 0; r < G; ++r) {
    capP = std::max(capP, all[r].max_tokens);
    if (!all[r].want) ok = 0;
    all[r].bus[sizeof(all[r].bus) - 1] = 0;
    if (cudaDeviceGetByPCIBusId(&ord[r], all[r].bus) != cudaSuccess) {
      cudaGetLastError();
      ok = 0;
      continue;
    }
    if (r != me) {
      int can = 0;
      if (cudaDeviceCanAccessPeer(&can, h->dev, ord[r]) != cudaSuccess || !can) ok = 0;
    }
  }
  cudaGetLastError();
  CKR(allreduce_min(h, &ok));
  if (!ok) return NOOR_MOE_OK;

  // this rank's buffers, cleared before any rank can see them
  capP = round_up(capP, 128);
  const int64_t cap_rows = (int64_t)G * capP * k;
  if (cap_rows > INT32_MAX) return fail(NOOR_MOE_ERR_INVALID, "expert-parallel capacity overflows");
  int rc = NOOR_MOE_OK;
  auto alloc = [&]() -> int {
    CKR(h->pxrecv.ensure(cap_rows * d * 2));
    CKR(h->py.ensure(capP * k * d * 2));
    CKR(h->prowmap.ensure(cap_rows * 4));
    CKR(h->psync.ensure(round_up(P::kCountsOff + (int64_t)G * E * 8, 4096)));
    CKR(h->pseq.ensure(8));
    CKR(h->pstatus.ensure(4));
    CKR(h->dest_base.ensure(E * 4));
    CKR(h->grp_orank.ensure(E * 4));
    CKR(h->grp_oshift.ensure(E * 4));
    CKR(h->grp_row.ensure((E + 1) * 4));
    CKR(h->grp_mtile.ensure((E + 1) * 4));
    CKR(h->grp_widx.ensure((E + 1) * 4));
    CKR(h->h.ensure(cap_rows * h->ff * 2));
    CK(cudaMemset(h->psync.p, 0, h->psync.bytes));
    CK(cudaMemset(h->pseq.p, 0, 8));
    CK(cudaMemset(h->pstatus.p, 0, 4));
    CK(cudaDeviceSynchronize());
    return NOOR_MOE_OK;
  };
  rc = alloc();
  int64_t ok2 = rc == NOOR_MOE_OK ? 1 : 0;
  CKR(allreduce_min(h, &ok2));
  if (!ok2) {
    peer_release(h);
    return rc != NOOR_MOE_OK ? rc : NOOR_MOE_OK;
  }

  // exchange the buffers' IPC handles (and raw addresses, for ranks that
  // share this process) and map the other ranks' buffers
  struct Handles {
    cudaIpcMemHandle_t x, y, sy, rm;
    uint64_t px, py, ps, prm;
  };
  Handles hm{};
  int64_t ok3 = 1;
  if (cudaIpcGetMemHandle(&hm.x, h->pxrecv.p) != cudaSuccess || cudaIpcGetMemHandle(&hm.y, h->py.p) != cudaSuccess ||
      cudaIpcGetMemHandle(&hm.sy, h->psync.p) != cudaSuccess ||
      cudaIpcGetMemHandle(&hm.rm, h->prowmap.p) != cudaSuccess) {
    cudaGetLastError();
    ok3 = 0;
  }
  hm.px = reinterpret_cast<uint64_t>(h->pxrecv.p);
  hm.py = reinterpret_cast<uint64_t>(h->py.p);
  hm.ps = reinterpret_cast<uint64_t>(h->psync.p);
  hm.prm = reinterpret_cast<uint64_t>(h->prowmap.p);
  std::vector<Handles> hs(G);
  CKR(allgather_bytes(h, &hm, hs.data(), sizeof(Handles)));
  P::Peers peers{};
  peers.G = G;
  peers.me = me;
  const char* senv = std::getenv("NOOR_MOE_DISPATCH_SMS");
  h->dispatch_sms = std::max(0, std::min(senv ? std::atoi(senv) : kDispatchSMsDefault, h->num_sms / 2)) & ~1;
  const char* denv = std::getenv("NOOR_MOE_DISPATCH");
  h->dispatch_bulk = denv && std::strcmp(denv, "bulk") == 0 && (d * 2) % 16 == 0;
  const char* tenv = std::getenv("NOOR_MOE_PEER_TIMEOUT_MS");
  const int64_t tms = tenv ? std::max<int64_t>(1, std::atoll(tenv)) : 10000;
  peers.timeout_ns = tms * 1000000LL;
  for (int r = 0; r < G && ok3; ++r) {
    void *px = nullptr, *py = nullptr, *ps = nullptr, *prm = nullptr;
    if (r == me || all[r].pid == mine.pid) {
      if (r != me) {
        cudaError_t e = cudaDeviceEnablePeerAccess(ord[r], 0);
        if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled) ok3 = 0;
        cudaGetLastError();
      }
      px = reinterpret_cast<void*>(hs[r].px);
      py = reinterpret_cast<void*>(hs[r].py);
      ps = reinterpret_cast<void*>(hs[r].ps);
      prm = reinterpret_cast<void*>(hs[r].prm);
    } else {
      void* m[4] = {nullptr, nullptr, nullptr, nullptr};
      const cudaIpcMemHandle_t* src[4] = {&hs[r].x, &hs[r].y, &hs[r].sy, &hs[r].rm};
      for (int i = 0; i < 4; ++i) {
        if (cudaIpcOpenMemHandle(&m[i], *src[i], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
          cudaGetLastError();
          ok3 = 0;
          break;
        }
        h->ipc_opened.push_back(m[i]);
      }
      px = m[0];
      py = m[1];
      ps = m[2];
      prm = m[3];
    }
    peers.xrecv[r] = static_cast<uint8_t*>(px);
    peers.sync[r] = static_cast<uint8_t*>(ps);
    peers.rowmap[r] = static_cast<int32_t*>(prm);
    h->peer_y[r] = py;
  }
  CKR(allreduce_min(h, &ok3));
  if (!ok3) {
    peer_release(h);
    return NOOR_MOE_OK;
  }
  h->peers = peers;
  h->capP = capP;
  h->cap_recv = std::max(h->cap_recv, cap_rows);
  CKR(encode_kmajor(&h->tm_pxrecv, h->pxrecv.p, cap_rows, d, tc::BM));
  CKR(encode_kmajor(&h->tm_h, h->h.p, h->cap_recv, h->ff, tc::BM));
  h->peer = true;
  // the NCCL path's staging buffers are not used
  DevBuf* unused[] = {&h->xp, &h->y, &h->xrecv, &h->ysend, &h->cnt_recv};
  for (DevBuf* b : unused) b->release();
  return NOOR_MOE_OK;
}

// The layer step under expert parallelism over peer memory (BF16), without
// host synchronization, on one stream:
//   router -> plan (counts to every rank, barrier, tables) -> permute (rows
//   into the owners' receive buffers) -> dense/shared up projections (while
//   the other ranks' rows arrive) -> barrier -> expert GEMM 1 -> expert
//   GEMM 2 (outputs back to the senders) -> barrier -> dense down
//   projection with the fused combine.
// kForkSidePeer / kSplitPermutePeer move the side branches or the remote
// rows to a second stream instead (both measured no faster).
// Every rank runs the plan and both barriers, with or without tokens.
int run_forward_peer(noor_moe_handle* h, cudaStream_t s, const void* x, const CUtensorMap* tmx, void* out,
                     int64_t T) {
  namespace P = noor::peer;
  const int d = h->d, k = h->k, E = h->E;
  const bool poison = T > h->capP;
  int tpb = 0;
  if (T > 0 && !poison) CKR(run_router(h, s, x, tmx, T, &tpb));
  else CK(cudaMemsetAsync(h->counts64.p, 0, E * 8, s));
  const int64_t cap_rows = (int64_t)h->G * h->capP * k;
  P::PlanOut po{h->grp_row.as<int32_t>(), h->grp_mtile.as<int32_t>(), h->grp_widx.as<int32_t>(),
                h->grp_orank.as<int32_t>(), h->grp_oshift.as<int32_t>(), h->dest_base.as<int32_t>(),
                h->counts_glob.as<int64_t>(), h->pstatus.as<int>(), h->pseq.as<uint64_t>(), h->d_err,
                h->util.as<int64_t>(), k};
  CKR(launch(h, s, K_EP_PLAN, [&] {
    P::plan_kernel<<<1, P::kPlanThreads, 0, s>>>(h->peers, h->counts64.as<int64_t>(), E, h->El, h->tile_m, cap_rows,
                                                 poison ? 1 : 0, po);
  }));
  if (poison) {
    // every rank skips this step; leave this rank's error word clear
    CK(cudaEventRecord(h->ev_done, s));
    CKR(wait_event_deadline(h, h->ev_done, 120.0));
    CK(cudaMemset(h->d_err, 0, sizeof(int)));
    return fail(NOOR_MOE_ERR_INVALID,
                "%lld tokens exceed the %lld tokens per rank that the expert-parallel buffers hold (the largest "
                "max_tokens given at creation); every rank skipped this step",
                (long long)T, (long long)h->capP);
  }
  // The side branches (dense up projection, shared expert) need only x.
  const GluFfn dense{K_DENSE_GEMM1, K_DENSE_GEMM2, tmx, x, T, h->dff, h->desc.dense_act == NOOR_ACT_SILU,
                     &h->tm_dw1, &h->tm_dw2, &h->tm_dh, nullptr, nullptr, nullptr, h->dense_h.p};
  const GluFfn shared{K_SHARED_GEMM1, K_SHARED_GEMM2, tmx, x, T, h->ff, true, &h->tm_sw1, &h->tm_sw2, &h->tm_sh,
                      nullptr, nullptr, nullptr, h->shared_h.p};
  const bool side = T > 0 && (h->has_dense || h->has_shared);
  const bool fork = side && kForkSidePeer;
  cudaStream_t ss = fork ? h->aux : s;
  auto side_branches = [&]() -> int {
    if (h->has_dense) CKR(glu_up(h, ss, dense));
    if (h->has_shared) {
      CKR(glu_up(h, ss, shared));
      CKR(glu_down(h, ss, shared, h->shared_out.p, nullptr));
    }
    return NOOR_MOE_OK;
  };
  if (fork) {
    CK(cudaEventRecord(h->ev_fork, s));
    CK(cudaStreamWaitEvent(h->aux, h->ev_fork, 0));
    CKR(side_branches());
    CK(cudaEventRecord(h->ev_join, h->aux));
  }
  const int row_bytes = d * 2;
  const int bulk_slots = std::min(P::kBulkSlotsMax, kDispatchSmem / row_bytes);
  // the bulk permute on `blocks` one-warp blocks with kDispatchSmem of ring each
  auto permute_bulk = [&](cudaStream_t st, unsigned blocks) -> int {
    return launch(h, st, K_PERMUTE, [&] {
      P::permute_peer_bulk_kernel<<<blocks, 32, kDispatchSmem, st>>>(
          static_cast<const uint8_t*>(x), row_bytes, (int32_t)T, k, (int32_t)((T + tpb - 1) / tpb), tpb,
          h->idx.as<int32_t>(), h->lrank.as<int32_t>(), h->blk_base.as<int32_t>(), h->seg_start.as<int32_t>(),
          h->dest_base.as<int32_t>(), h->El, h->peers, h->pstatus.as<int>(), h->dst_row.as<int32_t>(), cap_rows,
          bulk_slots, h->d_err);
    });
  };
  const bool bulk = h->dispatch_bulk && bulk_slots >= 2;
  if (bulk) CKR(ensure_smem_limit(P::permute_peer_bulk_kernel, kDispatchSmem));
  auto permute = [&](cudaStream_t st, int part, bool persistent) -> int {
    if (bulk && part == P::PERMUTE_ALL) return permute_bulk(st, (unsigned)(2 * h->num_sms));
    return launch(h, st, K_PERMUTE, [&] {
      const int64_t blocks = (T + P::kPermuteWarps - 1) / P::kPermuteWarps;
      const unsigned grid = (unsigned)(persistent ? std::min<int64_t>(blocks, h->num_sms) : blocks);
      P::permute_peer_kernel<P::kPermuteWarps><<<grid, P::kPermuteWarps * 32, 0, st>>>(
          static_cast<const uint8_t*>(x), d * 2, (int32_t)T, k, (int32_t)((T + tpb - 1) / tpb), tpb,
          h->idx.as<int32_t>(), h->lrank.as<int32_t>(), h->blk_base.as<int32_t>(), h->seg_start.as<int32_t>(),
          h->dest_base.as<int32_t>(), h->El, h->peers, h->pstatus.as<int>(), h->dst_row.as<int32_t>(), part,
          cap_rows, h->d_err);
    });
  };
  const bool split = kSplitPermutePeer && !fork && T > 0;
  const bool overlap = h->dispatch_sms > 0 && !fork && !split && T > 0 && side;
  if (overlap) {
    // the dispatch on its own SMs (second stream), the dense/shared up
    // projections on the rest; joined before the barrier
    CK(cudaEventRecord(h->ev_fork, s));
    CK(cudaStreamWaitEvent(h->aux, h->ev_fork, 0));
    if (bulk) {
      CKR(permute_bulk(h->aux, (unsigned)(2 * h->dispatch_sms)));
    } else {
      // one 16-warp block per SM; kDispatchSmemSide keeps GEMM CTAs off those SMs
      CKR(ensure_smem_limit(P::permute_peer_kernel<P::kPermuteWarpsSide>, kDispatchSmemSide));
      CKR(launch(h, h->aux, K_PERMUTE, [&] {
        P::permute_peer_kernel<P::kPermuteWarpsSide>
            <<<h->dispatch_sms, P::kPermuteWarpsSide * 32, kDispatchSmemSide, h->aux>>>(
            static_cast<const uint8_t*>(x), row_bytes, (int32_t)T, k, (int32_t)((T + tpb - 1) / tpb), tpb,
            h->idx.as<int32_t>(), h->lrank.as<int32_t>(), h->blk_base.as<int32_t>(), h->seg_start.as<int32_t>(),
            h->dest_base.as<int32_t>(), h->El, h->peers, h->pstatus.as<int>(), h->dst_row.as<int32_t>(),
            P::PERMUTE_ALL, cap_rows, h->d_err);
      }));
    }
    CK(cudaEventRecord(h->ev_join, h->aux));
    h->gemm_pair_cap = (h->num_sms - h->dispatch_sms) / 2;
    const int rc = side_branches();
    h->gemm_pair_cap = 0;
    CK(cudaStreamWaitEvent(s, h->ev_join, 0));  // joined on the error path too (a capture must not end forked)
    CKR(rc);
  } else if (split) {
    // remote rows on the second stream (persistent grid: it shares the SMs
    // with the GEMM beside it); local rows and the dense branch in line
    CK(cudaEventRecord(h->ev_fork, s));
    CK(cudaStreamWaitEvent(h->aux, h->ev_fork, 0));
    CKR(permute(h->aux, P::PERMUTE_REMOTE, true));
    CK(cudaEventRecord(h->ev_join, h->aux));
    CKR(permute(s, P::PERMUTE_LOCAL, false));
  } else if (T > 0) {
    CKR(permute(s, P::PERMUTE_ALL, fork));
  }
  if (side && !fork && !overlap) CKR(side_branches());  // in line, while the other ranks' rows arrive
  if (split) CK(cudaStreamWaitEvent(s, h->ev_join, 0));
  auto barrier = [&]() -> int {
    return launch(h, s, K_EP_BARRIER, [&] {
      P::barrier_kernel<<<1, 32, 0, s>>>(h->peers, h->pseq.as<uint64_t>(), h->pstatus.as<int>(), h->d_err);
    });
  };
  CKR(barrier());
  GroupTable gt;
  gt.row_start = h->grp_row.as<int32_t>();
  gt.mtile_start = h->grp_mtile.as<int32_t>();
  gt.weight_idx = h->grp_widx.as<int32_t>();
  gt.G = E;
  gt.dense_rows = -1;
  const int64_t max_mtiles = (cap_rows + h->tile_m - 1) / h->tile_m + E;
  const PeerOut pout{h->grp_orank.as<int32_t>(), h->grp_oshift.as<int32_t>(), h->peer_y, h->prowmap.as<int32_t>()};
  CKR(launch_gemm<tc::EPI_SWIGLU_BF16>(h, s, K_EXPERT_GEMM1, h->tm_pxrecv, h->tm_w1, gt, 2 * h->ff, d, h->h.p, h->ff,
                                       max_mtiles, nullptr, nullptr, h->cap_recv));
  CKR(launch_gemm<tc::EPI_STORE_BF16>(h, s, K_EXPERT_GEMM2, h->tm_h, h->tm_w2, gt, d, h->ff, nullptr, d, max_mtiles,
                                      nullptr, &pout, h->capP * k));
  CKR(barrier());
  if (T == 0) return NOOR_MOE_OK;
  if (fork) CK(cudaStreamWaitEvent(s, h->ev_join, 0));
  const float* shared_out = h->has_shared ? h->shared_out.as<float>() : nullptr;
  if (h->has_dense) {
    const CombineArgs comb{h->py.p, h->dst_row.as<int32_t>(), h->wts.as<float>(), shared_out, k, true, h->capP * k};
    return glu_down(h, s, dense, out, &comb);
  }
  return launch(h, s, K_COMBINE, [&] {
    const unsigned grid = (unsigned)((T + dispatch::kCombineWarps - 1) / dispatch::kCombineWarps);
    dispatch::combine_kernel<bf16, bf16><<<grid, dispatch::kCombineWarps * 32, 0, s>>>(
        h->py.as<bf16>(), nullptr, h->wts.as<float>(), nullptr, shared_out, (int32_t)T, d, k, (bf16*)out,
        h->capP * k, h->d_err);
  });
}

// ============================================================== forward

// x, out: device pointers of the layer dtype.  tmx: tensor map of x (BF16).
//
// One GPU: a single stream, in dependency order.  Expert parallel over peer
// memory: run_forward_peer.  Expert parallel over NCCL: the dense (and
// shared) up projections run on a second stream while the rows cross; the
// dense down projection waits for the returned expert rows.
int run_forward(noor_moe_handle* h, cudaStream_t s, const void* x, const CUtensorMap* tmx, void* out, int64_t T) {
  if (h->peer) return run_forward_peer(h, s, x, tmx, out, T);
  const int d = h->d, k = h->k, E = h->E;
  const int64_t b = h->bf16 ? 2 : 4;
  const GluFfn dense{K_DENSE_GEMM1, K_DENSE_GEMM2, tmx, x, T, h->dff, h->desc.dense_act == NOOR_ACT_SILU,
                     &h->tm_dw1, &h->tm_dw2, &h->tm_dh, h->dg32.as<float>(), h->du32.as<float>(),
                     h->dd32.as<float>(), h->dense_h.p};
  const GluFfn shared{K_SHARED_GEMM1, K_SHARED_GEMM2, tmx, x, T, h->ff, true, &h->tm_sw1, &h->tm_sw2, &h->tm_sh,
                      h->sg32.as<float>(), h->su32.as<float>(), h->sd32.as<float>(), h->shared_h.p};
  const bool fuse_combine = h->bf16 && h->has_dense;
  // BF16 on one GPU: the expert down projection writes y token-major (row
  // t*k + slot, through the permute's row map), so the combine reads each
  // token's k rows side by side.  The NCCL exchange returns rows in the
  // expert order and the combine gathers them through dst_row.
  const bool token_major = h->bf16 && h->G == 1;
  // The side branches (dense up projection, shared expert) run on a second
  // stream under the NCCL exchange, from the start, beside the transfers.  On
  // one GPU they run in line after the expert GEMMs unless kForkSideSingle.
  const bool side = (h->has_dense || h->has_shared) && T > 0 && (h->G > 1 || kForkSideSingle);
  const bool side_first = side && h->G > 1;
  cudaStream_t ss = side ? h->aux : s;  // stream of the side branches' up projections

  if (side_first) {
    CK(cudaEventRecord(h->ev_fork, s));
    CK(cudaStreamWaitEvent(h->aux, h->ev_fork, 0));
  }
  auto side_branches = [&]() -> int {
    if (T == 0) return NOOR_MOE_OK;
    if (h->has_dense) {
      CKR(glu_up(h, ss, dense));
      if (!fuse_combine) CKR(glu_down(h, ss, dense, h->dense_out.p, nullptr));
    }
    if (h->has_shared) {
      CKR(glu_up(h, ss, shared));
      CKR(glu_down(h, ss, shared, h->shared_out.p, nullptr));
    }
    if (side) CK(cudaEventRecord(h->ev_join, h->aux));
    return NOOR_MOE_OK;
  };
  if (side_first) CKR(side_branches());

  int tpb = 0;
  if (T == 0) {
    // A rank with no tokens still takes part in the exchange with zero counts.
    CK(cudaMemsetAsync(h->counts64.p, 0, E * 8, s));
  } else {
    CKR(run_router(h, s, x, tmx, T, &tpb, h->G == 1));
    if (side && !side_first) {
      CK(cudaEventRecord(h->ev_fork, s));
      CK(cudaStreamWaitEvent(h->aux, h->ev_fork, 0));
      CKR(side_branches());
    }
    CKR(launch(h, s, K_PERMUTE, [&] {
      // persistent beside the side branch's GEMM, else a block per 4 tokens
      const int64_t blocks = (T + dispatch::kPermuteWarps - 1) / dispatch::kPermuteWarps;
      const unsigned grid = (unsigned)(side ? std::min<int64_t>(blocks, h->num_sms) : blocks);
      dispatch::permute_rows_kernel<<<grid, dispatch::kPermuteWarps * 32, 0, s>>>(
          static_cast<const uint8_t*>(x), (int32_t)(d * b), (int32_t)T, k, (int32_t)((T + tpb - 1) / tpb), tpb,
          h->idx.as<int32_t>(), h->lrank.as<int32_t>(), h->blk_base.as<int32_t>(), h->seg_start.as<int32_t>(),
          h->xp.as<uint8_t>(), h->dst_row.as<int32_t>(), token_major ? h->ymap.as<int32_t>() : nullptr,
          h->capT * k, h->d_err);
    }));
  }

  GroupTable gt;
  const CUtensorMap* tA = &h->tm_xp;
  const void* A32 = h->xp.p;
  int64_t max_mtiles = 0;
  void* ybuf = h->y.p;  // rows the combine gathers from
  EpPlan plan;
  if (h->G == 1) {
    gt.row_start = h->seg_start.as<int32_t>();
    gt.mtile_start = h->mtile_start.as<int32_t>();
    gt.weight_idx = nullptr;
    gt.G = E;
    gt.dense_rows = -1;
    max_mtiles = (T * k + h->tile_m - 1) / h->tile_m + E;
  } else {
    CKR(ep_plan(h, s, plan));
    // global counts: the API's expert_counts and the layer's utilization
    CKN(noor::nccl().AllReduce(h->counts64.p, h->counts_glob.p, h->E, ncclInt64, ncclSum, h->comm, s));
    CKR(launch(h, s, K_SCAN, [&] {
      smebu::util_accumulate_kernel<<<1, 256, 0, s>>>(h->counts_glob.as<int64_t>(), E, k, h->util.as<int64_t>());
    }));
    CKR(ep_exchange(h, s, K_A2A_DISPATCH, plan, h->xp.p, h->xrecv.p, false));
    gt.row_start = h->grp_row.as<int32_t>();
    gt.mtile_start = h->grp_mtile.as<int32_t>();
    gt.weight_idx = h->grp_widx.as<int32_t>();
    gt.G = h->G * h->El;
    gt.dense_rows = -1;
    tA = &h->tm_xrecv;
    A32 = h->xrecv.p;
    max_mtiles = plan.mtiles;
    ybuf = h->ysend.p;
  }

  if (T > 0 && h->G == 1) max_mtiles = std::max<int64_t>(max_mtiles, 1);
  if (max_mtiles > 0) {
    if (h->bf16) {
      CKR(launch_gemm<tc::EPI_SWIGLU_BF16>(h, s, K_EXPERT_GEMM1, *tA, h->tm_w1, gt, 2 * h->ff, d, h->h.p, h->ff,
                                           max_mtiles, nullptr, nullptr, h->cap_recv));
      const PeerOut ytm{nullptr, nullptr, nullptr, h->ymap.as<int32_t>()};
      CKR(launch_gemm<tc::EPI_STORE_BF16>(h, s, K_EXPERT_GEMM2, h->tm_h, h->tm_w2, gt, d, h->ff, h->y.p, d,
                                          max_mtiles, nullptr, token_major ? &ytm : nullptr, h->cap_recv));
    } else {
      const int64_t ffd = (int64_t)d * h->ff;
      CKR((launch_simt<simt::EPI_SWIGLU>(h, s, K_EXPERT_GEMM1, gt, (const float*)A32, d, h->wg32.as<float>(),
                                         h->wu32.as<float>(), ffd, h->ff, d, h->h.as<float>(), h->ff, max_mtiles)));
      CKR((launch_simt<simt::EPI_STORE>(h, s, K_EXPERT_GEMM2, gt, h->h.as<float>(), h->ff, h->wd32.as<float>(), nullptr,
                                        ffd, d, h->ff, h->y.as<float>(), d, max_mtiles)));
    }
  }
  if (h->G > 1) CKR(ep_exchange(h, s, K_A2A_COMBINE, plan, h->y.p, h->ysend.p, true));

  if (side) CK(cudaStreamWaitEvent(s, h->ev_join, 0));
  else CKR(side_branches());  // nothing to do: no side branch or no tokens
  if (T == 0) return NOOR_MOE_OK;
  const float* shared_out = h->has_shared ? h->shared_out.as<float>() : nullptr;
  if (fuse_combine) {
    const int64_t y_rows = h->G > 1 ? h->capT * k : h->cap_recv;  // ysend (NCCL) or y
    const CombineArgs comb{ybuf, h->dst_row.as<int32_t>(), h->wts.as<float>(), shared_out, k, token_major, y_rows};
    return glu_down(h, s, dense, out, &comb);
  }
  return launch(h, s, K_COMBINE, [&] {
    const unsigned grid = (unsigned)((T + dispatch::kCombineWarps - 1) / dispatch::kCombineWarps);
    const float* dense_out = h->has_dense ? h->dense_out.as<float>() : nullptr;
    const int64_t y_rows = h->G > 1 ? h->capT * k : h->cap_recv;  // ysend (NCCL) or y
    if (h->bf16)
      dispatch::combine_kernel<bf16, bf16><<<grid, dispatch::kCombineWarps * 32, 0, s>>>(
          (const bf16*)ybuf, token_major ? nullptr : h->dst_row.as<int32_t>(), h->wts.as<float>(), dense_out,
          shared_out, (int32_t)T, d, k, (bf16*)out, y_rows, h->d_err);
    else
      dispatch::combine_kernel<float, float><<<grid, dispatch::kCombineWarps * 32, 0, s>>>(
          (const float*)ybuf, h->dst_row.as<int32_t>(), h->wts.as<float>(), dense_out, shared_out, (int32_t)T, d, k,
          (float*)out, y_rows, h->d_err);
  });
}

int global_counts(noor_moe_handle* h, cudaStream_t s, const int64_t** src) {
  if (h->G == 1) {
    *src = h->counts64.as<int64_t>();
    return NOOR_MOE_OK;
  }
  (void)s;  // summed in the forward: by the plan kernel (peer memory) or an all-reduce (NCCL)
  *src = h->counts_glob.as<int64_t>();
  return NOOR_MOE_OK;
}

int validate(const noor_moe_desc* d) {
  if (!d) return fail(NOOR_MOE_ERR_INVALID, "null descriptor");
  if (d->d_model <= 0 || d->n_experts <= 0 || d->top_k <= 0 || d->expert_ff <= 0)
    return fail(NOOR_MOE_ERR_INVALID, "sizes must be positive");
  if (d->dtype != NOOR_DTYPE_F32 && d->dtype != NOOR_DTYPE_BF16) return fail(NOOR_MOE_ERR_INVALID, "unknown dtype");
  if (d->dense_act != NOOR_ACT_GELU_TANH && d->dense_act != NOOR_ACT_SILU)
    return fail(NOOR_MOE_ERR_INVALID, "unknown dense activation");
  if (d->has_dense && d->dense_ff <= 0) return fail(NOOR_MOE_ERR_INVALID, "dense_ff must be positive");
  const int k = std::min(d->top_k, d->n_experts);
  if (k > router::kMaxTopK) return fail(NOOR_MOE_ERR_UNSUPPORTED, "top_k > %d", router::kMaxTopK);
  if (d->world_size < 1 || d->rank < 0 || d->rank >= d->world_size) return fail(NOOR_MOE_ERR_INVALID, "bad rank");
  if (d->n_experts % d->world_size != 0)
    return fail(NOOR_MOE_ERR_INVALID, "n_experts must be divisible by world_size");
  if (d->d_model % 8 != 0) return fail(NOOR_MOE_ERR_UNSUPPORTED, "d_model must be a multiple of 8");
  if (d->n_experts > 256) return fail(NOOR_MOE_ERR_UNSUPPORTED, "at most 256 experts");
  if (d->dtype == NOOR_DTYPE_BF16) {
    if (d->n_experts > router::kMaxExpertsTC)
      return fail(NOOR_MOE_ERR_UNSUPPORTED, "BF16 layers support at most %d experts", router::kMaxExpertsTC);
    if (d->d_model % 128 != 0 || d->expert_ff % 128 != 0 || (d->has_dense && d->dense_ff % 128 != 0))
      return fail(NOOR_MOE_ERR_UNSUPPORTED, "BF16 layers need d_model, expert_ff, dense_ff multiples of 128");
  }
  return NOOR_MOE_OK;
}

}  // namespace

// ============================================================== C ABI

extern "C" {

const char* noor_moe_last_error(void) { return g_last_error.c_str(); }

int noor_moe_create(const noor_moe_desc* desc, void* nccl_comm, noor_moe_handle** out) {
  if (!out) return fail(NOOR_MOE_ERR_INVALID, "null out");
  *out = nullptr;
  CKR(validate(desc));
  if (desc->world_size > 1 && !nccl_comm)
    return fail(NOOR_MOE_ERR_INVALID, "world_size > 1 needs an NCCL communicator");
  int ndev = 0;
  CK(cudaGetDeviceCount(&ndev));
  if (desc->device < 0 || desc->device >= ndev) return fail(NOOR_MOE_ERR_INVALID, "bad device %d", desc->device);
  DeviceGuard g(desc->device);
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, desc->device));
  if (desc->dtype == NOOR_DTYPE_BF16 && prop.major != 10)
    return fail(NOOR_MOE_ERR_UNSUPPORTED, "BF16 layers need an sm_100 GPU (found sm_%d%d)", prop.major, prop.minor);
  noor_moe_handle* h = new noor_moe_handle();
  h->desc = *desc;
  h->E = desc->n_experts;
  h->k = std::min(desc->top_k, desc->n_experts);
  h->d = desc->d_model;
  h->ff = desc->expert_ff;
  h->dff = desc->dense_ff;
  h->G = desc->world_size;
  h->rank = desc->rank;
  h->El = h->E / h->G;
  h->e0 = h->rank * h->El;
  h->bf16 = desc->dtype == NOOR_DTYPE_BF16;
  h->dev = desc->device;
  h->num_sms = prop.multiProcessorCount;
  h->comm = static_cast<ncclComm_t>(nccl_comm);
  h->has_dense = desc->has_dense != 0;
  h->has_shared = desc->has_shared != 0;
  h->Epad = (h->E + 7) / 8 * 8;
  h->bn2 = (h->d % 256 == 0) ? 256 : 128;
  h->pair2 = h->bf16 && h->d % 256 == 0;
  h->tile_m = h->pair2 ? tc::BM2 : (h->bf16 ? tc::BM : simt::BM);
  auto bail = [&](int rc) {
    noor_moe_destroy(h);
    return rc;
  };
  if (cudaStreamCreateWithFlags(&h->own, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&h->aux, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&h->ev_fork, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&h->ev_join, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&h->ev_done, cudaEventDisableTiming) != cudaSuccess ||
      cudaMalloc(&h->d_err, sizeof(int)) != cudaSuccess || cudaMemset(h->d_err, 0, sizeof(int)) != cudaSuccess)
    return bail(fail(NOOR_MOE_ERR_CUDA, "stream/event/flag setup failed"));
  if (h->G > 1) {
    const int ng = h->G * h->El;
    if (cudaMallocHost(&h->h_cnt, (h->E + ng) * 8) != cudaSuccess ||
        cudaMallocHost(&h->h_grp, 3 * (ng + 1) * 4) != cudaSuccess)
      return bail(fail(NOOR_MOE_ERR_OOM, "pinned host buffers"));
  }
  if (h->scan_done.ensure(sizeof(int)) != NOOR_MOE_OK || cudaMemset(h->scan_done.p, 0, sizeof(int)) != cudaSuccess ||
      h->seg_acc.ensure(h->E * 4) != NOOR_MOE_OK || cudaMemset(h->seg_acc.p, 0, h->E * 4) != cudaSuccess)
    return bail(fail(NOOR_MOE_ERR_CUDA, "scan counter setup failed"));
  if (h->util.ensure((h->E + 1) * 8) != NOOR_MOE_OK || cudaMemset(h->util.p, 0, (h->E + 1) * 8) != cudaSuccess ||
      h->smebu_m.ensure(h->E * 4) != NOOR_MOE_OK || cudaMemset(h->smebu_m.p, 0, h->E * 4) != cudaSuccess)
    return bail(fail(NOOR_MOE_ERR_CUDA, "utilization setup failed"));
  int rc = ensure_workspace(h, std::max<int64_t>(desc->max_tokens, 128));
  if (rc != NOOR_MOE_OK) return bail(rc);
  if (h->G > 1) {
    rc = peer_setup(h);
    if (rc != NOOR_MOE_OK) return bail(rc);
  }
  *out = h;
  return NOOR_MOE_OK;
}

int noor_moe_load_weights(noor_moe_handle* h, const float* gate, const float* bias, const float* scales,
                          const float* const* w_gate, const float* const* w_up, const float* const* w_down,
                          const float* const* shared, const float* const* dense) {
  if (!h || !gate || !bias || !scales || !w_gate || !w_up || !w_down)
    return fail(NOOR_MOE_ERR_INVALID, "null weight pointer");
  if (h->has_dense && (!dense || !dense[0] || !dense[1] || !dense[2]))
    return fail(NOOR_MOE_ERR_INVALID, "dense branch weights missing");
  if (h->has_shared && (!shared || !shared[0] || !shared[1] || !shared[2]))
    return fail(NOOR_MOE_ERR_INVALID, "shared expert weights missing");
  for (int le = 0; le < h->El; ++le)
    if (!w_gate[h->e0 + le] || !w_up[h->e0 + le] || !w_down[h->e0 + le])
      return fail(NOOR_MOE_ERR_INVALID, "expert %d weights missing", h->e0 + le);
  DeviceGuard g(h->dev);
  const int d = h->d, ff = h->ff, dff = h->dff, E = h->E, El = h->El;
  CKR(h->bias.ensure(E * 4));
  CKR(h->scales.ensure(E * 4));
  CK(cudaMemcpy(h->bias.p, bias, E * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(h->scales.p, scales, E * 4, cudaMemcpyHostToDevice));
  cudaStream_t s = h->own;
  if (!h->bf16) {
    const int64_t m = (int64_t)d * ff;
    CKR(h->gate.ensure((int64_t)d * E * 4));
    CK(cudaMemcpy(h->gate.p, gate, (int64_t)d * E * 4, cudaMemcpyHostToDevice));
    CKR(h->wg32.ensure(El * m * 4));
    CKR(h->wu32.ensure(El * m * 4));
    CKR(h->wd32.ensure(El * m * 4));
    for (int le = 0; le < El; ++le) {
      CK(cudaMemcpy(h->wg32.as<float>() + le * m, w_gate[h->e0 + le], m * 4, cudaMemcpyHostToDevice));
      CK(cudaMemcpy(h->wu32.as<float>() + le * m, w_up[h->e0 + le], m * 4, cudaMemcpyHostToDevice));
      CK(cudaMemcpy(h->wd32.as<float>() + le * m, w_down[h->e0 + le], m * 4, cudaMemcpyHostToDevice));
    }
    if (h->has_dense) {
      const int64_t md = (int64_t)d * dff;
      CKR(h->dg32.ensure(md * 4));
      CKR(h->du32.ensure(md * 4));
      CKR(h->dd32.ensure(md * 4));
      CK(cudaMemcpy(h->dg32.p, dense[0], md * 4, cudaMemcpyHostToDevice));
      CK(cudaMemcpy(h->du32.p, dense[1], md * 4, cudaMemcpyHostToDevice));
      CK(cudaMemcpy(h->dd32.p, dense[2], md * 4, cudaMemcpyHostToDevice));
    }
    if (h->has_shared) {
      CKR(h->sg32.ensure(m * 4));
      CKR(h->su32.ensure(m * 4));
      CKR(h->sd32.ensure(m * 4));
      CK(cudaMemcpy(h->sg32.p, shared[0], m * 4, cudaMemcpyHostToDevice));
      CK(cudaMemcpy(h->su32.p, shared[1], m * 4, cudaMemcpyHostToDevice));
      CK(cudaMemcpy(h->sd32.p, shared[2], m * 4, cudaMemcpyHostToDevice));
    }
    CK(cudaDeviceSynchronize());
    h->weights = true;
    return NOOR_MOE_OK;
  }

  // BF16: stage each f32 matrix on the device, then transpose + round.
  const int64_t stage_elems = std::max<int64_t>({(int64_t)d * ff, (int64_t)d * std::max(dff, 1), (int64_t)d * E});
  DevBuf stage;
  CKR(stage.ensure(stage_elems * 4));
  auto pack = [&](const float* src, int K, int N, bf16* dst, int group, int stride, int offset) -> int {
    CK(cudaMemcpyAsync(stage.p, src, (int64_t)K * N * 4, cudaMemcpyHostToDevice, s));
    dim3 grid((N + 31) / 32, (K + 31) / 32), block(32, 8);
    CKR(launch(h, s, K_PREPACK, [&] {
      prepack::transpose_to_bf16_kernel<<<grid, block, 0, s>>>(stage.as<float>(), K, N, dst, K, group, stride, offset);
    }));
    CK(cudaStreamSynchronize(s));  // the staging buffer is reused by the next matrix
    return NOOR_MOE_OK;
  };
  CKR(h->gate.ensure((int64_t)h->Epad * d * 2));
  CK(cudaMemset(h->gate.p, 0, (int64_t)h->Epad * d * 2));
  CKR(pack(gate, d, E, h->gate.as<bf16>(), E, E, 0));
  CKR(encode_kmajor(&h->tm_gate, h->gate.p, h->Epad, d, router::tc_npad(E)));
  // experts: W1 [El][2ff][d] with 128-row gate / up blocks interleaved; W2 [El][d][ff]
  CKR(h->w1.ensure((int64_t)El * 2 * ff * d * 2));
  CKR(h->w2.ensure((int64_t)El * d * ff * 2));
  for (int le = 0; le < El; ++le) {
    bf16* w1 = h->w1.as<bf16>() + (int64_t)le * 2 * ff * d;
    CKR(pack(w_gate[h->e0 + le], d, ff, w1, 128, 256, 0));
    CKR(pack(w_up[h->e0 + le], d, ff, w1, 128, 256, 128));
    CKR(pack(w_down[h->e0 + le], ff, d, h->w2.as<bf16>() + (int64_t)le * d * ff, d, d, 0));
  }
  const int bbox1 = h->pair2 ? 128 : 256, bbox2 = h->pair2 ? 128 : h->bn2;  // rows of B one CTA loads
  CKR(encode_kmajor(&h->tm_w1, h->w1.p, (int64_t)El * 2 * ff, d, bbox1));
  CKR(encode_kmajor(&h->tm_w2, h->w2.p, (int64_t)El * d, ff, bbox2));
  if (h->has_dense) {
    CKR(h->dw1.ensure((int64_t)2 * dff * d * 2));
    CKR(h->dw2.ensure((int64_t)d * dff * 2));
    CKR(pack(dense[0], d, dff, h->dw1.as<bf16>(), 128, 256, 0));
    CKR(pack(dense[1], d, dff, h->dw1.as<bf16>(), 128, 256, 128));
    CKR(pack(dense[2], dff, d, h->dw2.as<bf16>(), d, d, 0));
    CKR(encode_kmajor(&h->tm_dw1, h->dw1.p, 2 * dff, d, bbox1));
    CKR(encode_kmajor(&h->tm_dw2, h->dw2.p, d, dff, bbox2));
  }
  if (h->has_shared) {
    CKR(h->sw1.ensure((int64_t)2 * ff * d * 2));
    CKR(h->sw2.ensure((int64_t)d * ff * 2));
    CKR(pack(shared[0], d, ff, h->sw1.as<bf16>(), 128, 256, 0));
    CKR(pack(shared[1], d, ff, h->sw1.as<bf16>(), 128, 256, 128));
    CKR(pack(shared[2], ff, d, h->sw2.as<bf16>(), d, d, 0));
    CKR(encode_kmajor(&h->tm_sw1, h->sw1.p, 2 * ff, d, bbox1));
    CKR(encode_kmajor(&h->tm_sw2, h->sw2.p, d, ff, bbox2));
  }
  stage.release();
  h->weights = true;
  return NOOR_MOE_OK;
}

int noor_moe_set_bias(noor_moe_handle* h, const float* bias) {
  if (!h || !bias) return fail(NOOR_MOE_ERR_INVALID, "null argument");
  if (!h->weights) return fail(NOOR_MOE_ERR_STATE, "set_bias before load_weights");
  DeviceGuard g(h->dev);
  CK(cudaMemcpy(h->bias.p, bias, h->E * 4, cudaMemcpyHostToDevice));
  return NOOR_MOE_OK;
}

// Row-wise RMSNorm x sandwich depth scale (+ residual) over T rows of the
// layer dtype.
static int launch_norm(noor_moe_handle* h, cudaStream_t s, int kind, const void* x, const float* w,
                       const void* resid, int64_t T, void* out) {
  if (T == 0) return NOOR_MOE_OK;
  const unsigned grid = (unsigned)((T + norm::kWarps - 1) / norm::kWarps);
  const int smem = norm::staged_smem_bytes(h->bf16, h->d);  // BF16 rows staged in shared memory
  if (smem > 48 * 1024) {
    CKR(ensure_smem_limit(norm::rms_norm_rows_kernel<bf16, true, true>, smem));
    CKR(ensure_smem_limit(norm::rms_norm_rows_kernel<bf16, false, true>, smem));
  }
  return launch(h, s, kind, [&] {
    if (h->bf16) {
      const bf16* xb = (const bf16*)x;
      bf16* ob = (bf16*)out;
      if (smem > 0) {
        if (resid)
          norm::rms_norm_rows_kernel<bf16, true, true><<<grid, norm::kWarps * 32, smem, s>>>(
              xb, w, h->norm_eps, h->depth_scale, (const bf16*)resid, (int32_t)T, h->d, ob);
        else
          norm::rms_norm_rows_kernel<bf16, false, true><<<grid, norm::kWarps * 32, smem, s>>>(
              xb, w, h->norm_eps, h->depth_scale, nullptr, (int32_t)T, h->d, ob);
      } else {
        if (resid)
          norm::rms_norm_rows_kernel<bf16, true, false><<<grid, norm::kWarps * 32, 0, s>>>(
              xb, w, h->norm_eps, h->depth_scale, (const bf16*)resid, (int32_t)T, h->d, ob);
        else
          norm::rms_norm_rows_kernel<bf16, false, false><<<grid, norm::kWarps * 32, 0, s>>>(
              xb, w, h->norm_eps, h->depth_scale, nullptr, (int32_t)T, h->d, ob);
      }
    } else {
      if (resid)
        norm::rms_norm_rows_kernel<float, true, false><<<grid, norm::kWarps * 32, 0, s>>>(
            (const float*)x, w, h->norm_eps, h->depth_scale, (const float*)resid, (int32_t)T, h->d, (float*)out);
      else
        norm::rms_norm_rows_kernel<float, false, false><<<grid, norm::kWarps * 32, 0, s>>>(
            (const float*)x, w, h->norm_eps, h->depth_scale, nullptr, (int32_t)T, h->d, (float*)out);
    }
  });
}

// sublayer: the MoE block's FFN sublayer, out = x + post(layer(pre(x)))
// (block.rs:87-90), instead of the layer alone.
static int forward_impl(noor_moe_handle* h, const void* x, void* out, int64_t T, int32_t* topk_idx, float* topk_w,
                        int64_t* expert_counts, void* stream, bool route_only, bool sublayer = false) {
  if (!h) return fail(NOOR_MOE_ERR_INVALID, "null handle");
  if (!h->weights) return fail(NOOR_MOE_ERR_STATE, "forward before load_weights");
  if (h->comm_broken) return fail(NOOR_MOE_ERR_STATE, "communicator was aborted after a failed exchange");
  if (T < 0 || T > (int64_t)INT32_MAX / std::max(1, h->k * h->G))
    return fail(NOOR_MOE_ERR_INVALID, "token count %lld out of range", (long long)T);
  if (!x && T > 0) return fail(NOOR_MOE_ERR_INVALID, "null x");
  if (!route_only && !out && T > 0) return fail(NOOR_MOE_ERR_INVALID, "null out");
  DeviceGuard g(h->dev);
  CKR(ensure_workspace(h, std::max<int64_t>(T, 1)));
  const bool host = stream == nullptr;
  cudaStream_t s = host ? h->own : static_cast<cudaStream_t>(stream);
  const int64_t b = h->bf16 ? 2 : 4;
  const int64_t xbytes = T * h->d * b;
  if (T == 0 && h->G == 1) {
    if (expert_counts) {
      if (host) std::memset(expert_counts, 0, h->E * 8);
      else CK(cudaMemsetAsync(expert_counts, 0, h->E * 8, s));
    }
    return NOOR_MOE_OK;
  }
  const void* xd = x;
  const CUtensorMap* tmx = &h->tm_xin;
  if (host) {
    if (T > 0) CK(cudaMemcpyAsync(h->x_in.p, x, xbytes, cudaMemcpyHostToDevice, s));
    xd = h->x_in.p;
  } else if (h->bf16 && !sublayer && T > 0) {
    if (x != h->tm_user_ptr || T != h->tm_user_T) {
      CKR(encode_kmajor(&h->tm_user, x, T, h->d, tc::BM));
      h->tm_user_ptr = x;
      h->tm_user_T = T;
    }
    tmx = &h->tm_user;
  }
  if (route_only) {
    int tpb = 0;
    if (T > 0) CKR(run_router(h, s, xd, tmx, T, &tpb));
  } else {
    void* od = host ? h->out_buf.p : out;
    if (sublayer) {
      CKR(launch_norm(h, s, K_NORM_PRE, xd, h->pre_w.as<float>(), nullptr, T, h->xn.p));
      CKR(run_forward(h, s, h->xn.p, &h->tm_xn, h->ffn.p, T));
      CKR(launch_norm(h, s, K_NORM_POST, h->ffn.p, h->post_w.as<float>(), xd, T, od));
    } else {
      CKR(run_forward(h, s, xd, tmx, od, T));
    }
    if (host && T > 0) CK(cudaMemcpyAsync(out, od, xbytes, cudaMemcpyDeviceToHost, s));
  }
  const cudaMemcpyKind dk = host ? cudaMemcpyDeviceToHost : cudaMemcpyDeviceToDevice;
  if (topk_idx && T > 0) CK(cudaMemcpyAsync(topk_idx, h->idx.p, T * h->k * 4, dk, s));
  if (topk_w && T > 0) CK(cudaMemcpyAsync(topk_w, h->wts.p, T * h->k * 4, dk, s));
  if (expert_counts) {
    const int64_t* src = nullptr;
    if (route_only || h->G == 1) src = h->counts64.as<int64_t>();
    else CKR(global_counts(h, s, &src));
    CK(cudaMemcpyAsync(expert_counts, src, h->E * 8, dk, s));
  }
  if (host) {
    CK(cudaEventRecord(h->ev_done, s));
    CKR(wait_event_deadline(h, h->ev_done, 300.0));
    CKR(check_device_error(h));
  }
  return NOOR_MOE_OK;
}

int noor_moe_forward(noor_moe_handle* h, const void* x, void* out, int64_t T, int32_t* topk_idx, float* topk_w,
                     int64_t* expert_counts, void* stream) {
  return forward_impl(h, x, out, T, topk_idx, topk_w, expert_counts, stream, false);
}

int noor_moe_set_sandwich(noor_moe_handle* h, const float* pre_w, const float* post_w, double eps,
                          float depth_scale) {
  if (!h || !pre_w || !post_w) return fail(NOOR_MOE_ERR_INVALID, "null argument");
  if (!(eps >= 0.0) || !(depth_scale > 0.0f)) return fail(NOOR_MOE_ERR_INVALID, "bad eps or depth_scale");
  DeviceGuard g(h->dev);
  CKR(h->pre_w.ensure(h->d * 4));
  CKR(h->post_w.ensure(h->d * 4));
  CK(cudaMemcpy(h->pre_w.p, pre_w, h->d * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(h->post_w.p, post_w, h->d * 4, cudaMemcpyHostToDevice));
  h->norm_eps = eps;
  h->depth_scale = depth_scale;
  if (!h->sandwich) {
    h->sandwich = true;
    const int64_t b = h->bf16 ? 2 : 4;
    CKR(h->xn.ensure(h->capT * h->d * b));
    CKR(h->ffn.ensure(h->capT * h->d * b));
    if (h->bf16) CKR(encode_kmajor(&h->tm_xn, h->xn.p, h->capT, h->d, tc::BM));
  }
  return NOOR_MOE_OK;
}

int noor_gguf_tensor_info(const char* path, const char* name, int64_t* dims, int32_t* n_dims, int32_t* dtype) {
  if (!path || !name || !dims || !n_dims || !dtype) return fail(NOOR_MOE_ERR_INVALID, "null argument");
  noor::gguf::File f;
  if (!f.open(path)) return fail(NOOR_MOE_ERR_INVALID, "%s: %s", path, f.error().c_str());
  const noor::gguf::TensorInfo* t = f.find(name);
  if (!t) return fail(NOOR_MOE_ERR_INVALID, "%s: no tensor %s", path, name);
  *n_dims = (int32_t)t->dims.size();
  for (size_t i = 0; i < t->dims.size(); ++i) dims[i] = (int64_t)t->dims[i];
  *dtype = (int32_t)t->type;
  return NOOR_MOE_OK;
}

int noor_gguf_read_f32(const char* path, const char* name, float* out, int64_t n) {
  if (!path || !name || !out) return fail(NOOR_MOE_ERR_INVALID, "null argument");
  noor::gguf::File f;
  if (!f.open(path)) return fail(NOOR_MOE_ERR_INVALID, "%s: %s", path, f.error().c_str());
  const noor::gguf::TensorInfo* t = f.find(name);
  if (!t) return fail(NOOR_MOE_ERR_INVALID, "%s: no tensor %s", path, name);
  if ((uint64_t)n != t->numel) return fail(NOOR_MOE_ERR_INVALID, "tensor %s has %llu elements, not %lld", name,
                                           (unsigned long long)t->numel, (long long)n);
  std::vector<float> scratch;
  std::memcpy(out, f.f32(*t, scratch), t->numel * 4);
  return NOOR_MOE_OK;
}

int noor_moe_load_gguf(noor_moe_handle* h, const char* path, int32_t layer, double norm_eps) {
  if (!h || !path || layer < 0) return fail(NOOR_MOE_ERR_INVALID, "bad argument");
  noor::gguf::File f;
  if (!f.open(path)) return fail(NOOR_MOE_ERR_INVALID, "%s: %s", path, f.error().c_str());
  const std::string pre = "blocks." + std::to_string(layer) + ".";
  std::deque<std::vector<float>> scratch;  // f32 copies of F16 tensors
  auto get = [&](const std::string& name, std::initializer_list<uint64_t> shape, const float** out) -> int {
    const noor::gguf::TensorInfo* t = f.find(name);
    if (!t) return fail(NOOR_MOE_ERR_INVALID, "%s: no tensor %s", path, name.c_str());
    if (t->dims != std::vector<uint64_t>(shape)) {
      std::string want, got;
      for (uint64_t v : shape) want += (want.empty() ? "" : ",") + std::to_string(v);
      for (uint64_t v : t->dims) got += (got.empty() ? "" : ",") + std::to_string(v);
      return fail(NOOR_MOE_ERR_INVALID, "%s: tensor %s has shape [%s], the layer needs [%s]", path, name.c_str(),
                  got.c_str(), want.c_str());
    }
    scratch.emplace_back();
    *out = f.f32(*t, scratch.back());
    return NOOR_MOE_OK;
  };
  const uint64_t d = h->d, E = h->E, ff = h->ff, dff = h->dff;
  const float *gate = nullptr, *bias = nullptr, *scales = nullptr;
  CKR(get(pre + "moe.router.gate", {d, E}, &gate));
  CKR(get(pre + "moe.router.biases", {E}, &bias));
  CKR(get(pre + "moe.router.scales", {E}, &scales));
  std::vector<const float*> wg(E, nullptr), wu(E, nullptr), wd(E, nullptr);
  for (int e = h->e0; e < h->e0 + h->El; ++e) {  // this rank's experts only
    const std::string ex = pre + "moe.experts." + std::to_string(e) + ".";
    CKR(get(ex + "w_gate", {d, ff}, &wg[e]));
    CKR(get(ex + "w_up", {d, ff}, &wu[e]));
    CKR(get(ex + "w_down", {ff, d}, &wd[e]));
  }
  const float* shared[3] = {nullptr, nullptr, nullptr};
  if (h->has_shared) {
    CKR(get(pre + "moe.shared.w_gate", {d, ff}, &shared[0]));
    CKR(get(pre + "moe.shared.w_up", {d, ff}, &shared[1]));
    CKR(get(pre + "moe.shared.w_down", {ff, d}, &shared[2]));
  }
  const float* dense[3] = {nullptr, nullptr, nullptr};
  if (h->has_dense) {
    CKR(get(pre + "dense.w_gate", {d, dff}, &dense[0]));
    CKR(get(pre + "dense.w_up", {d, dff}, &dense[1]));
    CKR(get(pre + "dense.w_down", {dff, d}, &dense[2]));
  }
  const float *pre_w = nullptr, *post_w = nullptr;
  if (norm_eps >= 0.0) {
    CKR(get(pre + "ffn_norm.pre.weight", {d}, &pre_w));
    CKR(get(pre + "ffn_norm.post.weight", {d}, &post_w));
  }
  CKR(noor_moe_load_weights(h, gate, bias, scales, wg.data(), wu.data(), wd.data(), shared, dense));
  if (norm_eps >= 0.0) {
    const float depth_scale = 1.0f / std::sqrt((float)(layer + 1));  // norm.rs:44
    CKR(noor_moe_set_sandwich(h, pre_w, post_w, norm_eps, depth_scale));
  }
  return NOOR_MOE_OK;
}

int noor_moe_ffn_sublayer_forward(noor_moe_handle* h, const void* x, void* out, int64_t T, int32_t* topk_idx,
                                  float* topk_w, int64_t* expert_counts, void* stream) {
  if (h && !h->sandwich) return fail(NOOR_MOE_ERR_STATE, "ffn_sublayer_forward before set_sandwich");
  return forward_impl(h, x, out, T, topk_idx, topk_w, expert_counts, stream, false, true);
}

int noor_moe_route(noor_moe_handle* h, const void* x, int64_t T, int32_t* idx, float* w, int64_t* counts,
                   void* stream) {
  if (!idx || !w) return fail(NOOR_MOE_ERR_INVALID, "idx and w are required");
  return forward_impl(h, x, nullptr, T, idx, w, counts, stream, true);
}

int noor_moe_sync(noor_moe_handle* h, void* stream) {
  if (!h) return fail(NOOR_MOE_ERR_INVALID, "null handle");
  DeviceGuard g(h->dev);
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->own;
  CK(cudaEventRecord(h->ev_done, s));
  CKR(wait_event_deadline(h, h->ev_done, 300.0));
  return check_device_error(h);
}

void noor_moe_destroy(noor_moe_handle* h) {
  if (!h) return;
  {
    DeviceGuard g(h->dev);
    cudaDeviceSynchronize();
    peer_release(h);
    DevBuf* bufs[] = {&h->gate, &h->bias, &h->scales, &h->w1, &h->w2, &h->wg32, &h->wu32, &h->wd32, &h->dw1,
                      &h->dw2, &h->dg32, &h->du32, &h->dd32, &h->sw1, &h->sw2, &h->sg32, &h->su32, &h->sd32,
                      &h->x_in, &h->out_buf, &h->idx, &h->wts, &h->lrank, &h->dst_row, &h->blk_hist,
                      &h->blk_base, &h->counts64, &h->counts_glob, &h->seg_start, &h->mtile_start, &h->scores,
                      &h->xp, &h->h, &h->y, &h->ymap, &h->xrecv, &h->ysend, &h->dense_h, &h->dense_out, &h->shared_h,
                      &h->shared_out, &h->grp_row, &h->grp_mtile, &h->grp_widx, &h->cnt_recv, &h->scan_done,
                      &h->seg_acc,
                      &h->util, &h->smebu_m, &h->pre_w, &h->post_w, &h->xn, &h->ffn};
    for (DevBuf* b : bufs) b->release();
    if (h->h_cnt) cudaFreeHost(h->h_cnt);
    if (h->h_grp) cudaFreeHost(h->h_grp);
    if (h->d_err) cudaFree(h->d_err);
    for (cudaEvent_t e : h->prof_ev) cudaEventDestroy(e);
    if (h->ev_fork) cudaEventDestroy(h->ev_fork);
    if (h->ev_join) cudaEventDestroy(h->ev_join);
    if (h->ev_done) cudaEventDestroy(h->ev_done);
    if (h->own) cudaStreamDestroy(h->own);
    if (h->aux) cudaStreamDestroy(h->aux);
  }
  delete h;
}

int noor_matmul_f32(const float* a, const float* b, float* c, int64_t m, int64_t k, int64_t n) {
  if (!a || !b || !c) return fail(NOOR_MOE_ERR_INVALID, "null argument");
  if (m <= 0 || k <= 0 || n <= 0 || m > INT32_MAX || k > INT32_MAX || n > INT32_MAX)
    return fail(NOOR_MOE_ERR_INVALID, "bad shape");
  int dev = 0;
  CK(cudaGetDevice(&dev));
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, dev));
  DevBuf A, B, C;
  CKR(A.ensure(m * k * 4));
  CKR(B.ensure(k * n * 4));
  CKR(C.ensure(m * n * 4));
  CK(cudaMemcpy(A.p, a, m * k * 4, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(B.p, b, k * n * 4, cudaMemcpyHostToDevice));
  simt::Params p;
  p.groups = dense_group(m);
  p.A = A.as<float>();
  p.lda = k;
  p.Bg = B.as<float>();
  p.Bu = nullptr;
  p.b_stride = 0;
  p.N = (int32_t)n;
  p.K = (int32_t)k;
  p.n_tiles = (int32_t)((n + simt::BN - 1) / simt::BN);
  p.C = C.as<float>();
  p.ldc = n;
  const int64_t tiles = (m + simt::BM - 1) / simt::BM * p.n_tiles;
  const int grid = (int)std::min<int64_t>((int64_t)prop.multiProcessorCount * 8, tiles);
  simt::grouped_gemm_f32_kernel<simt::EPI_STORE><<<grid, simt::THREADS>>>(p);
  CK(cudaGetLastError());
  CK(cudaMemcpy(c, C.p, m * n * 4, cudaMemcpyDeviceToHost));
  return NOOR_MOE_OK;
}

int noor_moe_comm_id_size(void) { return (int)sizeof(ncclUniqueId); }

int noor_moe_comm_get_id(void* id_out) {
  if (!id_out) return fail(NOOR_MOE_ERR_INVALID, "null id");
  ncclUniqueId id;
  CKN(noor::nccl().GetUniqueId(&id));
  std::memcpy(id_out, &id, sizeof(id));
  return NOOR_MOE_OK;
}

int noor_moe_comm_init_rank(const void* id, int world_size, int rank, int device, void** comm_out) {
  if (!id || !comm_out) return fail(NOOR_MOE_ERR_INVALID, "null argument");
  DeviceGuard g(device);
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclComm_t comm;
  CKN(noor::nccl().CommInitRank(&comm, world_size, uid, rank));
  *comm_out = comm;
  return NOOR_MOE_OK;
}

int noor_moe_comm_destroy(void* comm) {
  if (!comm) return NOOR_MOE_OK;
  CKN(noor::nccl().CommDestroy(static_cast<ncclComm_t>(comm)));
  return NOOR_MOE_OK;
}

int noor_moe_profile_begin(noor_moe_handle* h, int max_launches) {
  if (!h || max_launches <= 0) return fail(NOOR_MOE_ERR_INVALID, "bad argument");
  DeviceGuard g(h->dev);
  while ((int)h->prof_ev.size() < 2 * max_launches) {
    cudaEvent_t e;
    CK(cudaEventCreate(&e));
    h->prof_ev.push_back(e);
  }
  h->prof_kind.assign(max_launches, 0);
  h->prof_cap = max_launches;
  h->prof_used = 0;
  h->prof_on = true;
  return NOOR_MOE_OK;
}

int noor_moe_profile_end(noor_moe_handle* h, char* names, float* total_ms, int32_t* launches, int n_slots,
                         int* n_out) {
  if (!h || !names || !total_ms || !launches || !n_out) return fail(NOOR_MOE_ERR_INVALID, "null argument");
  DeviceGuard g(h->dev);
  h->prof_on = false;
  float tot[K_NUM] = {0};
  int cnt[K_NUM] = {0};
  for (int i = 0; i < h->prof_used; ++i) {
    CK(cudaEventSynchronize(h->prof_ev[2 * i + 1]));
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, h->prof_ev[2 * i], h->prof_ev[2 * i + 1]));
    tot[h->prof_kind[i]] += ms;
    cnt[h->prof_kind[i]] += 1;
  }
  int n = 0;
  for (int kd = 0; kd < K_NUM && n < n_slots; ++kd) {
    if (!cnt[kd]) continue;
    std::snprintf(names + 32 * n, 32, "%s", kKindNames[kd]);
    total_ms[n] = tot[kd];
    launches[n] = cnt[kd];
    ++n;
  }
  *n_out = n;
  h->prof_used = 0;
  return NOOR_MOE_OK;
}

int64_t noor_moe_launch_count(const noor_moe_handle* h) { return h ? h->launches : 0; }

int noor_moe_utilization(noor_moe_handle* h, int64_t* counts, int64_t* tokens, int reset, void* stream) {
  if (!h) return fail(NOOR_MOE_ERR_INVALID, "null handle");
  DeviceGuard g(h->dev);
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->own;
  std::vector<int64_t> tmp(h->E + 1);
  CK(cudaMemcpyAsync(tmp.data(), h->util.p, (h->E + 1) * 8, cudaMemcpyDeviceToHost, s));
  if (reset) CK(cudaMemsetAsync(h->util.p, 0, (h->E + 1) * 8, s));
  CK(cudaEventRecord(h->ev_done, s));
  CKR(wait_event_deadline(h, h->ev_done, 300.0));
  if (counts) std::memcpy(counts, tmp.data(), h->E * 8);
  if (tokens) *tokens = tmp[h->E];
  return NOOR_MOE_OK;
}

int noor_moe_smebu_update(noor_moe_handle* h, float kappa, float beta, float lambda, void* stream) {
  if (!h) return fail(NOOR_MOE_ERR_INVALID, "null handle");
  if (!h->weights) return fail(NOOR_MOE_ERR_STATE, "smebu_update before load_weights");
  if (!(kappa > 0.0f)) return fail(NOOR_MOE_ERR_INVALID, "kappa must be positive");
  DeviceGuard g(h->dev);
  const bool host = stream == nullptr;
  cudaStream_t s = host ? h->own : static_cast<cudaStream_t>(stream);
  CKR(launch(h, s, K_SMEBU, [&] {
    smebu::smebu_update_kernel<<<1, std::max(32, (h->E + 31) / 32 * 32), 0, s>>>(
        h->util.as<int64_t>(), h->smebu_m.as<float>(), h->bias.as<float>(), h->E, kappa, beta, lambda);
  }));
  if (host) {
    CK(cudaEventRecord(h->ev_done, s));
    CKR(wait_event_deadline(h, h->ev_done, 300.0));
  }
  return NOOR_MOE_OK;
}

int noor_moe_smebu_momentum(noor_moe_handle* h, float* get, const float* set) {
  if (!h) return fail(NOOR_MOE_ERR_INVALID, "null handle");
  DeviceGuard g(h->dev);
  CK(cudaDeviceSynchronize());
  if (get) CK(cudaMemcpy(get, h->smebu_m.p, h->E * 4, cudaMemcpyDeviceToHost));
  if (set) CK(cudaMemcpy(h->smebu_m.p, set, h->E * 4, cudaMemcpyHostToDevice));
  return NOOR_MOE_OK;
}

int noor_moe_get_bias(noor_moe_handle* h, float* bias) {
  if (!h || !bias) return fail(NOOR_MOE_ERR_INVALID, "null argument");
  if (!h->weights) return fail(NOOR_MOE_ERR_STATE, "get_bias before load_weights");
  DeviceGuard g(h->dev);
  CK(cudaDeviceSynchronize());
  CK(cudaMemcpy(bias, h->bias.p, h->E * 4, cudaMemcpyDeviceToHost));
  return NOOR_MOE_OK;
}

int noor_moe_ep_transport(const noor_moe_handle* h) {
  if (!h) return -1;
  if (h->G == 1) return NOOR_MOE_EP_NONE;
  return h->peer ? NOOR_MOE_EP_PEER : NOOR_MOE_EP_NCCL;
}

}  // extern "C"

// ============================================================== routing without allocation
//
// noor_moe_route_static runs the router and the utilization histogram
// without a handle and without allocating: its working memory (per-pick
// ranks, per-block histograms and bases, the scan's tables and, for F32
// layers, the score matrix) lives in the file-scope device array below.  It is
// for callers that cannot call cudaMalloc: code recording a CUDA graph (an
// allocation is not allowed while a stream is being captured), and hosts that
// hand all device memory to their own pool up front and forbid allocation
// afterwards.  Every GPU that loads this library holds the array until exit.

static __device__ __align__(256) unsigned char g_route_scratch[NOOR_MOE_STATIC_SCRATCH_BYTES];

namespace {

std::mutex g_scratch_mu;
void* g_scratch_addr[256] = {nullptr};  // device address of g_route_scratch, per CUDA ordinal

// Looks up the array's device address once per device, with that device
// current.  In host code the name g_route_scratch is only a host-side stand-in,
// never a usable device address.  The address is kept for the life of the
// process: after cudaDeviceReset on a device the kept address no longer
// names the array, so a process that resets a device must not call
// noor_moe_route_static on it again.
int route_scratch_address(int dev, void** out) {
  if (dev < 0 || dev >= 256) return fail(NOOR_MOE_ERR_INVALID, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* ptr = nullptr;
    CK(cudaGetSymbolAddress(&ptr, g_route_scratch));
    g_scratch_addr[dev] = ptr;
  }
  *out = g_scratch_addr[dev];
  return NOOR_MOE_OK;
}

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

}  // namespace

extern "C" int noor_moe_route_static(const void* x, const void* gate, const float* bias, const float* scales,
                                     int64_t T, int32_t d, int32_t E, int32_t top_k, int32_t dtype,
                                     int32_t* idx, float* w, int64_t* counts, void* stream) {
  if (!x || !gate || !bias || !scales || !idx || !w || !counts)
    return fail(NOOR_MOE_ERR_INVALID, "null argument");
  if (dtype != NOOR_DTYPE_F32 && dtype != NOOR_DTYPE_BF16) return fail(NOOR_MOE_ERR_INVALID, "unknown dtype");
  if (T <= 0 || d <= 0 || E <= 0 || top_k <= 0) return fail(NOOR_MOE_ERR_INVALID, "sizes must be positive");
  const int k = std::min(top_k, E);
  if (k > router::kMaxTopK) return fail(NOOR_MOE_ERR_UNSUPPORTED, "top_k > %d", router::kMaxTopK);
  if (dtype == NOOR_DTYPE_BF16 && (E > router::kMaxExpertsTC || d % 128 != 0))
    return fail(NOOR_MOE_ERR_UNSUPPORTED, "BF16 routing needs E <= %d and d_model a multiple of 128",
                router::kMaxExpertsTC);
  if (dtype == NOOR_DTYPE_F32 && E > 256) return fail(NOOR_MOE_ERR_UNSUPPORTED, "at most 256 experts");
  if (T > INT32_MAX / k) return fail(NOOR_MOE_ERR_INVALID, "too many tokens");
  const int Epad = (E + 7) / 8 * 8;
  const int tpb = dtype == NOOR_DTYPE_BF16 ? router::kTcTPB : router::kTopkTPB;
  const int64_t nblk = (T + tpb - 1) / tpb;
  // carve the array: error word | ranks | block histograms | block bases | segment starts | tile starts |
  // [scores]
  const size_t off_err = 0;
  const size_t off_lrank = 256;
  const size_t off_hist = align256(off_lrank + (size_t)T * k * 4);
  const size_t off_base = align256(off_hist + (size_t)nblk * E * 4);
  const size_t off_seg = align256(off_base + (size_t)nblk * E * 4);
  const size_t off_mt = align256(off_seg + (size_t)(E + 1) * 4);
  const size_t off_scores = align256(off_mt + (size_t)(E + 1) * 4);
  const size_t need = off_scores + (dtype == NOOR_DTYPE_F32 ? (size_t)T * E * 4 : 0);
  if (need > (size_t)NOOR_MOE_STATIC_SCRATCH_BYTES)
    return fail(NOOR_MOE_ERR_INVALID,
                "noor_moe_route_static: %lld tokens x %d experts (top-%d) need %zu bytes of scratch, more than "
                "the fixed %d bytes; split the batch or use noor_moe_route",
                (long long)T, E, k, need, NOOR_MOE_STATIC_SCRATCH_BYTES);
  int dev = 0;
  CK(cudaGetDevice(&dev));
  void* base = nullptr;
  CKR(route_scratch_address(dev, &base));
  uint8_t* sb = static_cast<uint8_t*>(base);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The router records a bounded wait that gave up in the error word; the
  // scan then writes every count as -1.  The word starts each call at zero
  // (a memset allocates nothing).
  int* err = reinterpret_cast<int*>(sb + off_err);
  CK(cudaMemsetAsync(err, 0, sizeof(int), s));
  router::RouterOut ro{idx, w, reinterpret_cast<int32_t*>(sb + off_lrank), reinterpret_cast<int32_t*>(sb + off_hist)};
  float* scores = reinterpret_cast<float*>(sb + off_scores);
  const router::FusedScan nofs{nullptr, nullptr, nullptr, nullptr, nullptr, tc::BM, nullptr, nullptr, nullptr};
  if (dtype == NOOR_DTYPE_BF16) {
    // the same kernel as noor_moe_route, so the results are identical; the
    // tensor maps are encoded on the host for this call (no allocation)
    CUtensorMap tmx, tmg;
    CKR(encode_kmajor(&tmx, x, T, d, router::kTcTPB));
    CKR(encode_kmajor(&tmg, gate, Epad, d, router::tc_npad(E)));
    CKR(launch_route_tc(nullptr, s, tmx, tmg, bias, scales, T, d, E, k, ro, nofs, err));
  } else {
    const int64_t n = T * E;
    router::route_f32_scores_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
        static_cast<const float*>(x), static_cast<const float*>(gate), bias, (int32_t)T, d, E, scores);
    CK(cudaGetLastError());
    const size_t smem = router::topk_smem_bytes(E, k);
    if (smem > 48 * 1024)
      CK(cudaFuncSetAttribute(router::topk_from_scores_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    router::topk_from_scores_kernel<<<(unsigned)nblk, router::kTopkTPB, smem, s>>>(scores, scales, (int32_t)T, E, k,
                                                                                    ro, nofs);
  }
  CK(cudaGetLastError());
  dispatch::scan_segments_kernel<<<1, dispatch::kScanThreads, 0, s>>>(
      reinterpret_cast<const int32_t*>(sb + off_hist), (int32_t)nblk, E, tc::BM, counts,
      reinterpret_cast<int32_t*>(sb + off_seg), reinterpret_cast<int32_t*>(sb + off_base),
      reinterpret_cast<int32_t*>(sb + off_mt), err);
  CK(cudaGetLastError());
  return NOOR_MOE_OK;
}
