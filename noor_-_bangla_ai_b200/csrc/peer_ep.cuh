// peer_ep.cuh -- expert-parallel exchange over NVLink peer memory.
//
// Under expert parallelism rank r owns experts [r*El, (r+1)*El).  Instead of
// staging rows for an all-to-all, every rank maps the other ranks' receive
// buffers into its address space (CUDA IPC) and the kernels move the rows
// themselves:
//   plan     each rank stores its per-expert pick counts into every rank's
//            sync area, signals, waits for all ranks, then builds from the
//            full count matrix (identical on every rank) its receive group
//            table and the receive-row bases of its own picks;
//   permute  writes each picked row once, straight into the owner's receive
//            buffer (a local store or an NVLink store);
//   barrier  every rank's rows have landed;
//   GEMMs    the expert down projection's epilogue stores each output row
//            straight back into the buffer of the rank that sent the row, at
//            the token-major row t*k + slot the sender recorded beside the
//            row (the single-GPU layout of y);
//   barrier  every rank's outputs have landed; the combine gathers locally.
// Nothing waits on the host, so a whole layer step can be recorded in a CUDA
// graph.  Every wait is bounded; a rank that gives up writes an error code
// and marks the exchange failed, and the kernels after it skip their stores.
#pragma once

#include "common.cuh"

namespace noor {
namespace peer {

constexpr int kMaxRanks = 8;

// Each rank's peer-visible sync area:
//   bytes [0, 64)       uint64 flag[src]: last barrier number rank src reached
//   bytes [256, ...)    int64 cnt_all[src][E]: rank src's picks per expert
constexpr int kCountsOff = 256;

constexpr int STATUS_OK = 0;
constexpr int STATUS_PEER_INVALID = 1;  // a rank published an over-capacity batch
constexpr int STATUS_OVERFLOW = 2;      // a rank would receive more rows than its buffer holds
constexpr int STATUS_TIMEOUT = 3;       // a barrier gave up waiting

struct Peers {
  uint8_t* sync[kMaxRanks];   // every rank's sync area, as mapped in this process
  uint8_t* xrecv[kMaxRanks];  // every rank's receive buffer (rows of row_bytes)
  int32_t* rowmap[kMaxRanks]; // every rank's receive row map: for receive row j, the
                              // sender's token-major output row t*k + slot
  int32_t G;
  int32_t me;
  int64_t timeout_ns;         // bound of every wait on another rank
};

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Barrier number `seq` across the ranks, run by one full warp: lane r signals
// rank r (after a system-scope fence, so every store this rank made before
// is visible to whoever sees the signal), then waits, bounded, until rank r
// has signalled this rank.  Returns false on every lane if any wait gave up.
__device__ bool barrier_warp(const Peers& P, uint64_t seq) {
  const int lane = threadIdx.x & 31;
  __threadfence_system();
  if (lane < P.G) st_release_sys(reinterpret_cast<uint64_t*>(P.sync[lane]) + P.me, seq);
  bool ok = true;
  if (lane < P.G) {
    const uint64_t* f = reinterpret_cast<const uint64_t*>(P.sync[P.me]) + lane;
    const uint64_t t0 = global_ns();
    while (ld_acquire_sys(f) < seq) {
      if ((int64_t)(global_ns() - t0) > P.timeout_ns) {
        ok = false;
        break;
      }
    }
  }
  return __all_sync(0xffffffffu, ok);
}

// ---- the plan's arithmetic, shared by plan_kernel and the host-side
// noor_moe_peer_plan (so that it can be checked for any rank count on the
// CPU).  cnt[src * E + e]: picks of expert e made on rank src; pre[src *
// pre_ld + e]: sum of cnt[src][e' < e] (rank src keeps its picks of e from
// row pre[src][e] of its own layout, the single-GPU one).

struct PlanView {
  const int64_t* cnt;
  const int32_t* pre;
  int32_t pre_ld;
  int32_t G, E, El, me;
};

// Receive group j of this rank: (local expert le, source rank src) =
// (j / G, j % G).  Ordering the groups expert-major interleaves rows that
// return to other ranks with rows that stay here, so the GEMMs, which walk the
// tiles in order, keep NVLink busy for the whole down projection.
__host__ __device__ inline void plan_group(const PlanView& v, int j, int* src, int* le, int* e) {
  *le = j / v.G;
  *src = j - *le * v.G;
  *e = v.me * v.El + *le;
}

// First row, on expert e's owner r, of this rank's picks of e: the rows of
// the owner's groups before (le, me), i.e. experts r*El .. e-1 from every
// rank, then expert e from the ranks before this one.
__host__ __device__ inline int32_t plan_dest_base(const PlanView& v, int e) {
  const int r = e / v.El;
  int32_t base = 0;
  for (int src = 0; src < v.G; ++src) {
    base += v.pre[src * v.pre_ld + e] - v.pre[src * v.pre_ld + r * v.El];
    if (src < v.me) base += (int32_t)v.cnt[src * v.E + e];
  }
  return base;
}

// The receive group table: first row, first BM-row tile, local expert,
// source rank and output row shift of each group, [E+1] / [E] entries.
__host__ __device__ inline void plan_recv_table(const PlanView& v, int BM, int32_t* grp_row, int32_t* grp_mtile,
                                                int32_t* grp_widx, int32_t* grp_orank, int32_t* grp_oshift) {
  int32_t row = 0, tiles = 0;
  for (int j = 0; j < v.E; ++j) {
    int src, le, e;
    plan_group(v, j, &src, &le, &e);
    const int32_t c = (int32_t)v.cnt[src * v.E + e];
    grp_row[j] = row;
    grp_mtile[j] = tiles;
    grp_widx[j] = le;
    grp_orank[j] = src;
    grp_oshift[j] = v.pre[src * v.pre_ld + e] - row;  // back to row pre[src][e] on rank src
    row += c;
    tiles += (c + BM - 1) / BM;
  }
  grp_row[v.E] = row;
  grp_mtile[v.E] = tiles;
}

struct PlanOut {
  int32_t* grp_row;     // [E+1] receive group j = le*G + src: first row in xrecv
  int32_t* grp_mtile;   // [E+1] first BM-row tile of group j
  int32_t* grp_widx;    // [E]   local expert of group j
  int32_t* grp_orank;   // [E]   rank that sent group j's rows (its outputs go back there)
  int32_t* grp_oshift;  // [E]   output row on that rank minus the row in xrecv
  int32_t* dest_base;   // [E]   first row, on expert e's owner, of this rank's picks of e
  int64_t* counts_glob; // [E]   picks of expert e over all ranks
  int* status;          // STATUS_*
  uint64_t* seq;        // barrier counter of this rank
  int* err;             // device error word
  int64_t* util;        // nullable: utilization accumulator [E+1] (global counts, tokens)
  int32_t k;            // picks per token
};

constexpr int kPlanThreads = 256;

// One block.  counts: this rank's picks per expert (ignored when poison is
// set: the rank publishes -1 so that every rank skips this step).
// cap_rows: rows every rank's receive buffer holds (the same on all ranks).
__global__ void __launch_bounds__(kPlanThreads) plan_kernel(Peers P, const int64_t* __restrict__ counts, int32_t E,
                                                            int32_t El, int32_t BM, int64_t cap_rows, int32_t poison,
                                                            PlanOut o) {
  __shared__ int64_t s_cnt[kMaxRanks * 128];
  __shared__ int32_t s_pre[kMaxRanks][129];  // s_pre[src][e] = sum of cnt[src][e' < e]
  __shared__ int s_status;
  const int G = P.G, me = P.me;
  const int tid = threadIdx.x;
  // 1. publish this rank's counts in every rank's sync area
  for (int i = tid; i < G * E; i += blockDim.x) {
    const int r = i / E, e = i - r * E;
    const int64_t c = poison ? -1 : counts[e];
    reinterpret_cast<int64_t*>(P.sync[r] + kCountsOff)[me * E + e] = c;
  }
  __threadfence_system();
  __syncthreads();
  // 2. barrier
  if (tid < 32) {
    const uint64_t seq = *o.seq + 1;
    const bool ok = barrier_warp(P, seq);
    if (tid == 0) {
      *o.seq = seq;
      s_status = ok ? STATUS_OK : STATUS_TIMEOUT;
    }
  }
  __syncthreads();
  int status = s_status;
  // 3. read the full count matrix
  if (status == STATUS_OK) {
    const int64_t* all = reinterpret_cast<const int64_t*>(P.sync[me] + kCountsOff);
    for (int i = tid; i < G * E; i += blockDim.x) s_cnt[i] = __ldcv(all + i);
  }
  __syncthreads();
  if (status == STATUS_OK) {
    if (tid < G) {
      int32_t run = 0;
      bool bad = false;
      for (int e = 0; e < E; ++e) {
        s_pre[tid][e] = run;
        const int64_t c = s_cnt[tid * E + e];
        bad |= c < 0;
        run += c > 0 ? (int32_t)c : 0;
      }
      s_pre[tid][E] = run;
      if (bad) atomicMax(&s_status, STATUS_PEER_INVALID);
    }
    __syncthreads();
    // rows each rank would receive; every rank checks every rank, so all agree
    if (tid < G && s_status == STATUS_OK) {
      int64_t rows = 0;
      for (int src = 0; src < G; ++src) rows += s_pre[src][(tid + 1) * El] - s_pre[src][tid * El];
      if (rows > cap_rows) atomicMax(&s_status, STATUS_OVERFLOW);
    }
    __syncthreads();
    status = s_status;
  }
  if (status != STATUS_OK) {
    // an empty plan: the GEMMs find no tiles, the permute stores nothing
    for (int j = tid; j <= E; j += blockDim.x) {
      o.grp_row[j] = 0;
      o.grp_mtile[j] = 0;
      if (j < E) {
        o.grp_widx[j] = 0;
        o.grp_orank[j] = 0;
        o.grp_oshift[j] = 0;
        o.dest_base[j] = 0;
        o.counts_glob[j] = 0;
      }
    }
    if (tid == 0) {
      *o.status = status;
      atomicExch(o.err, status == STATUS_TIMEOUT ? DEV_TIMEOUT_PEER : DEV_PEER_PLAN);
    }
    return;
  }
  // 4. receive groups of this rank (plan_group order)
  const PlanView pv{s_cnt, &s_pre[0][0], 129, G, E, El, me};
  if (tid == 0) plan_recv_table(pv, BM, o.grp_row, o.grp_mtile, o.grp_widx, o.grp_orank, o.grp_oshift);
  // 5. where this rank's picks of each expert land on the expert's owner, and
  //    the global utilization counts
  for (int e = tid; e < E; e += blockDim.x) {
    int64_t tot = 0;
    for (int src = 0; src < G; ++src) tot += s_cnt[src * E + e];
    o.dest_base[e] = plan_dest_base(pv, e);
    o.counts_glob[e] = tot;
    if (o.util) o.util[e] += tot;
  }
  if (tid == 0) {
    if (o.util) {
      int64_t picks = 0;
      for (int src = 0; src < G; ++src) picks += s_pre[src][E];
      o.util[E] += picks / o.k;  // every token has exactly k picks
    }
    *o.status = STATUS_OK;
  }
}

// A barrier as its own launch (one warp).  Skipped, on every rank alike, when
// the step's plan failed.
__global__ void __launch_bounds__(32) barrier_kernel(Peers P, uint64_t* seq, int* status, int* err) {
  if (*status != STATUS_OK) return;
  const uint64_t s = *seq + 1;
  const bool ok = barrier_warp(P, s);
  if (threadIdx.x == 0) {
    *seq = s;
    if (!ok) {
      *status = STATUS_TIMEOUT;
      atomicExch(err, DEV_TIMEOUT_PEER);
    }
  }
}

// Dispatch under expert parallelism: each warp reads a token's row once
// (4 KB for d = 2048 in one batch of loads) and writes it to each pick's row
// in the receive buffer of the expert's owner.  dst_row[t, slot] is the pick's
// row in this rank's own (single-GPU) layout, where the owner returns the
// expert's output row.  The grid is persistent and small (one 4-warp block
// per SM, 48 registers a thread) so that it runs beside a tensor-core GEMM
// that holds the rest of each SM and its NVLink stores overlap that GEMM.
// part: PERMUTE_ALL, or one of two passes that together do the same work --
// PERMUTE_LOCAL (rows whose expert lives on this rank, plus every dst_row)
// and PERMUTE_REMOTE (rows bound for other ranks, over NVLink), which can run
// on different streams.
constexpr int kPermuteWarps = 4;       // in line: 4-warp blocks over the whole GPU
constexpr int kPermuteWarpsSide = 16;  // beside a GEMM: one 16-warp block per SM it is given
enum PermutePart : int { PERMUTE_ALL = 0, PERMUTE_LOCAL = 1, PERMUTE_REMOTE = 2 };

template <int W>
__global__ void __launch_bounds__(W * 32) permute_peer_kernel(
    const uint8_t* __restrict__ x, int32_t row_bytes, int32_t T, int32_t k, int32_t nblk, int32_t tpb,
    const int32_t* __restrict__ idx, const int32_t* __restrict__ lrank, const int32_t* __restrict__ blk_base,
    const int32_t* __restrict__ seg_start, const int32_t* __restrict__ dest_base, int32_t El, Peers P,
    const int* __restrict__ status, int32_t* __restrict__ dst_row, int32_t part, int64_t cap_rows, int* err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool store = *status == STATUS_OK;
  const int nvec = row_bytes >> 4;
  constexpr int U = 8;
  for (int32_t t = blockIdx.x * W + warp; t < T; t += gridDim.x * W) {
    uint8_t* dst[8];
    const int32_t* bb = blk_base + t / tpb;  // blk_base[e][block] is bb[e * nblk]
    bool any = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      dst[i] = nullptr;
      if (i < k) {
        const int32_t e = __ldg(idx + (int64_t)t * k + i);
        const int32_t in_seg = __ldg(bb + (int64_t)e * nblk) + __ldg(lrank + (int64_t)t * k + i);
        const int32_t local = __ldg(seg_start + e) + in_seg;
        if (lane == 0 && part != PERMUTE_REMOTE) dst_row[(int64_t)t * k + i] = local;
        const int32_t r = e / El;
        const bool mine = part == PERMUTE_ALL || ((r == P.me) == (part == PERMUTE_LOCAL));
        if (mine) {
          const int32_t remote = __ldg(dest_base + e) + in_seg;
          if (in_bounds(r >= 0 && r < P.G && remote >= 0 && remote < cap_rows, lane == 0 ? err : nullptr)) {
            dst[i] = P.xrecv[r] + (int64_t)remote * row_bytes;
            if (lane == 1 && store) P.rowmap[r][remote] = t * k + i;
            any = true;
          }
        }
      }
    }
    if (!store || !any) continue;
    const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)t * row_bytes);
    for (int base = lane; base < nvec; base += 32 * U) {
      uint4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (base + 32 * u < nvec) v[u] = __ldg(src + base + 32 * u);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i < k && dst[i] != nullptr) {
          uint4* d = reinterpret_cast<uint4*>(dst[i]);
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (base + 32 * u < nvec) d[base + 32 * u] = v[u];
        }
      }
    }
  }
  __threadfence_system();  // the rows are visible on their owners before the next barrier signals
}

// ---- the dispatch with bulk copies (TMA engine) instead of thread loads and
// stores: one warp per block; lane 0 moves whole rows through a ring of row
// slots in shared memory -- one bulk load per token, one bulk store per pick
// straight into the owner's receive buffer -- while lanes 0..k-1 compute the
// picks' rows and write the row maps.  Because the copy engine moves the
// bytes, a few SMs keep NVLink busy, and the kernel can run on SMs that a GEMM
// leaves free (it asks for the ring's shared memory, which keeps GEMM CTAs
// off its SMs).  Same results as permute_peer_kernel (PERMUTE_ALL).

__device__ __forceinline__ uint32_t bulk_smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Global -> shared, completing `bytes` on the barrier.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   bulk_smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(bulk_smem_addr(bar))
               : "memory");
}

// Shared -> global (this GPU's memory or a peer's), tracked by bulk groups.
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(bulk_smem_addr(src)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Every bulk group but the newest n (0 <= n <= 16) has finished reading
// shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read_c() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_read(int n) {
  switch (n) {
    case 0: bulk_wait_read_c<0>(); break;
    case 1: bulk_wait_read_c<1>(); break;
    case 2: bulk_wait_read_c<2>(); break;
    case 3: bulk_wait_read_c<3>(); break;
    case 4: bulk_wait_read_c<4>(); break;
    case 5: bulk_wait_read_c<5>(); break;
    case 6: bulk_wait_read_c<6>(); break;
    case 7: bulk_wait_read_c<7>(); break;
    case 8: bulk_wait_read_c<8>(); break;
    case 9: bulk_wait_read_c<9>(); break;
    case 10: bulk_wait_read_c<10>(); break;
    case 11: bulk_wait_read_c<11>(); break;
    case 12: bulk_wait_read_c<12>(); break;
    case 13: bulk_wait_read_c<13>(); break;
    case 14: bulk_wait_read_c<14>(); break;
    case 15: bulk_wait_read_c<15>(); break;
    default: bulk_wait_read_c<16>(); break;
  }
}

// Every bulk group has completed (its writes are performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

constexpr int kBulkSlotsMax = 32;

__global__ void __launch_bounds__(32) permute_peer_bulk_kernel(
    const uint8_t* __restrict__ x, int32_t row_bytes, int32_t T, int32_t k, int32_t nblk, int32_t tpb,
    const int32_t* __restrict__ idx, const int32_t* __restrict__ lrank, const int32_t* __restrict__ blk_base,
    const int32_t* __restrict__ seg_start, const int32_t* __restrict__ dest_base, int32_t El, Peers P,
    const int* __restrict__ status, int32_t* __restrict__ dst_row, int64_t cap_rows, int32_t nslots, int* err) {
  extern __shared__ __align__(128) uint8_t ring[];  // nslots rows
  __shared__ __align__(8) uint64_t full[kBulkSlotsMax];
  const int lane = threadIdx.x;
  const bool store = *status == STATUS_OK;
  const int32_t first = blockIdx.x;
  const int32_t n = first < T ? (T - 1 - first) / (int32_t)gridDim.x + 1 : 0;  // tokens of this block
  if (lane == 0) {
    for (int i = 0; i < nslots; ++i)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bulk_smem_addr(&full[i])) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  const int pending = nslots / 2 < 16 ? (nslots / 2 > 1 ? nslots / 2 : 1) : 16;  // store groups in flight
  int32_t issued = 0;  // tokens whose load lane 0 has issued
  auto load = [&](int32_t j) {  // token j of this block into slot j % nslots (lane 0)
    issued = j + 1;
    const int slot = j % nslots;
    const int32_t t = first + j * (int32_t)gridDim.x;
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bulk_smem_addr(&full[slot])),
                 "r"((uint32_t)row_bytes)
                 : "memory");
    bulk_load(ring + (int64_t)slot * row_bytes, x + (int64_t)t * row_bytes, (uint32_t)row_bytes, &full[slot]);
  };
  // lane 0: wait, bounded, until token j's row is in its slot
  auto wait_row = [&](int32_t j) -> bool {
    const uint32_t bar = bulk_smem_addr(&full[j % nslots]);
    const uint32_t parity = (uint32_t)((j / nslots) & 1);
    const uint64_t t0 = global_ns();
    uint32_t done = 0;
    while (!done) {
      asm volatile(
          "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
          : "=r"(done)
          : "r"(bar), "r"(parity)
          : "memory");
      if (!done && (int64_t)(global_ns() - t0) > P.timeout_ns) break;
    }
    return done != 0;
  };
  if (lane == 0 && store)
    for (int32_t j = 0; j < n && j < nslots; ++j) load(j);
  bool ok = true;
  int32_t waited = 0;  // tokens whose row lane 0 has seen arrive
  for (int32_t j = 0; j < n; ++j) {
    const int32_t t = first + j * (int32_t)gridDim.x;
    // lane i < k: pick i of token t -- its row here (dst_row), and where it
    // goes on the expert's owner (the owner's row map records t*k + i)
    uint8_t* dst = nullptr;
    if (lane < k) {
      const int32_t e = __ldg(idx + (int64_t)t * k + lane);
      const int32_t in_seg = __ldg(blk_base + (int64_t)e * nblk + t / tpb) + __ldg(lrank + (int64_t)t * k + lane);
      dst_row[(int64_t)t * k + lane] = __ldg(seg_start + e) + in_seg;
      const int32_t r = e / El;
      const int32_t remote = __ldg(dest_base + e) + in_seg;
      if (store && in_bounds(r >= 0 && r < P.G && remote >= 0 && remote < cap_rows, err)) {
        dst = P.xrecv[r] + (int64_t)remote * row_bytes;
        P.rowmap[r][remote] = t * k + lane;
      }
    }
    if (!store || !ok) continue;
    if (lane == 0) {
      if (wait_row(j)) {
        waited = j + 1;
      } else {
        atomicCAS(err, 0, DEV_TIMEOUT_PRODUCER);
        ok = false;
      }
    }
    ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
    if (!ok) continue;
    // lane 0 stores the row once per pick, reading each pick's target from its lane
    for (int i = 0; i < k; ++i) {
      uint8_t* d = reinterpret_cast<uint8_t*>(__shfl_sync(0xffffffffu, reinterpret_cast<uintptr_t>(dst), i));
      if (lane == 0 && d != nullptr) bulk_store(d, ring + (int64_t)(j % nslots) * row_bytes, (uint32_t)row_bytes);
    }
    if (lane == 0) {
      bulk_commit();
      // half the ring holds rows whose stores are in flight, the other half
      // rows being loaded: the slot of token f = j - pending + 1 is free once
      // its stores have read it (at most pending - 1 newer groups still
      // reading); it takes token f + nslots
      const int32_t f = j - pending + 1;
      if (f >= 0 && f + nslots < n) {
        bulk_wait_read(pending - 1);
        load(f + nslots);
      }
    }
    __syncwarp();
  }
  if (lane == 0) {
    // after a wait gave up, let the loads still in flight land (bounded)
    // before the block's shared memory is released
    for (int32_t j = waited; j < issued; ++j) (void)wait_row(j);
    bulk_wait_all();
    asm volatile("fence.proxy.async.global;" ::: "memory");  // the copies' writes before generic-proxy signals
  }
  __syncwarp();
  __threadfence_system();  // the rows are visible on their owners before the next barrier signals
}

}  // namespace peer
}  // namespace noor
