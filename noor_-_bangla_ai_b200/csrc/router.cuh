// router.cuh -- K1: sigmoid router + SMEBU bias + top-k + utilization histogram.
//
// Restates MoERouter::route (crates/noor-core/src/layers/moe.rs:79-107) for a
// whole batch of tokens, plus ExpertUtilization::record (moe.rs:40-45):
//   s_e = 1 / (1 + exp(-(sum_i x_i * gate[i, e] + bias_e)))
//   top-k by score, ties to the lower expert index (the reference's stable
//   descending sort), weight = s_e * scale_e (no renormalisation).
//
// Besides idx/w the router writes, for the permute step, the rank of every
// (token, slot) pick among the picks of the same expert inside its token
// block, and the block's per-expert histogram.  Picks are ordered
// (slot, token) inside a block, so the layout of the expert segments is
// deterministic.
//
// BF16 layers: router_tc.cuh (tcgen05 tensor cores, TMA-fed).
// F32 layers (below): each (token, expert) dot runs serially in the
// reference's order with separately rounded multiply and add, so scores match
// the reference bit for bit up to expf's last-place differences.
#pragma once

#include "common.cuh"
#include "dispatch.cuh"

namespace noor {
namespace router {

constexpr int kMaxTopK = 8;
constexpr int kMaxExpertsTC = 128;  // BF16 router: N = roundup(E, 16) <= 128 TMEM columns

// ------------------------------------------------------------------ ranking

// sel[slot * TPB + tok] holds the expert of each pick in the block (-1 for
// tokens past T).  Computes each pick's rank among the block's picks of the
// same expert in (slot, token) order and writes it to lrank_out[token*k +
// slot].  Then, per expert e with picks in the block, either
//   seg_acc == nullptr: the block histogram hist_out[e * hist_stride], for a
//                       later scan over all blocks (dispatch::scan_segments_*);
//   seg_acc != nullptr: the block claims its rows of expert e's segment with
//                       one atomicAdd on the running total seg_acc[e] and
//                       writes the first of them, relative to the segment
//                       start, to hist_out[e * hist_stride].
// The claim order between blocks varies from call to call, so the order of
// rows inside a segment does too; every row is computed on its own by the
// GEMMs and returns to its token through the row map, so the outputs do not
// depend on it.
__device__ void rank_block_picks(const int32_t* sel, int k, int TPB, int E, int T, int32_t tok_base,
                                 int32_t* chunk_cnt /* smem [nchunks][E] */,
                                 int32_t* intra /* smem [k*TPB] */, int32_t* lrank_out,
                                 int32_t* hist_out, int32_t hist_stride, int32_t* seg_acc = nullptr) {
  const int nchunks = (k * TPB + 31) / 32;  // sel is padded with -1 to whole warps
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  for (int i = threadIdx.x; i < nchunks * E; i += blockDim.x) chunk_cnt[i] = 0;
  __syncthreads();
  for (int c = warp; c < nchunks; c += nwarps) {
    const int a = c * 32 + lane;
    const int e = sel[a];
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int before = __popc(peers & ((1u << lane) - 1u));
    intra[a] = before;
    if (e >= 0 && before == 0) chunk_cnt[c * E + e] = __popc(peers);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int c = 0; c < nchunks; ++c) {
      const int v = chunk_cnt[c * E + e];
      chunk_cnt[c * E + e] = run;
      run += v;
    }
    if (seg_acc == nullptr) hist_out[(int64_t)e * hist_stride] = run;
    else if (run > 0) hist_out[(int64_t)e * hist_stride] = atomicAdd(seg_acc + e, run);
  }
  __syncthreads();
  for (int a = threadIdx.x; a < k * TPB; a += blockDim.x) {
    const int e = sel[a];
    if (e < 0) continue;
    const int slot = a / TPB, tok = a - slot * TPB;
    const int32_t t = tok_base + tok;
    lrank_out[(int64_t)t * k + slot] = chunk_cnt[(a >> 5) * E + e] + intra[a];
  }
}

// ------------------------------------------------------------------ outputs

struct RouterOut {
  int32_t* idx;      // [T, k]
  float* w;          // [T, k]
  int32_t* lrank;    // [T, k]
  int32_t* blk_hist; // [E, nblk], expert-major
};

// Segment tables built inside the router.  Every block claims its rows of
// each expert's segment from the running totals seg_acc (rank_block_picks),
// writing blk_base[e][block] relative to the segment start; the last block to
// finish turns the totals into the counts, the segment starts, the GEMM tile
// table and the utilization (finish_from_totals), and resets `done` and
// seg_acc to zero for the next call.
struct FusedScan {
  int* done;               // nullptr: no fused tables (the router writes block histograms)
  int64_t* counts;
  int32_t* seg_start;
  int32_t* blk_base;       // [E][nblk] first row of block b's picks of e, relative to seg_start[e]
  int32_t* mtile_start;
  int32_t BM;
  int64_t* util;           // nullable: utilization accumulator [E+1]
  int32_t* seg_acc;        // [E] running totals, zero between calls
  int* err;                // nullable: device error word (bounds checks of the debug build)
};

// The last router block: segment starts (exclusive prefix of the totals),
// counts, tile table and utilization; then the totals go back to zero.  All
// threads call it; s_warp: 32 ints, s_seg: E+1 ints (shared memory).
__device__ void finish_from_totals(const FusedScan& scan, int32_t E, int32_t k, int32_t T, int32_t* s_seg) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    int run = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int c = e < E ? __ldcg(scan.seg_acc + e) : 0;
      const int incl = dispatch::warp_inclusive_scan(c);
      if (e < E) s_seg[e] = run + incl - c;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      s_seg[E] = run;
      (void)in_bounds(run == T * k, scan.err);  // every token has exactly k picks
    }
  }
  __syncthreads();
  dispatch::finish_segments(E, scan.BM, s_seg, scan.counts, scan.seg_start, scan.mtile_start, scan.util, k);
  for (int e = threadIdx.x; e < E; e += blockDim.x) scan.seg_acc[e] = 0;
}

// ------------------------------------------------------------------ F32 router

// scores[t, e] = sigmoid(dot + bias), dot accumulated over i = 0..d-1 in order
// with separately rounded multiply and add (moe.rs:86-93).  One thread per
// (token, expert); threads of a warp share the token and read gate row-wise.
__global__ void route_f32_scores_kernel(const float* __restrict__ x, const float* __restrict__ gate,
                                        const float* __restrict__ bias, int32_t T, int32_t d, int32_t E,
                                        float* __restrict__ scores) {
  const int64_t gidx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gidx >= (int64_t)T * E) return;
  const int32_t t = (int32_t)(gidx / E);
  const int32_t e = (int32_t)(gidx - (int64_t)t * E);
  const float* xr = x + (int64_t)t * d;
  float dot = 0.0f;
  for (int32_t i = 0; i < d; ++i) dot = __fadd_rn(dot, __fmul_rn(__ldg(xr + i), __ldg(gate + (int64_t)i * E + e)));
  dot = __fadd_rn(dot, __ldg(bias + e));
  scores[gidx] = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-dot)));
}

// Top-k of precomputed scores, one thread per token, then block ranking (and,
// with `scan`, the segment scan in the last block).  The block's score tile
// is staged in shared memory with coalesced loads (rows padded by one float so
// each thread's row walk hits its own bank).  Dynamic shared memory:
// topk_smem_bytes(E, k).
constexpr int kTopkTPB = 128;

__host__ __device__ inline size_t topk_smem_bytes(int E, int k) {
  return (size_t)kTopkTPB * (E + 1) * 4 + (size_t)((k * kTopkTPB + 31) / 32) * E * 4;
}

__global__ void __launch_bounds__(kTopkTPB) topk_from_scores_kernel(const float* __restrict__ scores,
                                                                   const float* __restrict__ scales, int32_t T,
                                                                   int32_t E, int32_t k, RouterOut out,
                                                                   FusedScan scan) {
  __shared__ int32_t s_seg[257];
  __shared__ int s_last;
  __shared__ int32_t s_sel[kMaxTopK * kTopkTPB];
  __shared__ int32_t s_intra[kMaxTopK * kTopkTPB];
  extern __shared__ float s_dyn[];
  float* s_sc = s_dyn;                                                     // [TPB][E + 1]
  int32_t* s_cnt = reinterpret_cast<int32_t*>(s_dyn + kTopkTPB * (E + 1));  // [nchunks][E]
  const int32_t blk_tok0 = blockIdx.x * kTopkTPB;
  const int rows = min(kTopkTPB, T - blk_tok0);
  const float* src = scores + (int64_t)blk_tok0 * E;
  {
    // eight loads in flight per thread before their stores
    constexpr int U = 8;
    const int n = rows * E;
    for (int base = threadIdx.x; base < n; base += blockDim.x * U) {
      float v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = base + u * blockDim.x;
        if (i < n) v[u] = __ldg(src + i);
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int i = base + u * blockDim.x;
        if (i < n) {
          const int r = i / E;
          s_sc[r * (E + 1) + (i - r * E)] = v[u];
        }
      }
    }
  }
  __syncthreads();
  const int tok = threadIdx.x;
  const int32_t t = blk_tok0 + tok;
  if (t < T) {
    const float* sr = s_sc + tok * (E + 1);
    uint32_t taken[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // up to 256 experts
    for (int r = 0; r < k; ++r) {
      int best = -1;
      float bs = 0.f;
      for (int e = 0; e < E; ++e) {
        if (taken[e >> 5] & (1u << (e & 31))) continue;
        const float sv = sr[e];
        if (best < 0 || sv > bs) {  // strict: ties keep the lower index
          best = e;
          bs = sv;
        }
      }
      taken[best >> 5] |= 1u << (best & 31);
      s_sel[r * kTopkTPB + tok] = best;
      out.idx[(int64_t)t * k + r] = best;
      out.w[(int64_t)t * k + r] = __fmul_rn(bs, __ldg(scales + best));
    }
  } else {
    for (int r = 0; r < k; ++r) s_sel[r * kTopkTPB + tok] = -1;
  }
  __syncthreads();
  const bool fused = scan.done != nullptr;
  rank_block_picks(s_sel, k, kTopkTPB, E, T, blk_tok0, s_cnt, s_intra, out.lrank,
                   (fused ? scan.blk_base : out.blk_hist) + blockIdx.x, gridDim.x, fused ? scan.seg_acc : nullptr);
  if (!fused) return;
  __syncthreads();
  __threadfence();
  if (threadIdx.x == 0) s_last = atomicAdd(scan.done, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  finish_from_totals(scan, E, k, T, s_seg);
  if (threadIdx.x == 0) *scan.done = 0;
}

}  // namespace router
}  // namespace noor
