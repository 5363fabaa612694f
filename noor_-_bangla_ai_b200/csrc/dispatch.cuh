// dispatch.cuh -- segment scan, K2 permute (dispatch) and K4 gather-combine.
//
// The reference dispatches one token at a time (moe.rs:150-165): for every
// token it runs each selected expert on a 1-row tensor and accumulates
// out[s] += w_i * expert_i(x_s) in rank order.  Here the dispatch is a
// permutation: every (token, slot) pick gets a row in a buffer where the
// picks of each expert are contiguous, so the experts run as one grouped
// GEMM; the combine then gathers each token's k expert rows back in rank
// order and adds the dense branch (parallel_ffn.rs:30-36).
#pragma once

#include "common.cuh"

namespace noor {
namespace dispatch {

// ------------------------------------------------------------------ scan

constexpr int kScanThreads = 1024;

__device__ __forceinline__ int warp_inclusive_scan(int v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

// The per-expert tail of the scans below, with s_seg[0..E] holding the
// segment starts (shared memory): counts, segment starts, the BM-row tile
// starts (an exclusive warp scan) and the utilization, in parallel over the
// experts -- no serial chain of global loads.  All threads call it.
__device__ void finish_segments(int32_t E, int32_t BM, const int32_t* s_seg, int64_t* __restrict__ counts,
                                int32_t* __restrict__ seg_start, int32_t* __restrict__ mtile_start,
                                int64_t* __restrict__ util, int32_t k) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int c = s_seg[e + 1] - s_seg[e];
    counts[e] = c;
    seg_start[e] = s_seg[e];
    if (util) util[e] += c;
  }
  if (warp == 0) {
    int run = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int c = e < E ? s_seg[e + 1] - s_seg[e] : 0;
      const int t = (c + BM - 1) / BM;
      const int incl = warp_inclusive_scan(t);
      if (e < E) mtile_start[e] = run + incl - t;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      mtile_start[E] = run;
      seg_start[E] = s_seg[E];
      if (util) util[E] += s_seg[E] / k;
    }
  }
}

// From the per-token-block histograms, stored expert-major hist[E][nblk]:
//   blk_base[e][b]  = first row of block b's picks of expert e
//   seg_start[e]    = first row of expert e's segment, [E+1]
//   counts[e]       = picks of expert e (int64, the API's utilization counts)
//   mtile_start[e]  = first BM-row tile of expert e in the grouped GEMM, [E+1]
// Because the histograms are expert-major, blk_base is the exclusive prefix
// sum of the flattened array and seg_start[e] = blk_base[e][0].  Expert
// segments are laid out in expert order; under expert parallelism the experts
// of each rank are contiguous, so the rows bound for each rank are too.
// Runs in one thread block of any multiple of 32 threads (s_warp: 32 ints,
// s_seg: E+1 ints); hist is read through L2 (ld.cg), so a block may scan
// histograms that other blocks of the same grid have just written.
// util (nullable, [E+1]): the layer's utilization since its last reset,
// ExpertUtilization::record (moe.rs:40-45) for the whole batch: util[e] +=
// counts[e], util[E] += tokens (every token has exactly k picks).
__device__ void scan_segments_block(const int32_t* __restrict__ hist, int32_t nblk, int32_t E, int32_t BM,
                                    int64_t* __restrict__ counts, int32_t* __restrict__ seg_start,
                                    int32_t* __restrict__ blk_base, int32_t* __restrict__ mtile_start,
                                    int32_t* s_warp, int32_t* s_seg, int64_t* __restrict__ util = nullptr,
                                    int32_t k = 1) {
  const int N = E * nblk;
  const int nt = blockDim.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = nt >> 5;
  const int per = (N + nt - 1) / nt;
  const int i0 = min(N, (int)threadIdx.x * per), i1 = min(N, i0 + per);
  int sum = 0;
#pragma unroll 16
  for (int i = i0; i < i1; ++i) sum += __ldcg(hist + i);
  const int incl = warp_inclusive_scan(sum);
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int v = lane < nwarps ? s_warp[lane] : 0;
    const int vi = warp_inclusive_scan(v);
    if (lane < nwarps) s_warp[lane] = vi - v;
    if (lane == nwarps - 1) s_seg[E] = vi;  // total picks
  }
  __syncthreads();
  int run = s_warp[warp] + incl - sum;
#pragma unroll 16
  for (int i = i0; i < i1; ++i) {
    const int v = __ldcg(hist + i);
    blk_base[i] = run;
    run += v;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += nt) s_seg[e] = blk_base[(int64_t)e * nblk];
  __syncthreads();
  finish_segments(E, BM, s_seg, counts, seg_start, mtile_start, util, k);
}

// err (nullable): the router's device error word.  When it is set (a
// bounded wait in the router gave up, so some picks are placeholders), every
// count is written as -1 instead, so a caller without a handle sees the
// failure in the counts it reads anyway.
__global__ void __launch_bounds__(kScanThreads) scan_segments_kernel(const int32_t* __restrict__ hist, int32_t nblk,
                                                                     int32_t E, int32_t BM,
                                                                     int64_t* __restrict__ counts,
                                                                     int32_t* __restrict__ seg_start,
                                                                     int32_t* __restrict__ blk_base,
                                                                     int32_t* __restrict__ mtile_start,
                                                                     const int* __restrict__ err = nullptr) {
  __shared__ int32_t s_warp[32];
  __shared__ int32_t s_seg[1025];
  scan_segments_block(hist, nblk, E, BM, counts, seg_start, blk_base, mtile_start, s_warp, s_seg);
  if (err != nullptr) {
    __syncthreads();
    if (*reinterpret_cast<const volatile int*>(err) != 0)
      for (int e = threadIdx.x; e < E; e += blockDim.x) counts[e] = -1;
  }
}

// ------------------------------------------------------------------ permute

// Each warp takes tokens in a grid-stride loop: it reads the token's row once
// (up to 4 KB in one batch of 16-byte loads) and writes it to the row of each
// of its k picks -- seg_start[e] + blk_base[e][block] + lrank, the router's
// segment tables -- recording that row in dst_row[t, slot] and, when ymap is
// given, the inverse ymap[row] = t*k + slot (where the expert down
// projection puts that row's output: token-major, so the combine reads each
// token's k rows side by side).  Launched either with a block per 4 tokens,
// or persistent with one 4-warp block per SM (48 registers a thread) beside a
// tensor-core GEMM that holds the rest of each SM.
constexpr int kPermuteWarps = 4;

__global__ void __launch_bounds__(kPermuteWarps * 32) permute_rows_kernel(
    const uint8_t* __restrict__ x, int32_t row_bytes, int32_t T, int32_t k, int32_t nblk, int32_t tpb,
    const int32_t* __restrict__ idx, const int32_t* __restrict__ lrank, const int32_t* __restrict__ blk_base,
    const int32_t* __restrict__ seg_start, uint8_t* __restrict__ xp, int32_t* __restrict__ dst_row,
    int32_t* __restrict__ ymap, int64_t rows_cap, int* err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = row_bytes >> 4;
  constexpr int U = 8;
  for (int32_t t = blockIdx.x * kPermuteWarps + warp; t < T; t += gridDim.x * kPermuteWarps) {
    int32_t dst[8];
    const int32_t* bb = blk_base + t / tpb;  // blk_base[e][block] is bb[e * nblk]
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < k) {
        const int32_t e = __ldg(idx + (int64_t)t * k + i);
        dst[i] = __ldg(seg_start + e) + __ldg(bb + (int64_t)e * nblk) + __ldg(lrank + (int64_t)t * k + i);
        if (!in_bounds(e >= 0 && dst[i] >= 0 && dst[i] < rows_cap, lane == 0 ? err : nullptr)) dst[i] = -1;
        if (lane == 0) dst_row[(int64_t)t * k + i] = dst[i];
        if (lane == 1 && ymap != nullptr && dst[i] >= 0) ymap[dst[i]] = t * k + i;
      }
    }
    const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)t * row_bytes);
    for (int base = lane; base < nvec; base += 32 * U) {
      uint4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (base + 32 * u < nvec) v[u] = __ldg(src + base + 32 * u);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i < k && dst[i] >= 0) {
          uint4* d = reinterpret_cast<uint4*>(xp + (int64_t)dst[i] * row_bytes);
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (base + 32 * u < nvec) d[base + 32 * u] = v[u];
        }
      }
    }
  }
}

// ------------------------------------------------------------------ combine

// out[t] = (dense[t] + sum_i w[t,i] * y[dst_row[t,i]] (+ shared[t])) * 1/sqrt(2)
// with the sum taken in rank order starting from zero and every multiply and
// add rounded separately (moe.rs:159-173, parallel_ffn.rs:32-35).  Without a
// dense branch the result is the MoE sum alone (MoELayer::forward).
// YT / OUT: bf16 or float.  dense and shared are f32 (nullable).  dst_row
// null: y is token-major, pick (t, i) at row t*k + i.
template <typename T_>
struct Vec8;
template <>
struct Vec8<bf16> {
  __device__ static void load(const bf16* p, float (&v)[8]) {
    const uint4 r = *reinterpret_cast<const uint4*>(p);
    v[0] = bf16_lo(r.x); v[1] = bf16_hi(r.x); v[2] = bf16_lo(r.y); v[3] = bf16_hi(r.y);
    v[4] = bf16_lo(r.z); v[5] = bf16_hi(r.z); v[6] = bf16_lo(r.w); v[7] = bf16_hi(r.w);
  }
  __device__ static void store(bf16* p, const float (&v)[8]) {
    *reinterpret_cast<uint4*>(p) =
        make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
  }
};
template <>
struct Vec8<float> {
  __device__ static void load(const float* p, float (&v)[8]) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  }
  __device__ static void store(float* p, const float (&v)[8]) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
};

constexpr int kCombineWarps = 8;

template <typename YT, typename OT>
__global__ void __launch_bounds__(kCombineWarps * 32) combine_kernel(
    const YT* __restrict__ y, const int32_t* __restrict__ dst_row, const float* __restrict__ wts,
    const float* __restrict__ dense, const float* __restrict__ shared, int32_t T, int32_t d, int32_t k,
    OT* __restrict__ out, int64_t y_rows, int* err) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int32_t t = blockIdx.x * kCombineWarps + warp;
  if (t >= T) return;
  int32_t rows[8];
  float w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < k) {
      rows[i] = dst_row != nullptr ? __ldg(dst_row + (int64_t)t * k + i) : t * k + i;
      if (!in_bounds(rows[i] >= 0 && rows[i] < y_rows, lane == 0 ? err : nullptr)) rows[i] = -1;
      w[i] = __ldg(wts + (int64_t)t * k + i);
    }
  const float inv_sqrt2 = 0x1.6a09e6p-1f;  // 1.0f32 / 2.0f32.sqrt() = 0.70710677
  for (int c = lane * 8; c < d; c += 32 * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < k && rows[i] >= 0) {
        float v[8];
        Vec8<YT>::load(y + (int64_t)rows[i] * d + c, v);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = __fadd_rn(acc[j], __fmul_rn(w[i], v[j]));
      }
    }
    if (shared) {
      float v[8];
      Vec8<float>::load(shared + (int64_t)t * d + c, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = __fadd_rn(acc[j], v[j]);
    }
    if (dense) {
      float v[8];
      Vec8<float>::load(dense + (int64_t)t * d + c, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = __fmul_rn(__fadd_rn(v[j], acc[j]), inv_sqrt2);
    }
    Vec8<OT>::store(out + (int64_t)t * d + c, acc);
  }
}

}  // namespace dispatch
}  // namespace noor
