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
// BF16 layers: the dot products run on the tensor cores with mma.sync
// m16n8k16 (bf16 in, f32 accumulate); the router is bound by reading x from
// HBM, and the CUDA cores alone would make it compute-bound (E flops/byte).
// F32 layers: each (token, expert) dot runs serially in the reference's
// order with separately rounded multiply and add, so scores match the
// reference bit for bit up to expf's last-place differences.
#pragma once

#include "common.cuh"

namespace noor {
namespace router {

constexpr int kMaxTopK = 8;
constexpr int kMaxExpertsTC = 128;  // tensor-core router: up to 16 n-fragments

// ------------------------------------------------------------------ ranking

// sel[slot * TPB + tok] holds the expert of each pick in the block (-1 for
// tokens past T).  Computes each pick's rank among the block's picks of the
// same expert in (slot, token) order, writes it to lrank_out[token*k + slot],
// and writes the block histogram hist[E].
template <int TPB>
__device__ void rank_block_picks(const int32_t* sel, int k, int E, int T, int32_t tok_base,
                                 int32_t* chunk_cnt /* smem [nchunks][E] */,
                                 int32_t* intra /* smem [k*TPB] */, int32_t* lrank_out,
                                 int32_t* hist_out) {
  const int nchunks = k * TPB / 32;
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
    hist_out[e] = run;
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

// ------------------------------------------------------------------ BF16 router

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

struct RouterOut {
  int32_t* idx;      // [T, k]
  float* w;          // [T, k]
  int32_t* lrank;    // [T, k]
  int32_t* blk_hist; // [nblk, E]
};

// One warp routes 16*MF tokens; a block of 4 warps routes TPB = 64*MF tokens.
// gate_t is the router gate transposed to [NF*8, d] bf16 (rows >= E are zero).
// Each lane loads two 16-byte pieces of a row per 64-wide k-chunk (elements
// 8*t4 .. +7 and 32 + 8*t4 .. +7); the four k16 MMAs of a chunk consume them
// in an order that both A and B fragments follow, so the sum covers every k
// exactly once.
template <int NF, int MF>
__global__ void __launch_bounds__(128) route_bf16_kernel(const bf16* __restrict__ x, const bf16* __restrict__ gate_t,
                                                         const float* __restrict__ bias,
                                                         const float* __restrict__ scales, int32_t T, int32_t d,
                                                         int32_t E, int32_t k, RouterOut out) {
  constexpr int TPB = 64 * MF;
  __shared__ int32_t s_sel[kMaxTopK * TPB];
  __shared__ int32_t s_intra[kMaxTopK * TPB];
  __shared__ int32_t s_cnt[(kMaxTopK * TPB / 32) * kMaxExpertsTC];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, t4 = lane & 3;
  const int32_t blk_tok0 = blockIdx.x * TPB;
  const int32_t tok0 = blk_tok0 + warp * 16 * MF;

  float acc[MF][NF][4];
#pragma unroll
  for (int m = 0; m < MF; ++m)
#pragma unroll
    for (int n = 0; n < NF; ++n)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[m][n][j] = 0.f;

  const bf16* xrow[MF][2];
  bool rvalid[MF][2];
#pragma unroll
  for (int m = 0; m < MF; ++m)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int32_t r = tok0 + m * 16 + gid + 8 * h;
      rvalid[m][h] = r < T;
      xrow[m][h] = x + (int64_t)(rvalid[m][h] ? r : 0) * d;
    }
  const bf16* grow[NF];
#pragma unroll
  for (int n = 0; n < NF; ++n) grow[n] = gate_t + (int64_t)(n * 8 + gid) * d;

  for (int32_t kc = 0; kc < d; kc += 64) {
    uint4 a[MF][2][2];
#pragma unroll
    for (int m = 0; m < MF; ++m)
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int c = 0; c < 2; ++c)
          a[m][h][c] = rvalid[m][h] ? ldg_nc_v4(xrow[m][h] + kc + 32 * c + 8 * t4) : make_uint4(0, 0, 0, 0);
    uint4 b[NF][2];
#pragma unroll
    for (int n = 0; n < NF; ++n)
#pragma unroll
      for (int c = 0; c < 2; ++c) b[n][c] = __ldg(reinterpret_cast<const uint4*>(grow[n] + kc + 32 * c + 8 * t4));
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int c = q >> 1;
      const bool hi = q & 1;
#pragma unroll
      for (int m = 0; m < MF; ++m) {
        const uint32_t a0 = hi ? a[m][0][c].z : a[m][0][c].x;
        const uint32_t a2 = hi ? a[m][0][c].w : a[m][0][c].y;
        const uint32_t a1 = hi ? a[m][1][c].z : a[m][1][c].x;
        const uint32_t a3 = hi ? a[m][1][c].w : a[m][1][c].y;
#pragma unroll
        for (int n = 0; n < NF; ++n) {
          const uint32_t b0 = hi ? b[n][c].z : b[n][c].x;
          const uint32_t b1 = hi ? b[n][c].w : b[n][c].y;
          mma_bf16_16816(acc[m][n], a0, a1, a2, a3, b0, b1);
        }
      }
    }
  }

  // Scores and top-k.  Row (m, h) of this quad: lane holds experts
  // n*8 + 2*t4 + j (j = 0, 1) in acc[m][n][2h + j].  Keys order by score
  // (non-negative f32 bits are monotone) then by lower expert index.
#pragma unroll
  for (int m = 0; m < MF; ++m) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      unsigned long long key[2 * NF];
#pragma unroll
      for (int n = 0; n < NF; ++n)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int e = n * 8 + 2 * t4 + j;
          unsigned long long kv = 0ull;
          if (e < E) {
            const float dot = __fadd_rn(acc[m][n][2 * h + j], __ldg(bias + e));
            const float s = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-dot)));
            kv = ((unsigned long long)__float_as_uint(s) << 32) | (unsigned long long)(0xFFFFu - (unsigned)e);
          }
          key[2 * n + j] = kv;
        }
      const int tok_in_blk = warp * 16 * MF + m * 16 + gid + 8 * h;
      const int32_t t = blk_tok0 + tok_in_blk;
      for (int r = 0; r < k; ++r) {
        unsigned long long best = 0ull;
#pragma unroll
        for (int i = 0; i < 2 * NF; ++i) best = key[i] > best ? key[i] : best;
        unsigned long long o = __shfl_xor_sync(0xffffffffu, best, 1);
        best = o > best ? o : best;
        o = __shfl_xor_sync(0xffffffffu, best, 2);
        best = o > best ? o : best;
#pragma unroll
        for (int i = 0; i < 2 * NF; ++i)
          if (key[i] == best) key[i] = 0ull;
        const int e = (int)(0xFFFFu - (unsigned)(best & 0xFFFFFFFFull));
        if (t4 == 0) {
          const bool live = t < T;
          s_sel[r * TPB + tok_in_blk] = live ? e : -1;
          if (live) {
            const float s = __uint_as_float((uint32_t)(best >> 32));
            out.idx[(int64_t)t * k + r] = e;
            out.w[(int64_t)t * k + r] = __fmul_rn(s, __ldg(scales + e));
          }
        }
      }
    }
  }
  __syncthreads();
  rank_block_picks<TPB>(s_sel, k, E, T, blk_tok0, s_cnt, s_intra, out.lrank,
                        out.blk_hist + (int64_t)blockIdx.x * E);
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

// Top-k of precomputed scores, one thread per token, then block ranking.
constexpr int kTopkTPB = 128;
__global__ void __launch_bounds__(kTopkTPB) topk_from_scores_kernel(const float* __restrict__ scores,
                                                                   const float* __restrict__ scales, int32_t T,
                                                                   int32_t E, int32_t k, RouterOut out) {
  __shared__ int32_t s_sel[kMaxTopK * kTopkTPB];
  __shared__ int32_t s_intra[kMaxTopK * kTopkTPB];
  extern __shared__ int32_t s_cnt[];  // [(k*TPB/32) * E]
  const int32_t blk_tok0 = blockIdx.x * kTopkTPB;
  const int tok = threadIdx.x;
  const int32_t t = blk_tok0 + tok;
  if (t < T) {
    const float* sr = scores + (int64_t)t * E;
    uint32_t taken[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // up to 256 experts
    for (int r = 0; r < k; ++r) {
      int best = -1;
      float bs = 0.f;
      for (int e = 0; e < E; ++e) {
        if (taken[e >> 5] & (1u << (e & 31))) continue;
        const float s = sr[e];
        if (best < 0 || s > bs) {  // strict: ties keep the lower index
          best = e;
          bs = s;
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
  rank_block_picks<kTopkTPB>(s_sel, k, E, T, blk_tok0, s_cnt, s_intra, out.lrank,
                             out.blk_hist + (int64_t)blockIdx.x * E);
}

}  // namespace router
}  // namespace noor
