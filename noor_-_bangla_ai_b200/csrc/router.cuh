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
#include "dispatch.cuh"

namespace noor {
namespace router {

constexpr int kMaxTopK = 8;
constexpr int kMaxExpertsTC = 128;  // tensor-core router: up to 16 n-fragments

// ------------------------------------------------------------------ ranking

// sel[slot * TPB + tok] holds the expert of each pick in the block (-1 for
// tokens past T).  Computes each pick's rank among the block's picks of the
// same expert in (slot, token) order, writes it to lrank_out[token*k + slot],
// and writes the block histogram hist_out[e * hist_stride].
__device__ void rank_block_picks(const int32_t* sel, int k, int TPB, int E, int T, int32_t tok_base,
                                 int32_t* chunk_cnt /* smem [nchunks][E] */,
                                 int32_t* intra /* smem [k*TPB] */, int32_t* lrank_out,
                                 int32_t* hist_out, int32_t hist_stride) {
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
    hist_out[(int64_t)e * hist_stride] = run;
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
  int32_t* blk_hist; // [E, nblk], expert-major
};

// Optional scan fused into the router: the last block to finish turns the
// block histograms into the segment tables (dispatch::scan_segments_block).
// `done` is a zero-initialised counter the last block resets to zero.
struct FusedScan {
  int* done;               // nullptr: no fused scan
  int64_t* counts;
  int32_t* seg_start;
  int32_t* blk_base;
  int32_t* mtile_start;
  int32_t BM;
  int64_t* util;           // nullable: utilization accumulator [E+1] (dispatch::scan_segments_block)
};

// BF16 router: one block of W warps per SM-sized share of the batch; warp w
// owns 16 tokens (the block's token block is 16 W tokens).  The router gate is
// staged in shared memory K-chunk by K-chunk (kc_len columns, rows padded by
// 32 elements so the fragment reads hit distinct banks).  Each warp streams
// its tokens' x with mma.sync m16n8k16 over the whole K, keeping the next
// PF k-steps of x loads in flight while it multiplies the current ones.  Then,
// per token: sigmoid(dot + bias), top-k by quad shuffles on (score, ~index)
// keys, weights; per block: deterministic ranks and the histogram; the last
// block to finish runs the segment scan.
constexpr int kRouteMaxWarps = 8;
constexpr int kRouteMaxTPB = 16 * kRouteMaxWarps;

__host__ inline int route_chunk(int d, int nf) {
  // Largest chunk of K whose padded gate slice fits 96 KB: either all of K, or
  // a multiple of the 256-column load batch dividing d (so a batch never
  // straddles two chunks).  0 if none fits.
  int best = 0;
  for (int kc = 64; kc <= d; kc += 64)
    if (d % kc == 0 && (kc == d || kc % 256 == 0) && (size_t)nf * 8 * (kc + 32) * 2 <= 96 * 1024) best = kc;
  return best;
}

template <int NF>
__global__ void __launch_bounds__(32 * kRouteMaxWarps) route_bf16_kernel(
    const bf16* __restrict__ x, const bf16* __restrict__ gate_t, const float* __restrict__ bias,
    const float* __restrict__ scales, int32_t T, int32_t d, int32_t E, int32_t k, int32_t kc_len, RouterOut out,
    FusedScan scan) {
  constexpr int PF = 4;
  constexpr int SEL = kMaxTopK * kRouteMaxTPB;
  __shared__ int32_t s_sel[SEL];
  __shared__ int32_t s_intra[SEL];
  __shared__ int32_t s_cnt[(SEL / 32) * kMaxExpertsTC];
  __shared__ int32_t s_warp[32];
  __shared__ int32_t s_seg[kMaxExpertsTC + 1];
  __shared__ int s_last;
  extern __shared__ __align__(16) bf16 s_gate[];  // [NF*8][kc_len + 32]
  const int ld = kc_len + 32;
  const int nwarps = blockDim.x >> 5;
  const int TPB = 16 * nwarps;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, t4 = lane & 3;
  const int32_t blk_tok0 = blockIdx.x * TPB;
  const int32_t tok0 = blk_tok0 + warp * 16;
  const int32_t r0 = tok0 + gid, r1 = tok0 + gid + 8;
  const bool v0 = r0 < T, v1 = r1 < T;
  const bf16* x0 = x + (int64_t)(v0 ? r0 : 0) * d;
  const bf16* x1 = x + (int64_t)(v1 ? r1 : 0) * d;

  // S independent partial sums per output (split by the 16-byte piece c and
  // the fragment half of each MMA) so consecutive MMAs rarely wait on the
  // same accumulator; they are added in a fixed order at the end.
  constexpr int S = NF <= 4 ? 4 : (NF <= 8 ? 2 : 1);
  float part[S][NF][4];
#pragma unroll
  for (int q = 0; q < S; ++q)
#pragma unroll
    for (int n = 0; n < NF; ++n)
#pragma unroll
      for (int j = 0; j < 4; ++j) part[q][n][j] = 0.f;

  // x loads of PF k-steps starting at absolute column kk0 (zero past d)
  auto load_batch = [&](int32_t kk0, uint4 (&a)[PF][2][2]) {
#pragma unroll
    for (int pf = 0; pf < PF; ++pf) {
      const int32_t kk = kk0 + 64 * pf;
      const bool in = kk < d;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        a[pf][0][c] = (in && v0) ? ldg_nc_v4(x0 + kk + 32 * c + 8 * t4) : make_uint4(0, 0, 0, 0);
        a[pf][1][c] = (in && v1) ? ldg_nc_v4(x1 + kk + 32 * c + 8 * t4) : make_uint4(0, 0, 0, 0);
      }
    }
  };
  // the MMAs of PF k-steps; columns kk0 - k0 .. of the staged gate chunk
  auto mma_batch = [&](int32_t kk0, int32_t k0, const uint4 (&a)[PF][2][2]) {
    const bf16* g0 = s_gate + gid * ld;
#pragma unroll
    for (int pf = 0; pf < PF; ++pf) {
      const int32_t kk = kk0 + 64 * pf - k0;
      if (kk >= kc_len) break;
      uint4 b[2][NF];
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int n = 0; n < NF; ++n) b[c][n] = *reinterpret_cast<const uint4*>(g0 + n * 8 * ld + kk + 32 * c + 8 * t4);
#pragma unroll
      for (int c = 0; c < 2; ++c)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
#pragma unroll
          for (int n = 0; n < NF; ++n) {
            float (&acc)[4] = part[(2 * c + hh) % S][n];
            if (hh == 0)
              mma_bf16_16816(acc, a[pf][0][c].x, a[pf][1][c].x, a[pf][0][c].y, a[pf][1][c].y, b[c][n].x, b[c][n].y);
            else
              mma_bf16_16816(acc, a[pf][0][c].z, a[pf][1][c].z, a[pf][0][c].w, a[pf][1][c].w, b[c][n].z, b[c][n].w);
          }
    }
  };

  uint4 a_cur[PF][2][2], a_nxt[PF][2][2];
  load_batch(0, a_cur);  // in flight while the gate is staged
  for (int32_t k0 = 0; k0 < d; k0 += kc_len) {
    if (k0 > 0) __syncthreads();  // everyone is done with the previous chunk
    {
      // stage gate_t[:, k0 : k0 + kc_len], eight 16-byte loads in flight per thread
      const int pieces_per_row = kc_len / 8;
      const int pieces = NF * 8 * pieces_per_row;
      constexpr int U = 8;
      for (int base = threadIdx.x; base < pieces; base += blockDim.x * U) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = base + u * blockDim.x;
          if (i < pieces) {
            const int r = i / pieces_per_row, c = i - r * pieces_per_row;
            v[u] = __ldg(reinterpret_cast<const uint4*>(gate_t + (int64_t)r * d + k0 + c * 8));
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int i = base + u * blockDim.x;
          if (i < pieces) {
            const int r = i / pieces_per_row, c = i - r * pieces_per_row;
            *reinterpret_cast<uint4*>(s_gate + r * ld + c * 8) = v[u];
          }
        }
      }
    }
    __syncthreads();
    for (int32_t kk0 = k0; kk0 < k0 + kc_len; kk0 += 64 * PF) {
      load_batch(kk0 + 64 * PF, a_nxt);  // next batch (the next chunk's first one at a chunk end)
      mma_batch(kk0, k0, a_cur);
#pragma unroll
      for (int pf = 0; pf < PF; ++pf)
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
          for (int c = 0; c < 2; ++c) a_cur[pf][h][c] = a_nxt[pf][h][c];
    }
  }

  float acc[NF][4];
#pragma unroll
  for (int n = 0; n < NF; ++n)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float v = part[0][n][j];
#pragma unroll
      for (int q = 1; q < S; ++q) v = __fadd_rn(v, part[q][n][j]);
      acc[n][j] = v;
    }

  // Scores and top-k.  Row h of this quad: lane holds experts
  // n*8 + 2*t4 + j (j = 0, 1) in acc[n][2h + j].  Keys order by score
  // (non-negative f32 bits are monotone) then by lower expert index.
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
          const float dot = __fadd_rn(acc[n][2 * h + j], __ldg(bias + e));
          const float sc = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-dot)));
          kv = ((unsigned long long)__float_as_uint(sc) << 32) | (unsigned long long)(0xFFFFu - (unsigned)e);
        }
        key[2 * n + j] = kv;
      }
    const int tok_in_blk = warp * 16 + gid + 8 * h;
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
          const float sc = __uint_as_float((uint32_t)(best >> 32));
          out.idx[(int64_t)t * k + r] = e;
          out.w[(int64_t)t * k + r] = __fmul_rn(sc, __ldg(scales + e));
        }
      }
    }
  }
  for (int i = k * TPB + threadIdx.x; i < ((k * TPB + 31) / 32) * 32; i += blockDim.x) s_sel[i] = -1;  // padding
  __syncthreads();
  rank_block_picks(s_sel, k, TPB, E, T, blk_tok0, s_cnt, s_intra, out.lrank, out.blk_hist + blockIdx.x, gridDim.x);
  if (scan.done == nullptr) return;
  __syncthreads();
  __threadfence();
  if (threadIdx.x == 0) s_last = atomicAdd(scan.done, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  dispatch::scan_segments_block(out.blk_hist, gridDim.x, E, scan.BM, scan.counts, scan.seg_start, scan.blk_base,
                                scan.mtile_start, s_warp, s_seg, scan.util, k);
  if (threadIdx.x == 0) *scan.done = 0;
}

// Warps per block of route_bf16_kernel for T tokens: enough for one block per
// SM to cover the batch, at most kRouteMaxWarps.
__host__ inline int route_warps(int64_t T, int num_sms) {
  const int64_t units = (T + 15) / 16;
  return (int)std::min<int64_t>(kRouteMaxWarps, std::max<int64_t>(1, (units + num_sms - 1) / num_sms));
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
  __shared__ int32_t s_warp[32];
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
  rank_block_picks(s_sel, k, kTopkTPB, E, T, blk_tok0, s_cnt, s_intra, out.lrank, out.blk_hist + blockIdx.x,
                   gridDim.x);
  if (scan.done == nullptr) return;
  __syncthreads();
  __threadfence();
  if (threadIdx.x == 0) s_last = atomicAdd(scan.done, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  dispatch::scan_segments_block(out.blk_hist, gridDim.x, E, scan.BM, scan.counts, scan.seg_start, scan.blk_base,
                                scan.mtile_start, s_warp, s_seg, scan.util, k);
  if (threadIdx.x == 0) *scan.done = 0;
}

}  // namespace router
}  // namespace noor
