// router_tc.cuh -- K1 for BF16 layers on the tcgen05 tensor cores.
//
// The router's dot products are a GEMM with a narrow N: scores[T, E] =
// x[T, d] . gate_t[E, d]^T.  One CTA takes a tile of 128 tokens:
//   warp 0 lane 0   TMA producer: per 64-column k-block, the x tile (128 rows,
//                   16 KB) and the gate tile (NPAD rows) into a ring of up
//                   to 8 stages (128-byte swizzle)
//   warp 1 lane 0   MMA issuer: tcgen05.mma.cta_group::1.kind::f16, M = 128,
//                   N = NPAD (E rounded up to 16), f32 accumulator in TMEM
//   warps 2..5      epilogue: thread i owns token row i (TMEM lane i): it
//                   reads its E dot products with tcgen05.ld, adds the bias,
//                   applies the sigmoid and keeps its top k on (score, ~index)
//                   keys in registers -- MoERouter::route (moe.rs:79-107) for
//                   one token per thread, no shuffles
// then all 6 warps rank the block's picks and claim the block's rows of each
// expert's segment (rank_block_picks), and the last block to finish turns
// the per-expert totals into the segment tables (finish_from_totals).
// x is read from HBM exactly once, by TMA; the gate (E x d BF16) stays in L2.
#pragma once

#include "dispatch.cuh"
#include "router.cuh"
#include "tc_gemm.cuh"

namespace noor {
namespace router {

constexpr int kTcTPB = 128;       // tokens per CTA
constexpr int kTcMaxStages = 8;
constexpr int kTcRingBytes = 192 * 1024;     // stage ring budget, E <= 32: one CTA per SM
constexpr int kTcRingBytesWide = 72 * 1024;  // E > 32: two CTAs per SM, so that one streams x while the
                                             // other runs its (longer) epilogue
constexpr int kTcThreads = 192;   // producer, MMA, 4 epilogue warps
constexpr int kTcXBytes = kTcTPB * 64 * 2;  // one k-block of the x tile

__host__ __device__ constexpr int tc_npad(int E) { return (E + 15) / 16 * 16; }
__host__ __device__ constexpr int tc_stage_bytes(int npad) { return kTcXBytes + npad * 64 * 2; }
// As many stages as fit the ring budget, at most kTcMaxStages: each CTA
// streams 512 KB of x per 128 tokens (d = 2048), and the ring depth is what
// keeps its TMA -> MMA -> release chain from being latency-bound.
__host__ __device__ constexpr int tc_ring_budget(int npad) { return npad <= 32 ? kTcRingBytes : kTcRingBytesWide; }
__host__ __device__ constexpr int tc_stages(int npad) {
  return tc_ring_budget(npad) / tc_stage_bytes(npad) < kTcMaxStages ? tc_ring_budget(npad) / tc_stage_bytes(npad)
                                                                     : kTcMaxStages;
}
// For E > 32 the epilogue stages the tile's scores (kTcTPB rows of npad + 1
// floats) in the ring once every copy into it has retired.
__host__ __device__ constexpr int tc_scores_bytes(int npad) { return kTcTPB * (npad + 1) * 4; }
__host__ constexpr int tc_smem_bytes(int npad) {
  return (tc_stages(npad) * tc_stage_bytes(npad) > tc_scores_bytes(npad) ? tc_stages(npad) * tc_stage_bytes(npad)
                                                                         : tc_scores_bytes(npad)) +
         1024;
}
__host__ __device__ constexpr uint32_t tc_tmem_cols(int npad) {
  return npad <= 32 ? 32u : (npad <= 64 ? 64u : 128u);
}

// NL: 32-column TMEM loads covering NPAD = roundup(E, 16) columns.
template <int NL>
__global__ void __launch_bounds__(kTcThreads, 1) route_tc_kernel(
    const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmG,
    const float* __restrict__ bias, const float* __restrict__ scales, int32_t T, int32_t d, int32_t E, int32_t k,
    RouterOut out, FusedScan scan, int* err) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int npad = tc_npad(E);
  const int stage_bytes = tc_stage_bytes(npad);
  const int nstages = tc_stages(npad);
  const uint32_t tmem_cols = tc_tmem_cols(npad);
  // instruction descriptor: f32 accumulate, BF16 A and B, K-major, N = npad, M = 128
  const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(npad >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

  constexpr int SEL = kMaxTopK * kTcTPB;
  __shared__ __align__(8) uint64_t full_bar[kTcMaxStages];
  __shared__ __align__(8) uint64_t empty_bar[kTcMaxStages];
  __shared__ __align__(8) uint64_t accf_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  __shared__ int32_t s_sel[SEL];
  __shared__ int32_t s_intra[SEL];
  __shared__ int32_t s_cnt[(SEL / 32) * kMaxExpertsTC];
  __shared__ float s_bias[kMaxExpertsTC];
  __shared__ float s_scale[kMaxExpertsTC];
  __shared__ int32_t s_seg[kMaxExpertsTC + 1];
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int32_t tok0 = blockIdx.x * kTcTPB;
  const int num_kb = d / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < nstages; ++s) {
      tc::mbar_init(&full_bar[s], 1);
      tc::mbar_init(&empty_bar[s], 1);
    }
    tc::mbar_init(&accf_bar, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc::tma_prefetch_desc(&tmX);
    tc::tma_prefetch_desc(&tmG);
  }
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    s_bias[e] = bias[e];
    s_scale[e] = scales[e];
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc::smem_addr(&tmem_slot)),
                 "r"(tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem_base = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!tc::mbar_wait(&empty_bar[stage], phase ^ 1u, &abort_flag, err, DEV_TIMEOUT_PRODUCER)) break;
        uint8_t* st = smem + stage * stage_bytes;
        tc::mbar_arrive_expect_tx(&full_bar[stage], (uint32_t)stage_bytes);
        tc::tma_load_2d(st, &tmX, &full_bar[stage], kb * 64, tok0);
        tc::tma_load_2d(st + kTcXBytes, &tmG, &full_bar[stage], kb * 64, 0);
        if (++stage == nstages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!tc::mbar_wait(&full_bar[stage], phase, &abort_flag, err, DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc::tc_fence_after();
        const uint32_t a0 = tc::smem_addr(smem + stage * stage_bytes);
        const uint32_t b0 = a0 + kTcXBytes;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc::umma_bf16(tmem_base, tc::sdesc_sw128(a0 + kk * 32), tc::sdesc_sw128(b0 + kk * 32), idesc,
                        (kb | kk) != 0 ? 1u : 0u);
        tc::umma_commit(&empty_bar[stage]);
        if (++stage == nstages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      // the accumulator is complete once every issued MMA retires (also on
      // the abort path, so that the epilogue's wait ends and TMEM is idle)
      (void)ok;
      tc::umma_commit(&accf_bar);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue: thread i <-> token row i = TMEM lane i
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int32_t t = tok0 + row;
    const bool live = t < T;
    unsigned long long best[kMaxTopK];
    // If the wait gives up (the error word is set and the call fails), the
    // picks are experts 0..k-1 with score 0: garbage, but valid indices, so
    // the kernels after this one stay in bounds.
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r) best[r] = r < k ? (unsigned long long)(0xFFFFu - (unsigned)r) : 0ull;
    if (tc::mbar_wait(&accf_bar, 0, &abort_flag, err, DEV_TIMEOUT_EPILOGUE)) {
#pragma unroll
      for (int r = 0; r < kMaxTopK; ++r) best[r] = 0ull;
      tc::tc_fence_after();
      if constexpr (NL == 1) {
        // up to 32 experts: one TMEM load, and the insertion of every key
        // unrolled (fits the instruction cache, no dependent loop)
        uint32_t v[32];
        tc::tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16), v);
        tc::tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          if (e < E) {
            const float dot = __fadd_rn(__uint_as_float(v[e]), s_bias[e]);
            const float sc = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-dot)));
            unsigned long long kv =
                ((unsigned long long)__float_as_uint(sc) << 32) | (unsigned long long)(0xFFFFu - (unsigned)e);
#pragma unroll
            for (int r = 0; r < kMaxTopK; ++r) {
              if (r < k && kv > best[r]) {
                const unsigned long long tmp = best[r];
                best[r] = kv;
                kv = tmp;
              }
            }
          }
        }
      } else {
      // Phase 1: the row's sigmoid scores from TMEM into shared memory.  The
      // stage ring is idle once the accumulator is complete (every MMA, and
      // so every copy into the ring, has retired); rows are padded by one
      // float so that a warp's accesses to one expert hit 32 banks.
      float* s_sc = reinterpret_cast<float*>(smem);
      const int ld = npad + 1;
#pragma unroll 1
      for (int c = 0; c < NL; ++c) {
        uint32_t v[32];
        tc::tmem_ld32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 32), v);
        tc::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int e = c * 32 + j;
          if (e < E) {
            const float dot = __fadd_rn(__uint_as_float(v[j]), s_bias[e]);
            s_sc[row * ld + e] = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-dot)));
          }
        }
      }
      // Phase 2: the top k in a compact loop (an unrolled walk over 128
      // experts would not fit the instruction cache): most keys fail the test
      // against the current k-th key and cost a compare.
      unsigned long long kth = 0ull;  // best[k - 1]
#pragma unroll 1
      for (int e = 0; e < E; ++e) {
        unsigned long long kv = ((unsigned long long)__float_as_uint(s_sc[row * ld + e]) << 32) |
                                (unsigned long long)(0xFFFFu - (unsigned)e);
        if (kv > kth) {
          // keep best[0..k) sorted descending: bubble the new key in
#pragma unroll
          for (int r = 0; r < kMaxTopK; ++r) {
            if (r < k && kv > best[r]) {
              const unsigned long long tmp = best[r];
              best[r] = kv;
              kv = tmp;
            }
          }
#pragma unroll
          for (int r = 0; r < kMaxTopK; ++r)
            if (r == k - 1) kth = best[r];
        }
      }
      }
    }
#pragma unroll
    for (int r = 0; r < kMaxTopK; ++r) {
      if (r < k) {
        const int e = (int)(0xFFFFu - (unsigned)(best[r] & 0xFFFFFFFFull));
        s_sel[r * kTcTPB + row] = (live && e >= 0 && e < E) ? e : -1;
        if (live) {
          const float sc = __uint_as_float((uint32_t)(best[r] >> 32));
          out.idx[(int64_t)t * k + r] = e;
          out.w[(int64_t)t * k + r] = __fmul_rn(sc, s_scale[e < E ? e : 0]);
        }
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols)
                 : "memory");
  }
  const bool fused = scan.done != nullptr;
  rank_block_picks(s_sel, k, kTcTPB, E, T, tok0, s_cnt, s_intra, out.lrank,
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
#endif
}

}  // namespace router
}  // namespace noor
