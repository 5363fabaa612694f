// simt_gemm.cuh -- grouped f32 GEMM on the CUDA cores, for F32 layers.
//
// The reference computes every layer in f32 (crates/noor-core/src/tensor.rs,
// "All compute happens in f32").  F32 layers must match it to rel-L2 1e-5,
// which TF32 tensor cores cannot, so their GEMMs run here in full f32 with
// FFMA.  B keeps the reference's [K, N] row-major layout (one matrix per
// weight index); the gated form reads the gate and up matrices and applies
// act(gate) * up in the epilogue (ffn.rs:24-34, 62-68).
#pragma once

#include "common.cuh"

namespace noor {
namespace simt {

constexpr int BM = 64, BN = 64, BK = 16, THREADS = 256;

enum Epilogue : int { EPI_STORE = 0, EPI_SWIGLU = 1, EPI_GEGLU = 2 };

struct Params {
  GroupTable groups;
  const float* A;
  int64_t lda;
  const float* Bg;   // [W][K][N]
  const float* Bu;   // [W][K][N] (gated only)
  int64_t b_stride;  // elements between weight matrices
  int32_t N, K;
  int32_t n_tiles;
  float* C;
  int64_t ldc;
};

template <int EPI>
__global__ void __launch_bounds__(THREADS) grouped_gemm_f32_kernel(const Params p) {
  constexpr bool GATED = EPI != EPI_STORE;
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN];
  __shared__ float Us[GATED ? BK : 1][GATED ? BN : 1];
  const int tid = threadIdx.x;
  const int ty = tid >> 4, tx = tid & 15;
  const int32_t total = group_total_mtiles(p.groups, BM) * p.n_tiles;
  for (int32_t tile = blockIdx.x; tile < total; tile += gridDim.x) {
    const TileCoord tc = decode_tile(p.groups, tile, p.n_tiles, BM);
    const int32_t n0 = tc.nt * BN;
    const float* Bg = p.Bg + (int64_t)tc.widx * p.b_stride;
    const float* Bu = GATED ? p.Bu + (int64_t)tc.widx * p.b_stride : nullptr;
    float acc[4][4], accu[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = accu[i][j] = 0.f;
    for (int32_t k0 = 0; k0 < p.K; k0 += BK) {
      // A tile: 64 rows x 16 k, 4 elements per thread
      {
        const int r = tid >> 2, kq = (tid & 3) * 4;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int32_t kk = k0 + kq + j;
          As[kq + j][r] = (r < tc.rows && kk < p.K) ? p.A[(int64_t)(tc.row0 + r) * p.lda + kk] : 0.f;
        }
      }
      // B tile: 16 k x 64 n
      {
        const int kr = tid >> 4, c = (tid & 15) * 4;
        const int32_t kk = k0 + kr;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int32_t n = n0 + c + j;
          const bool ok = kk < p.K && n < p.N;
          Bs[kr][c + j] = ok ? Bg[(int64_t)kk * p.N + n] : 0.f;
          if constexpr (GATED) Us[kr][c + j] = ok ? Bu[(int64_t)kk * p.N + n] : 0.f;
        }
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < BK; ++kk) {
        float a[4], b[4], u[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          b[j] = Bs[kk][tx * 4 + j];
          if constexpr (GATED) u[j] = Us[kk][tx * 4 + j];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
            if constexpr (GATED) accu[i][j] = fmaf(a[i], u[j], accu[i][j]);
          }
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = ty * 4 + i;
      if (r >= tc.rows) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int32_t n = n0 + tx * 4 + j;
        if (n >= p.N) continue;
        float v = acc[i][j];
        if constexpr (EPI == EPI_SWIGLU) v = __fmul_rn(act_silu(v), accu[i][j]);
        if constexpr (EPI == EPI_GEGLU) v = __fmul_rn(act_gelu_tanh(v), accu[i][j]);
        p.C[(int64_t)(tc.row0 + r) * p.ldc + n] = v;
      }
    }
  }
}

}  // namespace simt
}  // namespace noor
