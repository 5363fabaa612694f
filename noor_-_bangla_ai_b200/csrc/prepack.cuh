// prepack.cuh -- weight layout conversion at load time.
//
// The reference stores every projection [K, N] row-major in f32
// (crates/noor-core/src/layers/ffn.rs:5-12, 43-50; moe.rs:7).  The tensor-core
// GEMM wants each weight K-major ([N, K]) in BF16, and the gate/up projection
// of a GLU FFN fused into one matrix whose 256-row n-tiles hold 128 gate rows
// followed by the 128 matching up rows, so one accumulator tile carries both
// halves into the SwiGLU / GeGLU epilogue.
#pragma once

#include "common.cuh"

namespace noor {
namespace prepack {

// dst[row(n)][k] = bf16_rne(src[k][n]) with row(n) = (n / group) * stride + n % group + offset.
// 32x32 tiles through shared memory so both sides stay coalesced.
__global__ void transpose_to_bf16_kernel(const float* __restrict__ src, int32_t K, int32_t N, bf16* __restrict__ dst,
                                         int64_t dst_ld, int32_t group, int32_t stride, int32_t offset) {
  __shared__ float tile[32][33];
  const int32_t k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int32_t k = k0 + i, n = n0 + threadIdx.x;
    tile[i][threadIdx.x] = (k < K && n < N) ? src[(int64_t)k * N + n] : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int32_t n = n0 + i, k = k0 + threadIdx.x;
    if (n < N && k < K) {
      const int64_t row = (int64_t)(n / group) * stride + (n % group) + offset;
      dst[row * dst_ld + k] = __float2bfloat16_rn(tile[threadIdx.x][i]);
    }
  }
}

// Elementwise f32 -> bf16 (RNE), for activations handed over in f32.
__global__ void f32_to_bf16_kernel(const float* __restrict__ src, bf16* __restrict__ dst, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = __float2bfloat16_rn(src[i]);
}

}  // namespace prepack
}  // namespace noor
