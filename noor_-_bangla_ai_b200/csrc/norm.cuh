// norm.cuh -- the sandwich norm around the MoE block's FFN sublayer.
//
// MoEBlock::forward (block.rs:87-90) wraps ParallelFFN in a SandwichNorm
// (norm.rs:31-60):
//   normed = rms_norm(h, w_pre) * depth_scale
//   out    = h + rms_norm(ParallelFFN(normed), w_post) * depth_scale
// with rms_norm as tensor.rs:462-490: the sum of squares and the division by
// the RMS in f64, the result rounded to f32; Tensor::scale and tensor::add
// (tensor.rs:222-229, 280-288) are plain f32 multiplies and adds.
//
// One warp per row.  The row is read twice (the second read hits L1/L2):
// once for the sum of squares, once to normalise.  Each lane sums its
// elements in f64 in order and the lanes are combined by a fixed butterfly,
// so the result is deterministic; its association differs from the
// reference's single running sum only in the last bits of an f64.
#pragma once

#include "common.cuh"

namespace noor {
namespace norm {

constexpr int kWarps = 8;

template <typename T_>
struct Row8;
template <>
struct Row8<bf16> {
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
struct Row8<float> {
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

// out[t] = (resid[t] +) f32(f64(x[t]) / rms * f64(w)) * depth_scale.
// d must be a multiple of 8 and rows 16-byte aligned.
template <typename T_, bool RESID>
__global__ void __launch_bounds__(kWarps * 32) rms_norm_rows_kernel(const T_* __restrict__ x,
                                                                    const float* __restrict__ w, double eps,
                                                                    float depth_scale, const T_* __restrict__ resid,
                                                                    int32_t T, int32_t d, T_* __restrict__ out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int32_t t = blockIdx.x * kWarps + warp;
  if (t >= T) return;
  const T_* row = x + (int64_t)t * d;
  double ss = 0.0;
  for (int c = lane * 8; c < d; c += 256) {
    float v[8];
    Row8<T_>::load(row + c, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) ss = __dadd_rn(ss, __dmul_rn((double)v[j], (double)v[j]));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  const double rms = __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)d), eps));
  for (int c = lane * 8; c < d; c += 256) {
    float v[8], o[8];
    Row8<T_>::load(row + c, v);
    const float4 wa = __ldg(reinterpret_cast<const float4*>(w + c));
    const float4 wb = __ldg(reinterpret_cast<const float4*>(w + c + 4));
    const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
    for (int j = 0; j < 8; ++j)
      o[j] = __fmul_rn(__double2float_rn(__dmul_rn(__ddiv_rn((double)v[j], rms), (double)wv[j])), depth_scale);
    if constexpr (RESID) {
      float r[8];
      Row8<T_>::load(resid + (int64_t)t * d + c, r);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = __fadd_rn(r[j], o[j]);
    }
    Row8<T_>::store(out + (int64_t)t * d + c, o);
  }
}

}  // namespace norm
}  // namespace noor
