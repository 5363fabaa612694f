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
// One warp per row.  Each lane sums its elements in f64 in order and the
// lanes are combined by a fixed butterfly, so the result is deterministic;
// its association differs from the reference's single running sum only in
// the last bits of an f64.
#pragma once

#include "common.cuh"

namespace noor {
namespace norm {

constexpr int kWarps = 8;
// At least 3 blocks (24 warps) per SM: the kernel is latency-bound per warp
// (a serial f64 sum, then the square root), so it needs warps in flight more
// than registers; this caps it at 85 registers a thread.
constexpr int kMinBlocks = 3;

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

// x / rms in f64, correctly rounded, without a divide per element:
// Markstein's correction (P. Markstein, "Computation of elementary functions
// on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990): with
// r = RN(1/rms), q = RN(x r) and the exact residual e = x - q rms (one FMA),
// RN(q + e r) = RN(x / rms) for operands away from overflow and underflow,
// which holds here (rms >= sqrt(eps) > 0, x finite).
__device__ __forceinline__ double div_by_rms(double x, double rms, double r) {
  const double q = __dmul_rn(x, r);
  const double e = __fma_rn(-q, rms, x);
  return __fma_rn(e, r, q);
}

// One element of the output: f32(x / rms * w) * depth_scale (+ resid).
__device__ __forceinline__ float norm_one(float x, double rms, double r, float w, float depth_scale) {
  return __fmul_rn(__double2float_rn(__dmul_rn(div_by_rms((double)x, rms, r), (double)w)), depth_scale);
}

// out[t] = (resid[t] +) f32(f64(x[t]) / rms * f64(w)) * depth_scale, rms =
// sqrt(sum_i x_i^2 / d + eps) in f64 (x_i^2 is exact in f64, so a fused
// multiply-add equals the reference's multiply then add).  d a multiple of 8,
// rows 16-byte aligned.
// STAGE (BF16 rows): each warp keeps its row in shared memory (dynamic,
// kWarps * d * 2 bytes), so the row is read from memory once and each
// thread's state stays small; without it the row is read twice (the second
// time from L1/L2).  Either way lane l sums elements 8l + 256j .. +7 in that
// order.
template <typename T_, bool RESID, bool STAGE>
__global__ void __launch_bounds__(kWarps * 32, kMinBlocks) rms_norm_rows_kernel(const T_* __restrict__ x,
                                                                                const float* __restrict__ w,
                                                                                double eps, float depth_scale,
                                                                                const T_* __restrict__ resid,
                                                                                int32_t T, int32_t d,
                                                                                T_* __restrict__ out) {
  extern __shared__ uint4 s_rows[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int32_t t = blockIdx.x * kWarps + warp;
  if (t >= T) return;
  const T_* row = x + (int64_t)t * d;
  double ss = 0.0;
  if constexpr (STAGE) {
    static_assert(sizeof(T_) == 2, "staged rows are BF16");
    const int nvec = d >> 3;  // 16-byte pieces of the row
    uint4* srow = s_rows + (int64_t)warp * nvec;
    const uint4* gx = reinterpret_cast<const uint4*>(row);
#pragma unroll 4
    for (int i = lane; i < nvec; i += 32) {
      const uint4 v = __ldg(gx + i);
      srow[i] = v;
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const double a = (double)bf16_lo(u[j]), bb = (double)bf16_hi(u[j]);
        ss = __fma_rn(a, a, ss);
        ss = __fma_rn(bb, bb, ss);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const double rms = __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)d), eps));
    const double r = __drcp_rn(rms);
#pragma unroll 2
    for (int i = lane; i < nvec; i += 32) {
      const int c = i * 8;
      const uint4 v = srow[i];
      const float4 wa = __ldg(reinterpret_cast<const float4*>(w + c));
      const float4 wb = __ldg(reinterpret_cast<const float4*>(w + c + 4));
      const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
      const uint32_t u[4] = {v.x, v.y, v.z, v.w};
      float o[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        o[2 * j] = norm_one(bf16_lo(u[j]), rms, r, wv[2 * j], depth_scale);
        o[2 * j + 1] = norm_one(bf16_hi(u[j]), rms, r, wv[2 * j + 1], depth_scale);
      }
      if constexpr (RESID) {
        float rr[8];
        Row8<T_>::load(resid + (int64_t)t * d + c, rr);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = __fadd_rn(rr[j], o[j]);
      }
      Row8<T_>::store(out + (int64_t)t * d + c, o);
    }
  } else {
    for (int c = lane * 8; c < d; c += 256) {
      float v[8];
      Row8<T_>::load(row + c, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = __fma_rn((double)v[j], (double)v[j], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __dadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const double rms = __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)d), eps));
    const double r = __drcp_rn(rms);
    for (int c = lane * 8; c < d; c += 256) {
      float v[8], o[8];
      Row8<T_>::load(row + c, v);
      const float4 wa = __ldg(reinterpret_cast<const float4*>(w + c));
      const float4 wb = __ldg(reinterpret_cast<const float4*>(w + c + 4));
      const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = norm_one(v[j], rms, r, wv[j], depth_scale);
      if constexpr (RESID) {
        float rr[8];
        Row8<T_>::load(resid + (int64_t)t * d + c, rr);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = __fadd_rn(rr[j], o[j]);
      }
      Row8<T_>::store(out + (int64_t)t * d + c, o);
    }
  }
}

// Shared memory of the staged BF16 form (0 when rows are read twice).
inline int staged_smem_bytes(bool bf16, int d) {
  const int bytes = kWarps * d * 2;
  return bf16 && bytes <= 64 * 1024 ? bytes : 0;
}

}  // namespace norm
}  // namespace noor
