// smebu.cuh -- expert utilization on the device and the SMEBU bias update.
//
// The reference keeps, per MoE layer, an ExpertUtilization (moe.rs:25-65):
// record() adds each token's k picks to counts[E] and 1 to total_tokens; once
// per training step the model reads fractions() = counts / total_tokens and
// resets it (model.rs:180-183), SMEBU::update turns the fractions into new
// router biases (smebu.rs:36-48) and apply_to_router writes them into the
// router (smebu.rs:56-61, training_loop.rs:290-301).  Here the utilization
// lives in device memory as util[E+1] (counts, then tokens), accumulated by
// the kernels that already hold each batch's counts (the router's fused scan
// on one GPU, the exchange plan under expert parallelism, where the counts are
// the global ones), and one small kernel applies the update straight to the
// bias the router reads, so the step's bias refresh never leaves the GPU.
#pragma once

#include "common.cuh"

namespace noor {
namespace smebu {

// util[e] += counts[e]; util[E] += sum(counts) / k.  One block of >= E threads.
__global__ void util_accumulate_kernel(const int64_t* __restrict__ counts, int32_t E, int32_t k,
                                       int64_t* __restrict__ util) {
  __shared__ int64_t s_sum;
  if (threadIdx.x == 0) s_sum = 0;
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int64_t c = counts[e];
    util[e] += c;
    atomicAdd(reinterpret_cast<unsigned long long*>(&s_sum), (unsigned long long)c);
  }
  __syncthreads();
  if (threadIdx.x == 0) util[E] += s_sum / k;
}

// SMEBU::update on fractions = counts / total_tokens (ExpertUtilization::
// fractions: all zero when no token was recorded), with each f32 operation
// rounded separately as the reference's scalar code does:
//   f_target = 1 / E
//   m = beta * m + lambda * (f_target - f)
//   b = kappa * tanh(m / kappa)
// b is written to the router's bias; the utilization is reset.  One block of
// >= E threads.
__global__ void smebu_update_kernel(int64_t* __restrict__ util, float* __restrict__ momentum,
                                    float* __restrict__ bias, int32_t E, float kappa, float beta, float lambda) {
  const int64_t tokens = util[E];
  __syncthreads();  // every thread has read the token count before it is reset
  const float f_target = __fdiv_rn(1.0f, (float)E);
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const float f = tokens == 0 ? 0.0f : __fdiv_rn(__ll2float_rn(util[e]), __ll2float_rn(tokens));
    const float m = __fadd_rn(__fmul_rn(beta, momentum[e]), __fmul_rn(lambda, __fsub_rn(f_target, f)));
    momentum[e] = m;
    bias[e] = __fmul_rn(kappa, tanhf(__fdiv_rn(m, kappa)));
    util[e] = 0;
  }
  if (threadIdx.x == 0) util[E] = 0;
}

}  // namespace smebu
}  // namespace noor
