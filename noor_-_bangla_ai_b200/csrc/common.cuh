// common.cuh -- shared device helpers for the Noor MoE kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace noor {

typedef __nv_bfloat16 bf16;

// Device-side error codes written to the handle's error word.  A bounded wait
// that gives up writes its code and returns instead of hanging the GPU.
enum DevError : int {
  DEV_OK = 0,
  DEV_TIMEOUT_PRODUCER = 1,
  DEV_TIMEOUT_MMA = 2,
  DEV_TIMEOUT_EPILOGUE = 3,
  DEV_BAD_INDEX = 4,
  DEV_TIMEOUT_PEER = 5,  // a wait on another rank gave up
  DEV_PEER_PLAN = 6,     // the expert-parallel plan was refused (over-capacity batch)
};

// Bounds checks of the debug build (compiled with -DNOOR_CHECK): a
// data-dependent index outside its buffer records DEV_BAD_INDEX in the
// device error word (err, nullable) and the caller skips the access -- no
// trap, so the context stays usable and the host reports the error.  Without
// NOOR_CHECK the check is compiled out and always passes.
__device__ __forceinline__ bool in_bounds(bool ok, int* err) {
#ifdef NOOR_CHECK
  if (!ok && err != nullptr) atomicCAS(err, 0, DEV_BAD_INDEX);
  return ok;
#else
  (void)ok;
  (void)err;
  return true;
#endif
}

// ~2 s at the B200's 1.9 GHz boost clock; no healthy wait comes close.
constexpr long long kWaitLimitCycles = 4000000000LL;

// Group table of a grouped GEMM: rows [row_start[g], row_start[g+1]) of the
// A and C buffers use weight matrix weight_idx[g]; their BM-row tiles are
// numbered from mtile_start[g].  A negative dense_rows means "read the
// table"; otherwise there is one group of dense_rows rows using weight 0.
struct GroupTable {
  const int32_t* row_start;    // [G+1]
  const int32_t* mtile_start;  // [G+1]
  const int32_t* weight_idx;   // [G] or nullptr for identity
  int32_t G;
  int32_t dense_rows;
};

struct TileCoord {
  int32_t row0;   // first A/C row of the tile
  int32_t rows;   // valid rows (<= BM)
  int32_t widx;   // weight matrix index
  int32_t nt;     // n-tile index
  int32_t g;      // group index (0 for a dense table)
};

__device__ __forceinline__ int32_t group_total_mtiles(const GroupTable& gt, int BM) {
  if (gt.dense_rows >= 0) return (gt.dense_rows + BM - 1) / BM;
  return gt.mtile_start[gt.G];
}

// Map a flat tile id (m-tile major, n-tile minor) to its group coordinates.
// The table pointers may point to global or shared memory.
__device__ __forceinline__ TileCoord decode_tile(const GroupTable& gt, int32_t tile, int32_t n_tiles,
                                                 int BM) {
  TileCoord c;
  const int32_t mt = tile / n_tiles;
  c.nt = tile - mt * n_tiles;
  if (gt.dense_rows >= 0) {
    c.row0 = mt * BM;
    c.rows = min(BM, gt.dense_rows - c.row0);
    c.widx = 0;
    c.g = 0;
    return c;
  }
  // last g with mtile_start[g] <= mt (groups with no tiles are skipped)
  int lo = 0, hi = gt.G;  // invariant: mtile_start[lo] <= mt < mtile_start[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (gt.mtile_start[mid] <= mt) lo = mid; else hi = mid;
  }
  const int32_t local = mt - gt.mtile_start[lo];
  const int32_t rs = gt.row_start[lo];
  const int32_t re = gt.row_start[lo + 1];
  c.row0 = rs + local * BM;
  c.rows = min(BM, re - c.row0);
  c.widx = gt.weight_idx ? gt.weight_idx[lo] : lo;
  c.g = lo;
  return c;
}

// Copy a group table of up to kSmemGroups groups into shared memory
// (s_tab: 3 * (kSmemGroups + 1) ints) so that per-tile decoding costs
// shared-memory latency, not a chain of global loads; larger tables stay in
// global memory.  All threads of the block call it; it ends with
// __syncthreads().
// A layer has at most 256 experts and every group table (one GPU: E
// experts; expert parallel: G*E/G = E (source rank, local expert) groups) has
// at most E groups.
constexpr int kSmemGroups = 256;
__device__ __forceinline__ GroupTable stage_group_table(const GroupTable& gt, int32_t* s_tab) {
  GroupTable out = gt;
  if (gt.dense_rows < 0 && gt.G <= kSmemGroups) {
    int32_t* rs = s_tab;
    int32_t* mt = s_tab + (kSmemGroups + 1);
    int32_t* wi = s_tab + 2 * (kSmemGroups + 1);
    for (int i = threadIdx.x; i <= gt.G; i += blockDim.x) {
      rs[i] = __ldg(gt.row_start + i);
      mt[i] = __ldg(gt.mtile_start + i);
      if (i < gt.G) wi[i] = gt.weight_idx ? __ldg(gt.weight_idx + i) : i;
    }
    out.row_start = rs;
    out.mtile_start = mt;
    out.weight_idx = wi;
  }
  __syncthreads();
  return out;
}

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);  // RNE, as tensor.rs:23-28
  return *reinterpret_cast<uint32_t*>(&p);
}

// Activations, written as the reference writes them (tensor.rs:438-459):
// silu(x) = x / (1 + exp(-x)); gelu(x) = 0.5x(1 + tanh(sqrt(2/pi)(x + 0.044715x^3))).
__device__ __forceinline__ float act_silu(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, expf(-x))); }

// SiLU for outputs rounded to BF16 (tensor-core epilogues): the fast
// exponential and approximate divide are within a few f32 ulp, far below the
// BF16 rounding (2^-8 relative) that follows.  exp(-x) overflowing to +inf
// for x < -88 gives x / inf = -0, the limit of silu.
__device__ __forceinline__ float act_silu_bf16out(float x) { return __fdividef(x, 1.0f + __expf(-x)); }

// GELU (tanh form) for outputs rounded to BF16: 0.5 (1 + tanh u) equals the
// logistic 1 / (1 + exp(-2u)) exactly, so gelu(x) = x / (1 + exp(-2u)) with
// u = sqrt(2/pi) (x + 0.044715 x^3) as the reference forms it; the fast
// exponential and divide stay within a few f32 ulp, far below the BF16
// rounding that follows (the same bound as act_silu_bf16out).
__device__ __forceinline__ float act_gelu_tanh_bf16out(float x) {
  const float sqrt_2_pi = 0x1.988452p-1f;
  const float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
  const float inner = __fmul_rn(sqrt_2_pi, __fadd_rn(x, cube));
  return __fdividef(x, 1.0f + __expf(-2.0f * inner));
}

__device__ __forceinline__ float act_gelu_tanh(float x) {
  // (2.0f32 / PI).sqrt() evaluated in f32, as the reference does: 0x1.988452p-1
  const float sqrt_2_pi = 0x1.988452p-1f;
  float cube = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, x), x), x);
  float inner = __fmul_rn(sqrt_2_pi, __fadd_rn(x, cube));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(inner)));
}

}  // namespace noor
