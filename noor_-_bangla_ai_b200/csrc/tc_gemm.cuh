// tc_gemm.cuh -- grouped BF16 GEMM on sm_100a tensor cores (tcgen05 + TMA).
//
// C[rows of group g, :] = epilogue( A[rows of g, :K] . B[weight_idx[g]]^T )
//
// A is [rows, K] bf16 row-major (K-major); B holds one [N, K] bf16 K-major
// matrix per weight index (the library prepacks the reference's [K, N]
// row-major weights transposed).  This one kernel runs all four GEMMs of the
// layer: the expert gate/up projection with the SwiGLU epilogue, the expert
// down projection, and the dense branch's gate/up (GeGLU epilogue) and down
// projections (crates/noor-core/src/layers/ffn.rs:24-34, 62-68).
//
// Design (one persistent CTA per SM, warp-specialised):
//   warp 0 lane 0 : TMA producer, STAGES-deep ring of (A, B) k-blocks in smem
//   warp 1 lane 0 : tcgen05.mma issuer, M=128 x N=BN x K=16 per instruction,
//                   f32 accumulator in TMEM, double-buffered (2 x BN columns)
//   warps 2..9    : epilogue, tcgen05.ld TMEM -> registers -> activation ->
//                   global; warp w reads TMEM lanes 32*(w%4) .. +31, warps
//                   2..5 the first half of the tile's columns, 6..9 the second
// Every mbarrier wait is bounded: after kWaitLimitCycles it records an error
// code in the handle's device error word, raises a CTA-wide abort flag, and
// all roles leave their loops; TMEM is always released before exit.
//
// Every CTA loads its own tiles from global memory; no load is shared across
// a cluster.
#pragma once

#include <cuda.h>
#include "common.cuh"

namespace noor {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one 128B swizzle row
constexpr int STAGES = 4;
#ifndef NOOR_GEMM_EPI_WARPS
#define NOOR_GEMM_EPI_WARPS 8
#endif
// Epilogue warps: EPI_PARTS per TMEM lane quarter, each on 1/EPI_PARTS of the
// tile's columns.
constexpr int EPI_WARPS = NOOR_GEMM_EPI_WARPS;
constexpr int EPI_PARTS = EPI_WARPS / 4;
static_assert(EPI_WARPS % 4 == 0 && (EPI_PARTS == 1 || EPI_PARTS == 2 || EPI_PARTS == 4), "epilogue warps");
constexpr int NUM_THREADS = 64 + 32 * EPI_WARPS;
// The SM-pair kernel sets its epilogue warp count per epilogue: the plain
// and gated epilogues (one TMEM read and a store per chunk) with
// NOOR_GEMM_EPI_WARPS_PLAIN warps, the fused combine (gathers that need
// warps in flight) with EPI_WARPS.
#ifndef NOOR_GEMM_EPI_WARPS_PLAIN
#define NOOR_GEMM_EPI_WARPS_PLAIN 8
#endif

enum Epilogue : int {
  EPI_STORE_BF16 = 0,   // C = acc (bf16)
  EPI_STORE_F32 = 1,    // C = acc (f32)
  EPI_SWIGLU_BF16 = 2,  // C[:, j] = silu(acc[:, j]) * acc[:, BN/2 + j]   (per n-tile)
  EPI_GEGLU_BF16 = 3,   // C[:, j] = gelu_tanh(acc[:, j]) * acc[:, BN/2 + j]
  EPI_COMBINE_BF16 = 4, // C[t, :] = (acc[t, :] + sum_i w[t,i] y[dst[t,i], :] (+ shared[t, :])) / sqrt 2
};

__host__ __device__ constexpr bool epi_gated(int e) { return e == EPI_SWIGLU_BF16 || e == EPI_GEGLU_BF16; }

template <int BN>
struct Cfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;  // + alignment slack
  static constexpr uint32_t TMEM_COLS = 2 * BN;                    // two accumulators
  // Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A bf16 (bits 7-9 = 1),
  // B bf16 (bits 10-12 = 1), both K-major (bits 15/16 = 0), N>>3 at bit 17,
  // M>>4 at bit 24.
  static constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) |
                                    ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128");
  static_assert(TMEM_COLS <= 512, "TMEM holds 512 columns");
};

struct Params {
  GroupTable groups;
  int32_t N;        // columns of each weight matrix (rows of B per weight index)
  int32_t K;
  int32_t n_tiles;  // N / BN
  void* C;
  int64_t ldc;      // elements
  int* err;         // device error word
  // EPI_COMBINE_BF16 only: the layer's gather-combine, fused into the dense
  // branch's down projection (rows are tokens; acc is the dense output).
  const bf16* y;          // [rows picked][ldc] expert outputs
  const int32_t* dst_row; // [T][k]
  const float* wts;       // [T][k]
  const float* shared;    // [T][ldc] f32 shared-expert output, nullable
  int32_t k;
  // Expert parallelism over peer memory (EPI_STORE_BF16): when out_rank is
  // set, the output rows of group g go to rank out_rank[g]'s buffer
  // out_peer[out_rank[g]] (mapped into this process) at row + out_shift[g],
  // instead of to C.
  const int32_t* out_rank;
  const int32_t* out_shift;
  void* out_peer[8];
  // EPI_STORE_BF16: when set, output row of the tile's row r is out_rowmap[r]
  // (the token-major row t*k + slot of the pick that row holds) instead of
  // r + shift, so the combine finds each token's k rows side by side.
  const int32_t* out_rowmap;
  // EPI_COMBINE_BF16: y is token-major (pick (t, i) at row t*k + i) and
  // dst_row is not read.
  int32_t y_token_major;
  // Rows of the output buffer(s) and of y, for the bounds checks of the debug
  // build (0: unchecked).
  int64_t out_rows;
  int64_t y_rows;
};

// Output base and row shift of the tile's group.
__device__ __forceinline__ void tile_output(const Params& p, int32_t g, void** C, int32_t* shift) {
  if (p.out_rank) {
    *C = p.out_peer[__ldg(p.out_rank + g)];
    *shift = __ldg(p.out_shift + g);
  } else {
    *C = p.C;
    *shift = 0;
  }
}

// ---------------------------------------------------------------- PTX helpers

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// The same test with a suspend-time hint: the thread sleeps in the wait until
// the phase completes or about 20 us pass, instead of taking issue slots from
// the producer and MMA threads while it polls.  Used by the epilogue warps,
// which wait a whole tile's mainloop for each accumulator.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns
// false (after recording `code` in *err, when err is not null) if the CTA is
// aborting or the limit passed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long start = clock64();
  while (true) {
    if (code == DEV_TIMEOUT_EPILOGUE ? mbar_try_wait_sleep(bar, parity) : mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - start > kWaitLimitCycles) {
      *abort_flag = 1;
      if (err) atomicCAS(err, 0, code);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                            int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar)), "r"(x), "r"(y)
      : "memory");
}

// Bring a tile into L2 ahead of its TMA load (no shared memory, no barrier).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Shared-memory matrix descriptor for a K-major operand laid out by TMA with
// 128-byte swizzle: rows of 128 bytes, 8-row atoms 1024 bytes apart (SBO),
// LBO unused for swizzled K-major (encoded 1), version 1 (bit 46),
// layout SWIZZLE_128B (2 at bits 61-63).  The atom base must be 1024-aligned.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 lanes x 32 consecutive f32 columns: thread i of the warp gets lane
// (base lane + i), columns col .. col+31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- epilogue

// Activation of one 32-column chunk of a row, packed to BF16 pairs.
template <int EPI>
__device__ __forceinline__ void activate_chunk32(const uint32_t (&v)[32], const uint32_t (&u)[32],
                                                 uint32_t (&p)[16]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    float a = __uint_as_float(v[2 * j]), b = __uint_as_float(v[2 * j + 1]);
    if constexpr (EPI == EPI_SWIGLU_BF16) {
      a = __fmul_rn(act_silu_bf16out(a), __uint_as_float(u[2 * j]));
      b = __fmul_rn(act_silu_bf16out(b), __uint_as_float(u[2 * j + 1]));
    } else if constexpr (EPI == EPI_GEGLU_BF16) {
      a = __fmul_rn(act_gelu_tanh_bf16out(a), __uint_as_float(u[2 * j]));
      b = __fmul_rn(act_gelu_tanh_bf16out(b), __uint_as_float(u[2 * j + 1]));
    }
    p[j] = pack_bf16(a, b);
  }
}

// One thread writes its row's 32 BF16 values (64 bytes) straight to global.
__device__ __forceinline__ void write_chunk32_direct(void* C, int64_t ldc, int row, int col, const uint32_t (&p)[16]) {
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(C) + (int64_t)row * ldc + col);
#pragma unroll
  for (int j = 0; j < 4; ++j) dst[j] = make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
}

// Warp-collective write of a 32-row x 32-column BF16 chunk (lane i holds row
// row0 + i): the rows pass through a 2 KB shared-memory buffer (16-byte
// pieces XOR-swizzled by (row >> 1) & 3, so both the row-wise writes and the
// piece-wise reads are free of bank conflicts) and leave as 16-byte stores in
// which 4 consecutive lanes cover one row's 64 bytes, 8 rows per instruction,
// instead of 32 rows per instruction.  Rows >= rows_valid are not written.
__device__ __forceinline__ void write_chunk32_staged(void* C, int64_t ldc, int row0, int rows_valid, int col,
                                                     const uint32_t (&p)[16], uint8_t* stage, int lane) {
  const int sw = (lane >> 1) & 3;
#pragma unroll
  for (int j = 0; j < 4; ++j)
    *reinterpret_cast<uint4*>(stage + lane * 64 + ((j ^ sw) << 4)) =
        make_uint4(p[4 * j], p[4 * j + 1], p[4 * j + 2], p[4 * j + 3]);
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int piece = lane + 32 * j;
    const int r = piece >> 2, part = piece & 3;
    const uint4 v = *reinterpret_cast<const uint4*>(stage + r * 64 + ((part ^ ((r >> 1) & 3)) << 4));
    if (r < rows_valid)
      *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(C) + (int64_t)(row0 + r) * ldc + col + part * 8) = v;
  }
  __syncwarp();  // the buffer is reused by the next chunk
}

// The same for a 32-row x 64-column chunk (lane i holds row row0 + i: p0 =
// columns col..col+31, p1 = col+32..col+63) through a 4 KB buffer: 8
// consecutive lanes store one row's 128 bytes, whole 128-byte lines, 4 rows
// per instruction.  For rows that cross NVLink to another GPU whole lines
// travel in fewer, fuller packets than 64-byte pieces.
__device__ __forceinline__ void write_chunk64_staged(void* C, int64_t ldc, int row0, int rows_valid, int col,
                                                     const uint32_t (&p0)[16], const uint32_t (&p1)[16],
                                                     uint8_t* stage, int lane) {
  const int sw = lane & 7;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    *reinterpret_cast<uint4*>(stage + lane * 128 + ((j ^ sw) << 4)) =
        make_uint4(p0[4 * j], p0[4 * j + 1], p0[4 * j + 2], p0[4 * j + 3]);
    *reinterpret_cast<uint4*>(stage + lane * 128 + (((j + 4) ^ sw) << 4)) =
        make_uint4(p1[4 * j], p1[4 * j + 1], p1[4 * j + 2], p1[4 * j + 3]);
  }
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int piece = lane + 32 * j;
    const int r = piece >> 3, part = piece & 7;
    const uint4 v = *reinterpret_cast<const uint4*>(stage + r * 128 + ((part ^ (r & 7)) << 4));
    if (r < rows_valid)
      *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(C) + (int64_t)(row0 + r) * ldc + col + part * 8) = v;
  }
  __syncwarp();  // the buffer is reused by the next chunk
}

// write_chunk64_staged with a row map: lane i's row (tile row row0 + i)
// leaves at output row myrow (-1: not written).  Each 128-byte piece takes
// its row from the lane that holds it.
__device__ __forceinline__ void write_chunk64_staged_mapped(void* C, int64_t ldc, int32_t myrow, int col,
                                                            const uint32_t (&p0)[16], const uint32_t (&p1)[16],
                                                            uint8_t* stage, int lane) {
  // myrow < 0: not written (a row past the tile's end, or one that failed a bounds check)
  const int sw = lane & 7;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    *reinterpret_cast<uint4*>(stage + lane * 128 + ((j ^ sw) << 4)) =
        make_uint4(p0[4 * j], p0[4 * j + 1], p0[4 * j + 2], p0[4 * j + 3]);
    *reinterpret_cast<uint4*>(stage + lane * 128 + (((j + 4) ^ sw) << 4)) =
        make_uint4(p1[4 * j], p1[4 * j + 1], p1[4 * j + 2], p1[4 * j + 3]);
  }
  __syncwarp();
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int piece = lane + 32 * j;
    const int r = piece >> 3, part = piece & 7;
    const int32_t orow = __shfl_sync(0xffffffffu, myrow, r);
    const uint4 v = *reinterpret_cast<const uint4*>(stage + r * 128 + ((part ^ (r & 7)) << 4));
    if (orow >= 0)
      *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(C) + (int64_t)orow * ldc + col + part * 8) = v;
  }
  __syncwarp();  // the buffer is reused by the next chunk
}

template <int EPI>
__device__ __forceinline__ void store_chunk32(void* C, int64_t ldc, int row, int col, const uint32_t (&v)[32],
                                              const uint32_t (&u)[32]) {
  if constexpr (EPI == EPI_STORE_F32) {
    float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(C) + (int64_t)row * ldc + col);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      dst[j] = make_float4(__uint_as_float(v[4 * j]), __uint_as_float(v[4 * j + 1]),
                           __uint_as_float(v[4 * j + 2]), __uint_as_float(v[4 * j + 3]));
  } else {
    uint32_t p[16];
    activate_chunk32<EPI>(v, u, p);
    write_chunk32_direct(C, ldc, row, col, p);
  }
}

// One 32-byte read-only load (a 256-bit vector load: half the instructions,
// and so half the L1 wavefronts, of 16-byte loads when the lanes' addresses
// fall in different rows).  p must be 32-byte aligned.
__device__ __forceinline__ void ldg256(const void* p, uint32_t (&r)[8]) {
  asm volatile("ld.global.nc.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "l"(p));
}

// The expert part of one 32-column chunk of the fused combine for token row
// `row`: moe = sum_i w_i * y_i in rank order from zero, each multiply and add
// rounded separately (moe.rs:159-165), then + shared (moe.rs:168-173).  Runs
// before the chunk's accumulator is read, so only these registers are live
// while the gathers are in flight.
__device__ __forceinline__ void combine_moe32(const Params& p, int row, int col, bool valid, const int32_t (&dst)[8],
                                              const float (&wv)[8], float (&moe)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) moe[j] = 0.f;
  if (!valid) return;
  // picks in pairs: both picks' loads are issued before either is used, so a
  // chunk waits for memory once per pair (batches of 4 spill at the 168
  // registers that 10 warps leave a thread, and measured slower)
  constexpr int KB = 2;
#pragma unroll
  for (int i0 = 0; i0 < 8; i0 += KB) {
    if (i0 < p.k) {
      uint32_t yv[KB][16];
#pragma unroll
      for (int b = 0; b < KB; ++b) {
        if (i0 + b < p.k) {
          const bf16* yp = p.y + (int64_t)dst[i0 + b] * p.ldc + col;
          ldg256(yp, *reinterpret_cast<uint32_t(*)[8]>(&yv[b][0]));
          ldg256(yp + 16, *reinterpret_cast<uint32_t(*)[8]>(&yv[b][8]));
        }
      }
#pragma unroll
      for (int b = 0; b < KB; ++b) {
        if (i0 + b < p.k) {
          const float wi = wv[i0 + b];
#pragma unroll
          for (int r = 0; r < 16; ++r) {
            moe[2 * r] = __fadd_rn(moe[2 * r], __fmul_rn(wi, bf16_lo(yv[b][r])));
            moe[2 * r + 1] = __fadd_rn(moe[2 * r + 1], __fmul_rn(wi, bf16_hi(yv[b][r])));
          }
        }
      }
    }
  }
  if (p.shared) {
    const float* sp = p.shared + (int64_t)row * p.ldc + col;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t v[8];
      ldg256(sp + 8 * q, v);
#pragma unroll
      for (int r = 0; r < 8; ++r) moe[8 * q + r] = __fadd_rn(moe[8 * q + r], __uint_as_float(v[r]));
    }
  }
}

// out = (dense + moe) * (1/sqrt 2) as BF16 pairs (parallel_ffn.rs:32-35).
__device__ __forceinline__ void combine_finish32(const uint32_t (&acc)[32], const float (&moe)[32],
                                                 uint32_t (&o)[16]) {
  const float inv_sqrt2 = 0x1.6a09e6p-1f;  // 1.0f32 / 2.0f32.sqrt()
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float a = __fmul_rn(__fadd_rn(__uint_as_float(acc[2 * j]), moe[2 * j]), inv_sqrt2);
    const float b = __fmul_rn(__fadd_rn(__uint_as_float(acc[2 * j + 1]), moe[2 * j + 1]), inv_sqrt2);
    o[j] = pack_bf16(a, b);
  }
}

// Epilogue of one accumulator tile, run by one epilogue warp: TMEM lanes
// 32*q .. +31 (the tile's rows row0 + 32*q + lane), column half `part`.
// With `stage` (4 KB of shared memory for this warp) BF16 outputs leave
// through write_chunk32_staged (write_chunk64_staged for the plain store);
// without it each thread stores its own row.
// The fused combine's per-token inputs for one epilogue warp's rows of a
// tile: each pick's row of y and weight, and an L2 prefetch of the warp's
// column range of those rows.  The epilogue calls it before it waits for the
// tile's accumulator, so the gathers of y overlap the tile's MMAs and the
// chunk loop finds them in L2.
template <int BN, int PARTS = EPI_PARTS>
__device__ __forceinline__ void combine_prepare(const Params& p, int32_t row0, int32_t rows, int32_t nt, int q,
                                                int part, int lane, int32_t (&dst)[8], float (&wv)[8]) {
  constexpr int SPAN = BN / PARTS;
  const int row_in_tile = q * 32 + lane;
  const bool valid = row_in_tile < rows;
  const int row = row0 + row_in_tile;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    dst[i] = 0;
    wv[i] = 0.f;
    if (valid && i < p.k) {
      dst[i] = p.y_token_major ? row * p.k + i : __ldg(p.dst_row + (int64_t)row * p.k + i);
      wv[i] = __ldg(p.wts + (int64_t)row * p.k + i);
      if (!in_bounds(p.y_rows == 0 || (dst[i] >= 0 && dst[i] < p.y_rows), p.err)) {
        dst[i] = 0;
        wv[i] = 0.f;
      }
    }
  }
  if (valid) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < p.k) {
        const char* yrow = reinterpret_cast<const char*>(p.y + (int64_t)dst[i] * p.ldc + nt * BN + part * SPAN);
#pragma unroll
        for (int off = 0; off < SPAN * 2; off += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(yrow + off));
      }
    }
  }
}

// Outputs go to rows + shift of C (the combine reads its inputs at the
// unshifted rows).  cdst / cwv: the combine's inputs from combine_prepare.
template <int BN, int EPI, int PARTS = EPI_PARTS>
__device__ __forceinline__ void epilogue_tile(const Params& p, void* C, int32_t shift, uint32_t t_base, int32_t row0,
                                              int32_t rows, int32_t nt, int q, int part, int lane, uint8_t* stage,
                                              const int32_t (&cdst)[8], const float (&cwv)[8]) {
  const int row_in_tile = q * 32 + lane;
  const bool valid = row_in_tile < rows;
  const int row = row0 + row_in_tile;
  const int orow = row + shift;
  const int wrow0 = row0 + q * 32 + shift;
  const int wrows = max(0, min(32, rows - q * 32));
  // the tile rows this warp writes (the row-mapped store checks its own rows)
  const bool rows_ok =
      in_bounds(p.out_rows == 0 || p.out_rowmap != nullptr || wrows == 0 || (wrow0 >= 0 && wrow0 + wrows <= p.out_rows),
                lane == 0 ? p.err : nullptr);
  if constexpr (epi_gated(EPI)) {
    constexpr int HALF = BN / 2;
    constexpr int SPAN = HALF / PARTS;
#pragma unroll 1
    for (int c = part * SPAN; c < (part + 1) * SPAN; c += 32) {
      uint32_t g[32], u[32];
      tmem_ld32(t_base + c, g);
      tmem_ld32(t_base + HALF + c, u);
      tmem_ld_wait();
      uint32_t pk[16];
      activate_chunk32<EPI>(g, u, pk);
      if (!rows_ok) continue;
      if (stage) write_chunk32_staged(C, p.ldc, wrow0, wrows, nt * HALF + c, pk, stage, lane);
      else if (valid) write_chunk32_direct(C, p.ldc, orow, nt * HALF + c, pk);
    }
  } else if constexpr (EPI == EPI_COMBINE_BF16) {
    constexpr int SPAN = BN / PARTS;
#pragma unroll 1
    for (int c = part * SPAN; c < (part + 1) * SPAN; c += 32) {
      float moe[32];
      combine_moe32(p, row, nt * BN + c, valid, cdst, cwv, moe);
      uint32_t g[32];
      tmem_ld32(t_base + c, g);
      tmem_ld_wait();
      uint32_t pk[16];
      combine_finish32(g, moe, pk);
      if (!rows_ok) continue;
      if (stage) write_chunk32_staged(C, p.ldc, wrow0, wrows, nt * BN + c, pk, stage, lane);
      else if (valid) write_chunk32_direct(C, p.ldc, orow, nt * BN + c, pk);
    }
  } else {
    constexpr int SPAN = BN / PARTS;
    if constexpr (EPI == EPI_STORE_BF16) {
      if (stage) {
        int32_t myrow = !valid ? -1 : (p.out_rowmap ? __ldg(p.out_rowmap + row) : orow);
        if (myrow >= 0 && !in_bounds(p.out_rows == 0 || myrow < p.out_rows, p.err)) myrow = -1;
#pragma unroll 1
        for (int c = part * SPAN; c < (part + 1) * SPAN; c += 64) {
          uint32_t g0[32], g1[32];
          tmem_ld32(t_base + c, g0);
          tmem_ld32(t_base + c + 32, g1);
          tmem_ld_wait();
          uint32_t pk0[16], pk1[16];
          activate_chunk32<EPI>(g0, g0, pk0);
          activate_chunk32<EPI>(g1, g1, pk1);
          if (p.out_rowmap) write_chunk64_staged_mapped(C, p.ldc, myrow, nt * BN + c, pk0, pk1, stage, lane);
          else if (rows_ok) write_chunk64_staged(C, p.ldc, wrow0, wrows, nt * BN + c, pk0, pk1, stage, lane);
        }
        return;
      }
    }
    // the plain BF16 store may send rows through the row map (token-major y)
    const int32_t orow_m = (EPI == EPI_STORE_BF16 && p.out_rowmap && valid) ? __ldg(p.out_rowmap + row) : orow;
#pragma unroll 1
    for (int c = part * SPAN; c < (part + 1) * SPAN; c += 32) {
      uint32_t g[32];
      tmem_ld32(t_base + c, g);
      tmem_ld_wait();
      if constexpr (EPI == EPI_STORE_F32) {
        if (valid && rows_ok) store_chunk32<EPI>(C, p.ldc, orow, nt * BN + c, g, g);
      } else {
        uint32_t pk[16];
        activate_chunk32<EPI>(g, g, pk);
        if (stage) {
          if (rows_ok) write_chunk32_staged(C, p.ldc, wrow0, wrows, nt * BN + c, pk, stage, lane);
        } else if (valid && in_bounds(p.out_rows == 0 || (orow_m >= 0 && orow_m < p.out_rows), p.err)) {
          write_chunk32_direct(C, p.ldc, orow_m, nt * BN + c, pk);
        }
      }
    }
  }
}

// ---------------------------------------------------------------- kernel

template <int BN, int EPI>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const Params p) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;                        // STAGES x A_BYTES
  uint8_t* smB = smem + STAGES * C::A_BYTES;  // STAGES x B_BYTES

  __shared__ __align__(8) uint64_t full_bar[STAGES];
  __shared__ __align__(8) uint64_t empty_bar[STAGES];
  __shared__ __align__(8) uint64_t accf_bar[2];
  __shared__ __align__(8) uint64_t acce_bar[2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf_bar[a], 1);
      mbar_init(&acce_bar[a], EPI_WARPS);  // one arrive per epilogue warp
    }
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_slot)),
                 "r"(C::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;

  __shared__ int32_t s_tab[3 * (kSmemGroups + 1)];
  const GroupTable groups = stage_group_table(p.groups, s_tab);
  const int32_t total_tiles = group_total_mtiles(groups, BM) * p.n_tiles;
  const int32_t num_kb = (p.K + BK - 1) / BK;

  if (warp == 0) {
    if (lane == 0) {
    // ---------------- TMA producer
    int stage = 0;
    uint32_t phase = 0;
    for (int32_t tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
      const TileCoord tc = decode_tile(groups, tile, p.n_tiles, BM);
      const int32_t brow = tc.widx * p.N + tc.nt * BN;
      bool ok = true;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, &abort_flag, p.err, DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full_bar[stage], C::STAGE_BYTES);
        tma_load_2d(smA + stage * C::A_BYTES, &tmA, &full_bar[stage], kb * BK, tc.row0);
        tma_load_2d(smB + stage * C::B_BYTES, &tmB, &full_bar[stage], kb * BK, brow);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
    }
    }
    __syncwarp();  // lanes 1..31 wait here so the warp reaches the block barrier converged
  } else if (warp == 1) {
    if (lane == 0) {
    // ---------------- MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool issued = false;
    for (int32_t tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
      if (!mbar_wait(&acce_bar[acc], acc_phase ^ 1u, &abort_flag, p.err, DEV_TIMEOUT_MMA)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
      bool ok = true;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&full_bar[stage], phase, &abort_flag, p.err, DEV_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_addr(smA + stage * C::A_BYTES);
        const uint32_t b0 = smem_addr(smB + stage * C::B_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          // advance 16 bf16 (32 bytes) along K inside the 128-byte swizzle row
          umma_bf16(d_tmem, sdesc_sw128(a0 + kk * 32), sdesc_sw128(b0 + kk * 32), C::IDESC,
                    (kb | kk) != 0 ? 1u : 0u);
        }
        issued = true;
        umma_commit(&empty_bar[stage]);  // frees the smem stage once these MMAs retire
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      umma_commit(&accf_bar[acc]);  // accumulator ready for the epilogue
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (issued) {
      // Retire every MMA this thread issued before TMEM is released.
      umma_commit(&drain_bar);
      const long long start = clock64();
      while (!mbar_try_wait(&drain_bar, 0) && clock64() - start < kWaitLimitCycles) {
      }
    }
    }
    __syncwarp();
  } else if (warp >= 2) {
    // ---------------- epilogue: warp w owns TMEM lanes 32*(w%4) .. +31 and
    // one half of the tile's columns
    const int q = warp & 3;
    const int part = (warp - 2) >> 2;  // which 1/EPI_PARTS of the columns
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int32_t tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
      const TileCoord tc = decode_tile(groups, tile, p.n_tiles, BM);
      int32_t cdst[8];
      float cwv[8];
      if constexpr (EPI == EPI_COMBINE_BF16) combine_prepare<BN>(p, tc.row0, tc.rows, tc.nt, q, part, lane, cdst, cwv);
      if (!mbar_wait(&accf_bar[acc], acc_phase, &abort_flag, p.err, DEV_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const uint32_t t_base = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      void* Ct;
      int32_t shift;
      tile_output(p, tc.g, &Ct, &shift);
      epilogue_tile<BN, EPI>(p, Ct, shift, t_base, tc.row0, tc.rows, tc.nt, q, part, lane, nullptr, cdst, cwv);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce_bar[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (p.out_rank) __threadfence_system();  // peer stores land before the next barrier signals
  }

  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(C::TMEM_COLS)
                 : "memory");
  }
#endif
}

// ---------------------------------------------------------------- 2-CTA kernel
//
// The same GEMM on an SM pair (a cluster of two CTAs): one tcgen05.mma
// .cta_group::2 computes a 256 x 256 x 16 tile, M split across the pair.
// CTA r loads, with its own TMA copies, A rows [row0 + 128r, +128) and B rows
// [n0 + 128r, +128) of the 256-column n-tile; the pair's MMA multiplies each
// CTA's A half by both B halves, so each SM reads 8 KB of shared memory per
// k16 step instead of 12 KB, for the same FLOPs.  Each CTA's TMEM holds its
// own 128 x 256 accumulator rows, so the epilogue is the one-CTA epilogue.
//
// Synchronisation: both CTAs' TMA copies complete on the leader's (CTA 0)
// full barrier; the leader alone issues MMAs and commits to the empty and
// accumulator-full barriers of both CTAs; both CTAs' epilogue warps arrive on
// the leader's accumulator-empty barrier.  Tiles are 256 rows: the group
// table's tile numbering must use BM2 = 256.
constexpr int BM2 = 256;
// Operand ring depth requested (build-time; each stage is 32 KB a CTA) and
// how many k-blocks ahead the producer prefetches its tiles into L2 (0: off).
#ifndef NOOR_GEMM_STAGES
#define NOOR_GEMM_STAGES 5
#endif
#ifndef NOOR_GEMM_PREFETCH_KB
#define NOOR_GEMM_PREFETCH_KB 0
#endif
constexpr int kMaxStages2 = 8;
constexpr int kPrefetchKB = NOOR_GEMM_PREFETCH_KB;
constexpr int kSmemLimit = 227 * 1024;
constexpr int kStaticSmemMargin = 4096;  // group table, barriers

template <int EPI>
struct Cfg2 {
  static constexpr int WARPS = EPI == EPI_COMBINE_BF16 ? EPI_WARPS : NOOR_GEMM_EPI_WARPS_PLAIN;  // epilogue warps
  static constexpr int PARTS = WARPS / 4;
  static_assert(WARPS % 4 == 0 && (PARTS == 1 || PARTS == 2 || PARTS == 4), "epilogue warps");
  static constexpr int THREADS = 64 + 32 * WARPS;
  static constexpr int A_BYTES = 128 * BK * 2;  // this CTA's A half
  static constexpr int B_BYTES = 128 * BK * 2;  // this CTA's B half
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // per epilogue warp: 4 KB for write_chunk64_staged (plain store), else 2 KB
  // for write_chunk32_staged (less shared memory leaves more L1 for the
  // combine's gathers)
  static constexpr int STAGE_OUT_BYTES = EPI == EPI_STORE_BF16 ? 4096 : 2048;
  // the requested depth, or as many stages as fit beside the output staging
  static constexpr int FIT = (kSmemLimit - kStaticSmemMargin - WARPS * STAGE_OUT_BYTES - 1024) / STAGE_BYTES;
  static constexpr int STAGES = NOOR_GEMM_STAGES < FIT ? NOOR_GEMM_STAGES : FIT;
  static_assert(STAGES >= 2 && STAGES <= kMaxStages2, "operand ring depth");
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + WARPS * STAGE_OUT_BYTES + 1024;
  static constexpr uint32_t TMEM_COLS = 512;  // two 256-column accumulators
  static constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(256 >> 3) << 17) |
                                    ((uint32_t)(256 >> 4) << 24);
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// TMA load into this CTA's shared memory whose completion is counted on the
// leader CTA's barrier (clearing the peer bit of the barrier's address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                                 int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_addr(bar) & 0xFEFFFFFFu), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the barrier at this smem offset in both CTAs of the pair once the
// MMAs issued so far retire.
__device__ __forceinline__ void umma_commit_pair_both(uint64_t* bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_addr(bar)),
      "h"(mask)
      : "memory");
}

__device__ __forceinline__ void umma_commit_pair_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

// Arrive on the barrier at this smem offset in CTA `rank` of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t* bar, uint32_t rank) {
  asm volatile(
      "{\n\t.reg .b32 remAddr32;\n\t"
      "mapa.shared::cluster.u32 remAddr32, %0, %1;\n\t"
      "mbarrier.arrive.shared::cluster.b64 _, [remAddr32];\n\t}" ::"r"(smem_addr(bar)),
      "r"(rank)
      : "memory");
}

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Cfg2<EPI>::THREADS, 1)
    grouped_gemm_2cta_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                             const Params p) {
#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ >= 1000)
  using C = Cfg2<EPI>;
  constexpr int BN = 256;
  constexpr int STAGES2 = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smA = smem;
  uint8_t* smB = smem + STAGES2 * C::A_BYTES;
  uint8_t* smOut = smem + STAGES2 * C::STAGE_BYTES;  // C::WARPS x STAGE_OUT_BYTES

  __shared__ __align__(8) uint64_t full_bar[kMaxStages2];
  __shared__ __align__(8) uint64_t empty_bar[kMaxStages2];
  __shared__ __align__(8) uint64_t accf_bar[2];
  __shared__ __align__(8) uint64_t acce_bar[2];
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES2; ++s) {
      mbar_init(&full_bar[s], 1);   // the leader's expect_tx; both CTAs' bytes
      mbar_init(&empty_bar[s], 1);  // the leader's commit, delivered to both CTAs
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&accf_bar[a], 1);
      mbar_init(&acce_bar[a], 2 * C::WARPS);  // epilogue warps of both CTAs (leader's copy is used)
    }
    mbar_init(&drain_bar, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&tmem_slot)),
                 "r"(C::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the peer's barriers exist before anyone signals them
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;

  const int32_t nclusters = gridDim.x >> 1;
  const int32_t cid = blockIdx.x >> 1;
  __shared__ int32_t s_tab[3 * (kSmemGroups + 1)];
  const GroupTable groups = stage_group_table(p.groups, s_tab);
  const int32_t total_tiles = group_total_mtiles(groups, BM2) * p.n_tiles;
  const int32_t num_kb = (p.K + BK - 1) / BK;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer (both CTAs)
      int stage = 0;
      uint32_t phase = 0;
      for (int32_t tile = cid; tile < total_tiles; tile += nclusters) {
        const TileCoord tc = decode_tile(groups, tile, p.n_tiles, BM2);
        const int32_t arow = tc.row0 + 128 * (int32_t)rank;
        const int32_t brow = tc.widx * p.N + tc.nt * BN + 128 * (int32_t)rank;
        // L2 prefetch cursor kPrefetchKB k-blocks ahead, into the next tile
        [[maybe_unused]] int32_t next_arow = -1, next_brow = 0;
        if constexpr (kPrefetchKB > 0) {
          if (tile + nclusters < total_tiles) {
            const TileCoord nc = decode_tile(groups, tile + nclusters, p.n_tiles, BM2);
            next_arow = nc.row0 + 128 * (int32_t)rank;
            next_brow = nc.widx * p.N + nc.nt * BN + 128 * (int32_t)rank;
          }
        }
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if constexpr (kPrefetchKB > 0) {
            const int pkb = kb + kPrefetchKB;
            if (pkb < num_kb) {
              tma_prefetch_l2_2d(&tmA, pkb * BK, arow);
              tma_prefetch_l2_2d(&tmB, pkb * BK, brow);
            } else if (next_arow >= 0 && pkb - num_kb < num_kb) {
              tma_prefetch_l2_2d(&tmA, (pkb - num_kb) * BK, next_arow);
              tma_prefetch_l2_2d(&tmB, (pkb - num_kb) * BK, next_brow);
            }
          }
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, &abort_flag, p.err, DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(&full_bar[stage], 2 * C::STAGE_BYTES);
          tma_load_2d_pair(smA + stage * C::A_BYTES, &tmA, &full_bar[stage], kb * BK, arow);
          tma_load_2d_pair(smB + stage * C::B_BYTES, &tmB, &full_bar[stage], kb * BK, brow);
          if (++stage == STAGES2) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (leader CTA only)
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool issued = false;
      for (int32_t tile = cid; tile < total_tiles; tile += nclusters) {
        if (!mbar_wait(&acce_bar[acc], acc_phase ^ 1u, &abort_flag, p.err, DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, &abort_flag, p.err, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_addr(smA + stage * C::A_BYTES);
          const uint32_t b0 = smem_addr(smB + stage * C::B_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_bf16_pair(d_tmem, sdesc_sw128(a0 + kk * 32), sdesc_sw128(b0 + kk * 32), C::IDESC,
                           (kb | kk) != 0 ? 1u : 0u);
          issued = true;
          umma_commit_pair_both(&empty_bar[stage]);
          if (++stage == STAGES2) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair_both(&accf_bar[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (issued) {
        umma_commit_pair_local(&drain_bar);
        const long long start = clock64();
        while (!mbar_try_wait(&drain_bar, 0) && clock64() - start < kWaitLimitCycles) {
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (both CTAs): this CTA's 128 rows of the pair tile
    const int q = warp & 3;
    const int part = (warp - 2) >> 2;  // which 1/C::PARTS of the columns
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int32_t tile = cid; tile < total_tiles; tile += nclusters) {
      const TileCoord tc = decode_tile(groups, tile, p.n_tiles, BM2);
      const int32_t row0 = tc.row0 + 128 * (int32_t)rank, rows = tc.rows - 128 * (int32_t)rank;
      int32_t cdst[8];
      float cwv[8];
      if constexpr (EPI == EPI_COMBINE_BF16) combine_prepare<BN, C::PARTS>(p, row0, rows, tc.nt, q, part, lane, cdst, cwv);
      if (!mbar_wait(&accf_bar[acc], acc_phase, &abort_flag, p.err, DEV_TIMEOUT_EPILOGUE)) break;
      tc_fence_after();
      const uint32_t t_base = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      void* Ct;
      int32_t shift;
      tile_output(p, tc.g, &Ct, &shift);
      epilogue_tile<BN, EPI, C::PARTS>(p, Ct, shift, t_base, row0, rows, tc.nt, q, part, lane,
                                       smOut + (warp - 2) * C::STAGE_OUT_BYTES, cdst, cwv);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader) mbar_arrive(&acce_bar[acc]);
        else mbar_arrive_cluster(&acce_bar[acc], 0);
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (p.out_rank) __threadfence_system();  // peer stores land before the next barrier signals
  }

  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its peer may still signal it
  if (warp == 0) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(C::TMEM_COLS)
                 : "memory");
  }
#endif
}

}  // namespace tc
}  // namespace noor
