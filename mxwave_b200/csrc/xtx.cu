// K3: full X^T X of bf16 calibration activations on the tcgen05 tensor cores.
//
// G[i, j] += sum_n X[n, i] * X[n, j] for X [tokens, cols] row-major bf16.  As a
// GEMM, M = N = cols and the reduction runs over tokens; both operands are
// slices of X whose contiguous dimension is the output (MN) dimension, so they
// are consumed "MN-major" straight from the TMA tiles -- no transpose pass.
//
// CTA tile 128 (i) x 256 (j), 64 tokens per pipeline stage:
//   warp 0      TMA producer: A = X[n0:n0+64, i0:i0+128] (2 boxes of 64x64),
//               B = X[n0:n0+64, j0:j0+256] (4 boxes), 128-byte swizzle
//   warp 1      TMEM owner + single-thread tcgen05.mma issuer
//               (kind::f16, bf16 x bf16 -> fp32, M=128 N=256 K=16, 4 per stage)
//   warps 2..9  epilogue: each owns 32 TMEM lanes (rows) x 128 columns
// Symmetry: G is symmetric, so only the tiles that reach the upper triangle
// (column >= row somewhere in the tile) are computed -- 420 of 800 tiles at
// 5120 channels.  A tile adds its entries with column >= row to G and the
// transpose of those with column > row below the diagonal; for one column the
// transposed entries are consecutive rows, so each warp's stores stay
// coalesced.  Every entry of G is written by exactly one tile.
// Accuracy: the tensor core's fp32 accumulation is not round-to-nearest (its
// error grows with the number of K steps in one accumulator).  So tokens are
// accumulated in chunks of 1024 (64 K steps) in one of two TMEM buffers (2 x
// 256 columns); while the MMA warp fills one buffer, the epilogue warps add the
// other into round-to-nearest fp32 totals held in registers.  The totals are
// added into the caller's Gram once, at the end.  Measured on B200 against a
// float64 Gram (max |G - G64| / sqrt(G64_ii G64_jj), heavy-channel bf16
// activations): 1.2e-6 with 256-token chunks, 2.7-3.2e-6 with 1024 (65,536 and
// 262,144 tokens), 6e-6 with 2048; 1024 is as fast as 4096 (each chunk
// boundary costs a TMEM drain and a buffer hand-off) and ~10 % faster than 256.
// Shared-memory descriptors (MN-major, SWIZZLE_128B): the 16-byte-unit layout
// is ((8, n), (8, k)) : ((1, LBO), (8, SBO)) -- 64 contiguous channels per
// 128-byte row, LBO = bytes between 64-channel boxes, SBO = 1024 bytes
// between groups of 8 tokens.
#include <cuda.h>
#include <cuda_bf16.h>

#include <cooperative_groups.h>

#include "common.cuh"
#include "runtime.h"
#include "tcgen05.cuh"
#include "tma.cuh"

namespace cg = cooperative_groups;

namespace mxw {

constexpr int kXtxBM = 128;
constexpr int kXtxBN = 256;
constexpr int kXtxBK = 64;  // tokens per stage
constexpr int kXtxStages = 4;
constexpr int kXtxBoxBytes = kXtxBK * 128;                    // 64 tokens x 64 channels bf16
constexpr int kXtxABytes = (kXtxBM / 64) * kXtxBoxBytes;      // 16 KB
constexpr int kXtxBBytes = (kXtxBN / 64) * kXtxBoxBytes;      // 32 KB
constexpr int kXtxStageBytes = kXtxABytes + kXtxBBytes;       // 48 KB
constexpr int kXtxEpiWarps = 8;
constexpr int kXtxThreads = (2 + kXtxEpiWarps) * 32;
constexpr int kXtxChunkStages = 16;  // block Gram: 1024 tokens per TMEM accumulation chunk
constexpr int kXtxAccumStages = 16;  // full X^T X: 1024 tokens per TMEM accumulation chunk
constexpr uint32_t kXtxTmemCols = 512;  // two 128 x 256 fp32 accumulators
constexpr int64_t kXtxMaxTokens = 262144;  // tokens per launch

struct XtxParams {
  int64_t tokens, cols, ldg, n_kblocks;
  int64_t n_col_tiles;  // 256-column tiles per row of tiles
  float* gram;
  float* packed;  // non-null: add each tile's totals to its slot here instead of into gram
  uint32_t* flags;
};

// ------------------------------------------------------------------- kernel

constexpr int kXtxTileFloats = kXtxBM * kXtxBN;

// Tile `t` of the upper triangle, row by row: row tile `by` (128 rows) holds
// the column tiles bx >= by / 2 (256 columns each), the first that reach
// column >= row.  Returns (i0, j0), the tile's first row and column.
__device__ __forceinline__ void xtx_tile_origin(int64_t t, int64_t n_col_tiles, int64_t& i0, int64_t& j0) {
  int64_t by = 0;
  for (;; ++by) {
    const int64_t in_row = n_col_tiles - (by >> 1);
    if (t < in_row) break;
    t -= in_row;
  }
  i0 = by * kXtxBM;
  j0 = ((by >> 1) + t) * kXtxBN;
}

// Adds one thread's 128 tile totals (row i0 + 32*quarter + lane, columns
// j0 + 128*half ..) into G: the entries with column >= row in place, and the
// transposes of those with column > row.  For one column the warp's 32 rows
// are consecutive, so the transposed stores coalesce.
__device__ __forceinline__ void add_tile_rows(float* gram, int64_t ldg, int64_t cols, int64_t i0, int64_t j0,
                                              int quarter, int half, int lane, const float (&total)[128]) {
  const int64_t r = i0 + 32 * quarter + lane;  // this thread's row of G
  const int64_t cbase = j0 + 128 * half;        // its first column
  if (cbase >= cols || cbase + 127 < i0 + 32 * quarter) return;
  float* grow = gram + r * ldg + cbase;
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    const int64_t c = cbase + 4 * k;
    if (c >= r) {
      float4 o = reinterpret_cast<float4*>(grow)[k];
      o.x = __fadd_rn(o.x, total[4 * k]);
      o.y = __fadd_rn(o.y, total[4 * k + 1]);
      o.z = __fadd_rn(o.z, total[4 * k + 2]);
      o.w = __fadd_rn(o.w, total[4 * k + 3]);
      reinterpret_cast<float4*>(grow)[k] = o;
    } else if (c + 3 >= r) {
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (c + u >= r) grow[4 * k + u] = __fadd_rn(grow[4 * k + u], total[4 * k + u]);
    }
  }
#pragma unroll
  for (int k = 0; k < 128; ++k) {
    const int64_t c = cbase + k;
    if (c > r) {
      float* g = gram + c * ldg + r;
      *g = __fadd_rn(*g, total[k]);
    }
  }
}

__global__ void __launch_bounds__(kXtxThreads, 1)
    xtx_kernel(const __grid_constant__ CUtensorMap map, const XtxParams P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align_smem<1024>(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kXtxStages * kXtxStageBytes);
  uint64_t* empty = full + kXtxStages;
  uint64_t* tfull = empty + kXtxStages;  // [2] accumulator buffer ready
  uint64_t* tempty = tfull + 2;          // [2] accumulator buffer drained
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  int* fail = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Tile blockIdx.x of the upper triangle, row by row: row tile `by` (128
  // rows) holds the column tiles bx >= by / 2 (256 columns each), the first
  // that reach column >= row.
  int64_t i0, j0;
  xtx_tile_origin(blockIdx.x, P.n_col_tiles, i0, j0);
  const int64_t n_chunks = (P.n_kblocks + kXtxAccumStages - 1) / kXtxAccumStages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kXtxStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kXtxEpiWarps);
    }
    *fail = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kXtxTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&map);
      int64_t kb = 0;
      bool ok = true;
      for (; kb < P.n_kblocks; ++kb) {
        const int s = static_cast<int>(kb % kXtxStages);
        if (kb >= kXtxStages && !mbar_wait(&empty[s], static_cast<uint32_t>((kb / kXtxStages - 1) & 1))) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * kXtxStageBytes;
        const int32_t y = static_cast<int32_t>(kb * kXtxBK);
        mbar_arrive_expect_tx(&full[s], kXtxStageBytes);
#pragma unroll
        for (int q = 0; q < kXtxBM / 64; ++q)
          tma_load_2d(st + q * kXtxBoxBytes, &map, &full[s], static_cast<int32_t>(i0 + 64 * q), y);
#pragma unroll
        for (int q = 0; q < kXtxBN / 64; ++q)
          tma_load_2d(st + kXtxABytes + q * kXtxBoxBytes, &map, &full[s], static_cast<int32_t>(j0 + 64 * q), y);
      }
      for (int64_t j = (kb > kXtxStages ? kb - kXtxStages : 0); j < kb; ++j)
        if (!mbar_wait(&full[j % kXtxStages], static_cast<uint32_t>((j / kXtxStages) & 1))) ok = false;
      if (!ok) atomicOr(fail, 1);
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16_f32_mn(kXtxBM, kXtxBN);
      bool ok = true;
      int64_t kb = 0;
      int64_t c = 0;
      for (; c < n_chunks && ok; ++c) {
        const int buf = static_cast<int>(c & 1);
        if (c >= 2 && !mbar_wait(&tempty[buf], static_cast<uint32_t>((c / 2 - 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(buf * kXtxBN);
        const int64_t kb_end = (c + 1) * kXtxAccumStages < P.n_kblocks ? (c + 1) * kXtxAccumStages : P.n_kblocks;
        for (int64_t first = kb; kb < kb_end; ++kb) {
          const int s = static_cast<int>(kb % kXtxStages);
          if (!mbar_wait(&full[s], static_cast<uint32_t>((kb / kXtxStages) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + s * kXtxStageBytes);
          const uint32_t b_base = a_base + kXtxABytes;
#pragma unroll
          for (int kk = 0; kk < kXtxBK / 16; ++kk) {
            // 16 tokens = two 8-row swizzle atoms = 2048 bytes further along K.
            const uint64_t ad = make_smem_desc_mn_sw128(a_base + kk * 2048, kXtxBoxBytes, 1024);
            const uint64_t bd = make_smem_desc_mn_sw128(b_base + kk * 2048, kXtxBoxBytes, 1024);
            mma_bf16_f32(d_tmem, ad, bd, idesc, (kb > first || kk > 0) ? 1u : 0u);
          }
          mma_commit(&empty[s]);  // stage reusable once these MMAs have read it
        }
        mma_commit(&tfull[buf]);  // chunk accumulated (or nothing more in flight)
      }
      if (!ok) {
        atomicOr(fail, 1);
        // Let any epilogue warp still waiting on a chunk see it "ready" so the
        // CTA unwinds; the fail flag keeps the data from being used.
        for (; c < n_chunks; ++c) mma_commit(&tfull[c & 1]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - 2;
    const int quarter = warp & 3;     // TMEM lanes 32*quarter .. +31 (hardware rule)
    const int half = e >> 2;          // columns 128*half .. +127 of the tile
    float total[128];
#pragma unroll
    for (int k = 0; k < 128; ++k) total[k] = 0.0f;
    bool ok = true;
    for (int64_t c = 0; c < n_chunks; ++c) {
      const int buf = static_cast<int>(c & 1);
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[buf], static_cast<uint32_t>((c / 2) & 1)))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t base = tmem + (static_cast<uint32_t>(32 * quarter) << 16) +
                            static_cast<uint32_t>(buf * kXtxBN + 128 * half);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float v[16];
        tmem_ld_32x32b_x16(base + static_cast<uint32_t>(16 * q), v);
#pragma unroll
        for (int k = 0; k < 16; ++k) total[16 * q + k] = __fadd_rn(total[16 * q + k], v[k]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
    if (!ok) atomicOr(fail, 1);
    // All epilogue warps agree before writing (named barrier 1, 256 threads).
    asm volatile("bar.sync 1, 256;" ::: "memory");
    if (*reinterpret_cast<volatile int*>(fail) == 0) {
      if (P.packed) {
        // This tile's totals, row-major 128 x 256, at its place in the packed buffer.
        float4* pt = reinterpret_cast<float4*>(P.packed + static_cast<int64_t>(blockIdx.x) * kXtxTileFloats +
                                               (32 * quarter + lane) * kXtxBN + 128 * half);
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          float4 o = pt[k];
          o.x = __fadd_rn(o.x, total[4 * k]);
          o.y = __fadd_rn(o.y, total[4 * k + 1]);
          o.z = __fadd_rn(o.z, total[4 * k + 2]);
          o.w = __fadd_rn(o.w, total[4 * k + 3]);
          pt[k] = o;
        }
      } else {
        add_tile_rows(P.gram, P.ldg, P.cols, i0, j0, quarter, half, lane, total);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kXtxTmemCols);
  }
  if (threadIdx.x == 0 && *fail && P.flags) atomicOr(P.flags, MXW_FLAG_TIMEOUT);
}

// Adds packed tile totals (the layout xtx_kernel writes with P.packed) into G:
// tiles first_tile + blockIdx.x, read from packed + blockIdx.x * tile.
__global__ void __launch_bounds__(256) xtx_unpack_kernel(const float* __restrict__ packed, int64_t cols,
                                                         int64_t n_col_tiles, float* gram, int64_t ldg,
                                                         int64_t first_tile) {
  int64_t i0, j0;
  xtx_tile_origin(first_tile + blockIdx.x, n_col_tiles, i0, j0);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quarter = warp & 3, half = warp >> 2;
  const float4* src = reinterpret_cast<const float4*>(packed + static_cast<int64_t>(blockIdx.x) * kXtxTileFloats +
                                                      (32 * quarter + lane) * kXtxBN + 128 * half);
  float total[128];
#pragma unroll
  for (int k = 0; k < 32; ++k) {
    const float4 v = src[k];
    total[4 * k] = v.x;
    total[4 * k + 1] = v.y;
    total[4 * k + 2] = v.z;
    total[4 * k + 3] = v.w;
  }
  add_tile_rows(gram, ldg, cols, i0, j0, quarter, half, lane, total);
}

static int64_t xtx_tiles(int64_t cols) {
  const int64_t n_col_tiles = (cols + kXtxBN - 1) / kXtxBN;
  int64_t n = 0;
  for (int64_t by = 0; by < cols / kXtxBM; ++by) n += n_col_tiles - (by >> 1);
  return n;
}

// ------------------------------------------------ block-diagonal Gram
//
// The diagonal 32x32 blocks of X^T X (the reference's block Hessian,
// mxwave/calibration.py:233-236) on the tensor cores.  A CTA owns one strip
// of 128 channels (four 32-channel blocks) and one contiguous token slice.
// Each stage is one TMA tile X[n0:n0+64, c0:c0+128]; it is both MMA operands
// (A = B: the 128 x 128 tile X_s^T X_s, M = N = 128, K = 16 per instruction,
// 4 per stage), accumulated in TMEM in chunks of 1024 tokens (two 128-column
// buffers).  Four epilogue warps read only the diagonal 32x32 sub-blocks
// (warp quarter q: TMEM lanes 32q.., columns 32q..) and add each chunk into
// round-to-nearest fp32 totals in registers, as the full X^T X kernel does.
// The CTAs of one strip form a thread-block cluster; rank 0 sums the ranks'
// totals over distributed shared memory in rank order and adds them into the
// caller's blocks, so the result is deterministic.  The other three quarters
// of each tile's MMA work are discarded: the tensor core has far more
// throughput than this HBM-bound pass needs.

constexpr int kBgStages = 8;
constexpr int kBgStageBytes = 2 * kXtxBoxBytes;  // 64 tokens x 128 channels
constexpr int kBgThreads = 6 * 32;               // producer, MMA, 4 epilogue warps
constexpr uint32_t kBgTmemCols = 256;            // two 128 x 128 fp32 accumulators
constexpr int kBgMaxSlices = 8;

struct BgParams {
  int64_t tokens, cols;
  float* gram_blocks;
  uint32_t* flags;
};

template <bool F16>
__global__ void __launch_bounds__(kBgThreads, 1)
    block_gram_tc_kernel(const __grid_constant__ CUtensorMap map, const BgParams P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = align_smem<1024>(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBgStages * kBgStageBytes);
  uint64_t* empty = full + kBgStages;
  uint64_t* tfull = empty + kBgStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  int* fail = reinterpret_cast<int*>(tmem_slot + 1);
  // This CTA's totals for the cluster fold: [quarter][lane][32] (16 KB), in
  // stage 0 once the pipeline has drained (read by rank 0 over DSMEM).
  float* part = reinterpret_cast<float*>(smem);

  cg::cluster_group cluster = cg::this_cluster();
  const unsigned rank = cluster.block_rank();
  const unsigned nrank = cluster.num_blocks();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c0 = static_cast<int64_t>(blockIdx.x) * 128;
  const int64_t n_kb = (P.tokens + kXtxBK - 1) / kXtxBK;
  const int64_t kb_begin = n_kb * rank / nrank, kb_end = n_kb * (rank + 1) / nrank;
  const int64_t n_chunks = (kb_end - kb_begin + kXtxChunkStages - 1) / kXtxChunkStages;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kBgStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    *fail = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kBgTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  float total[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) total[k] = 0.0f;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&map);
      bool ok = true;
      int64_t i = 0;
      for (int64_t kb = kb_begin; kb < kb_end; ++kb, ++i) {
        const int s = static_cast<int>(i % kBgStages);
        if (i >= kBgStages && !mbar_wait(&empty[s], static_cast<uint32_t>((i / kBgStages - 1) & 1))) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * kBgStageBytes;
        mbar_arrive_expect_tx(&full[s], kBgStageBytes);
        tma_load_2d(st, &map, &full[s], static_cast<int32_t>(c0), static_cast<int32_t>(kb * kXtxBK));
        tma_load_2d(st + kXtxBoxBytes, &map, &full[s], static_cast<int32_t>(c0 + 64),
                    static_cast<int32_t>(kb * kXtxBK));
      }
      for (int64_t j = (i > kBgStages ? i - kBgStages : 0); j < i; ++j)
        if (!mbar_wait(&full[j % kBgStages], static_cast<uint32_t>((j / kBgStages) & 1))) ok = false;
      if (!ok) atomicOr(fail, 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_bf16_f32_mn(128, 128) & (F16 ? ~((7u << 7) | (7u << 10)) : ~0u);
      bool ok = true;
      int64_t i = 0;
      int64_t c = 0;
      for (; c < n_chunks && ok; ++c) {
        const int buf = static_cast<int>(c & 1);
        if (c >= 2 && !mbar_wait(&tempty[buf], static_cast<uint32_t>((c / 2 - 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(buf * 128);
        const int64_t i_end = std::min<int64_t>((c + 1) * kXtxChunkStages, kb_end - kb_begin);
        for (const int64_t first = i; i < i_end; ++i) {
          const int s = static_cast<int>(i % kBgStages);
          if (!mbar_wait(&full[s], static_cast<uint32_t>((i / kBgStages) & 1))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t base = smem_u32(smem + s * kBgStageBytes);
#pragma unroll
          for (int kk = 0; kk < kXtxBK / 16; ++kk) {
            const uint64_t d = make_smem_desc_mn_sw128(base + kk * 2048, kXtxBoxBytes, 1024);
            mma_bf16_f32(d_tmem, d, d, idesc, (i > first || kk > 0) ? 1u : 0u);
          }
          mma_commit(&empty[s]);
        }
        mma_commit(&tfull[buf]);
      }
      if (!ok) {
        atomicOr(fail, 1);
        for (; c < n_chunks; ++c) mma_commit(&tfull[c & 1]);
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lanes 32q.. (hardware rule) = block q of the strip
    bool ok = true;
    for (int64_t c = 0; c < n_chunks; ++c) {
      const int buf = static_cast<int>(c & 1);
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[buf], static_cast<uint32_t>((c / 2) & 1)))) {
        ok = false;
        break;
      }
      tc_fence_after();
      float v[32];
      tmem_ld_32x32b_x32(tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(buf * 128 + 32 * q), v);
#pragma unroll
      for (int k = 0; k < 32; ++k) total[k] = __fadd_rn(total[k], v[k]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
    if (!ok) atomicOr(fail, 1);
  }
  tc_fence_before();
  __syncthreads();  // the pipeline has drained: stage memory is free for the totals
  if (warp >= 2) {
    float4* dst = reinterpret_cast<float4*>(part + ((warp & 3) * 32 + lane) * 32);
#pragma unroll
    for (int k = 0; k < 8; ++k) dst[k] = make_float4(total[4 * k], total[4 * k + 1], total[4 * k + 2], total[4 * k + 3]);
  }
  // Every thread of every CTA reaches both cluster barriers once (all waits above are bounded).
  cluster_sync_all();
  if (rank == 0 && warp >= 2) {
    bool failed = false;
    for (unsigned r = 0; r < nrank; ++r) failed |= *cluster.map_shared_rank(fail, r) != 0;
    const int q = warp & 3;
    if (failed) {
      if (P.flags && lane == 0 && q == 0) atomicOr(P.flags, MXW_FLAG_TIMEOUT);
    } else {
      float sum[32];
#pragma unroll
      for (int k = 0; k < 32; ++k) sum[k] = total[k];
      for (unsigned r = 1; r < nrank; ++r) {
        const float4* src = reinterpret_cast<const float4*>(cluster.map_shared_rank(part, r) + (q * 32 + lane) * 32);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float4 o = src[k];
          sum[4 * k] = __fadd_rn(sum[4 * k], o.x);
          sum[4 * k + 1] = __fadd_rn(sum[4 * k + 1], o.y);
          sum[4 * k + 2] = __fadd_rn(sum[4 * k + 2], o.z);
          sum[4 * k + 3] = __fadd_rn(sum[4 * k + 3], o.w);
        }
      }
      float4* g = reinterpret_cast<float4*>(P.gram_blocks + ((4 * blockIdx.x + q) * 32 + lane) * 32);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float4 o = g[k];
        o.x = __fadd_rn(o.x, sum[4 * k]);
        o.y = __fadd_rn(o.y, sum[4 * k + 1]);
        o.z = __fadd_rn(o.z, sum[4 * k + 2]);
        o.w = __fadd_rn(o.w, sum[4 * k + 3]);
        g[k] = o;
      }
    }
  }
  cluster_sync_all();  // keep every rank's totals alive until rank 0 has read them
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kBgTmemCols);
  }
}

// Token slices per strip: enough CTAs to cover the SMs, at least 16 K-blocks
// (1024 tokens) per slice.
static int bg_slices(int64_t strips, int64_t kblocks) {
  int s = static_cast<int>(std::max<int64_t>(1, num_sms() / std::max<int64_t>(strips, 1)));
  s = std::min<int>(s, kBgMaxSlices);
  while (s > 1 && kblocks / s < 16) --s;
  return s;
}

// Launches block_gram_tc_kernel for 2-byte activations whose layout suits TMA
// and the 128-channel strips; returns MXW_EUNSUPPORTED otherwise (the caller
// then uses the CUDA-core statistics kernel).
int accumulate_block_gram_tc(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ld,
                             float* gram_blocks, uint32_t* flags, cudaStream_t stream) {
  if ((dtype != MXW_BF16 && dtype != MXW_F16) || cols % 128 != 0 || ld % 8 != 0 ||
      reinterpret_cast<uintptr_t>(x) % 16 != 0 || reinterpret_cast<uintptr_t>(gram_blocks) % 16 != 0 ||
      tokens >= (int64_t(1) << 31) || cols >= (int64_t(1) << 31))
    return MXW_EUNSUPPORTED;
  const size_t smem = 1024 + kBgStages * kBgStageBytes + (2 * kBgStages + 4) * sizeof(uint64_t) + 16;
  auto kern = dtype == MXW_F16 ? block_gram_tc_kernel<true> : block_gram_tc_kernel<false>;
  const int rc = set_max_smem(reinterpret_cast<const void*>(kern), smem);
  if (rc != MXW_OK) return rc;
  const int64_t strips = cols / 128;
  for (int64_t t0 = 0; t0 < tokens; t0 += kXtxMaxTokens) {
    const int64_t n = std::min<int64_t>(kXtxMaxTokens, tokens - t0);
    CUtensorMap map;
    const CUtensorMapDataType dt = dtype == MXW_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    if (make_tensor_map_2d(&map, dt, static_cast<const uint16_t*>(x) + t0 * ld, cols, n, ld * 2, 64, kXtxBK,
                           CU_TENSOR_MAP_SWIZZLE_128B) != MXW_OK)
      return MXW_ECUDA;
    BgParams P{n, cols, gram_blocks, flags};
    const int S = bg_slices(strips, (n + kXtxBK - 1) / kXtxBK);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(strips), static_cast<unsigned>(S), 1);
    cfg.blockDim = dim3(kBgThreads, 1, 1);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = static_cast<unsigned>(S);
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&cfg, kern, map, P);
    if (err != cudaSuccess) return record_cuda_error(err);
    const int st = check_launch();
    if (st != MXW_OK) return st;
  }
  return MXW_OK;
}

}  // namespace mxw

using namespace mxw;

static int accumulate_xtx(const void* x, int64_t tokens, int64_t cols, int64_t ld, float* gram, int64_t ldg,
                          float* packed, uint32_t* flags, void* stream) {
  if (tokens < 0 || cols <= 0 || cols % 128 != 0 || ld < cols || ld % 8 != 0) return MXW_EINVAL;
  if (!packed && (ldg < cols || ldg % 4 != 0)) return MXW_EINVAL;
  if (tokens == 0) return MXW_OK;
  if (!x || (!gram && !packed)) return MXW_EINVAL;
  if (reinterpret_cast<uintptr_t>(x) % 16 != 0 || reinterpret_cast<uintptr_t>(gram ? gram : packed) % 16 != 0)
    return MXW_EINVAL;
  if (tokens >= (int64_t(1) << 31) || cols >= (int64_t(1) << 31)) return MXW_EINVAL;
  const size_t smem = 1024 + kXtxStages * kXtxStageBytes + (2 * kXtxStages + 4) * sizeof(uint64_t) + 16;
  const int rc = set_max_smem(reinterpret_cast<const void*>(xtx_kernel), smem);
  if (rc != MXW_OK) return rc;
  // One launch per slice of at most kXtxMaxTokens tokens: every on-device wait
  // stays far below the timeout, and each slice's TMEM accumulator is folded
  // into the fp32 Gram before the next one starts.  Only the tiles that reach
  // the upper triangle run.
  const int64_t n_col_tiles = (cols + kXtxBN - 1) / kXtxBN;
  const dim3 grid(static_cast<unsigned>(xtx_tiles(cols)));
  for (int64_t t0 = 0; t0 < tokens; t0 += kXtxMaxTokens) {
    const int64_t n = std::min<int64_t>(kXtxMaxTokens, tokens - t0);
    CUtensorMap map;
    if (make_tensor_map_2d(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, static_cast<const uint16_t*>(x) + t0 * ld, cols,
                           n, ld * 2, 64, kXtxBK, CU_TENSOR_MAP_SWIZZLE_128B) != MXW_OK)
      return MXW_ECUDA;
    XtxParams P{};
    P.tokens = n;
    P.cols = cols;
    P.ldg = ldg;
    P.n_kblocks = (n + kXtxBK - 1) / kXtxBK;
    P.n_col_tiles = n_col_tiles;
    P.gram = gram;
    P.packed = packed;
    P.flags = flags;
    xtx_kernel<<<grid, kXtxThreads, smem, static_cast<cudaStream_t>(stream)>>>(map, P);
    const int st = check_launch();
    if (st != MXW_OK) return st;
  }
  return MXW_OK;
}

extern "C" int mxw_accumulate_xtx(const void* x, int64_t tokens, int64_t cols, int64_t ld, float* gram,
                                  int64_t ldg, uint32_t* flags, void* stream) {
  if (!gram && tokens > 0) return MXW_EINVAL;
  return accumulate_xtx(x, tokens, cols, ld, gram, ldg, nullptr, flags, stream);
}

extern "C" size_t mxw_xtx_packed_floats(int64_t cols) {
  if (cols <= 0 || cols % 128 != 0 || cols >= (int64_t(1) << 31)) return 0;
  return static_cast<size_t>(xtx_tiles(cols)) * kXtxTileFloats;
}

extern "C" int mxw_accumulate_xtx_packed(const void* x, int64_t tokens, int64_t cols, int64_t ld, float* packed,
                                         uint32_t* flags, void* stream) {
  if (!packed && tokens > 0) return MXW_EINVAL;
  return accumulate_xtx(x, tokens, cols, ld, nullptr, 0, packed, flags, stream);
}

extern "C" int mxw_xtx_unpack(const float* packed, int64_t cols, float* gram, int64_t ldg, void* stream) {
  if (cols <= 0 || cols % 128 != 0 || cols >= (int64_t(1) << 31) || ldg < cols || ldg % 4 != 0) return MXW_EINVAL;
  if (!packed || !gram) return MXW_EINVAL;
  if (reinterpret_cast<uintptr_t>(packed) % 16 != 0 || reinterpret_cast<uintptr_t>(gram) % 16 != 0) return MXW_EINVAL;
  xtx_unpack_kernel<<<static_cast<unsigned>(xtx_tiles(cols)), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      packed, cols, (cols + kXtxBN - 1) / kXtxBN, gram, ldg, 0);
  return check_launch();
}

extern "C" int64_t mxw_xtx_packed_tiles(int64_t cols) {
  if (cols <= 0 || cols % 128 != 0 || cols >= (int64_t(1) << 31)) return 0;
  return xtx_tiles(cols);
}

extern "C" int mxw_xtx_unpack_tiles(const float* packed, int64_t first_tile, int64_t n_tiles, int64_t cols,
                                    float* gram, int64_t ldg, void* stream) {
  if (cols <= 0 || cols % 128 != 0 || cols >= (int64_t(1) << 31) || ldg < cols || ldg % 4 != 0) return MXW_EINVAL;
  if (first_tile < 0 || n_tiles < 0) return MXW_EINVAL;
  const int64_t total = xtx_tiles(cols);
  n_tiles = std::min<int64_t>(n_tiles, std::max<int64_t>(0, total - first_tile));  // padding tiles past the end
  if (n_tiles == 0) return MXW_OK;
  if (!packed || !gram) return MXW_EINVAL;
  if (reinterpret_cast<uintptr_t>(packed) % 16 != 0 || reinterpret_cast<uintptr_t>(gram) % 16 != 0) return MXW_EINVAL;
  xtx_unpack_kernel<<<static_cast<unsigned>(n_tiles), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      packed, cols, (cols + kXtxBN - 1) / kXtxBN, gram, ldg, first_tile);
  return check_launch();
}
