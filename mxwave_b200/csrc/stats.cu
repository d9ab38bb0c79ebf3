// K2: per-channel moments (sum |x|, sum x^2) and the diagonal 32x32 blocks of
// X^T X of calibration activations, in one pass over X.
//
// Replaces ActivationCollector.update (mxwave/calibration.py:206-236): the
// reference casts x to fp32 and forms values.abs().sum(0), values.square()
// .sum(0) and einsum("nbi,nbj->bij") per hooked call.  Here each CTA owns one
// 32-channel strip (= one MXFP4 block column) for all tokens, streams it
// through shared memory with TMA, keeps fp32 partial sums per 256-token tile
// and folds them into fp64 accumulators, then adds the strip's totals into
// the caller's fp32 buffers.  Every output element is written by exactly one
// CTA in a fixed order, so the result is deterministic run to run.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "runtime.h"
#include "tma.cuh"

namespace mxw {

constexpr int kStatConsumers = 8;
constexpr int kStatThreads = (kStatConsumers + 1) * 32;
constexpr int kStatStages = 4;
constexpr int kStatTileBytes = 16384;  // one stage: 256 rows x 64 B (2-byte types) or 128 x 128 B

template <int DT>
struct StatElem {
  static constexpr int kBytes = DT == MXW_F32 ? 4 : 2;
  static constexpr int kTileRows = kStatTileBytes / (32 * kBytes);
};

template <int DT>
__device__ __forceinline__ float load_elem(const uint8_t* row, int c) {
  if constexpr (DT == MXW_BF16) return bits_f32(static_cast<uint32_t>(reinterpret_cast<const uint16_t*>(row)[c]) << 16);
  if constexpr (DT == MXW_F16) return __half2float(reinterpret_cast<const __half*>(row)[c]);
  return reinterpret_cast<const float*>(row)[c];
}

struct StatParams {
  int64_t tokens, cols, n_tiles;
  float* sum_abs;
  float* sum_sq;
  float* gram_blocks;
  uint32_t* flags;
};

template <int DT, bool MOMENTS, bool GRAM>
__global__ void __launch_bounds__(kStatThreads, 1)
    activation_stats_kernel(const __grid_constant__ CUtensorMap map, const StatParams P) {
  constexpr int TR = StatElem<DT>::kTileRows;
  constexpr int RB = 32 * StatElem<DT>::kBytes;  // bytes per tile row
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStatStages * kStatTileBytes);
  uint64_t* empty = full + kStatStages;
  double* red = reinterpret_cast<double*>(empty + kStatStages);  // [256][16] doubles for the final reduction

  __shared__ int s_fail;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t col0 = static_cast<int64_t>(blockIdx.x) * 32;
  if (threadIdx.x == 0) {
    s_fail = 0;
    for (int s = 0; s < kStatStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kStatConsumers);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kStatConsumers) {
    if (lane == 0) {
      prefetch_tensormap(&map);
      bool ok = true;
      int64_t i = 0;
      for (; i < P.n_tiles; ++i) {
        const int s = static_cast<int>(i % kStatStages);
        if (i >= kStatStages && !mbar_wait(&empty[s], static_cast<uint32_t>((i / kStatStages - 1) & 1))) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], kStatTileBytes);
        tma_load_2d(stages + s * kStatTileBytes, &map, &full[s], static_cast<int32_t>(col0),
                    static_cast<int32_t>(i * TR));
      }
      for (int64_t j = (i > kStatStages ? i - kStatStages : 0); j < i; ++j)
        if (!mbar_wait(&full[j % kStatStages], static_cast<uint32_t>((j / kStatStages) & 1))) ok = false;
      if (!ok && P.flags) atomicOr(P.flags, MXW_FLAG_TIMEOUT);
    }
    return;
  }

  const int t = threadIdx.x;  // 0..255
  // Moments: channel pair p (columns 2p, 2p+1), token residue g (16 groups).
  const int mp = t & 15, mg = t >> 4;
  double macc_abs[2] = {0.0, 0.0}, macc_sq[2] = {0.0, 0.0};
  // Gram: 4x4 sub-block (i0, j0) of the 32x32 block, token residue gg (4 groups).
  const int gi0 = 4 * ((t & 63) >> 3), gj0 = 4 * (t & 7), gg = t >> 6;
  double gacc[16];
#pragma unroll
  for (int k = 0; k < 16; ++k) gacc[k] = 0.0;

  bool ok = true;
  for (int64_t i = 0; i < P.n_tiles; ++i) {
    const int s = static_cast<int>(i % kStatStages);
    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], static_cast<uint32_t>((i / kStatStages) & 1)))) {
      ok = false;
      break;
    }
    const uint8_t* tile = stages + s * kStatTileBytes;
    const int64_t remaining = P.tokens - i * TR;
    const int valid = remaining < TR ? static_cast<int>(remaining) : TR;  // rows past the end are TMA zero-fill
    if constexpr (MOMENTS) {
      float a0 = 0.f, a1 = 0.f, q0 = 0.f, q1 = 0.f;
      for (int r = mg; r < valid; r += 16) {
        const float x0 = load_elem<DT>(tile + r * RB, 2 * mp), x1 = load_elem<DT>(tile + r * RB, 2 * mp + 1);
        a0 = __fadd_rn(a0, fabsf(x0));
        a1 = __fadd_rn(a1, fabsf(x1));
        q0 = __fmaf_rn(x0, x0, q0);
        q1 = __fmaf_rn(x1, x1, q1);
      }
      macc_abs[0] += a0;
      macc_abs[1] += a1;
      macc_sq[0] += q0;
      macc_sq[1] += q1;
    }
    if constexpr (GRAM) {
      float acc[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) acc[k] = 0.f;
      for (int r = gg; r < valid; r += 4) {
        const uint8_t* row = tile + r * RB;
        float xi[4], xj[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          xi[k] = load_elem<DT>(row, gi0 + k);
          xj[k] = load_elem<DT>(row, gj0 + k);
        }
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int b = 0; b < 4; ++b) acc[a * 4 + b] = __fmaf_rn(xi[a], xj[b], acc[a * 4 + b]);
      }
#pragma unroll
      for (int k = 0; k < 16; ++k) gacc[k] += acc[k];
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
  // Every consumer warp leaves the loop (all waits are bounded); agree on the
  // verdict before any write-back so a timed-out CTA writes nothing.
  if (!ok && lane == 0) atomicOr(&s_fail, 1);
  asm volatile("bar.sync 1, 256;" ::: "memory");
  if (s_fail) {
    if (P.flags && t == 0) atomicOr(P.flags, MXW_FLAG_TIMEOUT);
    return;
  }

  // Fixed-order reductions across the token residues, then one add into the
  // caller's fp32 accumulators (these CTAs own their columns exclusively).
  // Named barrier 1 synchronises the 256 consumer threads only.
  if constexpr (MOMENTS) {
    red[t * 4 + 0] = macc_abs[0];
    red[t * 4 + 1] = macc_abs[1];
    red[t * 4 + 2] = macc_sq[0];
    red[t * 4 + 3] = macc_sq[1];
    asm volatile("bar.sync 1, 256;" ::: "memory");
    if (t < 16) {
      double sa0 = 0, sa1 = 0, sq0 = 0, sq1 = 0;
      for (int g = 0; g < 16; ++g) {
        const double* v = red + (g * 16 + t) * 4;
        sa0 += v[0];
        sa1 += v[1];
        sq0 += v[2];
        sq1 += v[3];
      }
      const int64_t c = col0 + 2 * t;
      if (P.sum_abs) {
        if (c < P.cols) P.sum_abs[c] += static_cast<float>(sa0);
        if (c + 1 < P.cols) P.sum_abs[c + 1] += static_cast<float>(sa1);
      }
      if (P.sum_sq) {
        if (c < P.cols) P.sum_sq[c] += static_cast<float>(sq0);
        if (c + 1 < P.cols) P.sum_sq[c + 1] += static_cast<float>(sq1);
      }
    }
    asm volatile("bar.sync 1, 256;" ::: "memory");
  }
  if constexpr (GRAM) {
#pragma unroll
    for (int k = 0; k < 16; ++k) red[t * 16 + k] = gacc[k];
    asm volatile("bar.sync 1, 256;" ::: "memory");
    if (t < 64) {
      float* G = P.gram_blocks + blockIdx.x * 1024;
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        double v = 0.0;
        for (int g = 0; g < 4; ++g) v += red[(g * 64 + t) * 16 + k];
        const int a = k >> 2, b = k & 3;
        G[(gi0 + a) * 32 + gj0 + b] += static_cast<float>(v);
      }
    }
  }
}

// Plain-load fallback (unaligned base or row stride): one thread per channel
// for the moments, one thread per Gram element.
template <int DT>
__global__ void stats_plain_kernel(const void* __restrict__ x, int64_t ld, StatParams P) {
  const int64_t col0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int t = threadIdx.x;
  const uint8_t* base = static_cast<const uint8_t*>(x);
  constexpr int EB = StatElem<DT>::kBytes;
  if (t < 32 && col0 + t < P.cols && (P.sum_abs || P.sum_sq)) {
    double sa = 0.0, sq = 0.0;
    for (int64_t r = 0; r < P.tokens; ++r) {
      const float v = load_elem<DT>(base + (r * ld + col0) * EB, t);
      sa += fabsf(v);
      sq += static_cast<double>(v) * v;
    }
    if (P.sum_abs) P.sum_abs[col0 + t] += static_cast<float>(sa);
    if (P.sum_sq) P.sum_sq[col0 + t] += static_cast<float>(sq);
  }
  if (P.gram_blocks) {
    for (int e = t; e < 1024; e += blockDim.x) {
      const int a = e >> 5, b = e & 31;
      double acc = 0.0;
      for (int64_t r = 0; r < P.tokens; ++r) {
        const uint8_t* row = base + (r * ld + col0) * EB;
        acc += static_cast<double>(load_elem<DT>(row, a)) * load_elem<DT>(row, b);
      }
      P.gram_blocks[blockIdx.x * 1024 + e] += static_cast<float>(acc);
    }
  }
}

template <int DT, bool M, bool G>
static int launch_stats_tma(const void* x, int64_t ld, const StatParams& P, cudaStream_t stream) {
  constexpr int TR = StatElem<DT>::kTileRows;
  const size_t smem = 1024 + kStatStages * kStatTileBytes + 2 * kStatStages * sizeof(uint64_t) +
                      256 * 16 * sizeof(double);
  CUtensorMap map;
  const CUtensorMapDataType dt = DT == MXW_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : DT == MXW_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  if (make_tensor_map_2d(&map, dt, x, P.cols, P.tokens, ld * StatElem<DT>::kBytes, 32, TR,
                         CU_TENSOR_MAP_SWIZZLE_NONE) != MXW_OK)
    return MXW_ECUDA;
  auto kern = activation_stats_kernel<DT, M, G>;
  const int rc = set_max_smem(reinterpret_cast<const void*>(kern), smem);
  if (rc != MXW_OK) return rc;
  StatParams Q = P;
  Q.n_tiles = (P.tokens + TR - 1) / TR;
  kern<<<static_cast<unsigned>((P.cols + 31) / 32), kStatThreads, smem, stream>>>(map, Q);
  return check_launch();
}

template <int DT>
static int launch_stats(const void* x, int64_t ld, const StatParams& P, bool moments, bool gram,
                        cudaStream_t stream) {
  const bool tma_ok = reinterpret_cast<uintptr_t>(x) % 16 == 0 && (ld * StatElem<DT>::kBytes) % 16 == 0 &&
                      P.tokens < (int64_t(1) << 31);
  if (!tma_ok) {
    stats_plain_kernel<DT><<<static_cast<unsigned>((P.cols + 31) / 32), 256, 0, stream>>>(x, ld, P);
    return check_launch();
  }
  if (moments && gram) return launch_stats_tma<DT, true, true>(x, ld, P, stream);
  if (moments) return launch_stats_tma<DT, true, false>(x, ld, P, stream);
  return launch_stats_tma<DT, false, true>(x, ld, P, stream);
}

}  // namespace mxw

using namespace mxw;

// One pass: any subset of sum_abs / sum_sq / gram_blocks (non-NULL ones).
extern "C" int mxw_accumulate_activation_stats(const void* x, int dtype, int64_t tokens, int64_t cols,
                                               int64_t ld, float* sum_abs, float* sum_sq,
                                               float* gram_blocks, uint32_t* flags, void* stream) {
  if (tokens < 0 || cols <= 0 || ld < cols) return MXW_EINVAL;
  if (dtype != MXW_BF16 && dtype != MXW_F16 && dtype != MXW_F32) return MXW_EINVAL;
  if (gram_blocks && cols % 32 != 0) return MXW_EINVAL;
  if (tokens == 0 || (!sum_abs && !sum_sq && !gram_blocks)) return MXW_OK;
  if (!x) return MXW_EINVAL;
  StatParams P{};
  P.tokens = tokens;
  P.cols = cols;
  P.sum_abs = sum_abs;
  P.sum_sq = sum_sq;
  P.gram_blocks = gram_blocks;
  P.flags = flags;
  const bool moments = sum_abs || sum_sq;
  const bool gram = gram_blocks != nullptr;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case MXW_BF16:
      return launch_stats<MXW_BF16>(x, ld, P, moments, gram, s);
    case MXW_F16:
      return launch_stats<MXW_F16>(x, ld, P, moments, gram, s);
    default:
      return launch_stats<MXW_F32>(x, ld, P, moments, gram, s);
  }
}

extern "C" int mxw_accumulate_moments(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ld,
                                      float* sum_abs, float* sum_sq, void* stream) {
  return mxw_accumulate_activation_stats(x, dtype, tokens, cols, ld, sum_abs, sum_sq, nullptr, nullptr, stream);
}

extern "C" int mxw_accumulate_block_gram(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ld,
                                         float* gram_blocks, void* stream) {
  if (!gram_blocks) return MXW_EINVAL;
  return mxw_accumulate_activation_stats(x, dtype, tokens, cols, ld, nullptr, nullptr, gram_blocks, nullptr,
                                         stream);
}
