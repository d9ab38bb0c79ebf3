// K2: per-channel moments (sum |x|, sum x^2) and the diagonal 32x32 blocks of
// X^T X of calibration activations, in one pass over X.
//
// Replaces ActivationCollector.update (mxwave/calibration.py:206-236): the
// reference casts x to fp32 and forms values.abs().sum(0), values.square()
// .sum(0) and einsum("nbi,nbj->bij") per hooked call.  Here a thread-block
// cluster owns one 32-channel strip (= one MXFP4 block column); each CTA of
// the cluster streams one contiguous token slice of the strip through shared
// memory with TMA, keeps fp32 partial sums per 256-token tile and folds them
// into fp64 accumulators.  CTA rank 0 then reads every rank's partials over
// distributed shared memory in rank order and adds the strip's totals into
// the caller's fp32 buffers.  Every output element is written by exactly one
// CTA with a fixed summation order, so the result is deterministic run to
// run, and no global scratch memory is needed.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "runtime.h"
#include "tma.cuh"

#include <cooperative_groups.h>

namespace cg = cooperative_groups;

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

// Shared-memory doubles per CTA: the reduction buffer (per thread) and this
// CTA's partials; the moments-only kernel needs far less, so more CTAs fit.
template <bool GRAM>
struct StatSmem {
  static constexpr int kRed = GRAM ? 16 : 4;
  static constexpr int kRes = 1 + 64 + (GRAM ? 1024 : 0);
  static constexpr size_t kBytes = 128 + kStatStages * kStatTileBytes + 2 * kStatStages * sizeof(uint64_t) +
                                   (256 * kRed + kRes) * sizeof(double);
};

struct StatParams {
  int64_t tokens, cols, n_tiles;
  float* sum_abs;
  float* sum_sq;
  float* gram_blocks;
  uint32_t* flags;
};

template <int DT, bool MOMENTS, bool GRAM>
__global__ void __launch_bounds__(kStatThreads, GRAM ? 2 : 3)
    activation_stats_kernel(const __grid_constant__ CUtensorMap map, const StatParams P) {
  constexpr int TR = StatElem<DT>::kTileRows;
  constexpr int RB = 32 * StatElem<DT>::kBytes;  // bytes per tile row
  // Unswizzled TMA tiles need 128-byte aligned destinations.
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  uint8_t* stages = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStatStages * kStatTileBytes);
  uint64_t* empty = full + kStatStages;
  double* red = reinterpret_cast<double*>(empty + kStatStages);  // [256][16 or 4] doubles: the CTA reduction
  double* res = red + 256 * StatSmem<GRAM>::kRed;  // failure flag, 64 moment and 1024 Gram partials of this CTA

  cg::cluster_group cluster = cg::this_cluster();
  const unsigned rank = cluster.block_rank();  // this CTA's token slice of the strip
  const unsigned nrank = cluster.num_blocks();
  __shared__ int s_fail;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t col0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int64_t i_begin = P.n_tiles * rank / nrank, i_end = P.n_tiles * (rank + 1) / nrank;
  if (threadIdx.x == 0) {
    s_fail = 0;
    for (int s = 0; s < kStatStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kStatConsumers);
    }
    fence_mbar_init();
  }
  __syncthreads();

  const int t = threadIdx.x;  // consumers: 0..255
  if (warp == kStatConsumers) {
    if (lane == 0) {
      prefetch_tensormap(&map);
      bool ok = true;
      int64_t n = 0;
      for (int64_t i = i_begin; i < i_end; ++i, ++n) {
        const int s = static_cast<int>(n % kStatStages);
        if (n >= kStatStages && !mbar_wait(&empty[s], static_cast<uint32_t>((n / kStatStages - 1) & 1))) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], kStatTileBytes);
        tma_load_2d(stages + s * kStatTileBytes, &map, &full[s], static_cast<int32_t>(col0),
                    static_cast<int32_t>(i * TR));
      }
      // Never leave copies in flight: wait for the last issued stages.
      for (int64_t j = (n > kStatStages ? n - kStatStages : 0); j < n; ++j)
        if (!mbar_wait(&full[j % kStatStages], static_cast<uint32_t>((j / kStatStages) & 1))) ok = false;
      if (!ok) atomicOr(&s_fail, 1);
    }
  } else {
    // Moments: channel pair p (columns 2p, 2p+1), token residue g (16 groups).
    const int mp = t & 15, mg = t >> 4;
    double macc_abs[2] = {0.0, 0.0}, macc_sq[2] = {0.0, 0.0};
    // Gram: 4x4 sub-block (i0, j0) of the 32x32 block, token residue gg (4 groups).
    const int gi0 = 4 * ((t & 63) >> 3), gj0 = 4 * (t & 7), gg = t >> 6;
    double gacc[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) gacc[k] = 0.0;

    bool ok = true;
    int64_t n = 0;
    for (int64_t i = i_begin; i < i_end; ++i, ++n) {
      const int s = static_cast<int>(n % kStatStages);
      if (!__all_sync(0xffffffffu, mbar_wait(&full[s], static_cast<uint32_t>((n / kStatStages) & 1)))) {
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
    if (!ok && lane == 0) atomicOr(&s_fail, 1);

    // Fixed-order reductions across the token residues into this CTA's
    // partials `res` (named barrier 1: the 256 consumer threads only).
    if constexpr (MOMENTS) {
      red[t * 4 + 0] = macc_abs[0];
      red[t * 4 + 1] = macc_abs[1];
      red[t * 4 + 2] = macc_sq[0];
      red[t * 4 + 3] = macc_sq[1];
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (t < 16) {
        double v[4] = {0.0, 0.0, 0.0, 0.0};
        for (int g = 0; g < 16; ++g)
#pragma unroll
          for (int k = 0; k < 4; ++k) v[k] += red[(g * 16 + t) * 4 + k];
#pragma unroll
        for (int k = 0; k < 4; ++k) res[1 + t * 4 + k] = v[k];
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");
    }
    if constexpr (GRAM) {
#pragma unroll
      for (int k = 0; k < 16; ++k) red[t * 16 + k] = gacc[k];
      asm volatile("bar.sync 1, 256;" ::: "memory");
      if (t < 64) {
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          double v = 0.0;
          for (int g = 0; g < 4; ++g) v += red[(g * 64 + t) * 16 + k];
          res[65 + t * 16 + k] = v;
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) res[0] = s_fail ? 1.0 : 0.0;

  // Every thread of every CTA of the cluster reaches both cluster barriers
  // exactly once (every wait above is bounded), so neither waits forever.
  cluster_sync_all();
  if (rank == 0 && warp < kStatConsumers) {
    // The strip's totals in rank order 0..nrank-1 (a fixed order: the result is
    // deterministic).  A failed slice anywhere leaves the outputs untouched.
    bool failed = false;
    for (unsigned r = 0; r < nrank; ++r) failed |= cluster.map_shared_rank(res, r)[0] != 0.0;
    if (failed) {
      if (P.flags && t == 0) atomicOr(P.flags, MXW_FLAG_TIMEOUT);
    } else {
      if (MOMENTS && t < 16) {
        double v[4] = {0.0, 0.0, 0.0, 0.0};
        for (unsigned r = 0; r < nrank; ++r) {
          const double* rr = cluster.map_shared_rank(res, r);
#pragma unroll
          for (int k = 0; k < 4; ++k) v[k] += rr[1 + t * 4 + k];
        }
        const int64_t c = col0 + 2 * t;
        if (P.sum_abs) {
          if (c < P.cols) P.sum_abs[c] += static_cast<float>(v[0]);
          if (c + 1 < P.cols) P.sum_abs[c + 1] += static_cast<float>(v[1]);
        }
        if (P.sum_sq) {
          if (c < P.cols) P.sum_sq[c] += static_cast<float>(v[2]);
          if (c + 1 < P.cols) P.sum_sq[c + 1] += static_cast<float>(v[3]);
        }
      }
      if (GRAM && t < 64) {
        const int gi0 = 4 * ((t & 63) >> 3), gj0 = 4 * (t & 7);
        float* G = P.gram_blocks + blockIdx.x * 1024;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          double v = 0.0;
          for (unsigned r = 0; r < nrank; ++r) v += cluster.map_shared_rank(res, r)[65 + t * 16 + k];
          G[(gi0 + (k >> 2)) * 32 + gj0 + (k & 3)] += static_cast<float>(v);
        }
      }
    }
  }
  // Keep every CTA's shared memory alive until rank 0 has read it.
  cluster_sync_all();
}

// ------------------------------------------------ moments-only pass
//
// Per-channel sum |x| and / or sum x^2 without the block Gram.  This pass is
// pure streaming, so it reads X straight from global memory with 8-byte
// (2-byte types) or 16-byte (fp32) vector loads: every warp load covers one
// whole 256- or 512-byte row segment, with no shared-memory staging.  A
// thread-block cluster owns a 128-channel strip and CTA rank r streams token
// slice r of it.  Warp w takes rows w, w + 8, ... of the slice and lane l
// channels 4l .. 4l + 3, with 16 rows in flight per lane (a batch).  Each
// batch is summed in fp32 and added into fp64 accumulators; the CTA folds its
// eight warps in warp order and rank 0 folds the slices in rank order over
// distributed shared memory, so the result is deterministic run to run.  Only
// the requested sums are formed.

constexpr int kMomStrip = 128;
constexpr int kMomWarps = 8;
constexpr int kMomBatch = 16;
constexpr int kMomMaxSlices = 8;

template <int DT>
struct MomVec {  // four consecutive elements
  using T = uint2;
};
template <>
struct MomVec<MXW_F32> {
  using T = uint4;
};

__device__ __forceinline__ void mom_load(const uint8_t* p, uint2& v) {
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
}
__device__ __forceinline__ void mom_load(const uint8_t* p, uint4& v) {
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
}

template <int DT>
__device__ __forceinline__ void mom_unpack(const typename MomVec<DT>::T& v, float (&x)[4]) {
  if constexpr (DT == MXW_BF16) {
    x[0] = bits_f32(v.x << 16);
    x[1] = bits_f32(v.x & 0xffff0000u);
    x[2] = bits_f32(v.y << 16);
    x[3] = bits_f32(v.y & 0xffff0000u);
  } else if constexpr (DT == MXW_F16) {
    const __half2 a = *reinterpret_cast<const __half2*>(&v.x), b = *reinterpret_cast<const __half2*>(&v.y);
    x[0] = __low2float(a);
    x[1] = __high2float(a);
    x[2] = __low2float(b);
    x[3] = __high2float(b);
  } else {
    x[0] = __uint_as_float(v.x);
    x[1] = __uint_as_float(v.y);
    x[2] = __uint_as_float(v.z);
    x[3] = __uint_as_float(v.w);
  }
}

struct MomParams {
  const uint8_t* x;
  int64_t ld_bytes, tokens, cols;
  float* sum_abs;
  float* sum_sq;
};

template <int DT, bool ABS, bool SQ>
__global__ void __launch_bounds__(kMomWarps * 32, 3) moments_kernel(const MomParams P) {
  using V = typename MomVec<DT>::T;
  constexpr int EB = StatElem<DT>::kBytes;
  __shared__ double red[kMomWarps][kMomStrip][2];  // each warp's accumulators (16 KB)
  __shared__ double part[kMomStrip][2];            // this CTA's slice totals, read by rank 0
  cg::cluster_group cluster = cg::this_cluster();
  const unsigned rank = cluster.block_rank(), nrank = cluster.num_blocks();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t c = static_cast<int64_t>(blockIdx.x) * kMomStrip + 4 * lane;  // this lane's first channel
  const bool have = c < P.cols;  // cols % 4 == 0: all four channels or none
  const int64_t r0 = P.tokens * rank / nrank, r1 = P.tokens * (rank + 1) / nrank;
  const uint8_t* base = P.x + c * EB;
  double da[4] = {0.0, 0.0, 0.0, 0.0}, dq[4] = {0.0, 0.0, 0.0, 0.0};
  for (int64_t r = r0 + warp; r < r1; r += kMomWarps * kMomBatch) {
    V v[kMomBatch];
#pragma unroll
    for (int k = 0; k < kMomBatch; ++k) {
      const int64_t rr = r + k * kMomWarps;
      if (have && rr < r1) {
        mom_load(base + rr * P.ld_bytes, v[k]);
      } else {
        v[k] = V{};
      }
    }
    float fa[4] = {0.f, 0.f, 0.f, 0.f}, fq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int k = 0; k < kMomBatch; ++k) {
      float x[4];
      mom_unpack<DT>(v[k], x);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if constexpr (ABS) fa[j] = __fadd_rn(fa[j], fabsf(x[j]));
        if constexpr (SQ) fq[j] = __fmaf_rn(x[j], x[j], fq[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      da[j] += fa[j];
      dq[j] += fq[j];
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    red[warp][4 * lane + j][0] = da[j];
    red[warp][4 * lane + j][1] = dq[j];
  }
  __syncthreads();
  if (threadIdx.x < kMomStrip) {
    double a = 0.0, q = 0.0;
    for (int w = 0; w < kMomWarps; ++w) {
      a += red[w][threadIdx.x][0];
      q += red[w][threadIdx.x][1];
    }
    part[threadIdx.x][0] = a;
    part[threadIdx.x][1] = q;
  }
  // Every thread of every CTA of the cluster reaches both cluster barriers
  // exactly once (no waits above), so neither waits forever.
  cluster_sync_all();
  if (rank == 0 && threadIdx.x < kMomStrip) {
    const int64_t ch = static_cast<int64_t>(blockIdx.x) * kMomStrip + threadIdx.x;
    if (ch < P.cols) {
      double a = 0.0, q = 0.0;
      for (unsigned s = 0; s < nrank; ++s) {
        const double* pp = cluster.map_shared_rank(&part[0][0], s);
        a += pp[2 * threadIdx.x];
        q += pp[2 * threadIdx.x + 1];
      }
      if constexpr (ABS) P.sum_abs[ch] += static_cast<float>(a);
      if constexpr (SQ) P.sum_sq[ch] += static_cast<float>(q);
    }
  }
  // Keep every CTA's shared memory alive until rank 0 has read it.
  cluster_sync_all();
}

// Token slices per strip (the cluster size): about 512 tokens or more each,
// at most kMomMaxSlices.
static int mom_slices(int64_t tokens) {
  return static_cast<int>(std::min<int64_t>(kMomMaxSlices, std::max<int64_t>(1, tokens / 512)));
}

template <int DT, bool ABS, bool SQ>
static int launch_moments(const void* x, int64_t ld, const StatParams& P, cudaStream_t stream) {
  MomParams Q{static_cast<const uint8_t*>(x), ld * StatElem<DT>::kBytes, P.tokens, P.cols, P.sum_abs, P.sum_sq};
  const int S = mom_slices(P.tokens);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((P.cols + kMomStrip - 1) / kMomStrip), static_cast<unsigned>(S), 1);
  cfg.blockDim = dim3(kMomWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = static_cast<unsigned>(S);
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, moments_kernel<DT, ABS, SQ>, Q);
  if (err != cudaSuccess) return record_cuda_error(err);
  return check_launch();
}

template <int DT>
static int launch_moments_any(const void* x, int64_t ld, const StatParams& P, cudaStream_t stream) {
  if (P.sum_abs && P.sum_sq) return launch_moments<DT, true, true>(x, ld, P, stream);
  if (P.sum_abs) return launch_moments<DT, true, false>(x, ld, P, stream);
  return launch_moments<DT, false, true>(x, ld, P, stream);
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

// Token slices per strip (the cluster size).  Measured on B200 at 5120
// channels, bf16 moments, L2 flushed before each launch (slices: time):
//   4096 tokens (16 tiles):  2: 22.5 us
//   8192 tokens (32 tiles):  2: 32.8 us, 4: 38.9 us
//   16384 tokens (64 tiles): 2: 53.2 us, 4: 57.3 us
//   65536 tokens (256 tiles): 2: 176 us, 4: 152 us
// Four slices pay off only once each slice still has 32 tiles; below that the
// second partial wave of CTAs and the per-CTA set-up and cluster barriers
// cost more than the extra loads in flight gain.  One slice below 16 tiles.
static int stat_slices(int64_t tiles) {
  if (tiles < 16) return 1;
  return tiles < 128 ? 2 : 4;
}

template <int DT, bool M, bool G>
static int launch_stats_tma(const void* x, int64_t ld, const StatParams& P, cudaStream_t stream) {
  constexpr int TR = StatElem<DT>::kTileRows;
  const size_t smem = StatSmem<G>::kBytes;
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
  const int64_t strips = (P.cols + 31) / 32;
  const int S = stat_slices(Q.n_tiles);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(strips), static_cast<unsigned>(S), 1);
  cfg.blockDim = dim3(kStatThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = static_cast<unsigned>(S);
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err = cudaLaunchKernelEx(&cfg, kern, map, Q);
  if (err != cudaSuccess) {
    record_cuda_error(err);
    return MXW_ECUDA;
  }
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
  // Moments only: the vector-load pass when every lane's four channels are
  // aligned (8-byte loads for 2-byte types, 16-byte for fp32).
  constexpr int64_t kVecBytes = DT == MXW_F32 ? 16 : 8;
  if (moments && P.cols % 4 == 0 && reinterpret_cast<uintptr_t>(x) % kVecBytes == 0 &&
      (ld * StatElem<DT>::kBytes) % kVecBytes == 0)
    return launch_moments_any<DT>(x, ld, P, stream);
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
  bool moments = sum_abs || sum_sq;
  bool gram = gram_blocks != nullptr;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (gram) {
    // The block Gram on the tensor cores when the input qualifies (2-byte
    // activations, 128-channel strips, TMA layout); the moments, if asked
    // for, then take the CUDA-core pass of their own.
    const int rc = accumulate_block_gram_tc(x, dtype, tokens, cols, ld, gram_blocks, flags, s);
    if (rc != MXW_EUNSUPPORTED) {
      if (rc != MXW_OK || !moments) return rc;
      gram = false;
      P.gram_blocks = nullptr;
    }
  }
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
