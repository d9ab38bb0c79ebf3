// K1: fused MXFP4 scale search + E2M1 round-to-nearest-even + nibble/E8M0 pack.
//
// Reproduces mxwave.core.quantize_mxfp4 (mxwave/core.py:114-251) bit for bit:
// every fp32 operation of the reference's eager torch ops is replayed with the
// same rounding, and the two reductions keep the reference's CPU order:
//   * Tensor.mean/sum over the 32 elements of a block: lane partials
//     p[l] = ((x[l] + x[l+8]) + x[l+16]) + x[l+24], l = 0..7, then
//     p[0] + p[1] + ... + p[7] left to right (mean then divides by 32);
//   * einsum("obs,bsd->obd", dW, H) (core.py:228): per output d the fp32 FMA
//     chain over s = 0..31.
// Data layout: one thread owns one 32-element block.  A warp owns one block
// column and 32 consecutive rows, so gamma and the block's 32x32 Hessian are
// shared by the whole warp (register / shared-memory broadcast).
//
// Pipeline: persistent CTAs, one TMA producer warp + 8 consumer warps.  A tile
// is 32 rows x 256 columns (8 block columns), loaded by TMA with the 128-byte
// swizzle into a ring of shared-memory stages; with the swizzle, the 8 lanes
// of a shared-memory phase (8 consecutive rows, same chunk) hit 8 distinct
// bank groups.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "runtime.h"
#include "tma.cuh"

namespace mxw {

constexpr int kTileRows = 32;
constexpr int kTileBlocks = 8;
constexpr int kConsumerWarps = kTileBlocks;
constexpr int kQuantThreads = (kConsumerWarps + 1) * 32;
constexpr int kStages = 4;
constexpr int kBoxBytes = kTileRows * 128;  // one TMA box: 32 rows x 128 bytes

enum Obj { kObjNone = 0, kObjGamma = 1, kObjHess = 2, kObjRtn = 3 };
enum QMode { kQAmax = 0, kQTop2 = 1, kQGeneral = 2 };

struct QuantParams {
  int64_t rows, cols, nb, n_row_tiles;
  const float* gamma;
  const float* hessian;
  uint8_t* packed;
  uint8_t* scales;
  uint32_t* flags;
  int depth;
  int q_below, q_above, q_small;
  float q_w;
};

template <int DT>
struct Elem;
template <>
struct Elem<MXW_BF16> {
  static constexpr int kBytes = 2;
};
template <>
struct Elem<MXW_F16> {
  static constexpr int kBytes = 2;
};
template <>
struct Elem<MXW_F32> {
  static constexpr int kBytes = 4;
};

// ------------------------------------------------------------ block loading

// Read this thread's block (row `lane` of the tile, block column `w`) from a
// swizzled stage.  Produces 16 fp32 pairs (elements 2j, 2j+1), the block's
// largest and second-largest magnitude, and whether it holds a NaN/inf.
template <int DT, int QM>
__device__ __forceinline__ void read_block_smem(const uint8_t* stage, int w, int lane,
                                                unsigned long long (&t2)[16], float& amax,
                                                float& second, bool& nonfinite) {
  if constexpr (Elem<DT>::kBytes == 2) {
    const uint8_t* box = stage + (w >> 1) * kBoxBytes + lane * 128;
    uint32_t words[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = (4 * (w & 1) + j) ^ (lane & 7);
      uint4 v = *reinterpret_cast<const uint4*>(box + (c << 4));
      words[4 * j + 0] = v.x;
      words[4 * j + 1] = v.y;
      words[4 * j + 2] = v.z;
      words[4 * j + 3] = v.w;
    }
    // Magnitude order statistics on the raw 16-bit patterns (sign-magnitude:
    // the integer order of |bits| is the order of |value|; NaN/inf on top).
    uint32_t m1 = 0, m2 = 0;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const uint32_t a = words[k] & 0x7fff7fffu;
      if constexpr (QM == kQTop2) m2 = __vmaxu2(m2, __vminu2(m1, a));
      m1 = __vmaxu2(m1, a);
    }
    const uint32_t lo1 = m1 & 0xffffu, hi1 = m1 >> 16;
    const uint32_t top1 = max(lo1, hi1);
    uint32_t top2 = 0;
    if constexpr (QM == kQTop2) top2 = max(min(lo1, hi1), max(m2 & 0xffffu, m2 >> 16));
    if constexpr (DT == MXW_BF16) {
      nonfinite = top1 >= 0x7f80u;
      amax = bits_f32(top1 << 16);
      second = bits_f32(top2 << 16);
#pragma unroll
      for (int k = 0; k < 16; ++k) t2[k] = pack2(bits_f32(words[k] << 16), bits_f32(words[k] & 0xffff0000u));
    } else {
      nonfinite = top1 >= 0x7c00u;
      amax = __half2float(__ushort_as_half(static_cast<unsigned short>(top1)));
      second = __half2float(__ushort_as_half(static_cast<unsigned short>(top2)));
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        __half2 h = *reinterpret_cast<__half2*>(&words[k]);
        t2[k] = pack2(__low2float(h), __high2float(h));
      }
    }
  } else {
    const uint8_t* box = stage + w * kBoxBytes + lane * 128;
    uint32_t m1 = 0, m2 = 0;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int cs = c ^ (lane & 7);
      float4 v = *reinterpret_cast<const float4*>(box + (cs << 4));
      t2[2 * c] = pack2(v.x, v.y);
      t2[2 * c + 1] = pack2(v.z, v.w);
      const uint32_t a[4] = {f32_bits(v.x) & 0x7fffffffu, f32_bits(v.y) & 0x7fffffffu,
                             f32_bits(v.z) & 0x7fffffffu, f32_bits(v.w) & 0x7fffffffu};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if constexpr (QM == kQTop2) m2 = max(m2, min(m1, a[k]));
        m1 = max(m1, a[k]);
      }
    }
    nonfinite = m1 >= 0x7f800000u;
    amax = bits_f32(m1);
    second = bits_f32(m2);
  }
}

// k-th smallest magnitude (0-based) of the block, by rank counting.
__device__ __forceinline__ float kth_magnitude(const unsigned long long (&t2)[16], int k) {
  float a[32];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    f2 v = unpack2(t2[j]);
    a[2 * j] = fabsf(v.x);
    a[2 * j + 1] = fabsf(v.y);
  }
  float result = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    int lt = 0, le = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      lt += a[j] < a[i];
      le += a[j] <= a[i];
    }
    if (lt <= k && k < le) result = a[i];
  }
  return result;
}

// ------------------------------------------------------------- error kernels

// Error of one candidate exponent e for the unweighted / gamma objectives:
// mean over the block of dW^2 (times gamma^2), dW = RNE(clamp(t/2^e)) * 2^e - t
// (core.py:224-234).  Computed as -dW = q' * 2^e + t with q' = RNE(t * -2^-e):
// the product is exact, so the fused form rounds like the reference's
// separate multiply and subtract, except when q*2^e overflows (e >= 126),
// which takes the unfused path.
template <bool GAMMA>
__device__ __forceinline__ float candidate_error(const unsigned long long (&t2)[16], int e,
                                                 const unsigned long long (&g2)[16]) {
  const float s = exp2i(e);
  const float ninv = -exp2i(-e);
  const unsigned long long S2 = pack2(s, s), NI2 = pack2(ninv, ninv);
  const bool unfused = e >= 126;
  unsigned long long p[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
#pragma unroll
    for (int lp = 0; lp < 4; ++lp) {
      const int j = q * 4 + lp;
      const f2 y = unpack2(mul2(t2[j], NI2));
      const unsigned long long qv = e2m1x2_to_f32x2(e2m1x2(y.x, y.y));
      const unsigned long long d = unfused ? add2(mul2(qv, S2), t2[j]) : fma2(qv, S2, t2[j]);
      unsigned long long sq = mul2(d, d);
      if constexpr (GAMMA) sq = mul2(sq, g2[j]);
      p[lp] = (q == 0) ? sq : add2(p[lp], sq);
    }
  }
  float acc = unpack2(p[0]).x;
  acc = __fadd_rn(acc, unpack2(p[0]).y);
#pragma unroll
  for (int lp = 1; lp < 4; ++lp) {
    const f2 v = unpack2(p[lp]);
    acc = __fadd_rn(acc, v.x);
    acc = __fadd_rn(acc, v.y);
  }
  return __fmul_rn(acc, 0.03125f);
}

// Block-Hessian error of one candidate: sum_d (sum_s dW_s H[s,d]) dW_d with
// the inner sum as a sequential fp32 FMA chain over s (core.py:228-229).
// Evaluated on -dW: every product flips sign twice, so the result is equal.
__device__ __forceinline__ float candidate_error_hessian(const unsigned long long (&t2)[16], int e,
                                                         const float* __restrict__ Hs) {
  const float s = exp2i(e);
  const float ninv = -exp2i(-e);
  const unsigned long long S2 = pack2(s, s), NI2 = pack2(ninv, ninv);
  const bool unfused = e >= 126;
  float nd[32];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const f2 y = unpack2(mul2(t2[j], NI2));
    const unsigned long long qv = e2m1x2_to_f32x2(e2m1x2(y.x, y.y));
    const f2 d = unpack2(unfused ? add2(mul2(qv, S2), t2[j]) : fma2(qv, S2, t2[j]));
    nd[2 * j] = d.x;
    nd[2 * j + 1] = d.y;
  }
  unsigned long long w[16];
#pragma unroll
  for (int si = 0; si < 32; ++si) {
    const unsigned long long ds = pack2(nd[si], nd[si]);
    const ulonglong2* row = reinterpret_cast<const ulonglong2*>(Hs + si * 32);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const ulonglong2 h = row[k];
      if (si == 0) {
        w[2 * k] = mul2(ds, h.x);
        w[2 * k + 1] = mul2(ds, h.y);
      } else {
        w[2 * k] = fma2(ds, h.x, w[2 * k]);
        w[2 * k + 1] = fma2(ds, h.y, w[2 * k + 1]);
      }
    }
  }
  unsigned long long p[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
#pragma unroll
    for (int lp = 0; lp < 4; ++lp) {
      const int j = q * 4 + lp;
      const unsigned long long prod = mul2(w[j], pack2(nd[2 * j], nd[2 * j + 1]));
      p[lp] = (q == 0) ? prod : add2(p[lp], prod);
    }
  }
  float acc = unpack2(p[0]).x;
  acc = __fadd_rn(acc, unpack2(p[0]).y);
#pragma unroll
  for (int lp = 1; lp < 4; ++lp) {
    const f2 v = unpack2(p[lp]);
    acc = __fadd_rn(acc, v.x);
    acc = __fadd_rn(acc, v.y);
  }
  return acc;
}

// _rtn_scale_exponent (core.py:91-104).
__device__ __forceinline__ int rtn_exponent(float block_max) {
  if (!(block_max > 0.0f)) return -127;
  const float safe = fmaxf(block_max, 1.17549435e-38f);
  const int base = floor_log2_f32(safe);
  const float sig = __fdiv_rn(safe, exp2i(base));
  return base + (sig >= 1.75f ? 1 : 0) - 2;
}

// ------------------------------------------------------------- block driver

// Chooses the exponent and encodes one block.  Returns the E8M0 byte and
// writes 16 packed bytes.
template <int OBJ, int QM>
__device__ __forceinline__ uint32_t quantize_one_block(unsigned long long (&t2)[16], float amax,
                                                       float second, const QuantParams& P,
                                                       const unsigned long long (&g2)[16],
                                                       const float* Hs, uint4& packed) {
  int raw;
  if constexpr (OBJ == kObjRtn) {
    raw = rtn_exponent(amax);
  } else {
    float anchor;
    if constexpr (QM == kQAmax) {
      anchor = amax;
    } else {
      float lo, hi;
      if constexpr (QM == kQTop2) {
        lo = P.q_below == 31 ? amax : second;
        hi = P.q_above == 31 ? amax : second;
      } else {
        lo = kth_magnitude(t2, P.q_below);
        hi = (P.q_above == P.q_below) ? lo : kth_magnitude(t2, P.q_above);
      }
      const float d = __fsub_rn(hi, lo);
      anchor = P.q_small ? __fmaf_rn(P.q_w, d, lo) : __fmaf_rn(__fsub_rn(P.q_w, 1.0f), d, hi);
    }
    const bool near_zero = amax < 1e-6f;
    anchor = fmaxf(anchor, 1e-6f);
    const int floor_e = floor_log2_f32(__fdiv_rn(anchor, 6.0f));
    const int lo_e = max(-127, min(127, floor_e - P.depth));
    if (near_zero) {
      // t is replaced by zeros (core.py:194-195): every candidate has error 0
      // and the first candidate wins the strict-< argmin.
#pragma unroll
      for (int j = 0; j < 16; ++j) t2[j] = 0ull;
      raw = lo_e;
    } else {
      const int hi_e = max(-127, min(127, floor_e + 1));
      const int safe_e = max(-127, min(127, ceil_log2_f32(__fdiv_rn(fmaxf(amax, 1e-12f), 6.0f))));
      float best = __int_as_float(0x7f800000);
      raw = lo_e;
      int prev = -1000;
      // Candidates floor-depth .. floor+1 (clamped: equal neighbours are
      // skipped, their error would be identical and never strictly smaller),
      // then the no-clipping exponent unless it repeats one of them.
      for (int k = 0; k <= P.depth + 2; ++k) {
        int e;
        if (k <= P.depth + 1) {
          e = max(-127, min(127, floor_e - P.depth + k));
          if (e == prev) continue;
          prev = e;
        } else {
          e = safe_e;
          if (e >= lo_e && e <= hi_e) continue;
        }
        float err;
        if constexpr (OBJ == kObjHess) {
          err = candidate_error_hessian(t2, e, Hs);
        } else {
          err = candidate_error<OBJ == kObjGamma>(t2, e, g2);
        }
        if (err < best) raw = e;
        best = (isnan(err) || isnan(best)) ? __int_as_float(0x7fffffff) : fminf(best, err);
      }
    }
  }
  // Final encode (core.py:242-249): x = clamp(t / 2^raw) -> nibble, -0 -> code 0.
  const float inv = exp2i(-raw);
  const unsigned long long I2 = pack2(inv, inv);
  const unsigned long long Z2 = 0ull;
  uint32_t bytes[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const f2 x = unpack2(add2(mul2(t2[j], I2), Z2));
    bytes[j] = e2m1x2(x.x, x.y);
  }
  packed.x = bytes[0] | (bytes[1] << 8) | (bytes[2] << 16) | (bytes[3] << 24);
  packed.y = bytes[4] | (bytes[5] << 8) | (bytes[6] << 16) | (bytes[7] << 24);
  packed.z = bytes[8] | (bytes[9] << 8) | (bytes[10] << 16) | (bytes[11] << 24);
  packed.w = bytes[12] | (bytes[13] << 8) | (bytes[14] << 16) | (bytes[15] << 24);
  return static_cast<uint32_t>(raw + 127);
}

// --------------------------------------------------------------- TMA kernel

template <int DT, int OBJ, int QM>
__global__ void __launch_bounds__(kQuantThreads, 1)
    quantize_tma_kernel(const __grid_constant__ CUtensorMap map, const QuantParams P) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  constexpr int kBoxesPerStage = (kTileBlocks * kBlock * Elem<DT>::kBytes) / 128;
  constexpr int kStageBytes = kBoxesPerStage * kBoxBytes;
  // 1024-byte alignment for the 128B-swizzle atoms.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;
  float* Hs = reinterpret_cast<float*>(smem + kStages * kStageBytes);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes +
                                               (OBJ == kObjHess ? kTileBlocks * 1024 * 4 : 0));
  uint64_t* empty = full + kStages;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int strip = blockIdx.x;
  const int64_t col0 = static_cast<int64_t>(strip) * kTileBlocks * kBlock;
  const int64_t boxes_left = (P.cols - col0 + (128 / Elem<DT>::kBytes) - 1) / (128 / Elem<DT>::kBytes);
  const int boxes = boxes_left < kBoxesPerStage ? static_cast<int>(boxes_left) : kBoxesPerStage;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  if constexpr (OBJ == kObjHess) {
    // Stage the 8 block Hessians of this column strip (4 KB each).
    const int64_t b0 = static_cast<int64_t>(strip) * kTileBlocks;
    for (int i = threadIdx.x; i < kTileBlocks * 256; i += blockDim.x) {
      const int blk = i >> 8;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (b0 + blk < P.nb) v = reinterpret_cast<const float4*>(P.hessian + (b0 + blk) * 1024)[i & 255];
      reinterpret_cast<float4*>(Hs)[i] = v;
    }
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---------------- producer warp: one elected lane issues all TMA loads.
    if (lane == 0) {
      prefetch_tensormap(&map);
      int64_t issued = 0;
      bool ok = true;
      for (int64_t rt = blockIdx.y; rt < P.n_row_tiles; rt += gridDim.y, ++issued) {
        const int s = static_cast<int>(issued % kStages);
        if (issued >= kStages && !mbar_wait(&empty[s], static_cast<uint32_t>((issued / kStages - 1) & 1))) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[s], boxes * kBoxBytes);
        for (int k = 0; k < boxes; ++k)
          tma_load_2d(stages + s * kStageBytes + k * kBoxBytes, &map, &full[s],
                      static_cast<int32_t>(col0 + k * (128 / Elem<DT>::kBytes)),
                      static_cast<int32_t>(rt * kTileRows));
      }
      // Never leave with copies in flight: wait for the last issued stages.
      for (int64_t i = (issued > kStages ? issued - kStages : 0); i < issued; ++i) {
        if (!mbar_wait(&full[i % kStages], static_cast<uint32_t>((i / kStages) & 1))) ok = false;
      }
      if (!ok && P.flags) atomicOr(P.flags, MXW_FLAG_TIMEOUT);
    }
    return;
  }

  // ---------------- consumer warps: warp w owns block column strip*8 + w.
  const int64_t b = static_cast<int64_t>(strip) * kTileBlocks + warp;
  const bool valid_col = b < P.nb;
  unsigned long long g2[16];
  if constexpr (OBJ == kObjGamma) {
    if (valid_col) {
      const float4* gp = reinterpret_cast<const float4*>(P.gamma + b * kBlock);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 g = __ldg(gp + j);
        g2[2 * j] = pack2(__fmul_rn(g.x, g.x), __fmul_rn(g.y, g.y));
        g2[2 * j + 1] = pack2(__fmul_rn(g.z, g.z), __fmul_rn(g.w, g.w));
      }
    }
  }
  const float* Hb = Hs + warp * 1024;
  bool any_nonfinite = false;
  int64_t it = 0;
  for (int64_t rt = blockIdx.y; rt < P.n_row_tiles; rt += gridDim.y, ++it) {
    const int s = static_cast<int>(it % kStages);
    // Warp-uniform verdict: a lane that timed out takes the whole warp out.
    if (!__all_sync(0xffffffffu, mbar_wait(&full[s], static_cast<uint32_t>((it / kStages) & 1)))) {
      if (P.flags && lane == 0) atomicOr(P.flags, MXW_FLAG_TIMEOUT);
      break;
    }
    const int64_t r = rt * kTileRows + lane;
    if (valid_col) {
      unsigned long long t2[16];
      float amax, second;
      bool nonfinite;
      read_block_smem<DT, QM>(stages + s * kStageBytes, warp, lane, t2, amax, second, nonfinite);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (r < P.rows) {
        any_nonfinite |= nonfinite;
        uint4 pk;
        const uint32_t sc = quantize_one_block<OBJ, QM>(t2, amax, second, P, g2, Hb, pk);
        *reinterpret_cast<uint4*>(P.packed + r * (P.cols / 2) + b * 16) = pk;
        P.scales[r * P.nb + b] = static_cast<uint8_t>(sc);
      }
    } else {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
  if (P.flags && __any_sync(0xffffffffu, any_nonfinite) && lane == 0) atomicOr(P.flags, MXW_FLAG_NONFINITE);
}

// -------------------------------------------------- generic (unaligned) path

// One thread per block with plain loads: used when the input pointer or row
// stride cannot be described to TMA (16-byte rules).
template <int DT, int OBJ, int QM>
__global__ void __launch_bounds__(128) quantize_plain_kernel(const void* __restrict__ w, int64_t ld,
                                                             const QuantParams P) {
  const int64_t total = P.rows * P.nb;
  bool any_nonfinite = false;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / P.nb, b = idx % P.nb;
    unsigned long long t2[16];
    uint32_t m1 = 0, m2 = 0;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float x0, x1;
      if constexpr (DT == MXW_BF16) {
        const uint16_t* p = static_cast<const uint16_t*>(w) + r * ld + b * kBlock + 2 * j;
        x0 = bits_f32(static_cast<uint32_t>(p[0]) << 16);
        x1 = bits_f32(static_cast<uint32_t>(p[1]) << 16);
      } else if constexpr (DT == MXW_F16) {
        const __half* p = static_cast<const __half*>(w) + r * ld + b * kBlock + 2 * j;
        x0 = __half2float(p[0]);
        x1 = __half2float(p[1]);
      } else {
        const float* p = static_cast<const float*>(w) + r * ld + b * kBlock + 2 * j;
        x0 = p[0];
        x1 = p[1];
      }
      t2[j] = pack2(x0, x1);
      const uint32_t a0 = f32_bits(x0) & 0x7fffffffu, a1 = f32_bits(x1) & 0x7fffffffu;
      m2 = max(m2, min(m1, a0));
      m1 = max(m1, a0);
      m2 = max(m2, min(m1, a1));
      m1 = max(m1, a1);
    }
    any_nonfinite |= m1 >= 0x7f800000u;
    unsigned long long g2[16];
    if constexpr (OBJ == kObjGamma) {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float ga = P.gamma[b * kBlock + 2 * j], gb = P.gamma[b * kBlock + 2 * j + 1];
        g2[j] = pack2(__fmul_rn(ga, ga), __fmul_rn(gb, gb));
      }
    }
    uint4 pk;
    const uint32_t sc = quantize_one_block<OBJ, QM>(t2, bits_f32(m1), bits_f32(m2), P, g2,
                                                    P.hessian ? P.hessian + b * 1024 : nullptr, pk);
    uint8_t* dst = P.packed + r * (P.cols / 2) + b * 16;
    const uint32_t words[4] = {pk.x, pk.y, pk.z, pk.w};
#pragma unroll
    for (int k = 0; k < 16; ++k) dst[k] = static_cast<uint8_t>(words[k >> 2] >> (8 * (k & 3)));
    P.scales[r * P.nb + b] = static_cast<uint8_t>(sc);
  }
  if (P.flags && any_nonfinite) atomicOr(P.flags, MXW_FLAG_NONFINITE);
}

// --------------------------------------------------------------- host side

template <int DT, int OBJ, int QM>
static int launch_tma(const void* w, int64_t ld, const QuantParams& P, cudaStream_t stream) {
  constexpr int kBoxCols = 128 / Elem<DT>::kBytes;
  constexpr int kStageBytes = (kTileBlocks * kBlock * Elem<DT>::kBytes / 128) * kBoxBytes;
  const size_t smem = 1024 + kStages * kStageBytes + (OBJ == kObjHess ? kTileBlocks * 4096 : 0) +
                      2 * kStages * sizeof(uint64_t);
  CUtensorMap map;
  const CUtensorMapDataType dt = DT == MXW_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : DT == MXW_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  if (make_tensor_map_2d(&map, dt, w, P.cols, P.rows, ld * Elem<DT>::kBytes, kBoxCols, kTileRows,
                         CU_TENSOR_MAP_SWIZZLE_128B) != MXW_OK)
    return MXW_ECUDA;
  auto kern = quantize_tma_kernel<DT, OBJ, QM>;
  int rc = set_max_smem(reinterpret_cast<const void*>(kern), smem);
  if (rc != MXW_OK) return rc;
  const int strips = static_cast<int>((P.nb + kTileBlocks - 1) / kTileBlocks);
  int per_sm = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kQuantThreads, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const int64_t want = static_cast<int64_t>(num_sms()) * per_sm;
  int64_t splits = (want + strips - 1) / strips;
  splits = std::max<int64_t>(1, std::min<int64_t>(splits, P.n_row_tiles));
  dim3 grid(strips, static_cast<unsigned>(splits));
  kern<<<grid, kQuantThreads, smem, stream>>>(map, P);
  return check_launch();
}

template <int DT, int OBJ, int QM>
static int launch_plain(const void* w, int64_t ld, const QuantParams& P, cudaStream_t stream) {
  const int64_t total = P.rows * P.nb;
  const int64_t blocks = std::min<int64_t>((total + 127) / 128, static_cast<int64_t>(num_sms()) * 16);
  quantize_plain_kernel<DT, OBJ, QM><<<static_cast<unsigned>(std::max<int64_t>(blocks, 1)), 128, 0, stream>>>(w, ld, P);
  return check_launch();
}

template <int DT, int OBJ, int QM>
static int launch_any(const void* w, int64_t ld, const QuantParams& P, cudaStream_t stream) {
  const bool tma_ok = (reinterpret_cast<uintptr_t>(w) % 16 == 0) && ((ld * Elem<DT>::kBytes) % 16 == 0) &&
                      P.rows < (int64_t(1) << 31) && P.cols < (int64_t(1) << 31);
  if (tma_ok) return launch_tma<DT, OBJ, QM>(w, ld, P, stream);
  return launch_plain<DT, OBJ, QM>(w, ld, P, stream);
}

template <int DT, int OBJ>
static int dispatch_q(int qm, const void* w, int64_t ld, const QuantParams& P, cudaStream_t s) {
  if (qm == kQAmax) return launch_any<DT, OBJ, kQAmax>(w, ld, P, s);
  if (qm == kQTop2) return launch_any<DT, OBJ, kQTop2>(w, ld, P, s);
  return launch_any<DT, OBJ, kQGeneral>(w, ld, P, s);
}

template <int DT>
static int dispatch_obj(int obj, int qm, const void* w, int64_t ld, const QuantParams& P, cudaStream_t s) {
  switch (obj) {
    case kObjNone:
      return dispatch_q<DT, kObjNone>(qm, w, ld, P, s);
    case kObjGamma:
      return dispatch_q<DT, kObjGamma>(qm, w, ld, P, s);
    case kObjHess:
      return dispatch_q<DT, kObjHess>(qm, w, ld, P, s);
    default:
      return launch_any<DT, kObjRtn, kQAmax>(w, ld, P, s);
  }
}

}  // namespace mxw

using namespace mxw;

extern "C" int mxw_quantize_mxfp4(const void* weight, int dtype, int64_t rows, int64_t cols, int64_t ld,
                                  double scale_percentile, const float* gamma, const float* hessian,
                                  int method, int mse_clip_depth, uint8_t* packed, uint8_t* scales,
                                  uint32_t* flags, void* stream) {
  if (rows < 0 || cols <= 0 || cols % kBlock != 0 || ld < cols) return MXW_EINVAL;
  if (dtype != MXW_BF16 && dtype != MXW_F16 && dtype != MXW_F32) return MXW_EINVAL;
  if (method != MXW_METHOD_MSE && method != MXW_METHOD_RTN) return MXW_EINVAL;
  if (gamma && hessian) return MXW_EINVAL;
  if (method == MXW_METHOD_RTN && (gamma || hessian)) return MXW_EINVAL;
  if (!(scale_percentile > 0.0 && scale_percentile <= 100.0)) return MXW_EINVAL;
  if (mse_clip_depth < 0 || mse_clip_depth > 8) return MXW_EINVAL;
  if (rows == 0) return MXW_OK;
  if (!weight || !packed || !scales) return MXW_EINVAL;
  if (reinterpret_cast<uintptr_t>(packed) % 16 != 0) return MXW_EINVAL;
  if (gamma && reinterpret_cast<uintptr_t>(gamma) % 16 != 0) return MXW_EINVAL;
  if (hessian && reinterpret_cast<uintptr_t>(hessian) % 16 != 0) return MXW_EINVAL;

  QuantParams P{};
  P.rows = rows;
  P.cols = cols;
  P.nb = cols / kBlock;
  P.n_row_tiles = (rows + kTileRows - 1) / kTileRows;
  P.gamma = gamma;
  P.hessian = hessian;
  P.packed = packed;
  P.scales = scales;
  P.flags = flags;
  P.depth = mse_clip_depth;
  // torch.quantile(|b|, p/100) over 32 values: ranks = fp32(p/100) * 31,
  // linear interpolation between the order statistics below and above.
  const float q = static_cast<float>(scale_percentile / 100.0);
  const float rank = q * 31.0f;
  P.q_below = static_cast<int>(rank);
  P.q_above = static_cast<int>(std::ceil(rank));
  P.q_w = rank - static_cast<float>(P.q_below);
  P.q_small = std::fabs(P.q_w) < 0.5f;

  int obj, qm;
  if (method == MXW_METHOD_RTN) {
    obj = kObjRtn;
    qm = kQAmax;
  } else {
    obj = hessian ? kObjHess : (gamma ? kObjGamma : kObjNone);
    qm = scale_percentile >= 100.0 ? kQAmax : (P.q_below >= 30 ? kQTop2 : kQGeneral);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case MXW_BF16:
      return dispatch_obj<MXW_BF16>(obj, qm, weight, ld, P, s);
    case MXW_F16:
      return dispatch_obj<MXW_F16>(obj, qm, weight, ld, P, s);
    default:
      return dispatch_obj<MXW_F32>(obj, qm, weight, ld, P, s);
  }
}
