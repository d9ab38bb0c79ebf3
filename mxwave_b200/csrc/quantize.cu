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
// The unweighted and gamma errors only need dW^2, so they are evaluated on
// magnitudes: |dW| = q(|t|/2^e) * 2^e - |t|.  Per element pair and candidate:
// one packed multiply, the E2M1 round trip (cvt to e2m1x2, cvt back to an
// exact f16x2 in the same asm block), two f16->f32 conversions, and packed
// fp32 FMA / multiply / add.
//
// For 2-byte inputs with the unweighted or gamma objective and a top-2/amax
// anchor, a fast path evaluates only the f and f+1 candidates per block and
// rules out the rest with certified bounds (see quantize_block_fast); the
// Hessian objective, fp32 inputs and low percentiles evaluate every candidate.
//
// Data layout: one thread owns one 32-element block.  A warp owns one block
// column and 32 consecutive rows, so gamma and the block's 32x32 Hessian are
// shared by the whole warp (registers / shared-memory broadcast).
//
// Pipeline: persistent CTAs (one wave: #SMs x occupancy), each owning a
// contiguous range of tiles in strip-major order; one TMA producer warp + 8
// consumer warps.  A tile is 32 rows x 256 columns (8 block columns) loaded by
// TMA with the 128-byte swizzle into a ring of shared-memory stages; with the
// swizzle, the 8 lanes of a shared-memory phase (8 consecutive rows, same
// chunk) hit 8 distinct bank groups.  Outputs go the same way in reverse: each
// thread writes its 16 packed bytes into a swizzled 32 x 128-byte staging tile,
// one TMA store writes the tile, and one warp writes the 32 x 8 scale bytes.
#include "quantize_impl.cuh"

namespace mxw {
int quantize_dispatch_bf16(int obj, int qm, const void* w, int64_t ld, const QuantParams& P, cudaStream_t s);
int quantize_dispatch_f16(int obj, int qm, const void* w, int64_t ld, const QuantParams& P, cudaStream_t s);
int quantize_dispatch_f32(int obj, int qm, const void* w, int64_t ld, const QuantParams& P, cudaStream_t s);
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
  P.weight = weight;
  P.ld = ld;
  P.nb = cols / kBlock;
  P.n_row_tiles = (rows + kTileRows - 1) / kTileRows;
  P.gamma = gamma;
  P.hessian = hessian;
  P.packed = packed;
  P.scales = scales;
  P.flags = flags;
  P.depth = mse_clip_depth;
  P.zero = 0.0f;
  P.negzero = -0.0f;
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
      return quantize_dispatch_bf16(obj, qm, weight, ld, P, s);
    case MXW_F16:
      return quantize_dispatch_f16(obj, qm, weight, ld, P, s);
    default:
      return quantize_dispatch_f32(obj, qm, weight, ld, P, s);
  }
}
