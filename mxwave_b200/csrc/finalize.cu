// K4: finalisation of calibration statistics, and MXFP4 dequantisation.
#include <cuda_runtime.h>

#include "common.cuh"
#include "runtime.h"

namespace mxw {

// mean_abs = S1 / count, rms = sqrt(S2 / count) in fp32, as
// ActivationCollector.finalize (mxwave/calibration.py:262-266) computes them
// (division by the count converted to fp32, then an IEEE square root).
__global__ void finalize_moments_kernel(const float* __restrict__ s1, const float* __restrict__ s2, int64_t cols,
                                        float count, float* __restrict__ mean_abs, float* __restrict__ rms) {
  for (int64_t c = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; c < cols;
       c += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (mean_abs) mean_abs[c] = __fdiv_rn(s1[c], count);
    if (rms) rms[c] = __fsqrt_rn(__fdiv_rn(s2[c], count));
  }
}

// H_b = G_b / count, then diagonal damping (_damp_block_hessian, core.py:61-69).
// One CTA of 1024 threads per 32x32 block.
__global__ void finalize_block_hessian_kernel(const float* __restrict__ g, int full, int64_t ldg, float count,
                                              float damp, int mode, float* __restrict__ out) {
  __shared__ float diag[32];
  const int64_t b = blockIdx.x;
  const int i = threadIdx.x >> 5, j = threadIdx.x & 31;
  const float v = full ? g[(b * 32 + i) * ldg + b * 32 + j] : g[b * 1024 + threadIdx.x];
  const float h = __fdiv_rn(v, count);
  if (i == j) diag[i] = h;
  __syncthreads();
  float add = damp;
  if (mode == MXW_DAMP_RELATIVE) {
    float s = 0.0f;
    for (int k = 0; k < 32; ++k) s = __fadd_rn(s, diag[k]);
    add = __fmul_rn(__fdiv_rn(s, 32.0f), damp);
  }
  out[b * 1024 + threadIdx.x] = (i == j) ? __fadd_rn(h, add) : h;
}

// dequant_mxfp4 (core.py:254-278): sign * magnitude * 2^(scale - 127).
__global__ void dequant_kernel(const uint8_t* __restrict__ packed, const uint8_t* __restrict__ scales, int64_t rows,
                               int64_t cols, float* __restrict__ out) {
  const int64_t half = cols / 2, total = rows * half;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / half, cb = i % half;
    const uint32_t byte = packed[i];
    const float sc = exp2i(static_cast<int>(scales[r * (cols / 32) + (2 * cb) / 32]) - 127);
    const f2 q = unpack2(e2m1x2_to_f32x2(byte));
    out[r * cols + 2 * cb] = __fmul_rn(q.x, sc);
    out[r * cols + 2 * cb + 1] = __fmul_rn(q.y, sc);
  }
}

static unsigned grid_for(int64_t n, int threads) {
  const int64_t blocks = (n + threads - 1) / threads;
  return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(blocks, static_cast<int64_t>(num_sms()) * 32)));
}

}  // namespace mxw

using namespace mxw;

extern "C" int mxw_finalize_moments(const float* sum_abs, const float* sum_sq, int64_t cols, int64_t count,
                                    float* mean_abs, float* rms, void* stream) {
  if (cols <= 0 || count <= 0) return MXW_EINVAL;
  if ((mean_abs && !sum_abs) || (rms && !sum_sq)) return MXW_EINVAL;
  finalize_moments_kernel<<<grid_for(cols, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      sum_abs, sum_sq, cols, static_cast<float>(count), mean_abs, rms);
  return check_launch();
}

extern "C" int mxw_finalize_block_hessian(const float* gram, int full, int64_t cols, int64_t ldg, int64_t count,
                                          double damp, int mode, float* out, void* stream) {
  if (cols <= 0 || cols % 32 != 0 || count <= 0 || !gram || !out) return MXW_EINVAL;
  if (!(damp >= 0.0) || !std::isfinite(damp)) return MXW_EINVAL;
  if (mode != MXW_DAMP_ABSOLUTE && mode != MXW_DAMP_RELATIVE) return MXW_EINVAL;
  if (full && ldg < cols) return MXW_EINVAL;
  finalize_block_hessian_kernel<<<static_cast<unsigned>(cols / 32), 1024, 0, static_cast<cudaStream_t>(stream)>>>(
      gram, full, ldg, static_cast<float>(count), static_cast<float>(damp), mode, out);
  return check_launch();
}

extern "C" int mxw_dequant_mxfp4(const uint8_t* packed, const uint8_t* scales, int64_t rows, int64_t cols,
                                 float* out, void* stream) {
  if (rows < 0 || cols <= 0 || cols % 32 != 0) return MXW_EINVAL;
  if (rows == 0) return MXW_OK;
  if (!packed || !scales || !out) return MXW_EINVAL;
  dequant_kernel<<<grid_for(rows * cols / 2, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(packed, scales,
                                                                                                  rows, cols, out);
  return check_launch();
}
