// K7: lossless repack of compressed-tensors MXFP4 into ggml block_mxfp4.
//
// Replaces repack_mxfp4_blocks (mxwave/gguf.py:134-150).  Source: packed
// [rows, cols/2] (element 2j in the low nibble of byte j) and E8M0 scales
// [rows, cols/32].  Destination: per 32-element block 17 bytes, the scale byte
// then 16 code bytes where byte j holds element j (low nibble) and element
// j + 16 (high nibble).  Blocks are contiguous across rows, so block g lands at
// byte 17 g.  One thread per block: its two 8-byte halves hold elements 0-15
// and 16-31 as consecutive nibbles, and the output bytes are the nibble-wise
// interleave of the two halves.  A CTA stages its 17-byte records in shared
// memory and writes them out as consecutive bytes.
#include "common.cuh"
#include "runtime.h"

namespace mxw {

constexpr int kGgufThreads = 256;

// 8 nibbles of `v` -> the low nibbles of 8 bytes.
__device__ __forceinline__ unsigned long long spread_nibbles(uint32_t v) {
  unsigned long long x = v;
  x = (x | (x << 16)) & 0x0000ffff0000ffffull;
  x = (x | (x << 8)) & 0x00ff00ff00ff00ffull;
  x = (x | (x << 4)) & 0x0f0f0f0f0f0f0f0full;
  return x;
}

__global__ void __launch_bounds__(kGgufThreads) gguf_repack_kernel(const uint8_t* __restrict__ packed,
                                                                   const uint8_t* __restrict__ scales,
                                                                   int64_t nblocks, uint8_t* __restrict__ out) {
  __shared__ uint8_t stage[kGgufThreads * 17];
  const int64_t first = static_cast<int64_t>(blockIdx.x) * kGgufThreads;
  const int64_t g = first + threadIdx.x;
  if (g < nblocks) {
    const uint4 v = *reinterpret_cast<const uint4*>(packed + g * 16);  // 16-byte aligned: blocks are 16 bytes
    const unsigned long long lo = spread_nibbles(v.x) | (spread_nibbles(v.z) << 4);  // elements 0-7 | 16-23
    const unsigned long long hi = spread_nibbles(v.y) | (spread_nibbles(v.w) << 4);  // elements 8-15 | 24-31
    uint8_t* rec = stage + threadIdx.x * 17;
    rec[0] = scales[g];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      rec[1 + k] = static_cast<uint8_t>(lo >> (8 * k));
      rec[9 + k] = static_cast<uint8_t>(hi >> (8 * k));
    }
  }
  __syncthreads();
  const int64_t n = (nblocks - first < kGgufThreads ? nblocks - first : kGgufThreads) * 17;
  uint8_t* dst = out + first * 17;
  for (int64_t i = threadIdx.x; i < n; i += kGgufThreads) dst[i] = stage[i];
}

}  // namespace mxw

using namespace mxw;

extern "C" int mxw_repack_gguf_mxfp4(const uint8_t* packed, const uint8_t* scales, int64_t rows, int64_t cols,
                                     uint8_t* out, void* stream) {
  if (rows < 0 || cols <= 0 || cols % 32 != 0) return MXW_EINVAL;
  if (rows == 0) return MXW_OK;
  if (!packed || !scales || !out) return MXW_EINVAL;
  if (reinterpret_cast<uintptr_t>(packed) % 16 != 0) return MXW_EINVAL;
  const int64_t nblocks = rows * (cols / 32);
  const int64_t ctas = (nblocks + kGgufThreads - 1) / kGgufThreads;
  if (ctas > 0x7fffffff) return MXW_EUNSUPPORTED;
  gguf_repack_kernel<<<static_cast<unsigned>(ctas), kGgufThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      packed, scales, nblocks, out);
  return check_launch();
}
