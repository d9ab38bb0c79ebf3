// K5: quantization-error sums behind the SQNR family.
//
// Replaces the reductions of mxwave/verify.py:24-86 (sqnr,
// channel_weighted_sqnr, block_hessian_weighted_sqnr): for an original matrix
// o and its reconstruction r (a dense tensor, or the packed MXFP4 bytes and
// E8M0 scales decoded on the fly, as dequant_mxfp4 decodes them,
// core.py:254-278) one pass computes
//   sums[0] = sum o^2            sums[1] = sum (o - r)^2
//   sums[2] = weighted signal    sums[3] = weighted noise
// where "weighted" is gamma^2 per input channel (sum o^2 g^2, sum d^2 g^2) or
// the block quadratic form with the 32x32 Hessian of each block column
// (sum_b o_b^T H_b o_b, sum_b d_b^T H_b d_b), or absent.
//
// Layout: a warp owns one 32-element block (row r, block column b) at a time,
// lane = element, so loads are coalesced and the Hessian's row s is read
// across the lanes.  Accumulation is fp64.  Reduction is deterministic: lanes
// and warps are combined in a fixed order, every CTA writes its four partials
// to the workspace, and the last CTA to finish (a ticket counter) adds the
// partials of all CTAs in CTA order.  Nothing waits on another CTA.
#include <cuda_bf16.h>
#include <cuda_fp16.h>


#include "common.cuh"
#include "runtime.h"

namespace mxw {

constexpr int kErrWarps = 8;
constexpr int kErrThreads = kErrWarps * 32;
constexpr int kErrPacked = 3;  // "reconstruction" given as packed bytes + scales

struct ErrParams {
  int64_t rows, cols, nb;  // nb = blocks per row (last one may be ragged)
  const void* orig;
  int64_t ld;
  const void* recon;
  int64_t rld;
  const uint8_t* packed;
  const uint8_t* scales;
  const float* gamma;
  const float* hessian;
  double* partials;      // [gridDim.x][4]
  unsigned int* ticket;  // zero before the launch; zero again after it
  double* sums;          // [4], overwritten
};

template <int T>
__device__ __forceinline__ float load_any(const void* base, int64_t idx) {
  if constexpr (T == MXW_BF16) return bits_f32(static_cast<uint32_t>(static_cast<const uint16_t*>(base)[idx]) << 16);
  if constexpr (T == MXW_F16) return __half2float(static_cast<const __half*>(base)[idx]);
  return static_cast<const float*>(base)[idx];
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
  return v;  // lane 0 holds the sum
}

// W: 0 none, 1 gamma, 2 block Hessian.
template <int DT, int RT, int W>
__global__ void __launch_bounds__(kErrThreads) error_sums_kernel(const ErrParams P) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
  const int64_t nblocks = P.rows * P.nb;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * kErrWarps + warp; idx < nblocks;
       idx += static_cast<int64_t>(gridDim.x) * kErrWarps) {
    const int64_t r = idx / P.nb, b = idx % P.nb;
    const int64_t c = b * 32 + lane;
    const bool in = c < P.cols;
    float o = 0.0f, rec = 0.0f;
    if (in) {
      o = load_any<DT>(P.orig, r * P.ld + c);
      if constexpr (RT == kErrPacked) {
        const uint32_t byte = P.packed[r * (P.cols / 2) + c / 2];
        const f2 q = unpack2(e2m1x2_to_f32x2(byte));
        const float sc = exp2i(static_cast<int>(P.scales[r * P.nb + b]) - 127);
        rec = __fmul_rn((lane & 1) ? q.y : q.x, sc);
      } else {
        rec = load_any<RT>(P.recon, r * P.rld + c);
      }
    }
    const double od = o, dd = static_cast<double>(__fsub_rn(o, rec));
    s0 += od * od;
    s1 += dd * dd;
    if constexpr (W == 1) {
      const double g = in ? static_cast<double>(P.gamma[c]) : 0.0;
      const double g2 = g * g;
      s2 += od * od * g2;
      s3 += dd * dd * g2;
    } else if constexpr (W == 2) {
      // Lane l forms (H^T o)_l = sum_s o_s H[s][l] and (H^T d)_l, then
      // contributes o_l (H^T o)_l: the quadratic form summed over lanes.
      const float* H = P.hessian + b * 1024;
      double wo = 0.0, wd = 0.0;
#pragma unroll 8
      for (int s = 0; s < 32; ++s) {
        const double os = __shfl_sync(0xffffffffu, od, s), ds = __shfl_sync(0xffffffffu, dd, s);
        const double h = H[s * 32 + lane];
        wo = fma(os, h, wo);
        wd = fma(ds, h, wd);
      }
      s2 += od * wo;
      s3 += dd * wd;
    }
  }
  // Fixed-order reductions: lanes (shuffle tree), then warps in order.
  __shared__ double red[kErrWarps][4];
  __shared__ bool last;
  s0 = warp_sum(s0);
  s1 = warp_sum(s1);
  s2 = warp_sum(s2);
  s3 = warp_sum(s3);
  if (lane == 0) {
    red[warp][0] = s0;
    red[warp][1] = s1;
    red[warp][2] = s2;
    red[warp][3] = s3;
  }
  __syncthreads();
  if (threadIdx.x < 4) {
    double v = 0.0;
    for (int w = 0; w < kErrWarps; ++w) v += red[w][threadIdx.x];
    P.partials[blockIdx.x * 4 + threadIdx.x] = v;
    __threadfence();  // partials visible device-wide before the ticket
  }
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(P.ticket, 1u) == gridDim.x - 1;
  __syncthreads();
  if (last) {
    __threadfence();
    if (threadIdx.x < 4) {
      double v = 0.0;
      for (unsigned i = 0; i < gridDim.x; ++i) v += __ldcg(P.partials + i * 4 + threadIdx.x);
      P.sums[threadIdx.x] = v;
    }
    if (threadIdx.x == 0) *P.ticket = 0u;  // ready for the next call
  }
}

// CTAs per launch: enough warps for every block, at most 8 CTAs per SM.
static int64_t error_ctas(int64_t nblocks) {
  const int64_t want = (nblocks + kErrWarps - 1) / kErrWarps;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
  return want < 1 ? 1 : (want < cap ? want : cap);
}

template <int DT, int RT>
static int launch_err(const ErrParams& P, int w, cudaStream_t s, unsigned ctas) {
  switch (w) {
    case 1:
      error_sums_kernel<DT, RT, 1><<<ctas, kErrThreads, 0, s>>>(P);
      break;
    case 2:
      error_sums_kernel<DT, RT, 2><<<ctas, kErrThreads, 0, s>>>(P);
      break;
    default:
      error_sums_kernel<DT, RT, 0><<<ctas, kErrThreads, 0, s>>>(P);
  }
  return check_launch();
}

template <int DT>
static int launch_err_rt(int rt, const ErrParams& P, int w, cudaStream_t s, unsigned ctas) {
  switch (rt) {
    case MXW_BF16:
      return launch_err<DT, MXW_BF16>(P, w, s, ctas);
    case MXW_F16:
      return launch_err<DT, MXW_F16>(P, w, s, ctas);
    case MXW_F32:
      return launch_err<DT, MXW_F32>(P, w, s, ctas);
    default:
      return launch_err<DT, kErrPacked>(P, w, s, ctas);
  }
}

}  // namespace mxw

using namespace mxw;

extern "C" size_t mxw_error_sums_workspace_size(int64_t rows, int64_t cols) {
  if (rows < 0 || cols <= 0) return 0;
  const int64_t nblocks = rows * ((cols + 31) / 32);
  return 16 + static_cast<size_t>(error_ctas(nblocks)) * 4 * sizeof(double);
}

extern "C" int mxw_error_sums(const void* original, int dtype, int64_t rows, int64_t cols, int64_t ld,
                              const void* reconstructed, int rdtype, int64_t rld, const uint8_t* packed,
                              const uint8_t* scales, const float* gamma, const float* hessian, double* sums,
                              void* workspace, size_t workspace_bytes, void* stream) {
  if (rows < 0 || cols <= 0 || ld < cols || !sums) return MXW_EINVAL;
  if (dtype != MXW_BF16 && dtype != MXW_F16 && dtype != MXW_F32) return MXW_EINVAL;
  const bool dense = reconstructed != nullptr;
  if (dense == (packed != nullptr || scales != nullptr)) return MXW_EINVAL;  // exactly one reconstruction
  if (dense) {
    if (rdtype != MXW_BF16 && rdtype != MXW_F16 && rdtype != MXW_F32) return MXW_EINVAL;
    if (rld < cols) return MXW_EINVAL;
  } else if (!packed || !scales || cols % 32 != 0) {
    return MXW_EINVAL;
  }
  if (gamma && hessian) return MXW_EINVAL;
  if (hessian && cols % 32 != 0) return MXW_EINVAL;
  if (rows > 0 && !original) return MXW_EINVAL;
  if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 16 != 0) return MXW_EINVAL;
  if (workspace_bytes < mxw_error_sums_workspace_size(rows, cols)) return MXW_EINVAL;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (rows == 0) {
    const cudaError_t err = cudaMemsetAsync(sums, 0, 4 * sizeof(double), s);
    return err == cudaSuccess ? MXW_OK : record_cuda_error(err);
  }
  ErrParams P{};
  P.rows = rows;
  P.cols = cols;
  P.nb = (cols + 31) / 32;
  P.orig = original;
  P.ld = ld;
  P.recon = reconstructed;
  P.rld = rld;
  P.packed = packed;
  P.scales = scales;
  P.gamma = gamma;
  P.hessian = hessian;
  P.ticket = static_cast<unsigned int*>(workspace);
  P.partials = reinterpret_cast<double*>(static_cast<uint8_t*>(workspace) + 16);
  P.sums = sums;
  const int w = hessian ? 2 : (gamma ? 1 : 0);
  const int rt = dense ? rdtype : kErrPacked;
  const unsigned ctas = static_cast<unsigned>(error_ctas(rows * P.nb));
  switch (dtype) {
    case MXW_BF16:
      return launch_err_rt<MXW_BF16>(rt, P, w, s, ctas);
    case MXW_F16:
      return launch_err_rt<MXW_F16>(rt, P, w, s, ctas);
    default:
      return launch_err_rt<MXW_F32>(rt, P, w, s, ctas);
  }
}

// ------------------------------------------------ no-allocation variant
//
// mxw_error_sums_noalloc: the same sums for callers that cannot allocate
// device memory at call time -- processes that reserve their whole device
// memory budget up front and forbid later allocations (a serving process
// that has carved up HBM at start-up, or a host application whose own pool
// owns every device byte), and health checks that must still run when the
// device is out of memory.  Its scratch (the CTA ticket and the per-CTA
// partials) lives in the fixed array below, which every GPU that loads this
// library holds until the process exits.

namespace mxw {

constexpr int kNoAllocMaxCtas = 2048;  // 8 CTAs per SM on GPUs of up to 256 SMs
constexpr size_t kNoAllocScratchBytes = 16 + static_cast<size_t>(kNoAllocMaxCtas) * 4 * sizeof(double);  // 65,552

static __device__ __align__(256) unsigned char g_error_sums_scratch[kNoAllocScratchBytes];

// Device address of g_error_sums_scratch in the current device's context.
// In host code the array's name is only a host-side stand-in, so the address
// comes from cudaGetSymbolAddress.  It is looked up on every call rather than
// cached: a cached address would go stale after cudaDeviceReset or a new
// primary context, and once this module is loaded the lookup is a table
// search.  The first call in a context may also load this module onto the
// device.
static void* noalloc_scratch(int* status) {
  void* p = nullptr;
  const cudaError_t err = cudaGetSymbolAddress(&p, g_error_sums_scratch);
  if (err != cudaSuccess) {
    *status = record_cuda_error(err);
    return nullptr;
  }
  *status = MXW_OK;
  return p;
}

}  // namespace mxw

extern "C" int mxw_error_sums_noalloc(const void* original, int dtype, int64_t rows, int64_t cols, int64_t ld,
                                      const void* reconstructed, int rdtype, int64_t rld, const uint8_t* packed,
                                      const uint8_t* scales, const float* gamma, const float* hessian,
                                      double* sums, void* stream) {
  if (rows < 0 || cols <= 0) return MXW_EINVAL;
  if (mxw_error_sums_workspace_size(rows, cols) > kNoAllocScratchBytes) return MXW_EUNSUPPORTED;
  int status = MXW_OK;
  void* scratch = noalloc_scratch(&status);
  if (scratch == nullptr) return status;
  // The ticket (first 16 bytes) must be zero when the kernel starts.  Each
  // call leaves it zero, but clearing it on the caller's stream keeps every
  // call independent of how an earlier one ended.  The partials need no
  // clearing: every CTA overwrites its own before the fold reads them.
  const cudaError_t err = cudaMemsetAsync(scratch, 0, 16, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return record_cuda_error(err);
  return mxw_error_sums(original, dtype, rows, cols, ld, reconstructed, rdtype, rld, packed, scales, gamma, hessian,
                        sums, scratch, kNoAllocScratchBytes, stream);
}
