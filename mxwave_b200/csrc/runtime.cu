// Host runtime: error bookkeeping, device properties, TMA descriptor encoding
// and the status/version entry points of the C ABI.
#include <cudaTypedefs.h>

#include <mutex>

#include "runtime.h"

namespace mxw {

static thread_local int g_last_cuda_error = 0;

int record_cuda_error(cudaError_t err) {
  g_last_cuda_error = static_cast<int>(err);
  return MXW_ECUDA;
}

int check_launch() {
  const cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? MXW_OK : record_cuda_error(err);
}

int num_sms() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cached[dev] = n;
  }
  return cached[dev];
}

int set_max_smem(const void* kernel, size_t bytes) {
  cudaError_t err =
      cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (err != cudaSuccess) return record_cuda_error(err);
  // Ask for the whole unified L1/shared array as shared memory: these kernels
  // stage through shared memory (TMA) and barely use L1, and the default
  // carveout can leave room for only one CTA per SM.
  err = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                             static_cast<int>(cudaSharedmemCarveoutMaxShared));
  return err == cudaSuccess ? MXW_OK : record_cuda_error(err);
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int make_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, int64_t cols,
                       int64_t rows, int64_t row_bytes, int box_cols, int box_rows,
                       CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return record_cuda_error(cudaErrorNotSupported);
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? MXW_OK : record_cuda_error(cudaErrorInvalidValue);
}

}  // namespace mxw

extern "C" const char* mxw_status_string(int status) {
  switch (status) {
    case MXW_OK:
      return "ok";
    case MXW_EINVAL:
      return "invalid argument";
    case MXW_ENONFINITE:
      return "non-finite input";
    case MXW_ECUDA:
      return "CUDA error";
    case MXW_ETIMEOUT:
      return "device wait timed out";
    case MXW_EUNSUPPORTED:
      return "unsupported";
    default:
      return "unknown status";
  }
}

extern "C" int mxw_last_cuda_error(void) { return mxw::g_last_cuda_error; }

extern "C" const char* mxw_version(void) { return "mxwave_b200 0.1.0 (sm_100a)"; }
