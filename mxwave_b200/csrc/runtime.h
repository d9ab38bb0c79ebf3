// Host-side runtime helpers shared by the kernels' launchers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>

#include "../../include/mxwave_b200.h"

namespace mxw {

// Records a failing cudaError_t for mxw_last_cuda_error() and maps it to MXW_ECUDA.
int record_cuda_error(cudaError_t err);

// cudaGetLastError() after a launch -> MXW_OK / MXW_ECUDA.
int check_launch();

// Number of SMs of the current device (cached per device).
int num_sms();

// Raise a kernel's dynamic shared-memory limit (idempotent per kernel+device).
int set_max_smem(const void* kernel, size_t bytes);

// cuTensorMapEncodeTiled through the runtime's driver entry point.  2-D tensor
// [rows, cols] with a row stride of `row_bytes`, box [box_rows, box_cols].
int make_tensor_map_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, int64_t cols,
                       int64_t rows, int64_t row_bytes, int box_cols, int box_rows,
                       CUtensorMapSwizzle swizzle);

// Diagonal 32x32 blocks of X^T X on the tensor cores (xtx.cu) for 2-byte
// activations with cols % 128 == 0 and TMA-compatible layout; MXW_EUNSUPPORTED
// when the input does not qualify.
int accumulate_block_gram_tc(const void* x, int dtype, int64_t tokens, int64_t cols, int64_t ld,
                             float* gram_blocks, uint32_t* flags, cudaStream_t stream);

}  // namespace mxw
