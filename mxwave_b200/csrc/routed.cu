// K6: routing-weighted squared activations per expert (mixture-of-experts
// calibration).
//
// Replaces the index_add_ accumulations of RoutedLayerMoments.update_inputs /
// update_down (mxwave/routed_calibration.py:104-141): for every route (token
// row, expert e, router weight w) the reference adds fl(fl(x^2) * fl(w^2)) to
// row e of an fp32 accumulator, in route order.  Here the routes arrive
// grouped by expert (a stable sort on the host, so each group keeps route
// order) and one CTA owns one (expert, 256-column strip): every thread sums
// the same fp32 products for its column over the expert's routes in order,
// in fp64, and adds the total to the accumulator once.  No atomics: the
// result is deterministic run to run and independent of the launch shape.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "runtime.h"

namespace mxw {

constexpr int kRoutedCols = 256;

struct RoutedParams {
  const void* x;
  int64_t rows, ld, cols, experts, n_routes;
  const int64_t* route_rows;  // row of x for each route, grouped by expert
  const float* route_w2;      // squared router weight of each route, same order
  const int64_t* offsets;     // [experts + 1]: routes of expert e are [offsets[e], offsets[e+1])
  float* squares;             // [experts][cols], accumulated in place
  float* mass;                // [experts] sum of w^2, accumulated in place (may be null)
};

template <int DT>
__device__ __forceinline__ float routed_load(const void* base, int64_t idx) {
  if constexpr (DT == MXW_BF16) return bits_f32(static_cast<uint32_t>(static_cast<const uint16_t*>(base)[idx]) << 16);
  if constexpr (DT == MXW_F16) return __half2float(static_cast<const __half*>(base)[idx]);
  return static_cast<const float*>(base)[idx];
}

template <int DT>
__global__ void __launch_bounds__(kRoutedCols) routed_squares_kernel(const RoutedParams P) {
  const int64_t e = blockIdx.y;
  const int64_t c = static_cast<int64_t>(blockIdx.x) * kRoutedCols + threadIdx.x;
  // Offsets and rows come from the caller's device arrays: clamp the range
  // and skip a row outside x, so a malformed grouping cannot read out of bounds.
  const int64_t begin = max(int64_t(0), min(P.offsets[e], P.n_routes));
  const int64_t end = max(begin, min(P.offsets[e + 1], P.n_routes));
  if (begin >= end) return;
  if (c < P.cols) {
    double acc = 0.0;
    for (int64_t r = begin; r < end; ++r) {
      const int64_t row = P.route_rows[r];
      if (static_cast<uint64_t>(row) >= static_cast<uint64_t>(P.rows)) continue;
      const float x = routed_load<DT>(P.x, row * P.ld + c);
      acc += static_cast<double>(__fmul_rn(__fmul_rn(x, x), P.route_w2[r]));
    }
    P.squares[e * P.cols + c] += static_cast<float>(acc);
  }
  if (P.mass && blockIdx.x == 0 && threadIdx.x == 0) {
    double m = 0.0;
    for (int64_t r = begin; r < end; ++r) m += static_cast<double>(P.route_w2[r]);
    P.mass[e] += static_cast<float>(m);
  }
}

}  // namespace mxw

using namespace mxw;

extern "C" int mxw_accumulate_routed_squares(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld,
                                             const int64_t* route_rows, const float* route_w2, int64_t n_routes,
                                             const int64_t* offsets, int64_t experts, float* squares, float* mass,
                                             void* stream) {
  if (rows < 0 || cols <= 0 || ld < cols || experts <= 0 || n_routes < 0) return MXW_EINVAL;
  if (n_routes == 0) return MXW_OK;
  if (dtype != MXW_BF16 && dtype != MXW_F16 && dtype != MXW_F32) return MXW_EINVAL;
  if (!x || !route_rows || !route_w2 || !offsets || !squares) return MXW_EINVAL;
  if (experts > 65535) return MXW_EUNSUPPORTED;  // grid.y limit
  RoutedParams P{};
  P.x = x;
  P.rows = rows;
  P.n_routes = n_routes;
  P.ld = ld;
  P.cols = cols;
  P.experts = experts;
  P.route_rows = route_rows;
  P.route_w2 = route_w2;
  P.offsets = offsets;
  P.squares = squares;
  P.mass = mass;
  const dim3 grid(static_cast<unsigned>((cols + kRoutedCols - 1) / kRoutedCols), static_cast<unsigned>(experts));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case MXW_BF16:
      routed_squares_kernel<MXW_BF16><<<grid, kRoutedCols, 0, s>>>(P);
      break;
    case MXW_F16:
      routed_squares_kernel<MXW_F16><<<grid, kRoutedCols, 0, s>>>(P);
      break;
    default:
      routed_squares_kernel<MXW_F32><<<grid, kRoutedCols, 0, s>>>(P);
  }
  return check_launch();
}
