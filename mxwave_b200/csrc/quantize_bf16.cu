// K1 launchers for bf16 weights (one translation unit per input type, so the
// template instantiations compile in parallel).
#include "quantize_impl.cuh"

namespace mxw {

int quantize_dispatch_bf16(int obj, int qm, const void* w, int64_t ld, const QuantParams& P, cudaStream_t s) {
  return dispatch_obj<MXW_BF16>(obj, qm, w, ld, P, s);
}

}  // namespace mxw
