// sm_100a tensor-core path (placeholder until the tcgen05 kernels are in).
#include "sqb_sm100.cuh"

namespace sqb {

bool sm100_supported(const Problem&, std::initializer_list<TensorView>, const float*, const void*,
                     const void*) {
  return false;
}

int sm100_forward(const Problem&, TensorView, TensorView, TensorView, TensorView, float*, void*,
                  void*, uint8_t*, const WorkspaceLayout&, cudaStream_t) {
  return SQB_ERR_UNSUPPORTED;
}

int sm100_backward(const Problem&, TensorView, TensorView, TensorView, TensorView, TensorView,
                   const float*, const void*, const void*, TensorView, TensorView, TensorView,
                   uint8_t*, const WorkspaceLayout&, cudaStream_t) {
  return SQB_ERR_UNSUPPORTED;
}

}  // namespace sqb
