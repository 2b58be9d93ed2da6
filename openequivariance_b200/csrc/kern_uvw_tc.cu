// Tensor-core shared-weight uvw forward (tp_kernels_uvw_tc.cuh), float32.
#include "tp_kernels_uvw_tc.cuh"
namespace oeqb {
const void* uvw_tc_kernel_ptr(int kind) {
  return kind == 0 ? (const void*)tp_uvw_tc_fwd<float> : (const void*)tp_uvw_tc_prep<float>;
}
}  // namespace oeqb
