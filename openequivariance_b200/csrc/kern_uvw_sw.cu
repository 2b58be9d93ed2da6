// Shared-weight uvw backward (tp_kernels_uvw_sw.cuh), float32 and float64.
#include "tp_kernels_uvw_sw.cuh"
namespace oeqb {
// kind: 0 = dX / dY, 1 = dW, 2 = weight image W'^T
template <class T>
const void* uvw_sw_kernel_ptr(int kind) {
  return kind == 0 ? (const void*)tp_uvw_sw_dxy<T>
                   : kind == 1 ? (const void*)tp_uvw_sw_dw<T> : (const void*)tp_uvw_sw_prep<T>;
}
template const void* uvw_sw_kernel_ptr<float>(int);
template const void* uvw_sw_kernel_ptr<double>(int);
}  // namespace oeqb
