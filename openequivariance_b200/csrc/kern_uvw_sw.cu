// Shared-weight uvw backward (tp_kernels_uvw_sw.cuh), float32 and float64.
#include "tp_kernels_uvw_sw.cuh"
namespace oeqb {
// kind: 0 = dX / dY, 1 = dW, 2 = weight image W'^T, 3 = forward (CUDA cores)
template <class T>
const void* uvw_sw_kernel_ptr(int kind) {
  switch (kind) {
    case 0: return (const void*)tp_uvw_sw_dxy<T>;
    case 1: return (const void*)tp_uvw_sw_dw<T>;
    case 2: return (const void*)tp_uvw_sw_prep<T>;
    default: return (const void*)tp_uvw_sw_fwd<T>;
  }
}
template const void* uvw_sw_kernel_ptr<float>(int);
template const void* uvw_sw_kernel_ptr<double>(int);
}  // namespace oeqb
