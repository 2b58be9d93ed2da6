// Software-pipelined single-path convolution kernels (tp_kernels_edge_pipe.cuh), float32, one
// instantiation per unrolled degree triple; and the deterministic backward's banded pass B
// (tp_kernels_edge.cuh) for float32 and float64.
#include "tp_kernels_edge_pipe.cuh"

namespace oeqb {

// Deterministic backward pass B of the single-path class (conv_bwd_edge1_band and its fix-up),
// by the degree l1 of the sender rows; float32 for the pipelined kernels, float64 (and float32
// plans outside the pipelined class) for the generic ones.  nullptr for l1 > 3.
template <class T>
const void* edge1_band_kernel(int l1, bool fix) {
  switch (l1) {
    case 0: return fix ? reinterpret_cast<const void*>(conv_bwd_edge1_band_fix<T, 0>)
                       : reinterpret_cast<const void*>(conv_bwd_edge1_band<T, 0>);
    case 1: return fix ? reinterpret_cast<const void*>(conv_bwd_edge1_band_fix<T, 1>)
                       : reinterpret_cast<const void*>(conv_bwd_edge1_band<T, 1>);
    case 2: return fix ? reinterpret_cast<const void*>(conv_bwd_edge1_band_fix<T, 2>)
                       : reinterpret_cast<const void*>(conv_bwd_edge1_band<T, 2>);
    case 3: return fix ? reinterpret_cast<const void*>(conv_bwd_edge1_band_fix<T, 3>)
                       : reinterpret_cast<const void*>(conv_bwd_edge1_band<T, 3>);
    default: return nullptr;
  }
}
template const void* edge1_band_kernel<float>(int, bool);
template const void* edge1_band_kernel<double>(int, bool);

// kind 0 / 1: pipelined atomic forward (two edges per lane) / backward of the triple `code`;
// 4 / 5: deterministic forward (two edges per lane) / backward pass A; 6 / 7: deterministic backward pass B, the
// banded sums and their fix-up (by l1); 2 / 3: the row padding kernels.  nullptr for a triple
// without an unrolled contraction.
const void* edge1_pipe_kernel(int kind, int code) {
  if (kind == 2) return reinterpret_cast<const void*>(conv_pad_rows);
  if (kind == 3) return reinterpret_cast<const void*>(conv_unpad_rows);
  if (kind == 6 || kind == 7) return edge1_band_kernel<float>((code >> 8) & 15, kind == 7);
#define OEQB_PIPE_CASE(A, B, C)                                                               \
  if (code == triple_code(A, B, C)) {                                                         \
    switch (kind) {                                                                           \
      case 0: return reinterpret_cast<const void*>(conv_fwd_edge1_pipe2<A, B, C>);            \
      case 1: return reinterpret_cast<const void*>(conv_bwd_edge1_pipe<A, B, C, false>);      \
      case 4: return reinterpret_cast<const void*>(conv_fwd_edge1_det_pipe2<A, B, C>);        \
      case 5: return reinterpret_cast<const void*>(conv_bwd_edge1_pipe<A, B, C, true>);       \
      default: return nullptr;                                                                \
    }                                                                                         \
  }
  OEQB_FOR_EACH_TRIPLE(OEQB_PIPE_CASE)
#undef OEQB_PIPE_CASE
  return nullptr;
}

}  // namespace oeqb
