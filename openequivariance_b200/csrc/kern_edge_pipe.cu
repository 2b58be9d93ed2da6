// Software-pipelined single-path convolution kernels (tp_kernels_edge_pipe.cuh), float32.
#include "tp_kernels_edge_pipe.cuh"

namespace oeqb {

const void* edge1_pipe_kernel(int kind) {
  switch (kind) {
    case 0: return reinterpret_cast<const void*>(conv_fwd_edge1_pipe<float>);
    case 1: return reinterpret_cast<const void*>(conv_bwd_edge1_pipe<float>);
    default: return nullptr;
  }
}

}  // namespace oeqb
