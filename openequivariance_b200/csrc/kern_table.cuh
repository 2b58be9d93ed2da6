// Kernel-pointer tables: each translation unit instantiates one dtype x family so the
// unrolled kernels compile in parallel.  The host runtime (capi.cu) looks kernels up
// here and launches them with cudaLaunchKernel.
#pragma once
#include "tp_kernels.cuh"
#include "tp_kernels_edge.cuh"
#include "tp_kernels_lk.cuh"

namespace oeqb {

// kind: 0 = forward (or double-backward part A), 1 = backward (or part B)
template <class T>
const void* batch_kernel_ptr(int kind, bool uvw, bool db, int policy);

template <class T>
const void* det_kernel_ptr(int kind, bool uvw, bool db, bool kahan);

// Row-staged wide-uvu batch kernels (tp_kernels_row.cuh); kind 0 = forward, 1 = backward.
template <class T>
const void* row_kernel_ptr(int kind, int nwarps);

// Channelwise-uvu segment kernels (tp_kernels_seg.cuh); kind 0 = forward, 1 = backward.
template <class T>
const void* seg_kernel_ptr(int kind);
template <class T>
const void* lk_kernel_ptr(int cpl);  // cpl = channels per lane (1 or 2)
template <class T>
const void* lkf_kernel_ptr(int cpl);  // lockstep forward
// Edge-per-lane convolution for multiplicity-1 problems (tp_kernels_edge.cuh); kind 0/1 =
// forward/backward, 2/3 = the single-path variants, 4/5/6 = single-path deterministic
// forward, backward pass A (messages to the workspace) and pass B (sender-ordered sums).
template <class T>
const void* edge_kernel_ptr(int kind);

#define OEQB_PICK4(K, T, P)                                                     \
  (uvw ? (db ? (const void*)K<T, true, true, P> : (const void*)K<T, true, false, P>) \
       : (db ? (const void*)K<T, false, true, P> : (const void*)K<T, false, false, P>))

#define OEQB_DEFINE_BATCH_TABLE(T)                                              \
  template <>                                                                   \
  const void* batch_kernel_ptr<T>(int kind, bool uvw, bool db, int policy) {     \
    if (kind == 0)                                                              \
      return policy == kBatch ? OEQB_PICK4(tp_fwd_kernel, T, kBatch)            \
                              : OEQB_PICK4(tp_fwd_kernel, T, kConvAtomic);      \
    return policy == kBatch ? OEQB_PICK4(tp_bwd_kernel, T, kBatch)              \
                            : OEQB_PICK4(tp_bwd_kernel, T, kConvAtomic);        \
  }

#define OEQB_DEFINE_ROW_TABLE(T)                                                \
  template <>                                                                   \
  const void* row_kernel_ptr<T>(int kind, int nwarps) {                          \
    if (kind == 0) return (const void*)tp_fwd_row<T, 8>;                          \
    return nwarps == 16 ? (const void*)tp_bwd_row<T, 16> : (const void*)tp_bwd_row<T, 8>; \
  }

#define OEQB_DEFINE_CW_TABLE(T)                                                 \
  template <>                                                                   \
  const void* seg_kernel_ptr<T>(int kind) {                                     \
    return kind == 0 ? (const void*)tp_fwd_seg<T> : (const void*)tp_bwd_seg<T, 16>; \
  }                                                                               \
  template <>                                                                     \
  const void* lk_kernel_ptr<T>(int cpl) {                                        \
    return cpl == 2 ? (const void*)tp_bwd_lk<T, 2> : (const void*)tp_bwd_lk<T, 1>; \
  }                                                                               \
  template <>                                                                     \
  const void* lkf_kernel_ptr<T>(int cpl) {                                        \
    return cpl == 2 ? (const void*)tp_fwd_lk<T, 2> : (const void*)tp_fwd_lk<T, 1>; \
  }                                                                               \
  template <>                                                                     \
  const void* edge_kernel_ptr<T>(int kind) {                                      \
    switch (kind) {                                                               \
      case 0: return (const void*)conv_fwd_edge<T>;                               \
      case 1: return (const void*)conv_bwd_edge<T>;                               \
      case 2: return (const void*)conv_fwd_edge1<T>;                              \
      case 3: return (const void*)conv_bwd_edge1<T>;                              \
      case 4: return (const void*)conv_fwd_edge1_det<T>;                          \
      case 5: return (const void*)conv_bwd_edge1_msg<T>;                          \
      default: return nullptr;                                                    \
    }                                                                             \
  }

#define OEQB_DEFINE_DET_TABLE(T, WITH_KAHAN)                                    \
  template <>                                                                   \
  const void* det_kernel_ptr<T>(int kind, bool uvw, bool db, bool kahan) {       \
    if (WITH_KAHAN && kahan)                                                    \
      return kind == 0 ? OEQB_PICK4(conv_fwd_det, T, WITH_KAHAN)                \
                       : OEQB_PICK4(conv_bwd_det, T, WITH_KAHAN);               \
    return kind == 0 ? OEQB_PICK4(conv_fwd_det, T, false)                       \
                     : OEQB_PICK4(conv_bwd_det, T, false);                      \
  }

}  // namespace oeqb
