// C ABI of the symmetric contraction and of group_gemm (declared in include/oeqb200.h):
// argument checks, kernel selection by (dtype, k, dt) and launch configuration.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <set>
#include <string>

#include "oeqb200.h"
#include "sc_kernels.cuh"

namespace oeqb {
int set_error(int code, const std::string& msg);
}

using namespace oeqb;

namespace {

#define SC_CUDA(expr)                                                                    \
  do {                                                                                   \
    cudaError_t e_ = (expr);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return set_error(OEQB_ERR_CUDA, std::string(#expr " failed: ") + cudaGetErrorString(e_)); \
  } while (0)

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

template <class T, int K, int DT>
int sc_launch(int kind, const ArgsSc<T>& a, cudaStream_t s) {
  const unsigned cblocks = static_cast<unsigned>((a.channels + kScWarps - 1) / kScWarps);
  const long long ntiles = (a.nodes + 31) / 32;
  if (kind == 2) {
    if (a.num_elements * a.channels > 0) {
      sc_bwd_dcoef_kernel<T, K, DT><<<a.num_elements * a.channels, 256, 0, s>>>(a);
      SC_CUDA(cudaGetLastError());
    }
    return 0;
  }
  if (ntiles == 0) return 0;
  const void* fn = kind == 0 ? reinterpret_cast<const void*>(sc_fwd_kernel<T, K, DT>)
                             : reinterpret_cast<const void*>(sc_bwd_dx_kernel<T, K, DT>);
  const size_t smem = sc_smem_bytes<T, K, DT>(a.m, a.num_elements);
  int per_sm = 0;
  {
    static std::mutex mu;
    static std::set<std::pair<int, const void*>> done;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    if (!done.count({dev, fn})) {
      SC_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
      done.insert({dev, fn});
    }
  }
  if (smem > 200 * 1024) return set_error(OEQB_ERR_UNSUPPORTED, "symmetric contraction: shapes exceed shared memory");
  SC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kScWarps * 32, smem));
  if (per_sm <= 0) return set_error(OEQB_ERR_UNSUPPORTED, "symmetric contraction kernel does not fit");
  // Persistent over node tiles: resident CTAs per SM, spread across the channel blocks.
  const long long tiles = (a.nodes + 32 * sc_npl(sizeof(T)) - 1) / (32 * sc_npl(sizeof(T))) +
                          a.num_elements;
  const long long want = std::max<long long>(1, static_cast<long long>(per_sm) * sm_count() / cblocks);
  const dim3 grid(static_cast<unsigned>(std::min(tiles, want)), cblocks);
  void* params[] = {const_cast<ArgsSc<T>*>(&a)};
  SC_CUDA(cudaLaunchKernel(fn, grid, dim3(kScWarps * 32), params, smem, s));
  return 0;
}

template <class T>
int sc_dispatch(int kind, const ArgsSc<T>& a, int dt, cudaStream_t s) {
  if (a.k == 9 && dt == 4) return sc_launch<T, 9, 4>(kind, a, s);
  if (a.k == 4 && dt == 4) return sc_launch<T, 4, 4>(kind, a, s);
  // 16 padded outputs: float only (the double staging buffers exceed 48 KB of static smem).
  if constexpr (sizeof(T) == 4) {
    if (a.k == 9 && dt == 16) return sc_launch<T, 9, 16>(kind, a, s);
    if (a.k == 4 && dt == 16) return sc_launch<T, 4, 16>(kind, a, s);
  }
  return set_error(OEQB_ERR_UNSUPPORTED, "symmetric contraction: unsupported (k, dt) = (" +
                                             std::to_string(a.k) + ", " + std::to_string(dt) + ")");
}

template <class T>
int sc_common(ArgsSc<T>& a, int dt, int nout, const int* out_col, const int* out_step) {
  if (a.nodes < 0 || a.channels <= 0 || a.degree < 1 || a.degree > 3 || a.num_elements <= 0)
    return set_error(OEQB_ERR_INVALID, "symmetric contraction: bad sizes or degree (1..3)");
  if (dt != 4 && dt != 16) return set_error(OEQB_ERR_UNSUPPORTED, "symmetric contraction: dt must be 4 or 16");
  if (nout < 1 || nout > dt) return set_error(OEQB_ERR_INVALID, "symmetric contraction: nout must be in [1, dt]");
  a.m = sc_monomials(a.k, a.degree);
  a.nout = nout;
  for (int o = 0; o < kScMaxOut; ++o) {
    a.map.col[o] = o < nout ? out_col[o] : 0;
    a.map.step[o] = o < nout ? out_step[o] : 0;
  }
  return 0;
}

}  // namespace

extern "C" {

int oeqb_sc_forward(int dtype, int64_t nodes, int channels, int k, int degree, int dt, int nout,
                    const int* out_col, const int* out_step, int64_t out_dim, int num_elements,
                    const void* x, const int64_t* perm, const int64_t* elem_offsets,
                    const void* coef, void* out, void* stream) {
  auto run = [&](auto tag) -> int {
    using T = decltype(tag);
    ArgsSc<T> a{};
    a.x = static_cast<const T*>(x);
    a.perm = perm;
    a.eoff = elem_offsets;
    a.num_elements = num_elements;
    a.coef = static_cast<const T*>(coef);
    a.out = static_cast<T*>(out);
    a.nodes = nodes;
    a.channels = channels;
    a.k = k;
    a.degree = degree;
    a.out_dim = static_cast<int>(out_dim);
    if (int rc = sc_common(a, dt, nout, out_col, out_step)) return rc;
    return sc_dispatch<T>(0, a, dt, static_cast<cudaStream_t>(stream));
  };
  if (dtype == 1) return run(float{});
  if (dtype == 2) return run(double{});
  return set_error(OEQB_ERR_INVALID, "symmetric contraction: dtype must be 1 (f32) or 2 (f64)");
}

int oeqb_sc_backward(int dtype, int64_t nodes, int channels, int k, int degree, int dt, int nout,
                     const int* out_col, const int* out_step, int64_t out_dim, int num_elements,
                     const void* x, const int64_t* perm, const int64_t* elem_offsets,
                     const void* coef, const void* grad_out, void* grad_x, void* grad_coef,
                     void* stream) {
  auto run = [&](auto tag) -> int {
    using T = decltype(tag);
    ArgsSc<T> a{};
    a.x = static_cast<const T*>(x);
    a.gout = static_cast<const T*>(grad_out);
    a.perm = perm;
    a.eoff = elem_offsets;
    a.coef = static_cast<const T*>(coef);
    a.out = static_cast<T*>(grad_x);
    a.dcoef = static_cast<T*>(grad_coef);
    a.nodes = nodes;
    a.channels = channels;
    a.k = k;
    a.degree = degree;
    a.out_dim = static_cast<int>(out_dim);
    a.num_elements = num_elements;
    if (int rc = sc_common(a, dt, nout, out_col, out_step)) return rc;
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (grad_x)
      if (int rc = sc_dispatch<T>(1, a, dt, s)) return rc;
    if (grad_coef)
      if (int rc = sc_dispatch<T>(2, a, dt, s)) return rc;
    return 0;
  };
  if (dtype == 1) return run(float{});
  if (dtype == 2) return run(double{});
  return set_error(OEQB_ERR_INVALID, "symmetric contraction: dtype must be 1 (f32) or 2 (f64)");
}

int oeqb_group_gemm(int dtype, const void* A, const void* B, const int64_t* offsets,
                    int num_groups, int64_t rows, int batch, int m, int k, int ragged_inner,
                    void* C, void* stream) {
  if (num_groups < 0 || rows < 0 || batch < 0 || m < 0 || k < 0)
    return set_error(OEQB_ERR_INVALID, "group_gemm: negative size");
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto run = [&](auto tag) -> int {
    using T = decltype(tag);
    ArgsGg<T> a{static_cast<const T*>(A), static_cast<const T*>(B), offsets, static_cast<T*>(C),
                rows, num_groups, batch, m, k};
    if (ragged_inner == 0) {
      const long long items = rows * batch;
      if (items == 0 || m == 0) return 0;
      const size_t smem = sizeof(T) * static_cast<size_t>(k);
      if (smem > 48 * 1024) return set_error(OEQB_ERR_UNSUPPORTED, "group_gemm: k too large");
      const unsigned grid = static_cast<unsigned>(std::min<long long>(items, 16LL * sm_count()));
      group_gemm_rows_kernel<T><<<grid, 256, smem, s>>>(a);
    } else {
      const long long items = static_cast<long long>(num_groups) * batch;
      if (items == 0 || m == 0 || k == 0) return 0;
      const size_t smem = sizeof(T) * 32 * static_cast<size_t>(m + k);
      if (smem > 200 * 1024) return set_error(OEQB_ERR_UNSUPPORTED, "group_gemm: m + k too large");
      static std::mutex mu;
      static std::set<std::pair<int, const void*>> done;
      {
        int dev = 0;
        cudaGetDevice(&dev);
        std::lock_guard<std::mutex> g(mu);
        const void* fn = reinterpret_cast<const void*>(group_gemm_inner_kernel<T>);
        if (!done.count({dev, fn})) {
          SC_CUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024));
          done.insert({dev, fn});
        }
      }
      group_gemm_inner_kernel<T><<<static_cast<unsigned>(items), 256, smem, s>>>(a);
    }
    SC_CUDA(cudaGetLastError());
    return 0;
  };
  if (dtype == 1) return run(float{});
  if (dtype == 2) return run(double{});
  return set_error(OEQB_ERR_INVALID, "group_gemm: dtype must be 1 (f32) or 2 (f64)");
}

}  // extern "C"
