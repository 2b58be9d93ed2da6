// MACE symmetric contraction (reference: _torch/symmetric_contraction/SymmetricContraction.py
// and extension/group_mm.hpp).
//
// For node n of element e and channel c, the reference's contraction of correlation nu_max is
//     out[o] = sum_{i..} T_nu[e,c,o,i1..inu] x_i1 .. x_inu   summed over nu = 1..nu_max,
// with T_nu = W_nu U_nu (weights times the coupled product basis), evaluated as nested
// contractions over materialised [N, C, d_out * K^(nu-1)] intermediates.  Only the
// symmetric part of T_nu contributes, so this build contracts with the distinct monomials
// phi_m = x_a x_b x_c (a <= b <= c) instead:
//     out[o] = sum_m coef[e,c,m,o] phi_m(x),
// where coef (symmetrised T, built by the host with library GEMMs) has K + K(K+1)/2 +
// K(K+1)(K+2)/6 rows (219 for K = 9).  Monomials are enumerated by degree, then in
// lexicographic order of (a, b, c); the kernels walk the same nested loops.
//
// Work mapping (forward, dX): nodes are processed in element-sorted order (perm), a warp is
// one channel and its lanes are 32 consecutive sorted nodes, so the coefficients of (e, c)
// are warp-uniform broadcast loads; a tile that straddles two elements loops over them.
// x (and dZ) rows are staged through shared memory so global accesses are row-contiguous.
// Coefficient gradient: one CTA per (element, channel), each thread owns monomials and
// accumulates over the element's nodes in sorted order (deterministic).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace oeqb {

constexpr int kScWarps = 8;       // channels per CTA (one warp each)
constexpr int kScMaxOut = 16;     // padded output components per (node, channel)

struct ScOutMap {                 // output component o of channel c -> column col[o] + c*step[o]
  int col[kScMaxOut];
  int step[kScMaxOut];
};

template <class T>
struct ArgsSc {
  const T* x;              // [N, C, K]
  const T* gout;           // [N, out_dim] (backward)
  const int64_t* perm;     // sorted position -> node
  const int64_t* elem;     // sorted position -> element
  const int64_t* eoff;     // [E + 1] sorted offsets of each element (coefficient gradient)
  const T* coef;           // [E, C, M, DT]
  T* out;                  // forward: [N, out_dim]; backward: dX [N, C, K]
  T* dcoef;                // [E, C, M, DT]
  long long nodes;
  int channels, k, degree, m, nout, out_dim, num_elements;
  ScOutMap map;
};

__host__ __device__ constexpr int sc_monomials(int k, int degree) {
  return k + (degree >= 2 ? k * (k + 1) / 2 : 0) + (degree >= 3 ? k * (k + 1) * (k + 2) / 6 : 0);
}

// Coefficient row of monomial x_p x_q (p <= q) and x_p x_q x_r (p <= q <= r); the kernels
// call these with unrolled loop indices, so they fold to constants.
template <int K>
__host__ __device__ constexpr int sc_idx2(int p, int q) {
  return K + p * K - p * (p - 1) / 2 + (q - p);
}
template <int K>
__host__ __device__ constexpr int sc_idx3(int p, int q, int r) {
  int n = K + K * (K + 1) / 2;
  for (int pp = 0; pp < p; ++pp) n += (K - pp) * (K - pp + 1) / 2;
  for (int qq = p; qq < q; ++qq) n += K - qq;
  return n + (r - q);
}

// Broadcast load of the DT coefficients of one monomial (16-byte vector loads).
template <class T, int DT>
__device__ __forceinline__ void sc_ldcoef(T (&d)[DT], const T* p) {
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int q = 0; q < DT / 4; ++q) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(p) + q);
      d[4 * q] = t.x;
      d[4 * q + 1] = t.y;
      d[4 * q + 2] = t.z;
      d[4 * q + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int q = 0; q < DT / 2; ++q) {
      const double2 t = __ldg(reinterpret_cast<const double2*>(p) + q);
      d[2 * q] = t.x;
      d[2 * q + 1] = t.y;
    }
  }
}

// Stages rows [pos0, pos0 + 32) of the sorted order, channels [c0, c0 + kScWarps), into
// xs[32][kScWarps * K + 1] (the pad keeps lane-strided reads conflict-free).
template <class T, int K>
__device__ __forceinline__ void sc_stage_x(const ArgsSc<T>& a, T* xs, long long pos0, int c0) {
  constexpr int ROW = kScWarps * K;
  const int nc = min(kScWarps, a.channels - c0);
  for (int e = threadIdx.x; e < 32 * ROW; e += blockDim.x) {
    const int r = e / ROW, q = e - r * ROW;
    const long long pos = pos0 + r;
    T v = T(0);
    if (pos < a.nodes && q < nc * K) v = a.x[(a.perm[pos] * a.channels + c0) * K + q];
    xs[r * (ROW + 1) + q] = v;
  }
}

template <class T, int K, int DT>
__global__ void __launch_bounds__(kScWarps * 32, 2) sc_fwd_kernel(const ArgsSc<T> a) {
  constexpr int ROW = kScWarps * K;
  __shared__ T xs[32 * (ROW + 1)];
  __shared__ T os[32 * kScWarps * DT];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int c0 = blockIdx.y * kScWarps, c = c0 + wid;
  const long long ntiles = (a.nodes + 31) / 32;
  for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const long long pos0 = tile * 32, pos = pos0 + lane;
    __syncthreads();
    sc_stage_x<T, K>(a, xs, pos0, c0);
    __syncthreads();
    const bool live = pos < a.nodes && c < a.channels;
    const int my_e = live ? static_cast<int>(a.elem[pos]) : -1;
    T x[K];
#pragma unroll
    for (int i = 0; i < K; ++i) x[i] = xs[lane * (ROW + 1) + wid * K + i];
    T acc[DT];
#pragma unroll
    for (int o = 0; o < DT; ++o) acc[o] = T(0);
    // Loop over the distinct elements of this tile (one, except at element boundaries).
    unsigned pending = __ballot_sync(0xffffffffu, live);
    while (pending) {
      const int e = __shfl_sync(0xffffffffu, my_e, __ffs(pending) - 1);
      const bool mine = live && my_e == e;
      pending &= ~__ballot_sync(0xffffffffu, mine);
      const T* cf = a.coef + (static_cast<size_t>(e) * a.channels + c) * a.m * DT;
      if (mine) {
#pragma unroll
        for (int p = 0; p < K; ++p) {
          T cv[DT];
          sc_ldcoef<T, DT>(cv, cf + p * DT);
#pragma unroll
          for (int o = 0; o < DT; ++o) acc[o] += cv[o] * x[p];
          if (a.degree >= 2) {
#pragma unroll
            for (int q = p; q < K; ++q) {
              const T xpq = x[p] * x[q];
              sc_ldcoef<T, DT>(cv, cf + sc_idx2<K>(p, q) * DT);
#pragma unroll
              for (int o = 0; o < DT; ++o) acc[o] += cv[o] * xpq;
              if (a.degree >= 3) {
#pragma unroll
                for (int r = q; r < K; ++r) {
                  const T xpqr = xpq * x[r];
                  sc_ldcoef<T, DT>(cv, cf + sc_idx3<K>(p, q, r) * DT);
#pragma unroll
                  for (int o = 0; o < DT; ++o) acc[o] += cv[o] * xpqr;
                }
              }
            }
          }
        }
      }
    }
    // Stage [node][channel][o] and write each node's output columns.
#pragma unroll
    for (int o = 0; o < DT; ++o) os[(lane * kScWarps + wid) * DT + o] = acc[o];
    __syncthreads();
    const int nc = min(kScWarps, a.channels - c0);
    for (int e = threadIdx.x; e < 32 * kScWarps * a.nout; e += blockDim.x) {
      const int r = e / (kScWarps * a.nout), q = e - r * kScWarps * a.nout;
      const int o = q / kScWarps, cc = q - o * kScWarps;  // consecutive threads: channels
      const long long p = pos0 + r;
      if (p < a.nodes && cc < nc)
        a.out[a.perm[p] * a.out_dim + a.map.col[o] + (c0 + cc) * a.map.step[o]] =
            os[(r * kScWarps + cc) * DT + o];
    }
  }
}

template <class T, int K, int DT>
__global__ void __launch_bounds__(kScWarps * 32, 2) sc_bwd_dx_kernel(const ArgsSc<T> a) {
  constexpr int ROW = kScWarps * K;
  __shared__ T xs[32 * (ROW + 1)];
  __shared__ T gs[32 * kScWarps * DT];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int c0 = blockIdx.y * kScWarps, c = c0 + wid;
  const long long ntiles = (a.nodes + 31) / 32;
  const int nc = min(kScWarps, a.channels - c0);
  for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const long long pos0 = tile * 32, pos = pos0 + lane;
    __syncthreads();
    sc_stage_x<T, K>(a, xs, pos0, c0);
    for (int e = threadIdx.x; e < 32 * kScWarps * DT; e += blockDim.x) {
      const int r = e / (kScWarps * DT), q = e - r * kScWarps * DT;
      const int o = q / kScWarps, cc = q - o * kScWarps;
      const long long p = pos0 + r;
      T v = T(0);
      if (p < a.nodes && cc < nc && o < a.nout)
        v = a.gout[a.perm[p] * a.out_dim + a.map.col[o] + (c0 + cc) * a.map.step[o]];
      gs[(r * kScWarps + cc) * DT + o] = v;
    }
    __syncthreads();
    const bool live = pos < a.nodes && c < a.channels;
    const int my_e = live ? static_cast<int>(a.elem[pos]) : -1;
    T x[K], dx[K], g[DT];
#pragma unroll
    for (int i = 0; i < K; ++i) {
      x[i] = xs[lane * (ROW + 1) + wid * K + i];
      dx[i] = T(0);
    }
#pragma unroll
    for (int o = 0; o < DT; ++o) g[o] = gs[(lane * kScWarps + wid) * DT + o];
    unsigned pending = __ballot_sync(0xffffffffu, live);
    while (pending) {
      const int e = __shfl_sync(0xffffffffu, my_e, __ffs(pending) - 1);
      const bool mine = live && my_e == e;
      pending &= ~__ballot_sync(0xffffffffu, mine);
      const T* cf = a.coef + (static_cast<size_t>(e) * a.channels + c) * a.m * DT;
      if (mine) {
#pragma unroll
        for (int p = 0; p < K; ++p) {
          T cv[DT];
          sc_ldcoef<T, DT>(cv, cf + p * DT);
          T G = T(0);
#pragma unroll
          for (int o = 0; o < DT; ++o) G += cv[o] * g[o];
          dx[p] += G;
          if (a.degree >= 2) {
#pragma unroll
            for (int q = p; q < K; ++q) {
              sc_ldcoef<T, DT>(cv, cf + sc_idx2<K>(p, q) * DT);
              T G2 = T(0);
#pragma unroll
              for (int o = 0; o < DT; ++o) G2 += cv[o] * g[o];
              dx[p] += G2 * x[q];
              dx[q] += G2 * x[p];
              if (a.degree >= 3) {
                const T xpq = x[p] * x[q];
#pragma unroll
                for (int r = q; r < K; ++r) {
                  sc_ldcoef<T, DT>(cv, cf + sc_idx3<K>(p, q, r) * DT);
                  T G3 = T(0);
#pragma unroll
                  for (int o = 0; o < DT; ++o) G3 += cv[o] * g[o];
                  const T G3r = G3 * x[r];
                  dx[p] += G3r * x[q];
                  dx[q] += G3r * x[p];
                  dx[r] += G3 * xpq;
                }
              }
            }
          }
        }
      }
    }
    // Stage dX like x and write it row-contiguously.
    __syncthreads();
#pragma unroll
    for (int i = 0; i < K; ++i) xs[lane * (ROW + 1) + wid * K + i] = dx[i];
    __syncthreads();
    for (int e = threadIdx.x; e < 32 * ROW; e += blockDim.x) {
      const int r = e / ROW, q = e - r * ROW;
      const long long p = pos0 + r;
      if (p < a.nodes && q < nc * K) a.out[(a.perm[p] * a.channels + c0) * K + q] = xs[r * (ROW + 1) + q];
    }
  }
}

// dcoef[e, c, m, o] = sum over nodes of element e of g[o] phi_m(x).  One CTA per (e, c);
// thread t owns monomials t, t + blockDim, ...; nodes are consumed in chunks staged in
// shared memory, in sorted order.
template <class T, int K, int DT>
__global__ void __launch_bounds__(256) sc_bwd_dcoef_kernel(const ArgsSc<T> a) {
  constexpr int CH = 64;  // nodes per chunk
  __shared__ T xs[CH * K];
  __shared__ T gs[CH * DT];
  __shared__ unsigned char tri[sc_monomials(K, 3)][3];
  const int e = blockIdx.x / a.channels, c = blockIdx.x - e * a.channels;
  // Monomial index -> (a, b, c) factors (K marks "absent", x[K] = 1).
  for (int t = threadIdx.x; t < a.m; t += blockDim.x) {
    int idx = t, f0 = K, f1 = K, f2 = K;
    if (idx < K) {
      f0 = idx;
    } else if ((idx -= K) < K * (K + 1) / 2) {
      for (int p = 0, n = 0; p < K; ++p)
        for (int q = p; q < K; ++q, ++n)
          if (n == idx) { f0 = p; f1 = q; }
    } else {
      idx -= K * (K + 1) / 2;
      for (int p = 0, n = 0; p < K; ++p)
        for (int q = p; q < K; ++q)
          for (int r = q; r < K; ++r, ++n)
            if (n == idx) { f0 = p; f1 = q; f2 = r; }
    }
    tri[t][0] = static_cast<unsigned char>(f0);
    tri[t][1] = static_cast<unsigned char>(f1);
    tri[t][2] = static_cast<unsigned char>(f2);
  }
  constexpr int MPT = (sc_monomials(K, 3) + 255) / 256;  // monomials per thread
  T acc[MPT][DT];
#pragma unroll
  for (int j = 0; j < MPT; ++j)
#pragma unroll
    for (int o = 0; o < DT; ++o) acc[j][o] = T(0);
  const long long b0 = a.eoff[e], b1 = a.eoff[e + 1];
  for (long long base = b0; base < b1; base += CH) {
    const int n = static_cast<int>(min(static_cast<long long>(CH), b1 - base));
    __syncthreads();
    for (int t = threadIdx.x; t < n * K; t += blockDim.x) {
      const int r = t / K, i = t - r * K;
      xs[t] = a.x[(a.perm[base + r] * a.channels + c) * K + i];
    }
    for (int t = threadIdx.x; t < n * DT; t += blockDim.x) {
      const int r = t / DT, o = t - r * DT;
      gs[t] = o < a.nout ? a.gout[a.perm[base + r] * a.out_dim + a.map.col[o] + c * a.map.step[o]] : T(0);
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < MPT; ++j) {
      const int mi = threadIdx.x + j * 256;
      if (mi < a.m) {
        const int f0 = tri[mi][0], f1 = tri[mi][1], f2 = tri[mi][2];
        for (int r = 0; r < n; ++r) {
          const T* xr = xs + r * K;
          T phi = xr[f0];
          if (f1 < K) phi *= xr[f1];
          if (f2 < K) phi *= xr[f2];
#pragma unroll
          for (int o = 0; o < DT; ++o) acc[j][o] += phi * gs[r * DT + o];
        }
      }
    }
  }
  T* dst = a.dcoef + (static_cast<size_t>(e) * a.channels + c) * a.m * DT;
#pragma unroll
  for (int j = 0; j < MPT; ++j) {
    const int mi = threadIdx.x + j * 256;
    if (mi < a.m)
#pragma unroll
      for (int o = 0; o < DT; ++o) dst[mi * DT + o] = acc[j][o];
  }
}

// ---------------------------------------------------------------------------------------
// group_gemm (extension/group_mm.hpp:38-141), row-major restatement.
//   ragged_inner == 0:  C[r, b, i] = sum_j A[g(r), b, i, j] B[r, b, j]      C: [R, batch, m]
//   ragged_inner == 1:  C[g, b, i, j] = sum_{r in g} A[r, b, i] B[r, b, j] C: [G, batch, m, k]
// where rows are grouped contiguously by `offsets` ([G + 1], device).

template <class T>
struct ArgsGg {
  const T* A;
  const T* B;
  const int64_t* offsets;
  T* C;
  long long rows;
  int groups, batch, m, k;
};

// ragged_inner == 0: one CTA per (row, batch index); threads over the m outputs.
template <class T>
__global__ void __launch_bounds__(256) group_gemm_rows_kernel(const ArgsGg<T> a) {
  extern __shared__ __align__(16) unsigned char gg_smem[];
  T* bv = reinterpret_cast<T*>(gg_smem);
  const long long nb = a.rows * a.batch;
  for (long long item = blockIdx.x; item < nb; item += gridDim.x) {
    const long long r = item / a.batch;
    const int b = static_cast<int>(item - r * a.batch);
    int lo = 0, hi = a.groups;  // group of row r: offsets[g] <= r < offsets[g + 1]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (a.offsets[mid] <= r) lo = mid; else hi = mid;
    }
    __syncthreads();
    for (int j = threadIdx.x; j < a.k; j += blockDim.x) bv[j] = a.B[(r * a.batch + b) * a.k + j];
    __syncthreads();
    const T* Ag = a.A + (static_cast<size_t>(lo) * a.batch + b) * a.m * a.k;
    for (int i = threadIdx.x; i < a.m; i += blockDim.x) {
      T acc = T(0);
      for (int j = 0; j < a.k; ++j) acc += Ag[i * a.k + j] * bv[j];
      a.C[(r * a.batch + b) * a.m + i] = acc;
    }
  }
}

// ragged_inner == 1: one CTA per (group, batch index); threads over the m x k outputs, rows
// consumed in order in chunks staged in shared memory.
template <class T>
__global__ void __launch_bounds__(256) group_gemm_inner_kernel(const ArgsGg<T> a) {
  extern __shared__ __align__(16) unsigned char gg_smem[];
  constexpr int CH = 32;
  T* as = reinterpret_cast<T*>(gg_smem);
  T* bs = as + CH * a.m;
  const int g = blockIdx.x / a.batch, b = blockIdx.x - g * a.batch;
  const long long r0 = a.offsets[g], r1 = a.offsets[g + 1];
  const int nout = a.m * a.k;
  constexpr int OPT = 8;  // outputs per thread per pass
  for (int base = 0; base < nout; base += blockDim.x * OPT) {
    T acc[OPT];
#pragma unroll
    for (int q = 0; q < OPT; ++q) acc[q] = T(0);
    for (long long rr = r0; rr < r1; rr += CH) {
      const int n = static_cast<int>(min(static_cast<long long>(CH), r1 - rr));
      __syncthreads();
      for (int t = threadIdx.x; t < n * a.m; t += blockDim.x) {
        const int r = t / a.m, i = t - r * a.m;
        as[t] = a.A[((rr + r) * a.batch + b) * a.m + i];
      }
      for (int t = threadIdx.x; t < n * a.k; t += blockDim.x) {
        const int r = t / a.k, j = t - r * a.k;
        bs[t] = a.B[((rr + r) * a.batch + b) * a.k + j];
      }
      __syncthreads();
#pragma unroll
      for (int q = 0; q < OPT; ++q) {
        const int o = base + threadIdx.x + q * blockDim.x;
        if (o < nout) {
          const int i = o / a.k, j = o - i * a.k;
          for (int r = 0; r < n; ++r) acc[q] += as[r * a.m + i] * bs[r * a.k + j];
        }
      }
    }
#pragma unroll
    for (int q = 0; q < OPT; ++q) {
      const int o = base + threadIdx.x + q * blockDim.x;
      if (o < nout) a.C[(static_cast<size_t>(g) * a.batch + b) * nout + o] = acc[q];
    }
  }
}

}  // namespace oeqb
