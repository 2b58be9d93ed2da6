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
// Work mapping (forward, dX): nodes are processed in element-sorted order (perm) in tiles of
// 32 (float64) or 64 (float32) nodes of one element; a warp is one channel, its lanes the
// tile's nodes, and the warp's coefficients of (element, channel) sit in a shared-memory
// cache read by broadcast loads.  x (and dZ) rows are staged through shared memory so global
// accesses are row-contiguous.
// Coefficient gradient: one CTA per (element, channel), each thread owns monomials and
// accumulates over the element's nodes in sorted order (deterministic).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

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
  const int64_t* eoff;     // [E + 1] offsets of each element's range in the sorted order
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

// Stages rows [pos0, pos0 + R) of the sorted order, channels [c0, c0 + kScWarps), into
// xs[R][kScWarps * K + 1] (the pad keeps lane-strided reads conflict-free).
template <class T, int K, int R>
__device__ __forceinline__ void sc_stage_x(const ArgsSc<T>& a, T* xs, long long pos0, int nrows,
                                           int c0) {
  constexpr int ROW = kScWarps * K;
  const int nc = min(kScWarps, a.channels - c0);
  for (int e = threadIdx.x; e < R * ROW; e += blockDim.x) {
    const int r = e / ROW, q = e - r * ROW;
    T v = T(0);
    if (r < nrows && q < nc * K) v = a.x[(a.perm[pos0 + r] * a.channels + c0) * K + q];
    xs[r * (ROW + 1) + q] = v;
  }
}

// Copies the coefficients of (element e, channel c) into this warp's cache.
template <class T, int DT>
__device__ __forceinline__ void sc_load_coef(const ArgsSc<T>& a, T* cache, int e, int c, int lane) {
  const T* src = a.coef + (static_cast<size_t>(e) * a.channels + c) * a.m * DT;
  constexpr int V = 16 / sizeof(T);
  const int nvec = a.m * DT / V;
  for (int i = lane; i < nvec; i += 32)
    reinterpret_cast<uint4*>(cache)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
  __syncwarp();
}

// Broadcast load of the DT coefficients of one monomial from the warp's cache.
template <class T, int DT>
__device__ __forceinline__ void sc_ldcache(T (&d)[DT], const T* p) {
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int q = 0; q < DT / 4; ++q) {
      const float4 t = reinterpret_cast<const float4*>(p)[q];
      d[4 * q] = t.x;
      d[4 * q + 1] = t.y;
      d[4 * q + 2] = t.z;
      d[4 * q + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int q = 0; q < DT / 2; ++q) {
      const double2 t = reinterpret_cast<const double2*>(p)[q];
      d[2 * q] = t.x;
      d[2 * q + 1] = t.y;
    }
  }
}

__host__ __device__ constexpr int sc_npl(int elem) { return elem == 4 ? 2 : 1; }

// Staging area of the forward / dX kernels: R rows of x ([R][8K+1]) or of outputs / dZ
// ([R][8][DT]), whichever is larger; the per-warp coefficient caches follow it.
template <class T, int K, int DT>
__host__ __device__ constexpr int sc_stage_elems() {
  return 32 * sc_npl(sizeof(T)) *
         (kScWarps * K + 1 > kScWarps * DT ? kScWarps * K + 1 : kScWarps * DT);
}

// Layout: tile prefix (num_elements + 1 int64, padded to 16 bytes) | staging | caches.
__host__ __device__ constexpr size_t sc_prefix_bytes(int num_elements) {
  return (static_cast<size_t>(num_elements + 1) * 8 + 15) / 16 * 16;
}

template <class T, int K, int DT>
__host__ __device__ constexpr size_t sc_smem_bytes(int m, int num_elements) {
  return sc_prefix_bytes(num_elements) +
         sizeof(T) * (static_cast<size_t>(sc_stage_elems<T, K, DT>()) +
                      static_cast<size_t>(kScWarps) * m * DT);
}

// Compile-time loop: f(std::integral_constant<int, I>) for I in [B, E).  The monomial loops
// are triangular nests of up to 165 iterations; writing them this way keeps every register
// array index a constant (an unroll pragma alone is not applied that deep).
template <int B, int E, class F>
__device__ __forceinline__ void static_for(F&& f) {
  if constexpr (B < E) {
    f(std::integral_constant<int, B>{});
    static_for<B + 1, E>(f);
  }
}

// acc[j] += sum_m coef_m phi_m(x[j]) for the NPL nodes of this lane (one element).
template <class T, int K, int DT, int NPL>
__device__ __forceinline__ void sc_fwd_pass(const T (&x)[NPL][K], T (&acc)[NPL][DT], const T* cw,
                                            int degree) {
  static_for<0, K>([&](auto P) {
    constexpr int p = decltype(P)::value;
    T cv[DT];
    sc_ldcache<T, DT>(cv, cw + p * DT);
#pragma unroll
    for (int j = 0; j < NPL; ++j)
#pragma unroll
      for (int o = 0; o < DT; ++o) acc[j][o] += cv[o] * x[j][p];
    if (degree >= 2) {
      static_for<p, K>([&](auto Q) {
        constexpr int q = decltype(Q)::value;
        T xpq[NPL];
#pragma unroll
        for (int j = 0; j < NPL; ++j) xpq[j] = x[j][p] * x[j][q];
        T cq[DT];
        sc_ldcache<T, DT>(cq, cw + sc_idx2<K>(p, q) * DT);
#pragma unroll
        for (int j = 0; j < NPL; ++j)
#pragma unroll
          for (int o = 0; o < DT; ++o) acc[j][o] += cq[o] * xpq[j];
        if (degree >= 3) {
          static_for<q, K>([&](auto Rr) {
            constexpr int r = decltype(Rr)::value;
            T cr[DT];
            sc_ldcache<T, DT>(cr, cw + sc_idx3<K>(p, q, r) * DT);
#pragma unroll
            for (int j = 0; j < NPL; ++j) {
              const T xpqr = xpq[j] * x[j][r];
#pragma unroll
              for (int o = 0; o < DT; ++o) acc[j][o] += cr[o] * xpqr;
            }
          });
        }
      });
    }
  });
}

// dx[j] += d/dx sum_o g[j][o] sum_m coef_m,o phi_m(x[j]).
template <class T, int K, int DT, int NPL>
__device__ __forceinline__ void sc_dx_pass(const T (&x)[NPL][K], const T (&g)[NPL][DT],
                                           T (&dx)[NPL][K], const T* cw, int degree) {
  static_for<0, K>([&](auto P) {
    constexpr int p = decltype(P)::value;
    T cv[DT];
    sc_ldcache<T, DT>(cv, cw + p * DT);
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
      T G = T(0);
#pragma unroll
      for (int o = 0; o < DT; ++o) G += cv[o] * g[j][o];
      dx[j][p] += G;
    }
    if (degree >= 2) {
      static_for<p, K>([&](auto Q) {
        constexpr int q = decltype(Q)::value;
        T cq[DT];
        sc_ldcache<T, DT>(cq, cw + sc_idx2<K>(p, q) * DT);
#pragma unroll
        for (int j = 0; j < NPL; ++j) {
          T G2 = T(0);
#pragma unroll
          for (int o = 0; o < DT; ++o) G2 += cq[o] * g[j][o];
          dx[j][p] += G2 * x[j][q];
          dx[j][q] += G2 * x[j][p];
        }
        if (degree >= 3) {
          static_for<q, K>([&](auto Rr) {
            constexpr int r = decltype(Rr)::value;
            T cr[DT];
            sc_ldcache<T, DT>(cr, cw + sc_idx3<K>(p, q, r) * DT);
#pragma unroll
            for (int j = 0; j < NPL; ++j) {
              T G3 = T(0);
#pragma unroll
              for (int o = 0; o < DT; ++o) G3 += cr[o] * g[j][o];
              const T G3r = G3 * x[j][r];
              dx[j][p] += G3r * x[j][q];
              dx[j][q] += G3r * x[j][p];
              dx[j][r] += G3 * (x[j][p] * x[j][q]);
            }
          });
        }
      });
    }
  });
}

// Tiles never span two elements: element e's sorted range [eoff[e], eoff[e+1]) is cut into
// ceil(count / R) tiles of its own.  Every CTA builds the per-element tile prefix in shared
// memory and maps a tile index to (element, first position, rows) by binary search.
__device__ __forceinline__ void sc_tile_prefix(const int64_t* eoff, int num_elements, int R,
                                               long long* tp) {
  if (threadIdx.x == 0) {
    long long t = 0;
    tp[0] = 0;
    for (int e = 0; e < num_elements; ++e) {
      t += (eoff[e + 1] - eoff[e] + R - 1) / R;
      tp[e + 1] = t;
    }
  }
  __syncthreads();
}

__device__ __forceinline__ int sc_tile_element(const long long* tp, int num_elements, long long t) {
  int lo = 0, hi = num_elements;  // tp[lo] <= t < tp[hi]
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (tp[mid] <= t) lo = mid; else hi = mid;
  }
  return lo;
}

// Forward.  Lane l of warp w handles rows l + 32 j (j < NPL) of a tile, channel c0 + w,
// with the warp's coefficients of (element, channel) cached in shared memory.
template <class T, int K, int DT>
__global__ void __launch_bounds__(kScWarps * 32, 2) sc_fwd_kernel(const ArgsSc<T> a) {
  constexpr int NPL = sc_npl(sizeof(T)), R = 32 * NPL, ROW = kScWarps * K;
  extern __shared__ __align__(16) unsigned char sc_smem[];
  long long* tp = reinterpret_cast<long long*>(sc_smem);
  T* xs = reinterpret_cast<T*>(sc_smem + sc_prefix_bytes(a.num_elements));
  T* cache = xs + sc_stage_elems<T, K, DT>();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  T* cw = cache + static_cast<size_t>(wid) * a.m * DT;
  const int c0 = blockIdx.y * kScWarps, c = c0 + wid;
  const int nc = min(kScWarps, a.channels - c0);
  sc_tile_prefix(a.eoff, a.num_elements, R, tp);
  const long long ntiles = tp[a.num_elements];
  int cached = -1;
  for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int e = sc_tile_element(tp, a.num_elements, tile);
    const long long pos0 = a.eoff[e] + (tile - tp[e]) * R;
    const int nrows = static_cast<int>(min(static_cast<long long>(R), a.eoff[e + 1] - pos0));
    __syncthreads();
    sc_stage_x<T, K, R>(a, xs, pos0, nrows, c0);
    if (e != cached && c < a.channels) {
      sc_load_coef<T, DT>(a, cw, e, c, lane);
      cached = e;
    }
    __syncthreads();
    T x[NPL][K], acc[NPL][DT];
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
#pragma unroll
      for (int i = 0; i < K; ++i) x[j][i] = xs[(lane + 32 * j) * (ROW + 1) + wid * K + i];
#pragma unroll
      for (int o = 0; o < DT; ++o) acc[j][o] = T(0);
    }
    if (c < a.channels) sc_fwd_pass<T, K, DT, NPL>(x, acc, cw, a.degree);
    // Stage [row][channel][o] (reusing xs) and write each node's output columns.
    __syncthreads();
#pragma unroll
    for (int j = 0; j < NPL; ++j)
#pragma unroll
      for (int o = 0; o < DT; ++o) xs[((lane + 32 * j) * kScWarps + wid) * DT + o] = acc[j][o];
    __syncthreads();
    for (int t = threadIdx.x; t < nrows * kScWarps * a.nout; t += blockDim.x) {
      const int r = t / (kScWarps * a.nout), q = t - r * kScWarps * a.nout;
      const int o = q / kScWarps, cc = q - o * kScWarps;  // consecutive threads: channels
      if (cc < nc)
        a.out[a.perm[pos0 + r] * a.out_dim + a.map.col[o] + (c0 + cc) * a.map.step[o]] =
            xs[(r * kScWarps + cc) * DT + o];
    }
  }
}

// dX, same mapping as the forward.
template <class T, int K, int DT>
__global__ void __launch_bounds__(kScWarps * 32, 2) sc_bwd_dx_kernel(const ArgsSc<T> a) {
  constexpr int NPL = sc_npl(sizeof(T)), R = 32 * NPL, ROW = kScWarps * K;
  extern __shared__ __align__(16) unsigned char sc_smem[];
  long long* tp = reinterpret_cast<long long*>(sc_smem);
  T* xs = reinterpret_cast<T*>(sc_smem + sc_prefix_bytes(a.num_elements));
  T* cache = xs + sc_stage_elems<T, K, DT>();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  T* cw = cache + static_cast<size_t>(wid) * a.m * DT;
  const int c0 = blockIdx.y * kScWarps, c = c0 + wid;
  const int nc = min(kScWarps, a.channels - c0);
  sc_tile_prefix(a.eoff, a.num_elements, R, tp);
  const long long ntiles = tp[a.num_elements];
  int cached = -1;
  for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int e = sc_tile_element(tp, a.num_elements, tile);
    const long long pos0 = a.eoff[e] + (tile - tp[e]) * R;
    const int nrows = static_cast<int>(min(static_cast<long long>(R), a.eoff[e + 1] - pos0));
    T x[NPL][K], g[NPL][DT], dx[NPL][K];
    __syncthreads();
    sc_stage_x<T, K, R>(a, xs, pos0, nrows, c0);
    if (e != cached && c < a.channels) {
      sc_load_coef<T, DT>(a, cw, e, c, lane);
      cached = e;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < NPL; ++j)
#pragma unroll
      for (int i = 0; i < K; ++i) {
        x[j][i] = xs[(lane + 32 * j) * (ROW + 1) + wid * K + i];
        dx[j][i] = T(0);
      }
    // Stage dZ of the tile as [row][channel][o] in xs.
    __syncthreads();
    for (int t = threadIdx.x; t < R * kScWarps * DT; t += blockDim.x) {
      const int r = t / (kScWarps * DT), q = t - r * kScWarps * DT;
      const int o = q / kScWarps, cc = q - o * kScWarps;
      T v = T(0);
      if (r < nrows && cc < nc && o < a.nout)
        v = a.gout[a.perm[pos0 + r] * a.out_dim + a.map.col[o] + (c0 + cc) * a.map.step[o]];
      xs[(r * kScWarps + cc) * DT + o] = v;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < NPL; ++j)
#pragma unroll
      for (int o = 0; o < DT; ++o) g[j][o] = xs[((lane + 32 * j) * kScWarps + wid) * DT + o];
    if (c < a.channels) sc_dx_pass<T, K, DT, NPL>(x, g, dx, cw, a.degree);
    // Stage dX like x and write it row-contiguously.
    __syncthreads();
#pragma unroll
    for (int j = 0; j < NPL; ++j)
#pragma unroll
      for (int i = 0; i < K; ++i) xs[(lane + 32 * j) * (ROW + 1) + wid * K + i] = dx[j][i];
    __syncthreads();
    for (int t = threadIdx.x; t < nrows * ROW; t += blockDim.x) {
      const int r = t / ROW, q = t - r * ROW;
      if (q < nc * K) a.out[(a.perm[pos0 + r] * a.channels + c0) * K + q] = xs[r * (ROW + 1) + q];
    }
  }
}

// dcoef[e, c, m, o] = sum over nodes of element e of g[o] phi_m(x).  One CTA per (e, c);
// thread t owns monomials t, t + blockDim, ...; nodes are consumed in chunks staged in
// shared memory, in sorted order: the chunk's node indices first, then independent gathers of
// x and g.  A staged x row has K + 1 slots, the last one 1, so every monomial is
// x[f0] x[f1] x[f2] without branches (absent factors point at the 1); a node's DT output
// gradients are vector loads.
template <class T, int K, int DT>
__global__ void __launch_bounds__(256) sc_bwd_dcoef_kernel(const ArgsSc<T> a) {
  constexpr int CH = 256;     // nodes per chunk
  constexpr int XR = K + 1;   // staged x row: K values and a 1
  __shared__ T xs[CH * XR];
  __shared__ __align__(16) T gs[CH * DT];
  __shared__ long long ps[CH];  // the chunk's node indices
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
  // Zero rows (and the 1 slots) once: the unrolled loop reads up to 3 rows past a short last
  // chunk, which then hold zeros or an earlier chunk's x (finite), times zero gradients.
  for (int t = threadIdx.x; t < CH * XR; t += blockDim.x) xs[t] = t % XR == K ? T(1) : T(0);
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
    for (int r = threadIdx.x; r < n; r += blockDim.x) ps[r] = a.perm[base + r];
    __syncthreads();
#pragma unroll 4
    for (int t = threadIdx.x; t < n * K; t += blockDim.x) {
      const int r = t / K, i = t - r * K;
      xs[r * XR + i] = a.x[(ps[r] * a.channels + c) * K + i];
    }
#pragma unroll 4
    for (int t = threadIdx.x; t < n * DT; t += blockDim.x) {
      const int r = t / DT, o = t - r * DT;
      gs[t] = o < a.nout ? a.gout[ps[r] * a.out_dim + a.map.col[o] + c * a.map.step[o]] : T(0);
    }
    // Rows n..CH-1 of a short last chunk: zero gradients, so the unrolled loop adds nothing.
    for (int t = n * DT + threadIdx.x; t < CH * DT; t += blockDim.x) gs[t] = T(0);
    __syncthreads();
    const int nr = (n + 3) & ~3;  // rows rounded up to the unroll
#pragma unroll
    for (int j = 0; j < MPT; ++j) {
      const int mi = threadIdx.x + j * 256;
      if (mi < a.m) {
        const T* x0 = xs + tri[mi][0];
        const T* x1 = xs + tri[mi][1];
        const T* x2 = xs + tri[mi][2];
#pragma unroll 4
        for (int r = 0; r < nr; ++r) {
          const T phi = x0[r * XR] * x1[r * XR] * x2[r * XR];
          T gv[DT];
          if constexpr (sizeof(T) == 4 && DT % 4 == 0) {
#pragma unroll
            for (int o4 = 0; o4 < DT; o4 += 4) {
              const float4 q = reinterpret_cast<const float4*>(gs + r * DT + o4)[0];
              gv[o4] = q.x;
              gv[o4 + 1] = q.y;
              gv[o4 + 2] = q.z;
              gv[o4 + 3] = q.w;
            }
          } else {
#pragma unroll
            for (int o = 0; o < DT; ++o) gv[o] = gs[r * DT + o];
          }
#pragma unroll
          for (int o = 0; o < DT; ++o) acc[j][o] += phi * gv[o];
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
