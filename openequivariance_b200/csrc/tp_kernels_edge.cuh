// Edge-per-lane fused convolution for problems whose instructions all have multiplicity 1
// (the C3 class: e.g. 1x2e x 1x3e -> 1x2e), atomic mode.
//
// Reference semantics: z[rows[e]] += TP(x[cols[e]], y[e], W[e])
// (core/ConvolutionBase.py:300-309, templates/loop_unroll_conv_atomic.cuh:53-363).
//
// With multiplicity 1 a whole edge is one lane's work.  A warp takes 32 consecutive edges:
// Y and W rows (contiguous in memory) are copied into shared memory with coalesced loads, X
// rows are gathered per lane, and each instruction runs its unrolled CG contraction on the
// lane's slices.  Edges are receiver-sorted, so in the forward pass the lanes of a warp mostly
// share one receiver: a segmented shuffle reduction over equal receivers leaves one reduction
// per receiver segment instead of one per edge.  In the backward pass dY and dW are per edge
// (written back coalesced through shared memory) and dX goes to the senders, which differ
// across lanes: one reduction per edge, both written as aligned vector reductions (red_row).
#pragma once

#include "tp_kernels.cuh"

namespace oeqb {

constexpr int kEdgeWarps = 8;

struct EdgeLayout {  // padded per-lane row lengths (odd, so lane-strided accesses do not conflict)
  int l1p, l2p, l3p, wp;
};

__host__ __device__ constexpr int edge_pad(int n) { return n % 2 == 0 ? n + 1 : n; }

// Shared-memory elements of one warp's buffers (forward, backward).
__host__ __device__ constexpr int edge_warp_elems(const EdgeLayout& L, bool bwd) {
  return 32 * (L.l1p + L.l2p + L.l3p + L.wp + (bwd ? L.l1p + L.l2p + L.wp : 0));
}

// Adds n values (shared memory, stride 1) into a global row with the fewest reduction
// operations: 16-byte aligned runs of four go out as one red.global.add.v4.f32, 8-byte
// aligned pairs as .v2, the rest one by one.  The L2 reduction units, not the lanes, bound the
// atomic scatter, so fewer and wider operations are what counts.
template <class T>
__device__ __forceinline__ void red_row(T* dst, const T* src, int n) {
  if constexpr (sizeof(T) == 4) {
    int i = 0;
    while (i < n) {
      const unsigned long long ad = reinterpret_cast<unsigned long long>(dst + i);
      if ((ad & 15) == 0 && n - i >= 4) {
        asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"l"(dst + i),
                     "f"(src[i]), "f"(src[i + 1]), "f"(src[i + 2]), "f"(src[i + 3])
                     : "memory");
        i += 4;
      } else if ((ad & 7) == 0 && n - i >= 2) {
        asm volatile("red.global.add.v2.f32 [%0], {%1, %2};\n" ::"l"(dst + i), "f"(src[i]),
                     "f"(src[i + 1])
                     : "memory");
        i += 2;
      } else {
        atomic_add(dst + i, src[i]);
        i += 1;
      }
    }
  } else {
    for (int i = 0; i < n; ++i) atomic_add(dst + i, src[i]);
  }
}

template <class T>
__device__ __forceinline__ void edge_copy_rows(T* dst, int pitch, const T* src, int width,
                                               long long base, long long n, int lane) {
  for (int t = lane; t < 32 * width; t += 32) {
    const int r = t / width, j = t - r * width;
    dst[r * pitch + j] = base + r < n ? src[(base + r) * width + j] : T(0);
  }
}

template <class T>
__global__ void __launch_bounds__(kEdgeWarps * 32) conv_fwd_edge(const Args<T> a, const EdgeLayout L) {
  extern __shared__ __align__(16) unsigned char smem[];
  InstrD* ins = reinterpret_cast<InstrD*>(smem);
  for (int i = threadIdx.x; i < a.nins * static_cast<int>(sizeof(InstrD) / 4); i += blockDim.x)
    reinterpret_cast<int*>(ins)[i] = reinterpret_cast<const int*>(a.ins)[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  T* base_ptr = reinterpret_cast<T*>(smem + ((sizeof(InstrD) * a.nins + 15) & ~size_t(15)));
  T* xs = base_ptr + static_cast<size_t>(wid) * edge_warp_elems(L, false);
  T* ys = xs + 32 * L.l1p;
  T* zs = ys + 32 * L.l2p;
  T* ws = zs + 32 * L.l3p;
  const long long nw = static_cast<long long>(gridDim.x) * kEdgeWarps;
  for (long long base = (static_cast<long long>(blockIdx.x) * kEdgeWarps + wid) * 32;
       base < a.nitems; base += nw * 32) {
    const long long e = base + lane;
    bool valid = e < a.nitems;
    long long row = valid ? a.rows[e] : -1, col = valid ? a.cols[e] : 0;
    if (valid && (row < 0 || row >= a.nnodes || col < 0 || col >= a.nnodes)) {
      flag(a.status, 1);
      valid = false;
      row = -1;
      col = 0;
    }
    __syncwarp();
    edge_copy_rows(ys, L.l2p, a.Y, a.L2dim, base, a.nitems, lane);
    if (!a.shared_w) edge_copy_rows(ws, L.wp, a.W, a.wnumel, base, a.nitems, lane);
    for (int i = 0; i < a.L1dim; ++i) xs[lane * L.l1p + i] = valid ? a.X[col * a.L1dim + i] : T(0);
    for (int k = 0; k < a.L3dim; ++k) zs[lane * L.l3p + k] = T(0);
    __syncwarp();
    for (int n = 0; n < a.nins; ++n) {
      const InstrD in = ins[n];
      const int o1 = a.ir1[in.i1].off, o2 = a.ir2[in.i2].off, o3 = a.ir3[in.i3].off;
      const T w = (a.shared_w ? a.W[in.woff] : ws[lane * L.wp + in.woff]) * T(in.pw);
      dispatch_triple(in.code, [&]<int A, int B, int C>() {
        constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1, D3 = 2 * C + 1;
        T x[D1], y[D2], z[D3];
#pragma unroll
        for (int i = 0; i < D1; ++i) x[i] = xs[lane * L.l1p + o1 + i] * w;
#pragma unroll
        for (int j = 0; j < D2; ++j) y[j] = ys[lane * L.l2p + o2 + j];
#pragma unroll
        for (int k = 0; k < D3; ++k) z[k] = zs[lane * L.l3p + o3 + k];
        CG<A, B, C>::fwd(x, y, z);
#pragma unroll
        for (int k = 0; k < D3; ++k) zs[lane * L.l3p + o3 + k] = z[k];
      });
    }
    // Segmented suffix sums over equal receivers (rows are sorted), one atomic per segment.
    const int r32 = static_cast<int>(row);
    const int prev = __shfl_up_sync(0xffffffffu, r32, 1);
    const bool head = row >= 0 && (lane == 0 || prev != r32);
    for (int k = 0; k < a.L3dim; ++k) {
      T v = zs[lane * L.l3p + k];
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const T vo = __shfl_down_sync(0xffffffffu, v, off);
        const int ro = __shfl_down_sync(0xffffffffu, r32, off);
        if (lane + off < 32 && ro == r32) v += vo;
      }
      zs[lane * L.l3p + k] = v;  // the lane's own column: no other lane reads it
    }
    if (head) red_row(a.out0 + row * a.L3dim, zs + lane * L.l3p, a.L3dim);
  }
}

template <class T>
__global__ void __launch_bounds__(kEdgeWarps * 32) conv_bwd_edge(const Args<T> a, const EdgeLayout L) {
  extern __shared__ __align__(16) unsigned char smem[];
  InstrD* ins = reinterpret_cast<InstrD*>(smem);
  for (int i = threadIdx.x; i < a.nins * static_cast<int>(sizeof(InstrD) / 4); i += blockDim.x)
    reinterpret_cast<int*>(ins)[i] = reinterpret_cast<const int*>(a.ins)[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  T* base_ptr = reinterpret_cast<T*>(smem + ((sizeof(InstrD) * a.nins + 15) & ~size_t(15)));
  T* xs = base_ptr + static_cast<size_t>(wid) * edge_warp_elems(L, true);
  T* ys = xs + 32 * L.l1p;
  T* gs = ys + 32 * L.l2p;
  T* ws = gs + 32 * L.l3p;
  T* gxs = ws + 32 * L.wp;
  T* gys = gxs + 32 * L.l1p;
  T* gws = gys + 32 * L.l2p;
  const long long nw = static_cast<long long>(gridDim.x) * kEdgeWarps;
  for (long long base = (static_cast<long long>(blockIdx.x) * kEdgeWarps + wid) * 32;
       base < a.nitems; base += nw * 32) {
    const long long e = base + lane;
    bool valid = e < a.nitems;
    long long row = valid ? a.rows[e] : 0, col = valid ? a.cols[e] : 0;
    if (valid && (row < 0 || row >= a.nnodes || col < 0 || col >= a.nnodes)) {
      flag(a.status, 1);
      valid = false;
      row = col = 0;
    }
    __syncwarp();
    edge_copy_rows(ys, L.l2p, a.Y, a.L2dim, base, a.nitems, lane);
    if (!a.shared_w) edge_copy_rows(ws, L.wp, a.W, a.wnumel, base, a.nitems, lane);
    for (int i = 0; i < a.L1dim; ++i) {
      xs[lane * L.l1p + i] = valid ? a.X[col * a.L1dim + i] : T(0);
      gxs[lane * L.l1p + i] = T(0);
    }
    for (int k = 0; k < a.L3dim; ++k) gs[lane * L.l3p + k] = valid ? a.Gz[row * a.L3dim + k] : T(0);
    for (int j = 0; j < a.L2dim; ++j) gys[lane * L.l2p + j] = T(0);
    __syncwarp();
    for (int n = 0; n < a.nins; ++n) {
      const InstrD in = ins[n];
      const int o1 = a.ir1[in.i1].off, o2 = a.ir2[in.i2].off, o3 = a.ir3[in.i3].off;
      const T pw = T(in.pw);
      const T w = a.shared_w ? a.W[in.woff] : ws[lane * L.wp + in.woff];
      dispatch_triple(in.code, [&]<int A, int B, int C>() {
        constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1, D3 = 2 * C + 1;
        T x[D1], y[D2], g[D3], h[D1], ev[D2];
#pragma unroll
        for (int i = 0; i < D1; ++i) x[i] = xs[lane * L.l1p + o1 + i];
#pragma unroll
        for (int j = 0; j < D2; ++j) y[j] = ys[lane * L.l2p + o2 + j];
#pragma unroll
        for (int k = 0; k < D3; ++k) g[k] = gs[lane * L.l3p + o3 + k] * pw;
        CG<A, B, C>::hvec(g, y, h);
        CG<A, B, C>::evec(g, x, ev);
        T sdot = T(0);
#pragma unroll
        for (int i = 0; i < D1; ++i) {
          gxs[lane * L.l1p + o1 + i] += w * h[i];
          sdot += x[i] * h[i];
        }
#pragma unroll
        for (int j = 0; j < D2; ++j) gys[lane * L.l2p + o2 + j] += w * ev[j];
        if (a.shared_w) {
          // Warp sum of dW, one atomic per warp and instruction.
          T s = valid ? sdot : T(0);
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
          if (lane == 0) atomic_add(a.out2 + in.woff, s);
        } else {
          gws[lane * L.wp + in.woff] = sdot;
        }
      });
    }
    __syncwarp();
    // dY and dW rows back to global memory, coalesced.
    for (int t = lane; t < 32 * a.L2dim; t += 32) {
      const int r = t / a.L2dim, j = t - r * a.L2dim;
      if (base + r < a.nitems) a.out1[(base + r) * a.L2dim + j] = gys[r * L.l2p + j];
    }
    if (!a.shared_w)
      for (int t = lane; t < 32 * a.wnumel; t += 32) {
        const int r = t / a.wnumel, j = t - r * a.wnumel;
        if (base + r < a.nitems) a.out2[(base + r) * a.wnumel + j] = gws[r * L.wp + j];
      }
    if (valid) red_row(a.out0 + col * a.L1dim, gxs + lane * L.l1p, a.L1dim);
  }
}


// ---------------------------------------------------------------------------------------
// Single-path variant: one instruction whose three irreps are the whole X, Y and Z rows, all of
// multiplicity 1 (BASELINE C3: 1x2e x 1x3e -> 1x2e).  Everything stays in registers with
// compile-time sizes: each lane loads its edge's Y row, weight and the gathered X / dZ rows
// directly (the rows of a warp's 32 edges are contiguous, so the per-lane loads are served by
// the same few cache lines), and writes dY / dW directly.  The generic kernels above stage
// rows through shared memory with runtime offsets, which costs ~10x more instructions per edge.


// Register-array version of red_row: the alignment phase O = (address / 4) mod 4 of the row
// selects, at compile time, the sequence of v4 / v2 / scalar reductions.
template <int O, int I, int N>
__device__ __forceinline__ void red_vec_step(float* dst, const float (&v)[N]) {
  if constexpr (I < N) {
    constexpr int ph = (O + I) & 3;
    if constexpr (ph == 0 && I + 4 <= N) {
      asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"l"(dst + I), "f"(v[I]),
                   "f"(v[I + 1]), "f"(v[I + 2]), "f"(v[I + 3])
                   : "memory");
      red_vec_step<O, I + 4, N>(dst, v);
    } else if constexpr ((ph & 1) == 0 && I + 2 <= N) {
      asm volatile("red.global.add.v2.f32 [%0], {%1, %2};\n" ::"l"(dst + I), "f"(v[I]),
                   "f"(v[I + 1])
                   : "memory");
      red_vec_step<O, I + 2, N>(dst, v);
    } else {
      atomic_add(dst + I, v[I]);
      red_vec_step<O, I + 1, N>(dst, v);
    }
  }
}

template <class T, int N>
__device__ __forceinline__ void red_vec(T* dst, const T (&v)[N]) {
  if constexpr (sizeof(T) == 4) {
    switch ((reinterpret_cast<unsigned long long>(dst) >> 2) & 3) {
      case 0: red_vec_step<0, 0, N>(dst, v); break;
      case 1: red_vec_step<1, 0, N>(dst, v); break;
      case 2: red_vec_step<2, 0, N>(dst, v); break;
      default: red_vec_step<3, 0, N>(dst, v); break;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) atomic_add(dst + i, v[i]);
  }
}

struct Edge1 {
  int code;  // triple_code(l1, l2, l3)
  int woff;  // weight offset of the path (0 unless weights are shared with other paths)
  double pw;
};

template <class T, int A, int B, int C>
__device__ __forceinline__ void edge1_fwd_chunk(const Args<T>& a, const Edge1& p, long long e,
                                                bool valid, long long row, long long col,
                                                int lane) {
  constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1, D3 = 2 * C + 1;
  T z[D3];
#pragma unroll
  for (int k = 0; k < D3; ++k) z[k] = T(0);
  if (valid) {
    const T w = (a.shared_w ? a.W[p.woff] : a.W[e * a.wnumel + p.woff]) * T(p.pw);
    T x[D1], y[D2];
#pragma unroll
    for (int i = 0; i < D1; ++i) x[i] = a.X[col * D1 + i] * w;
#pragma unroll
    for (int j = 0; j < D2; ++j) y[j] = a.Y[e * D2 + j];
    CG<A, B, C>::fwd(x, y, z);
  }
  // Segmented suffix sums over equal receivers (rows are sorted), one reduction per segment.
  const int r32 = static_cast<int>(row);
  const int prev = __shfl_up_sync(0xffffffffu, r32, 1);
  const bool head = row >= 0 && (lane == 0 || prev != r32);
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int ro = __shfl_down_sync(0xffffffffu, r32, off);
    const bool take = lane + off < 32 && ro == r32;
#pragma unroll
    for (int k = 0; k < D3; ++k) {
      const T vo = __shfl_down_sync(0xffffffffu, z[k], off);
      if (take) z[k] += vo;
    }
  }
  if (head) red_vec(a.out0 + row * D3, z);
}

template <class T>
__global__ void __launch_bounds__(kEdgeWarps * 32) conv_fwd_edge1(const Args<T> a, const Edge1 p) {
  const int lane = threadIdx.x & 31;
  const long long nw = static_cast<long long>(gridDim.x) * kEdgeWarps;
  for (long long base = (static_cast<long long>(blockIdx.x) * kEdgeWarps + (threadIdx.x >> 5)) * 32;
       base < a.nitems; base += nw * 32) {
    const long long e = base + lane;
    bool valid = e < a.nitems;
    long long row = valid ? a.rows[e] : -1, col = valid ? a.cols[e] : 0;
    if (valid && (row < 0 || row >= a.nnodes || col < 0 || col >= a.nnodes)) {
      flag(a.status, 1);
      valid = false;
      row = -1;
      col = 0;
    }
    dispatch_triple(p.code, [&]<int A, int B, int C>() {
      edge1_fwd_chunk<T, A, B, C>(a, p, e, valid, row, col, lane);
    });
  }
}

template <class T, int A, int B, int C>
__device__ __forceinline__ void edge1_bwd_chunk(const Args<T>& a, const Edge1& p, long long e,
                                                bool valid, long long row, long long col,
                                                int lane) {
  constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1, D3 = 2 * C + 1;
  T sdot = T(0);
  if (valid) {
    const T w = a.shared_w ? a.W[p.woff] : a.W[e * a.wnumel + p.woff];
    const T pw = T(p.pw);
    T x[D1], y[D2], g[D3], h[D1], ev[D2];
#pragma unroll
    for (int i = 0; i < D1; ++i) x[i] = a.X[col * D1 + i];
#pragma unroll
    for (int j = 0; j < D2; ++j) y[j] = a.Y[e * D2 + j];
#pragma unroll
    for (int k = 0; k < D3; ++k) g[k] = a.Gz[row * D3 + k] * pw;
    CG<A, B, C>::hvec(g, y, h);
    CG<A, B, C>::evec(g, x, ev);
#pragma unroll
    for (int i = 0; i < D1; ++i) {
      sdot += x[i] * h[i];
      h[i] *= w;
    }
#pragma unroll
    for (int j = 0; j < D2; ++j) a.out1[e * D2 + j] = w * ev[j];
    if (!a.shared_w) a.out2[e * a.wnumel + p.woff] = sdot;
    red_vec(a.out0 + col * D1, h);
  }
  if (a.shared_w) {
    T s = sdot;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) atomic_add(a.out2 + p.woff, s);
  }
}

template <class T>
__global__ void __launch_bounds__(kEdgeWarps * 32) conv_bwd_edge1(const Args<T> a, const Edge1 p) {
  const int lane = threadIdx.x & 31;
  const long long nw = static_cast<long long>(gridDim.x) * kEdgeWarps;
  for (long long base = (static_cast<long long>(blockIdx.x) * kEdgeWarps + (threadIdx.x >> 5)) * 32;
       base < a.nitems; base += nw * 32) {
    const long long e = base + lane;
    bool valid = e < a.nitems;
    long long row = valid ? a.rows[e] : 0, col = valid ? a.cols[e] : 0;
    if (valid && (row < 0 || row >= a.nnodes || col < 0 || col >= a.nnodes)) {
      flag(a.status, 1);
      valid = false;
      row = col = 0;
    }
    dispatch_triple(p.code, [&]<int A, int B, int C>() {
      edge1_bwd_chunk<T, A, B, C>(a, p, e, valid, row, col, lane);
    });
  }
}

}  // namespace oeqb
