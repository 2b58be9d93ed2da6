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
// share one receiver: a segmented shuffle reduction over equal receivers leaves one atomic
// per (receiver segment, component) instead of one per edge.  In the backward pass dY and dW
// are per edge (written back coalesced through shared memory) and dX goes to the senders,
// which differ across lanes, with one atomic per (edge, component).
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
      if (head) atomic_add(a.out0 + row * a.L3dim + k, v);
    }
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
    if (valid)
      for (int i = 0; i < a.L1dim; ++i) atomic_add(a.out0 + col * a.L1dim + i, gxs[lane * L.l1p + i]);
  }
}

}  // namespace oeqb
