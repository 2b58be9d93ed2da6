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

// Row r (0..31) of a warp's D consecutive-row block, staged in shared memory at r * D.
// Global rows [base, base + 32) of width D start at base * D: 16-byte aligned when base is a
// multiple of 32 and the tensor is (float) / when D is even or base a multiple of 32 (double),
// so the block moves with 16-byte copies; the tail of the last block goes element-wise.
template <class T, int D>
__device__ __forceinline__ void e1_stage_in(T* dst, const T* src, long long base, long long n,
                                            int lane) {
  const long long rows = n - base < 32 ? n - base : 32;
  const int total = static_cast<int>(rows) * D;
  const T* g = src + base * D;
  constexpr int V = 16 / sizeof(T);
  const int nv = total / V;
  for (int q = lane; q < nv; q += 32) {
    if constexpr (sizeof(T) == 4) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(g) + q);
      dst[4 * q] = t.x;
      dst[4 * q + 1] = t.y;
      dst[4 * q + 2] = t.z;
      dst[4 * q + 3] = t.w;
    } else {
      const double2 t = __ldg(reinterpret_cast<const double2*>(g) + q);
      dst[2 * q] = t.x;
      dst[2 * q + 1] = t.y;
    }
  }
  for (int e = nv * V + lane; e < total; e += 32) dst[e] = g[e];
}

template <class T, int D>
__device__ __forceinline__ void e1_stage_out(T* dst, const T* src, long long base, long long n,
                                             int lane) {
  const long long rows = n - base < 32 ? n - base : 32;
  const int total = static_cast<int>(rows) * D;
  T* g = dst + base * D;
  constexpr int V = 16 / sizeof(T);
  const int nv = total / V;
  for (int q = lane; q < nv; q += 32) {
    if constexpr (sizeof(T) == 4)
      reinterpret_cast<float4*>(g)[q] =
          make_float4(src[4 * q], src[4 * q + 1], src[4 * q + 2], src[4 * q + 3]);
    else
      reinterpret_cast<double2*>(g)[q] = make_double2(src[2 * q], src[2 * q + 1]);
  }
  for (int e = nv * V + lane; e < total; e += 32) g[e] = src[e];
}

// Gathers row `node` (D values) of a [nodes, D] tensor: 16-byte loads of the aligned window
// that contains it (all D values in (D + 6) / 4 loads), element-wise where the window would
// pass the end of the tensor.
template <class T, int D>
__device__ __forceinline__ void e1_gather(T (&v)[D], const T* src, long long node, long long nodes) {
  if constexpr (sizeof(T) == 4) {
    constexpr int NW = (D + 6) / 4;
    const long long f = node * D;
    const int o = static_cast<int>(f & 3);
    const long long b4 = f - o;
    if (b4 + 4 * NW <= nodes * D) {
      float w[4 * NW];
#pragma unroll
      for (int q = 0; q < NW; ++q) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(src + b4) + q);
        w[4 * q] = t.x;
        w[4 * q + 1] = t.y;
        w[4 * q + 2] = t.z;
        w[4 * q + 3] = t.w;
      }
      switch (o) {
        case 0:
#pragma unroll
          for (int i = 0; i < D; ++i) v[i] = w[i];
          break;
        case 1:
#pragma unroll
          for (int i = 0; i < D; ++i) v[i] = w[i + 1];
          break;
        case 2:
#pragma unroll
          for (int i = 0; i < D; ++i) v[i] = w[i + 2];
          break;
        default:
#pragma unroll
          for (int i = 0; i < D; ++i) v[i] = w[i + 3];
          break;
      }
      return;
    }
  }
#pragma unroll
  for (int i = 0; i < D; ++i) v[i] = src[node * D + i];
}

// Per-lane edge record of one 32-edge block: receiver, sender, validity (bounds-checked).
struct E1Lane {
  long long e, row, col;
  bool valid;
};

// The index loads of a lane's edge, unchecked: the backward kernels and the deterministic
// forward issue them one 32-edge block ahead, so that only the dependent X / dZ row gathers wait on memory in each iteration (in the
// forward the four extra registers cost more occupancy than the overlap gains: 543 vs 527 us).
struct E1Raw {
  long long e, row, col;
};

template <class T>
__device__ __forceinline__ E1Raw e1_raw(const Args<T>& a, long long base, int lane) {
  E1Raw r;
  r.e = base + lane;
  const bool v = r.e < a.nitems;
  r.row = v ? a.rows[r.e] : -1;
  r.col = v ? a.cols[r.e] : 0;
  return r;
}

// Range check of the loaded indices (bad indices raise status 1 and drop the edge).
template <class T>
__device__ __forceinline__ E1Lane e1_check(const Args<T>& a, const E1Raw& r) {
  E1Lane l;
  l.e = r.e;
  l.valid = r.e < a.nitems;
  l.row = r.row;
  l.col = r.col;
  if (l.valid && (l.row < 0 || l.row >= a.nnodes || l.col < 0 || l.col >= a.nnodes)) {
    flag(a.status, 1);
    l.valid = false;
    l.row = -1;
    l.col = 0;
  }
  return l;
}

template <class T>
__device__ __forceinline__ E1Lane e1_lane(const Args<T>& a, long long base, int lane) {
  E1Lane l;
  l.e = base + lane;
  l.valid = l.e < a.nitems;
  l.row = l.valid ? a.rows[l.e] : -1;
  l.col = l.valid ? a.cols[l.e] : 0;
  if (l.valid && (l.row < 0 || l.row >= a.nnodes || l.col < 0 || l.col >= a.nnodes)) {
    flag(a.status, 1);
    l.valid = false;
    l.row = -1;
    l.col = 0;
  }
  return l;
}

// Forward message of one lane: z = w pw CG(x[col], y[e]).
template <class T, int A, int B, int C>
__device__ __forceinline__ void e1_message(const Args<T>& a, const Edge1& p, const E1Lane& l,
                                           const T* ys, int lane, T (&z)[2 * C + 1]) {
  constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1, D3 = 2 * C + 1;
#pragma unroll
  for (int k = 0; k < D3; ++k) z[k] = T(0);
  if (l.valid) {
    const T w = (a.shared_w ? a.W[p.woff] : a.W[l.e * a.wnumel + p.woff]) * T(p.pw);
    T x[D1], y[D2];
    e1_gather<T, D1>(x, a.X, l.col, a.nnodes);
#pragma unroll
    for (int i = 0; i < D1; ++i) x[i] *= w;
#pragma unroll
    for (int j = 0; j < D2; ++j) y[j] = ys[lane * D2 + j];
    CG<A, B, C>::fwd(x, y, z);
  }
}

// Suffix sums over runs of equal keys (keys sorted within the warp): afterwards the first lane
// of each run holds the run's sum.  The tree is fixed, so the result is deterministic.
template <class T, int D>
__device__ __forceinline__ void e1_seg_sum(T (&z)[D], int key, int lane) {
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int ko = __shfl_down_sync(0xffffffffu, key, off);
    const bool take = lane + off < 32 && ko == key;
#pragma unroll
    for (int k = 0; k < D; ++k) {
      const T vo = __shfl_down_sync(0xffffffffu, z[k], off);
      if (take) z[k] += vo;
    }
  }
}

template <class T>
__device__ __forceinline__ T* e1_warp_smem(unsigned char* smem, int elems) {
  return reinterpret_cast<T*>(smem) + static_cast<size_t>(threadIdx.x >> 5) * elems;
}

// ----------------------------------------------------------------------- atomic mode

template <class T>
__global__ void __launch_bounds__(kEdgeWarps * 32) conv_fwd_edge1(const Args<T> a, const Edge1 p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x & 31;
  const long long nw = static_cast<long long>(gridDim.x) * kEdgeWarps;
  dispatch_triple(p.code, [&]<int A, int B, int C>() {
    constexpr int D2 = 2 * B + 1, D3 = 2 * C + 1;
    T* ys = e1_warp_smem<T>(smem, 32 * D2);
    for (long long base = (static_cast<long long>(blockIdx.x) * kEdgeWarps + (threadIdx.x >> 5)) * 32;
         base < a.nitems; base += nw * 32) {
      const E1Lane l = e1_lane(a, base, lane);
      e1_stage_in<T, D2>(ys, a.Y, base, a.nitems, lane);
      __syncwarp();
      T z[D3];
      e1_message<T, A, B, C>(a, p, l, ys, lane, z);
      __syncwarp();
      const int r32 = static_cast<int>(l.row);
      const int prev = __shfl_up_sync(0xffffffffu, r32, 1);
      const bool head = l.row >= 0 && (lane == 0 || prev != r32);
      e1_seg_sum<T, D3>(z, r32, lane);
      if (head) red_vec(a.out0 + l.row * D3, z);
    }
  });
}

// Backward pieces of one lane: h (message to the sender, weight applied), dY (in ys_out),
// sdot = dW of the edge.
template <class T, int A, int B, int C>
__device__ __forceinline__ T e1_backward(const Args<T>& a, const Edge1& p, const E1Lane& l,
                                         const T* ys, T* ys_out, int lane, T (&h)[2 * A + 1]) {
  constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1, D3 = 2 * C + 1;
  T sdot = T(0);
  T ev[D2];
#pragma unroll
  for (int i = 0; i < D1; ++i) h[i] = T(0);
#pragma unroll
  for (int j = 0; j < D2; ++j) ev[j] = T(0);
  if (l.valid) {
    const T w = a.shared_w ? a.W[p.woff] : a.W[l.e * a.wnumel + p.woff];
    const T pw = T(p.pw);
    T x[D1], y[D2], g[D3];
    e1_gather<T, D1>(x, a.X, l.col, a.nnodes);
    e1_gather<T, D3>(g, a.Gz, l.row, a.nnodes);
#pragma unroll
    for (int k = 0; k < D3; ++k) g[k] *= pw;
#pragma unroll
    for (int j = 0; j < D2; ++j) y[j] = ys[lane * D2 + j];
    CG<A, B, C>::hvec(g, y, h);
    CG<A, B, C>::evec(g, x, ev);
#pragma unroll
    for (int i = 0; i < D1; ++i) {
      sdot += x[i] * h[i];
      h[i] *= w;
    }
#pragma unroll
    for (int j = 0; j < D2; ++j) ev[j] *= w;
  }
#pragma unroll
  for (int j = 0; j < D2; ++j) ys_out[lane * D2 + j] = ev[j];
  return sdot;
}

template <class T>
__device__ __forceinline__ void e1_write_dw(const Args<T>& a, const Edge1& p, const E1Lane& l,
                                            T sdot, int lane) {
  if (a.shared_w) {
    T s = l.valid ? sdot : T(0);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) atomic_add(a.out2 + p.woff, s);
  } else if (l.valid) {
    a.out2[l.e * a.wnumel + p.woff] = sdot;
  }
}

template <class T>
__global__ void __launch_bounds__(kEdgeWarps * 32) conv_bwd_edge1(const Args<T> a, const Edge1 p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x & 31;
  const long long nw = static_cast<long long>(gridDim.x) * kEdgeWarps;
  dispatch_triple(p.code, [&]<int A, int B, int C>() {
    constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1;
    T* ys = e1_warp_smem<T>(smem, 64 * D2);
    T* yo = ys + 32 * D2;
    long long base = (static_cast<long long>(blockIdx.x) * kEdgeWarps + (threadIdx.x >> 5)) * 32;
    E1Raw next = e1_raw(a, base, lane);
    for (; base < a.nitems; base += nw * 32) {
      const E1Lane l = e1_check(a, next);
      next = e1_raw(a, base + nw * 32, lane);
      e1_stage_in<T, D2>(ys, a.Y, base, a.nitems, lane);
      __syncwarp();
      T h[D1];
      const T sdot = e1_backward<T, A, B, C>(a, p, l, ys, yo, lane, h);
      __syncwarp();
      e1_stage_out<T, D2>(a.out1, yo, base, a.nitems, lane);
      e1_write_dw(a, p, l, sdot, lane);
      if (l.valid) red_vec(a.out0 + l.col * D1, h);
      __syncwarp();
    }
  });
}

// ----------------------------------------------------------------------- deterministic mode
//
// Forward: warp w owns the edges of whole receivers: its nominal range [w E / W, (w+1) E / W)
// moved forward to receiver boundaries.  It walks the range in 32-edge blocks; the sums of
// receivers that continue into the next block are carried in registers (carry + block sum, a
// fixed order), and every receiver row is written once with plain stores.
//
// Backward, two passes.  Pass A (receiver order, coalesced) writes dY, dW and each edge's
// message to its sender, h_e (D1 values) plus the sender index, into the workspace.  Pass B
// walks the sender-sorted positions t, reads h of edge transpose_perm[t] and sums runs of
// equal senders the same way as the forward, one plain store per sender row.

// First position >= p whose key differs from its predecessor's (or n).
template <class F>
__device__ __forceinline__ long long e1_snap(long long p, long long n, F&& key, int lane) {
  if (p <= 0) return 0;
  if (p >= n) return n;
  long long kp = key(p - 1);
  for (long long q = p; q < n; q += 32) {
    const long long t = q + lane;
    const bool brk = t < n && key(t) != kp;
    const unsigned m = __ballot_sync(0xffffffffu, brk);
    if (m) return q + __ffs(m) - 1;
  }
  return n;
}

template <class T, int D>
__device__ __forceinline__ void e1_store_row(T* dst, const T (&v)[D]) {
#pragma unroll
  for (int k = 0; k < D; ++k) dst[k] = v[k];
}

// Block-wise segmented sums with a carried tail segment.  key = -1 marks invalid lanes (past the
// range end).  `more` = the range continues after this block.
template <class T, int D>
__device__ __forceinline__ void e1_seg_block(T (&z)[D], long long key, long long next_key,
                                             bool more, T (&carry)[D], long long& carry_key,
                                             T* out, int lane) {
  const int k32 = static_cast<int>(key);
  const int prev = __shfl_up_sync(0xffffffffu, k32, 1);
  const bool head = key >= 0 && (lane == 0 || prev != k32);
  e1_seg_sum<T, D>(z, k32, lane);
  // The run holding lane 0 continues a carried run from the previous block.
  if (lane == 0 && key >= 0 && key == carry_key) {
#pragma unroll
    for (int k = 0; k < D; ++k) z[k] = carry[k] + z[k];
  }
  // Key of the last valid lane, and whether its run goes on into the next block.
  const unsigned vm = __ballot_sync(0xffffffffu, key >= 0);
  const int last = vm ? 31 - __clz(vm) : -1;
  const long long last_key = last >= 0 ? __shfl_sync(0xffffffffu, key, last) : -1;
  const bool cont = more && last == 31 && next_key == last_key;
  // Head lane of the last run.
  const unsigned hm = __ballot_sync(0xffffffffu, head);
  const int last_head = hm ? 31 - __clz(hm) : -1;
  if (head && !(cont && lane == last_head)) e1_store_row(out + key * D, z);
  carry_key = -2;
  if (cont) {
#pragma unroll
    for (int k = 0; k < D; ++k) carry[k] = __shfl_sync(0xffffffffu, z[k], last_head);
    carry_key = last_key;
  }
}

template <class T>
__global__ void __launch_bounds__(kEdgeWarps * 32) conv_fwd_edge1_det(const Args<T> a, const Edge1 p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x & 31;
  const long long nwarps = static_cast<long long>(gridDim.x) * kEdgeWarps;
  const long long wg = static_cast<long long>(blockIdx.x) * kEdgeWarps + (threadIdx.x >> 5);
  const long long n = a.nitems;
  auto key = [&](long long e) { return a.rows[e]; };
  const long long p0 = e1_snap(static_cast<long long>((static_cast<__int128>(n) * wg) / nwarps), n, key, lane);
  const long long p1 = e1_snap(static_cast<long long>((static_cast<__int128>(n) * (wg + 1)) / nwarps), n, key, lane);
  dispatch_triple(p.code, [&]<int A, int B, int C>() {
    constexpr int D2 = 2 * B + 1, D3 = 2 * C + 1;
    T* ys = e1_warp_smem<T>(smem, 32 * D2);
    T carry[D3];
    long long carry_key = -2;
    // Blocks start at the 4-aligned edge at or below p0 (lanes before p0 belong to the previous
    // warp and are masked), so the Y rows of a block start 16-byte aligned.
    // The index loads run one block ahead; the next block's first receiver (the key that
    // decides whether the last run continues) is lane 0's prefetched row.
    long long base = p0 & ~3LL;
    E1Raw next = e1_raw(a, base, lane);
    for (; base < p1; base += 32) {
      E1Lane l = e1_check(a, next);
      next = e1_raw(a, base + 32, lane);
      if (l.e >= p1 || l.e < p0) {
        l.valid = false;
        l.row = -1;
      }
      e1_stage_in<T, D2>(ys, a.Y, base, p1, lane);
      __syncwarp();
      T z[D3];
      e1_message<T, A, B, C>(a, p, l, ys, lane, z);
      __syncwarp();
      const bool more = base + 32 < p1;
      const long long nk0 = __shfl_sync(0xffffffffu, next.row, 0);
      const long long nk = more ? nk0 : -3;
      e1_seg_block<T, D3>(z, l.valid ? l.row : -1, nk, more, carry, carry_key, a.out0, lane);
    }
  });
}

// Workspace record of pass A, 8 values: h (D1 <= 7 values), and at index 7 the bits of the
// sender index (int32 in a float slot, int64 in a double slot).  32 bytes (float): one sector,
// 16-byte loads.
constexpr int kE1Rec = 8;

// Floats of side data per 32-position block in the banded deterministic pass B (a head and a
// tail slot of 8 floats each).
constexpr int kBandSlot = 16;

template <class T>
__device__ __forceinline__ T e1_key_bits(long long k) {
  if constexpr (sizeof(T) == 4)
    return __int_as_float(static_cast<int>(k));
  else
    return __longlong_as_double(k);
}

template <class T>
__device__ __forceinline__ long long e1_bits_key(T v) {
  if constexpr (sizeof(T) == 4)
    return __float_as_int(v);
  else
    return __double_as_longlong(v);
}

// 32-byte read-only load of 8 floats (ld.global.v8, sm_100); p must be 32-byte aligned.
__device__ __forceinline__ void ldg_v8(float (&v)[8], const float* p) {
  asm("ld.global.nc.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7])
      : "l"(p));
}

// One 8-value record: a 32-byte load for float (32-byte aligned), four 16-byte loads for double.
template <class T>
__device__ __forceinline__ void load_rec8(T (&r)[kE1Rec], const T* src) {
  if constexpr (sizeof(T) == 4) {
    ldg_v8(r, src);
  } else {
#pragma unroll
    for (int q = 0; q < kE1Rec / 2; ++q) {
      const double2 u = __ldg(reinterpret_cast<const double2*>(src) + q);
      r[2 * q] = u.x;
      r[2 * q + 1] = u.y;
    }
  }
}

// Deterministic backward pass B, banded.  transpose_perm lists the edges in sender order; pass
// B sums each sender's records (written by pass A in edge order) along it.  The positions are
// cut into absolute 32-position blocks, and warp w of W takes blocks w, w + W, w + 2W, ...: at
// any moment the warps work on one band of about W blocks, so the records of one cache line
// (consecutive edges of one receiver, whose senders are near one another in the node order)
// are read while the line is still in L2.  (Contiguous per-warp ranges spread the warps over
// the whole array at once, and nearly every record read then fetched its line from DRAM
// again.)
//
// Per block, the runs of equal senders are summed with a segmented shuffle tree.  A run that
// neither contains lane 0 nor lane 31 is complete and is stored into dX directly.  The run
// holding lane 0 goes to the block's head slot, the run holding lane 31 (if it is another run)
// to its tail slot; conv_bwd_edge1_band_fix joins the slots of consecutive blocks.  Every sum
// is taken in one fixed order (the tree inside each block, then the blocks left to right), so
// the result does not depend on the grid, the SM count or timing.
//
// Side slots: kBandSlot values per block, head at [0, 8), tail at [8, 16), the sum in the
// first D1 values and the sender key's bits in the last.  Head key -1: lane 0 holds no valid
// record.  Tail key -1: lane 31 holds none; -2: the head run reaches lane 31 (one run fills
// the block).  The transpose_perm entries are loaded two blocks ahead and the records one
// block ahead.  dX rows of nodes that send no edge are not written (the caller clears dX).
template <class T, int D1>
__device__ __forceinline__ void band_slot_store(T* dst, const T (&h)[D1], long long key) {
  T v[8];
#pragma unroll
  for (int i = 0; i < 7; ++i) v[i] = i < D1 ? h[i] : T(0);
  v[7] = e1_key_bits<T>(key);
  if constexpr (sizeof(T) == 4) {
    reinterpret_cast<float4*>(dst)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(dst)[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) reinterpret_cast<double2*>(dst)[q] = make_double2(v[2 * q], v[2 * q + 1]);
  }
}

template <class T, int A>
__global__ void __launch_bounds__(kEdgeWarps * 32) conv_bwd_edge1_band(const Args<T> a,
                                                                       const Edge1 p,
                                                                       const T* __restrict__ ws,
                                                                       T* __restrict__ side) {
  (void)p;
  constexpr int D1 = 2 * A + 1, R = kE1Rec;
  const int lane = threadIdx.x & 31;
  const long long nw = static_cast<long long>(gridDim.x) * kEdgeWarps;
  const long long n = a.nitems;
  const long long nb = (n + 31) / 32;
  long long b = static_cast<long long>(blockIdx.x) * kEdgeWarps + (threadIdx.x >> 5);
  if (b >= nb) return;
  // Edge at position 32 blk + lane, or -1 (past the end, or a bad permutation entry: status 2).
  auto edge_at = [&](long long blk) -> long long {
    const long long t = blk * 32 + lane;
    if (blk >= nb || t >= n) return -1;
    const long long e = a.perm[t];
    if (e < 0 || e >= n) {
      flag(a.status, 2);
      return -1;
    }
    return e;
  };
  auto load = [&](T (&r)[R], long long e) {
    if (e >= 0) {
      load_rec8<T>(r, ws + e * R);
    } else {
#pragma unroll
      for (int i = 0; i < R - 1; ++i) r[i] = T(0);
      r[R - 1] = e1_key_bits<T>(-1);
    }
  };
  long long e_c = edge_at(b);
  long long e_n = edge_at(b + nw);
  T rc[R];
  load(rc, e_c);
  for (; b < nb; b += nw) {
    const long long e_nn = edge_at(b + 2 * nw);  // two blocks ahead
    T rn[R];
    load(rn, e_n);  // one block ahead
    T h[D1];
#pragma unroll
    for (int i = 0; i < D1; ++i) h[i] = rc[i];
    const long long k64 = e1_bits_key<T>(rc[R - 1]);
    const int key = (k64 < 0 || k64 >= a.nnodes) ? -1 : static_cast<int>(k64);
    const int prev = __shfl_up_sync(0xffffffffu, key, 1);
    const bool head = key >= 0 && (lane == 0 || prev != key);
    e1_seg_sum<T, D1>(h, key, lane);
    const unsigned hm = __ballot_sync(0xffffffffu, head);
    const int last_head = hm ? 31 - __clz(hm) : -1;
    const bool v31 = __shfl_sync(0xffffffffu, key, 31) >= 0;
    T* hs = side + b * kBandSlot;
    if (head) {
      if (lane == 0)
        band_slot_store<T, D1>(hs, h, key);
      else if (lane == last_head && v31)
        band_slot_store<T, D1>(hs + 8, h, key);
      else
        e1_store_row(a.out0 + static_cast<long long>(key) * D1, h);
    }
    if (lane == 0) {
      if (!head) hs[7] = e1_key_bits<T>(-1);
      if (!v31)
        hs[15] = e1_key_bits<T>(-1);
      else if (last_head == 0)
        hs[15] = e1_key_bits<T>(-2);
    }
#pragma unroll
    for (int i = 0; i < R; ++i) rc[i] = rn[i];
    e_c = e_n;
    e_n = e_nn;
  }
}

// Joins the head / tail slots of conv_bwd_edge1_band, one thread per block b.  The run in b's
// head slot is written here if it starts in b (block b - 1 does not end with the same sender)
// and ends in b.  A run that starts in b and reaches lane 31 (b's tail slot, or its head slot
// when one run fills b) is summed with the head slots of the following blocks, left to right,
// as long as they continue it, and written.  Each run is written once.
template <class T, int A>
__global__ void __launch_bounds__(256) conv_bwd_edge1_band_fix(const Args<T> a,
                                                               const T* __restrict__ side) {
  constexpr int D1 = 2 * A + 1;
  const long long nb = (a.nitems + 31) / 32;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  auto hkey = [&](long long m) { return e1_bits_key<T>(side[m * kBandSlot + 7]); };
  auto tkey = [&](long long m) { return e1_bits_key<T>(side[m * kBandSlot + 15]); };
  for (long long b = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; b < nb;
       b += stride) {
    const long long k0 = hkey(b), t0 = tkey(b);
    long long prev_last = -1;
    if (b > 0) {
      const long long tp = tkey(b - 1);
      prev_last = tp >= 0 ? tp : (tp == -2 ? hkey(b - 1) : -1);
    }
    const bool starts = k0 >= 0 && prev_last != k0;
    const T* hs = side + b * kBandSlot;
    T s[D1];
    if (starts && t0 != -2) {
#pragma unroll
      for (int i = 0; i < D1; ++i) s[i] = hs[i];
      e1_store_row(a.out0 + k0 * D1, s);
    }
    long long k = -1;
    if (t0 >= 0) {
      k = t0;
#pragma unroll
      for (int i = 0; i < D1; ++i) s[i] = hs[8 + i];
    } else if (t0 == -2 && starts) {
      k = k0;
#pragma unroll
      for (int i = 0; i < D1; ++i) s[i] = hs[i];
    }
    if (k < 0) continue;
    for (long long m = b + 1; m < nb; ++m) {
      if (hkey(m) != k) break;
#pragma unroll
      for (int i = 0; i < D1; ++i) s[i] += side[m * kBandSlot + i];
      if (tkey(m) != -2) break;
    }
    e1_store_row(a.out0 + k * D1, s);
  }
}

template <class T>
__global__ void __launch_bounds__(kEdgeWarps * 32) conv_bwd_edge1_msg(const Args<T> a, const Edge1 p,
                                                                      T* ws) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x & 31;
  const long long nw = static_cast<long long>(gridDim.x) * kEdgeWarps;
  dispatch_triple(p.code, [&]<int A, int B, int C>() {
    constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1, R = kE1Rec;
    T* ys = e1_warp_smem<T>(smem, 64 * D2 + 32 * R);
    T* yo = ys + 32 * D2;
    T* hs = yo + 32 * D2;
    long long base = (static_cast<long long>(blockIdx.x) * kEdgeWarps + (threadIdx.x >> 5)) * 32;
    E1Raw next = e1_raw(a, base, lane);
    for (; base < a.nitems; base += nw * 32) {
      const E1Lane l = e1_check(a, next);
      next = e1_raw(a, base + nw * 32, lane);
      e1_stage_in<T, D2>(ys, a.Y, base, a.nitems, lane);
      __syncwarp();
      T h[D1];
      const T sdot = e1_backward<T, A, B, C>(a, p, l, ys, yo, lane, h);
#pragma unroll
      for (int i = 0; i < R - 1; ++i) hs[lane * R + i] = i < D1 ? h[i] : T(0);
      hs[lane * R + R - 1] = e1_key_bits<T>(l.valid ? l.col : -1);
      __syncwarp();
      e1_stage_out<T, D2>(a.out1, yo, base, a.nitems, lane);
      e1_stage_out<T, R>(ws, hs, base, a.nitems, lane);
      e1_write_dw(a, p, l, sdot, lane);
      __syncwarp();
    }
  });
}


}  // namespace oeqb
