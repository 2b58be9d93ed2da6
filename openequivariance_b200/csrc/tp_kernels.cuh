// Kernel templates for the batch tensor product and the fused graph convolution.
//
//   tp_fwd_kernel  : batch forward / conv forward with atomic scatter
//                    (reference: loop_unroll_batch.cuh:26-64, loop_unroll_conv_atomic.cuh:53-106)
//   tp_bwd_kernel  : batch backward / conv backward with atomic scatter of dX
//                    (reference: loop_unroll_batch.cuh:70-143, loop_unroll_conv_atomic.cuh:108-200)
//   conv_fwd_det   : receiver-sorted segmented reduction, one writer per output row
//   conv_bwd_det   : sender-ordered (through the transpose permutation) segmented
//                    reduction of dX, one writer per sender row
//                    (reference: loop_unroll_conv_det.cuh:97-294; the reference splits rows
//                    across warps and repairs them with a fixup pass, this build snaps each
//                    warp's edge range to row boundaries so no fixup is needed)
//
// DB = true turns the forward into part A of the double backward (three forward terms)
// and the backward into part B (two backward terms); see tp_core.cuh.
#pragma once

#include "tp_core.cuh"

namespace oeqb {

enum Policy { kBatch = 0, kConvAtomic = 1 };

template <class T>
__device__ __forceinline__ Lane<T> make_lane(const Args<T>& a, const SmemDesc& d) {
  Lane<T> L;
  L.lane = threadIdx.x & 31;
  L.lgG = a.lgG;
  L.G = 1 << a.lgG;
  L.gl = L.lane & (L.G - 1);
  L.gsub = L.lane >> a.lgG;
  L.ws = reinterpret_cast<T*>(d.end) + static_cast<size_t>(threadIdx.x >> 5) * a.ws_elems;
  return L;
}

__device__ __forceinline__ void flag(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// ---------------------------------------------------------------------------
// Forward chunk: one output block chunk (irrep r3, lanes c0..c0+G) of one item slot.
// L3 >= 0: unrolled output degree, L3 == -1: generic.  Instructions whose triple is not
// unrolled accumulate into a separate local array (zt) so that the register
// accumulator z is never address-taken.

template <class T, bool UVW, bool DB, int L3>
__device__ __forceinline__ void fwd_chunk(const Args<T>& a, const SmemDesc& d, const Lane<T>& L,
                                          const GroupD& gd, const IrrepD& r3, int c0, bool rv,
                                          const RowPtrs<T>& rp, T* stage_row) {
  constexpr int D3 = L3 >= 0 ? 2 * L3 + 1 : kDMax;
  const int wu = c0 + L.gl;
  const bool act = rv && wu < r3.mul;
  T z[D3];
  zero(z);
  T zt[kDMax];
  bool generic_used = false;
  T* ws_t = L.ws + a.off_t;
  T* ws_t2 = L.ws + a.off_t2;
  for (int ii = gd.first; ii < gd.first + gd.count; ++ii) {
    const InstrD& in = d.ins[ii];
    const IrrepD r1 = d.ir1[in.i1];
    const IrrepD r2 = d.ir2[in.i2];
    bool done = false;
    if constexpr (!UVW) {
      if (act) {
        if constexpr (L3 >= 0)
          done = dispatch_triple(in.code, [&]<int A, int B, int C>() {
            if constexpr (C == L3)
              uvu_fwd<T, A, B, C, DB>(in, r1, r2, rp, rp.w + in.woff + (wu & ~31) * in.m2, wu, z);
          });
        if (!done) {
          if (!generic_used) {
            for (int k = 0; k < kDMax; ++k) zt[k] = T(0);
            generic_used = true;
          }
          uvu_fwd_generic<T, DB>(in, r1, r2, a.cgtab, rp, wu, zt);
        }
      }
    } else {
      if constexpr (L3 >= 0)
        done = dispatch_triple(in.code, [&]<int A, int B, int C>() {
          if constexpr (C == L3)
            uvw_fwd<T, A, B, C, DB>(in, r1, r2, rp, rv, wu, act, L, ws_t, ws_t2, z);
        });
      if (!done) {
        if (!generic_used) {
          for (int k = 0; k < kDMax; ++k) zt[k] = T(0);
          generic_used = true;
        }
        uvw_fwd_generic<T, DB>(in, r1, r2, a.cgtab, rp, rv, wu, act, L.lgG, L.gl, L.gsub, ws_t,
                               ws_t2, zt);
      }
    }
  }
  if (generic_used) {
#pragma unroll
    for (int k = 0; k < D3; ++k) z[k] += zt[k];
  }
  if (act) {
    const int ulen = min(L.G, r3.mul - c0);
#pragma unroll
    for (int k = 0; k < D3; ++k)
      if (k < r3.dim) stage_row[stage_index(r3, ulen, L.gl, k)] = z[k];
  }
}

// Backward chunk: gradient of input irrep r1 (lanes c0..c0+G) for one item slot.
template <class T, bool UVW, bool DB, int L1>
__device__ __forceinline__ void bwd_chunk(const Args<T>& a, const SmemDesc& d, const Lane<T>& L,
                                          const GroupD& gd, const IrrepD& r1, int cidx, bool rv,
                                          const RowPtrs<T>& rp, const BwdOut<T>& bo,
                                          T* stage_row) {
  constexpr int D1 = L1 >= 0 ? 2 * L1 + 1 : kDMax;
  const int c0 = cidx << L.lgG;
  const int u = c0 + L.gl;
  const bool act = rv && u < r1.mul;
  T gx[D1];
  zero(gx);
  T gxt[kDMax];
  bool generic_used = false;
  T* ws_t = L.ws + a.off_t;
  T* ws_gz = L.ws + a.off_gz;
  for (int ii = gd.first; ii < gd.first + gd.count; ++ii) {
    const InstrD& in = d.ins[ii];
    const IrrepD r2 = d.ir2[in.i2];
    const IrrepD r3 = d.ir3[in.i3];
    bool done = false;
    if constexpr (L1 >= 0)
      done = dispatch_triple(in.code, [&]<int A, int B, int C>() {
        if constexpr (A == L1) {
          if constexpr (!UVW)
            uvu_bwd<T, A, B, C, DB>(in, r1, r2, r3, rp, rp.w + in.woff + (u & ~31) * in.m2, u,
                                    act, L, gx, bo);
          else
            uvw_bwd<T, A, B, C, DB>(in, r1, r2, r3, rp, rv, cidx, L, ws_t, ws_gz, gx, bo);
        }
      });
    if (!done) {
      if (!generic_used) {
        for (int k = 0; k < kDMax; ++k) gxt[k] = T(0);
        generic_used = true;
      }
      if constexpr (!UVW)
        uvu_bwd_generic<T, DB>(in, r1, r2, r3, a.cgtab, rp, u, act, L.lgG, L.gl, gxt, bo);
      else
        uvw_bwd_generic<T, DB>(in, r1, r2, r3, a.cgtab, rp, rv, cidx, L.lgG, L.gl, L.gsub, ws_t,
                               ws_gz, gxt, bo);
    }
  }
  if (generic_used) {
#pragma unroll
    for (int i = 0; i < D1; ++i) gx[i] += gxt[i];
  }
  if (act) {
    const int ulen = min(L.G, r1.mul - c0);
#pragma unroll
    for (int i = 0; i < D1; ++i)
      if (i < r1.dim) stage_row[stage_index(r1, ulen, L.gl, i)] = gx[i];
  }
}

// Dispatches a templated chunk body on the degree of irrep `l` (generic beyond the
// unrolled range).
template <class F>
__device__ __forceinline__ void with_degree(int l, F&& f) {
  if (!dispatch_l(l, f)) f.template operator()<-1>();
}

template <class T>
__device__ __forceinline__ RowPtrs<T> row_ptrs(const Args<T>& a, long long xr, long long it,
                                               long long gr) {
  RowPtrs<T> rp;
  rp.x = a.X + xr * a.L1dim;
  rp.y = a.Y + it * a.L2dim;
  rp.w = a.shared_w ? a.W : a.W + it * a.wnumel;
  rp.g = a.Gz ? a.Gz + gr * a.L3dim : nullptr;
  rp.a = a.dA ? a.dA + xr * a.L1dim : nullptr;
  rp.b = a.dB ? a.dB + it * a.L2dim : nullptr;
  rp.c = a.dC ? (a.shared_w ? a.dC : a.dC + it * a.wnumel) : nullptr;
  return rp;
}

// ---------------------------------------------------------------------------

template <class T, bool UVW, bool DB, int POLICY>
__global__ void __launch_bounds__(kThreads) tp_fwd_kernel(const Args<T> a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ long long s_dst[kWarps][32];
  const SmemDesc d = stage_desc(a, smem);
  const Lane<T> L = make_lane(a, d);
  const int wid = threadIdx.x >> 5;
  const int rpw = 32 >> a.lgG;
  const int sstride = L.G * kDMax;
  T* stage = L.ws;
  const long long nw = static_cast<long long>(gridDim.x) * kWarps;
  for (long long base = (static_cast<long long>(blockIdx.x) * kWarps + wid) * rpw; base < a.nitems;
       base += nw * rpw) {
    const long long item = base + L.gsub;
    bool rv = item < a.nitems;
    const long long it = rv ? item : 0;
    long long xr = it, orow = it;
    if constexpr (POLICY == kConvAtomic) {
      xr = a.cols[it];
      orow = a.rows[it];
      if (rv && (xr < 0 || xr >= a.nnodes || orow < 0 || orow >= a.nnodes)) {
        flag(a.status, 1);
        rv = false;
      }
      if (!rv) xr = orow = 0;
    }
    const RowPtrs<T> rp = row_ptrs(a, xr, it, 0);
    __syncwarp();
    if (L.gl == 0) s_dst[wid][L.gsub] = rv ? orow : -1;
    __syncwarp();
    for (int g = 0; g < a.ngrp; ++g) {
      const GroupD gd = d.grp[g];
      const IrrepD r3 = d.ir3[gd.irrep];
      const int nch = (r3.mul + L.G - 1) >> L.lgG;
      for (int c = 0; c < nch; ++c) {
        const int c0 = c << L.lgG;
        with_degree(r3.l, [&]<int L3>() {
          fwd_chunk<T, UVW, DB, L3>(a, d, L, gd, r3, c0, rv, rp, stage + L.gsub * sstride);
        });
        __syncwarp();
        flush_block<T, POLICY == kBatch ? 0 : 1>(L, stage, sstride, r3, c0, min(L.G, r3.mul - c0),
                                                 a.out0, s_dst[wid], a.L3dim);
        __syncwarp();
      }
    }
    if constexpr (POLICY == kBatch) {
      for (int z = 0; z < a.nzero; ++z) {
        const IrrepD r3 = d.ir3[d.zb[z]];
        const int n = r3.mul * r3.dim;
        for (int idx = L.lane; idx < rpw * n; idx += 32) {
          const int s = idx / n, e = idx - s * n;
          const long long r = s_dst[wid][s];
          if (r >= 0) a.out0[r * a.L3dim + block_addr(r3, 0, r3.mul, e)] = T(0);
        }
      }
    }
  }
}

template <class T, bool UVW, bool DB, int POLICY>
__global__ void __launch_bounds__(kThreads) tp_bwd_kernel(const Args<T> a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ long long s_dst[kWarps][32];
  __shared__ long long s_item[kWarps][32];
  const SmemDesc d = stage_desc(a, smem);
  const Lane<T> L = make_lane(a, d);
  const int wid = threadIdx.x >> 5;
  const int rpw = 32 >> a.lgG;
  const int sstride = L.G * kDMax;
  T* stage = L.ws;
  T* dys = L.ws + a.off_dy;
  const long long nw = static_cast<long long>(gridDim.x) * kWarps;
  for (long long base = (static_cast<long long>(blockIdx.x) * kWarps + wid) * rpw; base < a.nitems;
       base += nw * rpw) {
    const long long item = base + L.gsub;
    bool rv = item < a.nitems;
    const long long it = rv ? item : 0;
    long long xr = it, gr = it;
    if constexpr (POLICY == kConvAtomic) {
      xr = a.cols[it];
      gr = a.rows[it];
      if (rv && (xr < 0 || xr >= a.nnodes || gr < 0 || gr >= a.nnodes)) {
        flag(a.status, 1);
        rv = false;
      }
      if (!rv) xr = gr = 0;
    }
    const RowPtrs<T> rp = row_ptrs(a, xr, it, gr);
    __syncwarp();
    if (L.gl == 0) {
      s_dst[wid][L.gsub] = rv ? xr : -1;
      s_item[wid][L.gsub] = rv ? it : -1;
    }
    for (int e = L.lane; e < rpw * a.L2dim; e += 32) dys[e] = T(0);
    __syncwarp();
    BwdOut<T> bo;
    bo.dy_row = rv ? dys + L.gsub * a.L2dim : nullptr;
    bo.dw = a.shared_w ? a.out2 : a.out2 + it * a.wnumel;
    bo.shared_w = a.shared_w != 0;
    for (int g = 0; g < a.ngrp; ++g) {
      const GroupD gd = d.grp[g];
      const IrrepD r1 = d.ir1[gd.irrep];
      const int nch = (r1.mul + L.G - 1) >> L.lgG;
      for (int c = 0; c < nch; ++c) {
        with_degree(r1.l, [&]<int L1>() {
          bwd_chunk<T, UVW, DB, L1>(a, d, L, gd, r1, c, rv, rp, bo, stage + L.gsub * sstride);
        });
        __syncwarp();
        const int c0 = c << L.lgG;
        flush_block<T, POLICY == kBatch ? 0 : 1>(L, stage, sstride, r1, c0, min(L.G, r1.mul - c0),
                                                 a.out0, s_dst[wid], a.L1dim);
        __syncwarp();
      }
    }
    if constexpr (POLICY == kBatch) {
      for (int z = 0; z < a.nzero; ++z) {
        const IrrepD r1 = d.ir1[d.zb[z]];
        const int n = r1.mul * r1.dim;
        for (int idx = L.lane; idx < rpw * n; idx += 32) {
          const int s = idx / n, e = idx - s * n;
          const long long r = s_dst[wid][s];
          if (r >= 0) a.out0[r * a.L1dim + block_addr(r1, 0, r1.mul, e)] = T(0);
        }
      }
    }
    __syncwarp();
    for (int idx = L.lane; idx < rpw * a.L2dim; idx += 32) {
      const int s = idx / a.L2dim, e = idx - s * a.L2dim;
      const long long r = s_item[wid][s];
      if (r >= 0) a.out1[r * a.L2dim + e] = dys[idx];
    }
  }
}

// ---------------------------------------------------------------------------
// Deterministic convolution: each warp owns a contiguous range of positions whose ends
// are snapped to key boundaries, so every output row is produced by exactly one warp in
// a fixed order (bitwise reproducible).

template <class KeyF>
__device__ long long snap_to_key(long long p, long long n, KeyF key) {
  if (p <= 0) return 0;
  if (p >= n) return n;
  const long long kp = key(p - 1);
  if (key(p) != kp) return p;
  long long lo = p, hi = n;
  while (lo < hi) {
    const long long mid = lo + ((hi - lo) >> 1);
    if (key(mid) <= kp)
      lo = mid + 1;
    else
      hi = mid;
  }
  return lo;
}

// Running accumulator over a staged block row: element e = lane + 32*q.
template <class T, bool KAHAN>
struct SegAcc {
  T acc[kDMax];
  T comp[KAHAN ? kDMax : 1];
  long long cur;
  __device__ __forceinline__ void reset() {
#pragma unroll
    for (int q = 0; q < kDMax; ++q) {
      acc[q] = T(0);
      if constexpr (KAHAN) comp[q] = T(0);
    }
  }
  __device__ __forceinline__ void add(const T* src, int n, int lane) {
#pragma unroll
    for (int q = 0; q < kDMax; ++q) {
      const int e = lane + 32 * q;
      if (e < n) {
        const T v = src[e];
        if constexpr (KAHAN) {
          const T y = v - comp[q];
          const T t = acc[q] + y;
          comp[q] = (t - acc[q]) - y;
          acc[q] = t;
        } else {
          acc[q] += v;
        }
      }
    }
  }
  __device__ __forceinline__ void store(T* dst_row, const IrrepD& ir, int c0, int ulen, int n,
                                        int lane) {
#pragma unroll
    for (int q = 0; q < kDMax; ++q) {
      const int e = lane + 32 * q;
      if (e < n) dst_row[block_addr(ir, c0, ulen, e)] = acc[q];
    }
  }
};

template <class T, bool UVW, bool DB, bool KAHAN>
__global__ void __launch_bounds__(kThreads) conv_fwd_det(const Args<T> a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ long long s_key[kWarps][32];
  const SmemDesc d = stage_desc(a, smem);
  const Lane<T> L = make_lane(a, d);
  const int wid = threadIdx.x >> 5;
  const int rpw = 32 >> a.lgG;
  const int sstride = L.G * kDMax;
  T* stage = L.ws;
  const long long nw = static_cast<long long>(gridDim.x) * kWarps;
  const long long wg = static_cast<long long>(blockIdx.x) * kWarps + wid;
  const long long n = a.nitems;
  auto key = [&](long long p) { return a.rows[p]; };
  long long p0 = 0, p1 = 0;
  if (L.lane == 0) {
    p0 = snap_to_key(static_cast<long long>((static_cast<__int128>(n) * wg) / nw), n, key);
    p1 = snap_to_key(static_cast<long long>((static_cast<__int128>(n) * (wg + 1)) / nw), n, key);
  }
  p0 = __shfl_sync(0xffffffffu, p0, 0);
  p1 = __shfl_sync(0xffffffffu, p1, 0);
  if (p0 >= p1) return;
  for (int g = 0; g < a.ngrp; ++g) {
    const GroupD gd = d.grp[g];
    const IrrepD r3 = d.ir3[gd.irrep];
    const int nch = (r3.mul + L.G - 1) >> L.lgG;
    for (int c = 0; c < nch; ++c) {
      const int c0 = c << L.lgG;
      const int ulen = min(L.G, r3.mul - c0);
      const int nel = ulen * r3.dim;
      SegAcc<T, KAHAN> sa;
      sa.reset();
      sa.cur = -1;
      for (long long base = p0; base < p1; base += rpw) {
        const long long item = base + L.gsub;
        bool rv = item < p1;
        const long long it = rv ? item : p0;
        long long xr = a.cols[it], orow = a.rows[it];
        if (rv && (xr < 0 || xr >= a.nnodes || orow < 0 || orow >= a.nnodes)) {
          flag(a.status, 1);
          rv = false;
        }
        if (!rv) xr = orow = 0;
        const RowPtrs<T> rp = row_ptrs(a, xr, it, 0);
        __syncwarp();
        if (L.gl == 0) s_key[wid][L.gsub] = rv ? orow : -1;
        with_degree(r3.l, [&]<int L3>() {
          fwd_chunk<T, UVW, DB, L3>(a, d, L, gd, r3, c0, rv, rp, stage + L.gsub * sstride);
        });
        __syncwarp();
        for (int s = 0; s < rpw; ++s) {
          const long long k = s_key[wid][s];
          if (k < 0) continue;
          if (k != sa.cur) {
            if (sa.cur >= 0) sa.store(a.out0 + sa.cur * a.L3dim, r3, c0, ulen, nel, L.lane);
            sa.reset();
            sa.cur = k;
          }
          sa.add(stage + s * sstride, nel, L.lane);
        }
      }
      if (sa.cur >= 0) sa.store(a.out0 + sa.cur * a.L3dim, r3, c0, ulen, nel, L.lane);
      __syncwarp();
    }
  }
}

template <class T, bool UVW, bool DB, bool KAHAN>
__global__ void __launch_bounds__(kThreads) conv_bwd_det(const Args<T> a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ long long s_key[kWarps][32];
  const SmemDesc d = stage_desc(a, smem);
  const Lane<T> L = make_lane(a, d);
  const int wid = threadIdx.x >> 5;
  const int rpw = 32 >> a.lgG;
  const int sstride = L.G * kDMax;
  T* stage = L.ws;
  const long long nw = static_cast<long long>(gridDim.x) * kWarps;
  const long long wg = static_cast<long long>(blockIdx.x) * kWarps + wid;
  const long long n = a.nitems;
  const long long ne = a.nitems;
  // Sender of sender-ordered position p (clamped so a corrupt permutation cannot fault).
  auto key = [&](long long p) {
    long long e = a.perm[p];
    e = (e < 0 || e >= ne) ? 0 : e;
    return a.cols[e];
  };
  long long p0 = 0, p1 = 0;
  if (L.lane == 0) {
    p0 = snap_to_key(static_cast<long long>((static_cast<__int128>(n) * wg) / nw), n, key);
    p1 = snap_to_key(static_cast<long long>((static_cast<__int128>(n) * (wg + 1)) / nw), n, key);
  }
  p0 = __shfl_sync(0xffffffffu, p0, 0);
  p1 = __shfl_sync(0xffffffffu, p1, 0);
  if (p0 >= p1) return;
  for (int g = 0; g < a.ngrp; ++g) {
    const GroupD gd = d.grp[g];
    const IrrepD r1 = d.ir1[gd.irrep];
    const int nch = (r1.mul + L.G - 1) >> L.lgG;
    for (int c = 0; c < nch; ++c) {
      const int c0 = c << L.lgG;
      const int ulen = min(L.G, r1.mul - c0);
      const int nel = ulen * r1.dim;
      SegAcc<T, KAHAN> sa;
      sa.reset();
      sa.cur = -1;
      for (long long base = p0; base < p1; base += rpw) {
        const long long pos = base + L.gsub;
        bool rv = pos < p1;
        long long e = a.perm[rv ? pos : p0];
        if (rv && (e < 0 || e >= ne)) {
          flag(a.status, 2);
          rv = false;
        }
        if (!rv) e = 0;
        long long xr = a.cols[e], gr = a.rows[e];
        if (rv && (xr < 0 || xr >= a.nnodes || gr < 0 || gr >= a.nnodes)) {
          flag(a.status, 1);
          rv = false;
        }
        if (!rv) xr = gr = 0;
        const RowPtrs<T> rp = row_ptrs(a, xr, e, gr);
        BwdOut<T> bo;
        bo.dy_row = rv ? a.out1 + e * a.L2dim : nullptr;  // zero-initialised, one writer
        bo.dw = a.shared_w ? a.out2 : a.out2 + e * a.wnumel;
        bo.shared_w = a.shared_w != 0;
        __syncwarp();
        if (L.gl == 0) s_key[wid][L.gsub] = rv ? xr : -1;
        with_degree(r1.l, [&]<int L1>() {
          bwd_chunk<T, UVW, DB, L1>(a, d, L, gd, r1, c, rv, rp, bo, stage + L.gsub * sstride);
        });
        __syncwarp();
        for (int s = 0; s < rpw; ++s) {
          const long long k = s_key[wid][s];
          if (k < 0) continue;
          if (k != sa.cur) {
            if (sa.cur >= 0) sa.store(a.out0 + sa.cur * a.L1dim, r1, c0, ulen, nel, L.lane);
            sa.reset();
            sa.cur = k;
          }
          sa.add(stage + s * sstride, nel, L.lane);
        }
      }
      if (sa.cur >= 0) sa.store(a.out0 + sa.cur * a.L1dim, r1, c0, ulen, nel, L.lane);
      __syncwarp();
    }
  }
}

}  // namespace oeqb
