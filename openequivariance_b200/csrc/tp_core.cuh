// Core device code for the Clebsch-Gordan tensor-product kernels (sm_100a).
//
// Semantics follow the reference's generated kernels (templates/loop_unroll_tp.cuh:19-313
// for one row, templates/loop_unroll_batch.cuh:26-318 for the batch passes,
// templates/loop_unroll_conv_{atomic,det}.cuh for the fused convolution):
//
//   uvu:  Z[u,k] += pw * sum_v sum_(i,j,k) C_ijk X[u,i] (W[u,v] Y[v,j])
//   uvw:  Z[w,k] += pw * sum_(u,v) W[u,v,w] sum_(i,j) C_ijk X[u,i] Y[v,j]
//
// with weights in the reference's "oeq" order (multiplicities split into chunks of 32,
// uvu blocks [v][u], uvw blocks [v][u][w]; ComputationSchedule.py:653-714).
//
// Work mapping.  A warp processes RPW = 32/G items (batch rows or edges) at a time;
// each item owns a lane group of G lanes (G = power of two covering the largest
// multiplicity, capped at 32).  Lane gl of a group is the multiplicity index u (or w)
// within the current 32-wide chunk.  Instructions are grouped by the irrep whose
// gradient/output they produce (output irrep for the forward, first input irrep for
// the backward), so each lane keeps its accumulator in registers for a whole group and
// writes every output element exactly once.  Output blocks are staged in a per-warp
// shared-memory buffer and written with coalesced stores.  Reductions over u (dY) use
// an xor butterfly inside the lane group, which is deterministic.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "cg_unrolled.cuh"

namespace oeqb {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kDMax = 15;  // largest irrep dimension supported (l <= 7)

struct IrrepD {
  int mul, l, dim, off, su, si;  // element (u, i) of this irrep sits at off + u*su + i*si
};

struct InstrD {
  int i1, i2, i3, code;  // code = triple_code(l1,l2,l3) (dispatch key)
  int m1, m2, m3;
  int l1, l2, l3;
  int woff;              // offset of this instruction's weights (oeq order)
  int cg_off, cg_nnz;    // slice of the generic CG table
  int pad;
  double pw;             // path weight
};

struct GroupD {
  int irrep, first, count, pad;
};

struct CGEntry {
  int i, j, k, pad;
  double c;
};

template <class T>
struct Args {
  const IrrepD* ir1;
  const IrrepD* ir2;
  const IrrepD* ir3;
  const InstrD* ins;     // instruction order used by this kernel
  const GroupD* grp;
  const CGEntry* cgtab;
  const int* zero_blocks;  // irreps of the produced tensor that no instruction touches
  int n1, n2, n3, nins, ngrp, nzero;
  int L1dim, L2dim, L3dim, wnumel, shared_w;
  int lgG;               // log2 of the lane-group size
  int ws_elems;          // per-warp scratch, in elements of T
  int off_t, off_t2, off_gz, off_dy;  // sub-buffers of the per-warp scratch
  long long nitems;      // rows (batch) or edges (conv)
  long long nnodes;      // conv only
  const T* X;
  const T* Y;
  const T* W;
  const T* Gz;           // gradient of the output (backward passes)
  const T* dA;           // double backward: upstream gradient for dX
  const T* dB;           // ... for dY
  const T* dC;           // ... for dW
  T* out0;               // forward: Z; backward: dX
  T* out1;               // backward: dY
  T* out2;               // backward: dW
  const long long* rows;  // conv receivers
  const long long* cols;  // conv senders
  const long long* perm;  // conv: receiver-sorted index of each sender-sorted position
  int* status;            // device error flag (bounds violations), may be null
};

// ---------------------------------------------------------------------------
// small helpers

__device__ __forceinline__ int widx_uvu(int m1, int m2, int u, int v) {
  const int u0 = u & ~31;
  const int ul = min(32, m1 - u0);
  return u0 * m2 + v * ul + (u - u0);
}

__device__ __forceinline__ int widx_uvw(int m1, int m2, int m3, int u, int v, int w) {
  const int u0 = u & ~31, ul = min(32, m1 - u0);
  const int v0 = v & ~31, vl = min(32, m2 - v0);
  const int w0 = w & ~31, wl = min(32, m3 - w0);
  return u0 * m2 * m3 + ul * v0 * m3 + ul * vl * w0 + (v - v0) * ul * wl + (u - u0) * wl + (w - w0);
}

template <class T, int D>
__device__ __forceinline__ void ldv(T (&v)[D], const T* __restrict__ base, const IrrepD& ir, int u) {
  const T* p = base + ir.off + u * ir.su;
#pragma unroll
  for (int i = 0; i < D; ++i) v[i] = p[i * ir.si];
}

template <class T, int D>
__device__ __forceinline__ void zero(T (&v)[D]) {
#pragma unroll
  for (int i = 0; i < D; ++i) v[i] = T(0);
}

template <class T>
__device__ __forceinline__ T group_sum(T v, int lgG) {
  for (int o = (1 << lgG) >> 1; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double atomic_add(double* p, double v) { return atomicAdd(p, v); }
__device__ __forceinline__ float atomic_add(float* p, float v) { return atomicAdd(p, v); }

// Index of element e of a staged block (chunk c of irrep ir, ulen lanes wide) inside its
// row.  Staging order follows the global layout so that consecutive e are consecutive
// addresses for mul_ir (and consecutive within each component for ir_mul).
__device__ __forceinline__ int block_addr(const IrrepD& ir, int c0, int ulen, int e) {
  if (ir.si == 1) return ir.off + c0 * ir.su + e;  // mul_ir: contiguous run
  const int k = e / ulen, ul = e - k * ulen;        // ir_mul: [k][u]
  return ir.off + k * ir.si + c0 + ul;
}

__device__ __forceinline__ int stage_index(const IrrepD& ir, int ulen, int ul, int k) {
  return (ir.si == 1) ? ul * ir.dim + k : k * ulen + ul;
}

// ---------------------------------------------------------------------------
// generic (table-driven) CG contractions for degrees beyond the unrolled range.
// Arrays are indexed dynamically, so they live in local memory; these paths are
// correct for any degree up to kDMax but not tuned.

template <class T>
__device__ void g_fwd(const CGEntry* tab, int nnz, const T* x, const T* y, T* z) {
  for (int n = 0; n < nnz; ++n) {
    const CGEntry e = tab[n];
    z[e.k] += (T(e.c) * x[e.i]) * y[e.j];
  }
}

template <class T>
__device__ T g_bwd(const CGEntry* tab, int nnz, const T* p, const T* q, const T* gz, T* gx, T* gy,
                   const T* x1, const T* y1, const T* x2, const T* y2) {
  T s = T(0);
  for (int n = 0; n < nnz; ++n) {
    const CGEntry e = tab[n];
    const T t = T(e.c) * gz[e.k];
    gx[e.i] += t * q[e.j];
    gy[e.j] += t * p[e.i];
    s += t * (x1[e.i] * y1[e.j]);
    if (x2) s += t * (x2[e.i] * y2[e.j]);
  }
  return s;
}

template <class T>
__device__ void g_ldv(T* v, const T* base, const IrrepD& ir, int u) {
  const T* p = base + ir.off + u * ir.su;
  for (int i = 0; i < ir.dim; ++i) v[i] = p[i * ir.si];
}

// ---------------------------------------------------------------------------
// Per-warp context shared by the per-instruction routines.

template <class T>
struct Lane {
  int lane, gl, gsub, lgG, G;
  T* ws;  // per-warp scratch base
};

// Row pointers for one item.
template <class T>
struct RowPtrs {
  const T* x;
  const T* y;
  const T* w;
  const T* g;   // output gradient row (backward)
  const T* a;   // double-backward rows
  const T* b;
  const T* c;
};

// ---------------------------------------------------------------------------
// uvu, forward (and double-backward part A): z[D3] accumulates output index u.

// wblk: this chunk's weight block, indexed v*ul + (u - u0) (ul = chunk width, u0 = start).
template <class T, int A, int B, int C, bool DB>
__device__ __forceinline__ void uvu_fwd(const InstrD& in, const IrrepD& r1, const IrrepD& r2,
                                        const RowPtrs<T>& rp, const T* wblk, int u, T* z) {
  constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1;
  T x[D1];
  ldv(x, rp.x, r1, u);
  T xa[DB ? D1 : 1];
  if constexpr (DB) ldv(xa, rp.a, r1, u);
  const T pw = T(in.pw);
  const int u0 = u & ~31, ul = min(32, in.m1 - u0);
  for (int v = 0; v < in.m2; ++v) {
    const int wi = in.woff + widx_uvu(in.m1, in.m2, u, v);
    const T wp = wblk[v * ul + (u - u0)] * pw;
    T y[D2];
    ldv(y, rp.y, r2, v);
    if constexpr (!DB) {
#pragma unroll
      for (int j = 0; j < D2; ++j) y[j] *= wp;
      CG<A, B, C>::fwd(x, y, z);
    } else {
      T yb[D2];
      ldv(yb, rp.b, r2, v);
      const T cp = rp.c[wi] * pw;
      T q[D2];
#pragma unroll
      for (int j = 0; j < D2; ++j) {
        q[j] = wp * yb[j] + cp * y[j];
        y[j] *= wp;
      }
      CG<A, B, C>::fwd(xa, y, z);
      CG<A, B, C>::fwd(x, q, z);
    }
  }
}

// Table-driven uvu forward for triples outside the unrolled range; adds into zt[kDMax].
template <class T, bool DB>
__device__ __noinline__ void uvu_fwd_generic(const InstrD in, const IrrepD r1, const IrrepD r2,
                                             const CGEntry* cgtab, const RowPtrs<T> rp, int u,
                                             T* zt) {
  T x[kDMax], xa[kDMax], y[kDMax], q[kDMax];
  g_ldv(x, rp.x, r1, u);
  if (DB) g_ldv(xa, rp.a, r1, u);
  const T pw = T(in.pw);
  const CGEntry* tab = cgtab + in.cg_off;
  for (int v = 0; v < in.m2; ++v) {
    const int wi = in.woff + widx_uvu(in.m1, in.m2, u, v);
    const T wp = rp.w[wi] * pw;
    g_ldv(y, rp.y, r2, v);
    if (!DB) {
      for (int j = 0; j < r2.dim; ++j) y[j] *= wp;
      g_fwd(tab, in.cg_nnz, x, y, zt);
    } else {
      g_ldv(q, rp.b, r2, v);
      const T cp = rp.c[wi] * pw;
      for (int j = 0; j < r2.dim; ++j) {
        q[j] = wp * q[j] + cp * y[j];
        y[j] *= wp;
      }
      g_fwd(tab, in.cg_nnz, xa, y, zt);
      g_fwd(tab, in.cg_nnz, x, q, zt);
    }
  }
}

// ---------------------------------------------------------------------------
// uvu, backward (and double-backward part B) for lane u.  gx accumulates dX[u, :];
// the dY contribution is reduced over the lane group and added into the per-warp dY
// staging row by the group's first lane; dW is written (or atomically added when the
// weights are shared).

template <class T>
struct BwdOut {
  T* dy_row;   // per-warp smem staging for this item's dY (length L2dim)
  T* dw;       // dW row (global)
  bool shared_w;
  int dy_shift = 0;  // real irrep offset minus the offset of the (staged) view used to read Y
};

template <class T, int A, int B, int C, bool DB>
__device__ __forceinline__ void uvu_bwd(const InstrD& in, const IrrepD& r1, const IrrepD& r2,
                                        const IrrepD& r3, const RowPtrs<T>& rp, const T* wblk,
                                        int u, bool act, const Lane<T>& L, T* gx,
                                        const BwdOut<T>& bo) {
  constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1, D3 = 2 * C + 1;
  T x[D1], gz[D3];
  T xa[DB ? D1 : 1];
  if (act) {
    ldv(x, rp.x, r1, u);
    ldv(gz, rp.g, r3, u);
    if constexpr (DB) ldv(xa, rp.a, r1, u);
  }
  const T pw = T(in.pw);
  const int u0 = u & ~31, ul = min(32, in.m1 - u0);
  for (int v = 0; v < in.m2; ++v) {
    T gy[D2];
    zero(gy);
    if (act) {
      const int wi = in.woff + widx_uvu(in.m1, in.m2, u, v);
      const T wp = wblk[v * ul + (u - u0)] * pw;
      T y[D2];
      ldv(y, rp.y, r2, v);
      T s = T(0);
      if constexpr (!DB) {
        // h_i = sum c gz_k y_j:  dX_i += w h_i,  dW = sum_i x_i h_i;  e_j = sum c gz_k x_i.
        T h[D1];
        CG<A, B, C>::hvec(gz, y, h);
#pragma unroll
        for (int i = 0; i < D1; ++i) {
          gx[i] += wp * h[i];
          s += x[i] * h[i];
        }
        T e[D2];
        CG<A, B, C>::evec(gz, x, e);
#pragma unroll
        for (int j = 0; j < D2; ++j) gy[j] = wp * e[j];
      } else {
        T yb[D2];
        ldv(yb, rp.b, r2, v);
        const T cp = rp.c[wi] * pw;
        T hy[D1], hb[D1];
        CG<A, B, C>::hvec(gz, y, hy);
        CG<A, B, C>::hvec(gz, yb, hb);
#pragma unroll
        for (int i = 0; i < D1; ++i) {
          gx[i] += wp * hb[i] + cp * hy[i];
          s += xa[i] * hy[i] + x[i] * hb[i];
        }
        T ea[D2], ex[D2];
        CG<A, B, C>::evec(gz, xa, ea);
        CG<A, B, C>::evec(gz, x, ex);
#pragma unroll
        for (int j = 0; j < D2; ++j) gy[j] = wp * ea[j] + cp * ex[j];
      }
      if (bo.shared_w)
        atomic_add(bo.dw + wi, s * pw);
      else
        bo.dw[wi] = s * pw;
    }
#pragma unroll
    for (int j = 0; j < D2; ++j) {
      const T t = group_sum(gy[j], L.lgG);
      if (L.gl == 0 && bo.dy_row) bo.dy_row[r2.off + bo.dy_shift + v * r2.su + j * r2.si] += t;
    }
  }
}

// Table-driven uvu backward; adds dX into gxt[kDMax].  All lanes must call it.
template <class T, bool DB>
__device__ __noinline__ void uvu_bwd_generic(const InstrD in, const IrrepD r1, const IrrepD r2,
                                             const IrrepD r3, const CGEntry* cgtab,
                                             const RowPtrs<T> rp, int u, bool act, int lgG,
                                             int gl, T* gxt, const BwdOut<T> bo) {
  T x[kDMax], xa[kDMax], gz[kDMax], y[kDMax], yb[kDMax], p[kDMax], q[kDMax], gy[kDMax];
  if (act) {
    g_ldv(x, rp.x, r1, u);
    g_ldv(gz, rp.g, r3, u);
    if (DB) g_ldv(xa, rp.a, r1, u);
  }
  const T pw = T(in.pw);
  const CGEntry* tab = cgtab + in.cg_off;
  for (int v = 0; v < in.m2; ++v) {
    for (int j = 0; j < kDMax; ++j) gy[j] = T(0);
    if (act) {
      const int wi = in.woff + widx_uvu(in.m1, in.m2, u, v);
      const T wp = rp.w[wi] * pw;
      g_ldv(y, rp.y, r2, v);
      T s;
      if (!DB) {
        for (int i = 0; i < r1.dim; ++i) p[i] = wp * x[i];
        for (int j = 0; j < r2.dim; ++j) q[j] = wp * y[j];
        s = g_bwd<T>(tab, in.cg_nnz, p, q, gz, gxt, gy, x, y, nullptr, nullptr);
      } else {
        g_ldv(yb, rp.b, r2, v);
        const T cp = rp.c[wi] * pw;
        for (int i = 0; i < r1.dim; ++i) p[i] = wp * xa[i] + cp * x[i];
        for (int j = 0; j < r2.dim; ++j) q[j] = wp * yb[j] + cp * y[j];
        s = g_bwd<T>(tab, in.cg_nnz, p, q, gz, gxt, gy, xa, y, x, yb);
      }
      if (bo.shared_w)
        atomic_add(bo.dw + wi, s * pw);
      else
        bo.dw[wi] = s * pw;
    }
    for (int j = 0; j < r2.dim; ++j) {
      const T t = group_sum(gy[j], lgG);
      if (gl == 0 && bo.dy_row) bo.dy_row[r2.off + v * r2.su + j * r2.si] += t;
    }
  }
}

// ---------------------------------------------------------------------------
// uvw, forward.  All lanes of the warp must call this (it synchronises the warp).
// Phase A (lane = u) contracts X and Y into t[u][k] in the per-warp scratch; phase B
// (lane = w) accumulates z[k] += pw * sum_u W[u,v,w] t[u][k].  For the double backward,
// t1 = dX' (x) Y + X (x) dY' is weighted by W and t2 = X (x) Y by dW'.

template <class T, int A, int B, int C, bool DB>
__device__ __forceinline__ void uvw_fwd(const InstrD& in, const IrrepD& r1, const IrrepD& r2,
                                        const RowPtrs<T>& rp, bool rv, int w, bool actw,
                                        const Lane<T>& L, T* ws_t, T* ws_t2, T* z) {
  constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1, D3 = 2 * C + 1;
  const int G = L.G;
  const T pw = T(in.pw);
  const int nchu = (in.m1 + G - 1) >> L.lgG;
  T* tg = ws_t + L.gsub * G * D3;
  T* tg2 = ws_t2 + L.gsub * G * D3;
  for (int v = 0; v < in.m2; ++v) {
    for (int cu = 0; cu < nchu; ++cu) {
      const int u = (cu << L.lgG) + L.gl;
      T t1[D3], t2[DB ? D3 : 1];
      zero(t1);
      if constexpr (DB) zero(t2);
      if (rv && u < in.m1) {
        T x[D1], y[D2];
        ldv(x, rp.x, r1, u);
        ldv(y, rp.y, r2, v);
        if constexpr (!DB) {
          CG<A, B, C>::fwd(x, y, t1);
        } else {
          T xa[D1], yb[D2];
          ldv(xa, rp.a, r1, u);
          ldv(yb, rp.b, r2, v);
          CG<A, B, C>::fwd(xa, y, t1);
          CG<A, B, C>::fwd(x, yb, t1);
          CG<A, B, C>::fwd(x, y, t2);
        }
      }
      __syncwarp();
#pragma unroll
      for (int k = 0; k < D3; ++k) {
        tg[L.gl * D3 + k] = t1[k];
        if constexpr (DB) tg2[L.gl * D3 + k] = t2[k];
      }
      __syncwarp();
      if (actw) {
        const int ulen = min(G, in.m1 - (cu << L.lgG));
        for (int ul = 0; ul < ulen; ++ul) {
          const int wi = in.woff + widx_uvw(in.m1, in.m2, in.m3, (cu << L.lgG) + ul, v, w);
          const T wt = rp.w[wi] * pw;
#pragma unroll
          for (int k = 0; k < D3; ++k) z[k] += wt * tg[ul * D3 + k];
          if constexpr (DB) {
            const T ct = rp.c[wi] * pw;
#pragma unroll
            for (int k = 0; k < D3; ++k) z[k] += ct * tg2[ul * D3 + k];
          }
        }
      }
      __syncwarp();
    }
  }
}

// Table-driven uvw forward; adds into zt[kDMax].  All lanes must call it.
template <class T, bool DB>
__device__ __noinline__ void uvw_fwd_generic(const InstrD in, const IrrepD r1, const IrrepD r2,
                                             const CGEntry* cgtab, const RowPtrs<T> rp, bool rv,
                                             int w, bool actw, int lgG, int gl, int gsub,
                                             T* ws_t, T* ws_t2, T* zt) {
  const int G = 1 << lgG;
  const int d3 = 2 * in.l3 + 1;
  const T pw = T(in.pw);
  const int nchu = (in.m1 + G - 1) >> lgG;
  const CGEntry* tab = cgtab + in.cg_off;
  T* tg = ws_t + gsub * G * kDMax;
  T* tg2 = ws_t2 + gsub * G * kDMax;
  T x[kDMax], y[kDMax], xa[kDMax], yb[kDMax], t1[kDMax], t2[kDMax];
  for (int v = 0; v < in.m2; ++v) {
    for (int cu = 0; cu < nchu; ++cu) {
      const int u = (cu << lgG) + gl;
      for (int k = 0; k < kDMax; ++k) t1[k] = t2[k] = T(0);
      if (rv && u < in.m1) {
        g_ldv(x, rp.x, r1, u);
        g_ldv(y, rp.y, r2, v);
        if (!DB) {
          g_fwd(tab, in.cg_nnz, x, y, t1);
        } else {
          g_ldv(xa, rp.a, r1, u);
          g_ldv(yb, rp.b, r2, v);
          g_fwd(tab, in.cg_nnz, xa, y, t1);
          g_fwd(tab, in.cg_nnz, x, yb, t1);
          g_fwd(tab, in.cg_nnz, x, y, t2);
        }
      }
      __syncwarp();
      for (int k = 0; k < d3; ++k) {
        tg[gl * kDMax + k] = t1[k];
        if (DB) tg2[gl * kDMax + k] = t2[k];
      }
      __syncwarp();
      if (actw) {
        const int ulen = min(G, in.m1 - (cu << lgG));
        for (int ul = 0; ul < ulen; ++ul) {
          const int wi = in.woff + widx_uvw(in.m1, in.m2, in.m3, (cu << lgG) + ul, v, w);
          const T wt = rp.w[wi] * pw;
          const T ct = DB ? rp.c[wi] * pw : T(0);
          for (int k = 0; k < d3; ++k) {
            zt[k] += wt * tg[ul * kDMax + k];
            if (DB) zt[k] += ct * tg2[ul * kDMax + k];
          }
        }
      }
      __syncwarp();
    }
  }
}

// Stage the output-gradient block G[w][k] (all w of irrep r3) of each item slot.
template <class T>
__device__ __forceinline__ T* stage_gz(const InstrD& in, const IrrepD& r3, const RowPtrs<T>& rp,
                                       bool rv, int lgG, int gl, int gsub, T* ws_gz) {
  const int G = 1 << lgG;
  const int d3 = r3.dim;
  T* gzs = ws_gz + gsub * (in.m3 * d3);
  __syncwarp();
  for (int e = gl; e < in.m3 * d3; e += G) {
    const int w = e / d3, k = e - w * d3;
    gzs[e] = rv ? rp.g[r3.off + w * r3.su + k * r3.si] : T(0);
  }
  __syncwarp();
  return gzs;
}

// uvw, backward (and double-backward part B) for lane u of chunk cu.  All lanes call.
template <class T, int A, int B, int C, bool DB>
__device__ __forceinline__ void uvw_bwd(const InstrD& in, const IrrepD& r1, const IrrepD& r2,
                                        const IrrepD& r3, const RowPtrs<T>& rp, bool rv, int cu,
                                        const Lane<T>& L, T* ws_t, T* ws_gz, T* gx,
                                        const BwdOut<T>& bo) {
  constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1, D3 = 2 * C + 1;
  const int G = L.G;
  const int u = (cu << L.lgG) + L.gl;
  const bool actu = rv && u < in.m1;
  const T pw = T(in.pw);
  const T* gzs = stage_gz(in, r3, rp, rv, L.lgG, L.gl, L.gsub, ws_gz);
  T* tg = ws_t + L.gsub * G * D3;
  T x[D1];
  T xa[DB ? D1 : 1];
  if (actu) {
    ldv(x, rp.x, r1, u);
    if constexpr (DB) ldv(xa, rp.a, r1, u);
  }
  for (int v = 0; v < in.m2; ++v) {
    T gy[D2], t[D3];
    zero(gy);
    zero(t);
    if (actu) {
      T dtw[D3], dtc[DB ? D3 : 1];
      zero(dtw);
      if constexpr (DB) zero(dtc);
      for (int w = 0; w < in.m3; ++w) {
        const int wi = in.woff + widx_uvw(in.m1, in.m2, in.m3, u, v, w);
        const T wt = rp.w[wi] * pw;
#pragma unroll
        for (int k = 0; k < D3; ++k) dtw[k] += wt * gzs[w * D3 + k];
        if constexpr (DB) {
          const T ct = rp.c[wi] * pw;
#pragma unroll
          for (int k = 0; k < D3; ++k) dtc[k] += ct * gzs[w * D3 + k];
        }
      }
      T y[D2];
      ldv(y, rp.y, r2, v);
      T h[D1], e[D2];
      if constexpr (!DB) {
        CG<A, B, C>::hvec(dtw, y, h);
        CG<A, B, C>::evec(dtw, x, e);
#pragma unroll
        for (int i = 0; i < D1; ++i) gx[i] += h[i];
#pragma unroll
        for (int j = 0; j < D2; ++j) gy[j] += e[j];
        CG<A, B, C>::fwd(x, y, t);
      } else {
        T yb[D2];
        ldv(yb, rp.b, r2, v);
        CG<A, B, C>::hvec(dtw, yb, h);
        CG<A, B, C>::evec(dtw, xa, e);
#pragma unroll
        for (int i = 0; i < D1; ++i) gx[i] += h[i];
#pragma unroll
        for (int j = 0; j < D2; ++j) gy[j] += e[j];
        CG<A, B, C>::hvec(dtc, y, h);
        CG<A, B, C>::evec(dtc, x, e);
#pragma unroll
        for (int i = 0; i < D1; ++i) gx[i] += h[i];
#pragma unroll
        for (int j = 0; j < D2; ++j) gy[j] += e[j];
        CG<A, B, C>::fwd(xa, y, t);
        CG<A, B, C>::fwd(x, yb, t);
      }
    }
#pragma unroll
    for (int j = 0; j < D2; ++j) {
      const T s = group_sum(gy[j], L.lgG);
      if (L.gl == 0 && bo.dy_row) bo.dy_row[r2.off + v * r2.su + j * r2.si] += s;
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < D3; ++k) tg[L.gl * D3 + k] = t[k];
    __syncwarp();
    if (rv) {
      const int ulen = min(G, in.m1 - (cu << L.lgG));
      for (int w = L.gl; w < in.m3; w += G) {
        for (int ul = 0; ul < ulen; ++ul) {
          T s = T(0);
#pragma unroll
          for (int k = 0; k < D3; ++k) s += gzs[w * D3 + k] * tg[ul * D3 + k];
          const int wi = in.woff + widx_uvw(in.m1, in.m2, in.m3, (cu << L.lgG) + ul, v, w);
          if (bo.shared_w)
            atomic_add(bo.dw + wi, s * pw);
          else
            bo.dw[wi] = s * pw;
        }
      }
    }
    __syncwarp();
  }
}

// Table-driven uvw backward; adds dX into gxt[kDMax].  All lanes call.
template <class T, bool DB>
__device__ __noinline__ void uvw_bwd_generic(const InstrD in, const IrrepD r1, const IrrepD r2,
                                             const IrrepD r3, const CGEntry* cgtab,
                                             const RowPtrs<T> rp, bool rv, int cu, int lgG,
                                             int gl, int gsub, T* ws_t, T* ws_gz, T* gxt,
                                             const BwdOut<T> bo) {
  const int G = 1 << lgG;
  const int d2 = r2.dim, d3 = r3.dim;
  const int u = (cu << lgG) + gl;
  const bool actu = rv && u < in.m1;
  const T pw = T(in.pw);
  const CGEntry* tab = cgtab + in.cg_off;
  const T* gzs = stage_gz(in, r3, rp, rv, lgG, gl, gsub, ws_gz);
  T* tg = ws_t + gsub * G * kDMax;
  T x[kDMax], xa[kDMax], y[kDMax], yb[kDMax], gy[kDMax], t[kDMax], dtw[kDMax], dtc[kDMax];
  if (actu) {
    g_ldv(x, rp.x, r1, u);
    if (DB) g_ldv(xa, rp.a, r1, u);
  }
  for (int v = 0; v < in.m2; ++v) {
    for (int k = 0; k < kDMax; ++k) gy[k] = t[k] = dtw[k] = dtc[k] = T(0);
    if (actu) {
      for (int w = 0; w < in.m3; ++w) {
        const int wi = in.woff + widx_uvw(in.m1, in.m2, in.m3, u, v, w);
        const T wt = rp.w[wi] * pw;
        const T ct = DB ? rp.c[wi] * pw : T(0);
        for (int k = 0; k < d3; ++k) {
          dtw[k] += wt * gzs[w * d3 + k];
          if (DB) dtc[k] += ct * gzs[w * d3 + k];
        }
      }
      g_ldv(y, rp.y, r2, v);
      if (!DB) {
        g_bwd<T>(tab, in.cg_nnz, x, y, dtw, gxt, gy, x, y, nullptr, nullptr);
        g_fwd(tab, in.cg_nnz, x, y, t);
      } else {
        g_ldv(yb, rp.b, r2, v);
        g_bwd<T>(tab, in.cg_nnz, xa, yb, dtw, gxt, gy, x, y, nullptr, nullptr);
        g_bwd<T>(tab, in.cg_nnz, x, y, dtc, gxt, gy, x, y, nullptr, nullptr);
        g_fwd(tab, in.cg_nnz, xa, y, t);
        g_fwd(tab, in.cg_nnz, x, yb, t);
      }
    }
    for (int j = 0; j < d2; ++j) {
      const T s = group_sum(gy[j], lgG);
      if (gl == 0 && bo.dy_row) bo.dy_row[r2.off + v * r2.su + j * r2.si] += s;
    }
    __syncwarp();
    for (int k = 0; k < d3; ++k) tg[gl * kDMax + k] = t[k];
    __syncwarp();
    if (rv) {
      const int ulen = min(G, in.m1 - (cu << lgG));
      for (int w = gl; w < in.m3; w += G) {
        for (int ul = 0; ul < ulen; ++ul) {
          T s = T(0);
          for (int k = 0; k < d3; ++k) s += gzs[w * d3 + k] * tg[ul * kDMax + k];
          const int wi = in.woff + widx_uvw(in.m1, in.m2, in.m3, (cu << lgG) + ul, v, w);
          if (bo.shared_w)
            atomic_add(bo.dw + wi, s * pw);
          else
            bo.dw[wi] = s * pw;
        }
      }
    }
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// Shared-memory descriptor staging.

struct SmemDesc {
  IrrepD* ir1;
  IrrepD* ir2;
  IrrepD* ir3;
  InstrD* ins;
  GroupD* grp;
  int* zb;
  unsigned char* end;
};

template <class T>
__device__ __forceinline__ SmemDesc stage_desc(const Args<T>& a, unsigned char* sm) {
  SmemDesc d;
  unsigned char* p = sm;
  d.ins = reinterpret_cast<InstrD*>(p);
  p += sizeof(InstrD) * a.nins;
  d.ir1 = reinterpret_cast<IrrepD*>(p);
  p += sizeof(IrrepD) * a.n1;
  d.ir2 = reinterpret_cast<IrrepD*>(p);
  p += sizeof(IrrepD) * a.n2;
  d.ir3 = reinterpret_cast<IrrepD*>(p);
  p += sizeof(IrrepD) * a.n3;
  d.grp = reinterpret_cast<GroupD*>(p);
  p += sizeof(GroupD) * a.ngrp;
  d.zb = reinterpret_cast<int*>(p);
  p += sizeof(int) * a.nzero;
  p = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t(15));
  d.end = p;
  auto copy = [&](void* dst, const void* src, int bytes) {
    const int* s = reinterpret_cast<const int*>(src);
    int* t = reinterpret_cast<int*>(dst);
    for (int i = threadIdx.x; i < bytes / 4; i += blockDim.x) t[i] = s[i];
  };
  copy(d.ins, a.ins, sizeof(InstrD) * a.nins);
  copy(d.ir1, a.ir1, sizeof(IrrepD) * a.n1);
  copy(d.ir2, a.ir2, sizeof(IrrepD) * a.n2);
  copy(d.ir3, a.ir3, sizeof(IrrepD) * a.n3);
  copy(d.grp, a.grp, sizeof(GroupD) * a.ngrp);
  copy(d.zb, a.zero_blocks, sizeof(int) * a.nzero);
  __syncthreads();
  return d;
}

// Write a staged block (RPW items x ulen*dim elements) to its rows with coalesced stores.
// MODE 0: plain store; 1: atomic add.
template <class T, int MODE>
__device__ __forceinline__ void flush_block(const Lane<T>& L, const T* stage, int stride,
                                            const IrrepD& ir, int c0, int ulen, T* dst,
                                            const long long* dst_rows, int rowlen) {
  const int n = ulen * ir.dim;
  const int rpw = 32 >> L.lgG;
  for (int idx = L.lane; idx < rpw * n; idx += 32) {
    const int s = idx / n, e = idx - s * n;
    const long long r = dst_rows[s];
    if (r < 0) continue;
    T* p = dst + r * (long long)rowlen + block_addr(ir, c0, ulen, e);
    if constexpr (MODE == 0)
      *p = stage[s * stride + e];
    else
      atomic_add(p, stage[s * stride + e]);
  }
}

}  // namespace oeqb
