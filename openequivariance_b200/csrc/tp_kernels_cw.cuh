// Channelwise-uvu batch kernels: the MACE / NequIP interaction class.
//
// Eligible problems: uvu, mul_ir layout, every instruction with one copy of its Y irrep
// (m2 == 1), multiplicities that are multiples of 32, and one instruction per output
// irrep.  This is the shape of e3nn/MACE "channelwise" tensor products (BASELINE C2).
//
// Row staging and the mbarrier/TMA pipeline are those of tp_kernels_row.cuh.  What makes
// these kernels lean:
//   * all index arithmetic is compile-time (mul_ir, per-triple dimensions) plus one
//     precomputed record per item (instruction x 32-lane chunk);
//   * the CG contraction uses the row's Y once per item: P[i][k] = sum_j c_ijk y_j, then
//     z_k = w pw sum_i x_i P[i][k] (dense D1 x D3 FMAs instead of two per CG non-zero);
//   * forward items process two rows each, halving per-item overhead;
//   * backward dY accumulates in lane-private shared-memory columns and is reduced once per
//     row (no per-item butterfly); dX accumulates in per-warp partial rows; both are summed
//     in fixed order, so results are bitwise reproducible.
#pragma once

#include "tp_kernels_row.cuh"

namespace oeqb {

struct CwItem {
  int code;    // triple_code(l1, l2, l3)
  int x_off;   // X row offset of this chunk (irrep offset + c0 * d1)
  int y_off;   // Y row offset of the Y irrep
  int w_off;   // W row offset of this chunk (instruction offset + c0)
  int z_off;   // output row offset of this chunk (irrep offset + c0 * d3)
  int xp_off;  // offset of this chunk in the warp's dX partial (backward)
  int pad0, pad1;
  double pw;
};

// Backward dX reduction plan: per X irrep, where its chunks live in the warp partials.
struct CwXIrrep {
  int off, dim, nch, poff;  // row offset, irrep dim, chunks, offset of chunk slice in partials
};

template <class T>
struct ArgsCw {
  Args<T> a;
  const CwItem* items;
  const CwXIrrep* xirr;
  int nitems, nxirr;
  int nwarps;
  int chunk_mode;   // backward: 1 = warp w owns chunk w % nch_all; partials hold one chunk
  int nch_all;      // chunks per instruction (chunk mode)
  int dxn;          // elements of the per-warp dX partial
  int offY, offW, offG, row_elems;  // one row's layout in the row buffer
  int rows_per_buf;                 // forward: rows staged per buffer (consecutive rows)
  int use_tma;
  int ws_elems;                     // per-warp scratch
};

struct SmemCw {
  CwItem* items;
  CwXIrrep* xirr;
  unsigned long long* bars;
  unsigned char* rowbuf;
  unsigned char* warps;
};

template <class T>
__device__ __forceinline__ SmemCw stage_cw(const ArgsCw<T>& v, unsigned char* sm) {
  SmemCw s;
  unsigned char* p = sm;
  s.items = reinterpret_cast<CwItem*>(p);
  p += sizeof(CwItem) * v.nitems;
  s.xirr = reinterpret_cast<CwXIrrep*>(p);
  p += sizeof(CwXIrrep) * v.nxirr;
  p = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t(15));
  s.bars = reinterpret_cast<unsigned long long*>(p);
  p += 16;
  s.rowbuf = p;
  p += 2 * sizeof(T) * static_cast<size_t>(v.row_elems) * v.rows_per_buf;
  s.warps = p;
  const int* src = reinterpret_cast<const int*>(v.items);
  int* dst = reinterpret_cast<int*>(s.items);
  for (int i = threadIdx.x; i < static_cast<int>(sizeof(CwItem) / 4) * v.nitems; i += blockDim.x)
    dst[i] = src[i];
  const int* xs = reinterpret_cast<const int*>(v.xirr);
  int* xd = reinterpret_cast<int*>(s.xirr);
  for (int i = threadIdx.x; i < 4 * v.nxirr; i += blockDim.x) xd[i] = xs[i];
  if (threadIdx.x == 0) {
    mbar_init(&s.bars[0], 1);
    mbar_init(&s.bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  return s;
}

// Loads rows [row0, row0 + n) into buffer b.  Row r of the buffer holds X | Y | W (| dZ)
// at r * row_elems.  TMA: one bulk copy per tensor and row.
template <class T, bool BWD>
__device__ __forceinline__ void cw_load(const ArgsCw<T>& v, const SmemCw& s, int b, long long row0,
                                        int n) {
  const Args<T>& a = v.a;
  T* buf = reinterpret_cast<T*>(s.rowbuf) + static_cast<size_t>(b) * v.row_elems * v.rows_per_buf;
  if (v.use_tma) {
    if (threadIdx.x == 0) {
      unsigned bytes = 0;
      const int per_row = a.L1dim + a.L2dim + (a.shared_w ? 0 : a.wnumel) + (BWD ? a.L3dim : 0);
      bytes = static_cast<unsigned>(per_row * n * sizeof(T));
      mbar_expect_tx(&s.bars[b], bytes);
      for (int r = 0; r < n; ++r) {
        T* rb = buf + static_cast<size_t>(r) * v.row_elems;
        const long long row = row0 + r;
        bulk_g2s(rb, a.X + row * a.L1dim, a.L1dim * sizeof(T), &s.bars[b]);
        bulk_g2s(rb + v.offY, a.Y + row * a.L2dim, a.L2dim * sizeof(T), &s.bars[b]);
        if (!a.shared_w) bulk_g2s(rb + v.offW, a.W + row * a.wnumel, a.wnumel * sizeof(T), &s.bars[b]);
        if (BWD) bulk_g2s(rb + v.offG, a.Gz + row * a.L3dim, a.L3dim * sizeof(T), &s.bars[b]);
      }
    }
  } else {
    for (int r = 0; r < n; ++r) {
      T* rb = buf + static_cast<size_t>(r) * v.row_elems;
      const long long row = row0 + r;
      for (int e = threadIdx.x; e < a.L1dim; e += blockDim.x) rb[e] = a.X[row * a.L1dim + e];
      for (int e = threadIdx.x; e < a.L2dim; e += blockDim.x) rb[v.offY + e] = a.Y[row * a.L2dim + e];
      if (!a.shared_w)
        for (int e = threadIdx.x; e < a.wnumel; e += blockDim.x) rb[v.offW + e] = a.W[row * a.wnumel + e];
      if (BWD)
        for (int e = threadIdx.x; e < a.L3dim; e += blockDim.x) rb[v.offG + e] = a.Gz[row * a.L3dim + e];
    }
  }
}

// ---------------------------------------------------------------------------------------

template <class T>
__global__ void __launch_bounds__(256, 2) tp_fwd_cw(const ArgsCw<T> v) {
  extern __shared__ __align__(16) unsigned char smem[];
  const SmemCw s = stage_cw(v, smem);
  const Args<T>& a = v.a;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  T* stage0 = reinterpret_cast<T*>(s.warps) + static_cast<size_t>(wid) * v.ws_elems;
  int sb = 0;
  const int R = v.rows_per_buf;
  const long long B = a.nitems;
  const long long nblk = (B + R - 1) / R;
  auto rows_in = [&](long long blk) { return static_cast<int>(min(static_cast<long long>(R), B - blk * R)); };
  if (blockIdx.x < nblk) cw_load<T, false>(v, s, 0, blockIdx.x * R, rows_in(blockIdx.x));
  if (blockIdx.x + gridDim.x < nblk)
    cw_load<T, false>(v, s, 1, (blockIdx.x + gridDim.x) * R, rows_in(blockIdx.x + gridDim.x));
  if (!v.use_tma) __syncthreads();
  int it = 0;
  for (long long blk = blockIdx.x; blk < nblk; blk += gridDim.x, ++it) {
    const int b = it & 1;
    const int nr = rows_in(blk);
    if (v.use_tma) mbar_wait(&s.bars[b], (it >> 1) & 1, a.status);
    const T* buf = reinterpret_cast<const T*>(s.rowbuf) + static_cast<size_t>(b) * v.row_elems * R;
    const T* wsh = a.shared_w ? a.W : nullptr;
    for (int ii = wid; ii < v.nitems; ii += v.nwarps) {
      const CwItem it_ = s.items[ii];
      dispatch_triple(it_.code, [&]<int A, int Bd, int C>() {
        constexpr int D1 = 2 * A + 1, D2 = 2 * Bd + 1, D3 = 2 * C + 1;
        const T pw = T(it_.pw);
        for (int r = 0; r < nr; ++r) {
          const T* rb = buf + static_cast<size_t>(r) * v.row_elems;
          T y[D2];
#pragma unroll
          for (int j = 0; j < D2; ++j) y[j] = rb[v.offY + it_.y_off + j];
          T P[D1 * D3];
          CG<A, Bd, C>::pmat(y, P);
          const T* xs = rb + it_.x_off + lane * D1;
          T x[D1];
#pragma unroll
          for (int i = 0; i < D1; ++i) x[i] = xs[i];
          const T w = (a.shared_w ? wsh[it_.w_off + lane] : rb[v.offW + it_.w_off + lane]) * pw;
          T z[D3];
#pragma unroll
          for (int k = 0; k < D3; ++k) {
            T acc = T(0);
#pragma unroll
            for (int i = 0; i < D1; ++i) acc += x[i] * P[i * D3 + k];
            z[k] = acc * w;
          }
          T* stage = stage0 + sb * (32 * kDMax);
          sb ^= 1;
          if (lane == 0) bulk_wait_read<1>();
          __syncwarp();
#pragma unroll
          for (int k = 0; k < D3; ++k) stage[lane * D3 + k] = z[k];
          T* dst = a.out0 + (blk * R + r) * a.L3dim + it_.z_off;
          const unsigned bytes = 32 * D3 * sizeof(T);
          if (((reinterpret_cast<uintptr_t>(dst) | bytes) & 15) == 0) {
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
              bulk_s2g(dst, stage, bytes);
              bulk_commit();
            }
          } else {
            __syncwarp();
            for (int e = lane; e < 32 * D3; e += 32) dst[e] = stage[e];
          }
        }
      });
    }
    __syncthreads();
    const long long next = blk + 2LL * gridDim.x;
    if (next < nblk) cw_load<T, false>(v, s, b, next * R, rows_in(next));
    if (!v.use_tma) __syncthreads();
  }
  if (lane == 0) bulk_wait_all<0>();
}

template <class T, int NW>
__global__ void __launch_bounds__(NW * 32, 1) tp_bwd_cw(const ArgsCw<T> v) {
  extern __shared__ __align__(16) unsigned char smem[];
  const SmemCw s = stage_cw(v, smem);
  const Args<T>& a = v.a;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  // Per-warp scratch: dX partial (v.dxn elements) then dY lane columns [L2dim][32].
  T* dxp = reinterpret_cast<T*>(s.warps) + static_cast<size_t>(wid) * v.ws_elems;
  T* gyc = dxp + v.dxn;
  const long long B = a.nitems;
  if (blockIdx.x < B) cw_load<T, true>(v, s, 0, blockIdx.x, 1);
  if (blockIdx.x + gridDim.x < B) cw_load<T, true>(v, s, 1, blockIdx.x + gridDim.x, 1);
  if (!v.use_tma) __syncthreads();
  int it = 0;
  for (long long row = blockIdx.x; row < B; row += gridDim.x, ++it) {
    const int b = it & 1;
    for (int e = lane; e < v.dxn + a.L2dim * 32; e += 32) dxp[e] = T(0);
    if (v.use_tma) mbar_wait(&s.bars[b], (it >> 1) & 1, a.status);
    __syncwarp();
    const T* rb = reinterpret_cast<const T*>(s.rowbuf) + static_cast<size_t>(b) * v.row_elems;
    T* dwrow = a.shared_w ? a.out2 : a.out2 + row * a.wnumel;
    for (int ii = wid; ii < v.nitems; ii += NW) {
      const CwItem it_ = s.items[ii];
      dispatch_triple(it_.code, [&]<int A, int Bd, int C>() {
        constexpr int D1 = 2 * A + 1, D2 = 2 * Bd + 1, D3 = 2 * C + 1;
        const T pw = T(it_.pw);
        T y[D2];
#pragma unroll
        for (int j = 0; j < D2; ++j) y[j] = rb[v.offY + it_.y_off + j];
        T P[D1 * D3];
        CG<A, Bd, C>::pmat(y, P);
        T x[D1], gz[D3];
        const T* xs = rb + it_.x_off + lane * D1;
        const T* gs = rb + v.offG + it_.z_off + lane * D3;
#pragma unroll
        for (int i = 0; i < D1; ++i) x[i] = xs[i];
#pragma unroll
        for (int k = 0; k < D3; ++k) gz[k] = gs[k];
        const T wraw = a.shared_w ? a.W[it_.w_off + lane] : rb[v.offW + it_.w_off + lane];
        const T wp = wraw * pw;
        // h_i = sum_k P[i][k] gz_k: dX_i += w pw h_i, dW = pw sum_i x_i h_i.
        T sdot = T(0);
        T* gxr = dxp + it_.xp_off + lane * D1;
#pragma unroll
        for (int i = 0; i < D1; ++i) {
          T h = T(0);
#pragma unroll
          for (int k = 0; k < D3; ++k) h += P[i * D3 + k] * gz[k];
          gxr[i] += wp * h;
          sdot += x[i] * h;
        }
        if (a.shared_w)
          atomic_add(dwrow + it_.w_off + lane, sdot * pw);
        else
          dwrow[it_.w_off + lane] = sdot * pw;
        // dY_j += w pw sum_(i,k) c_ijk x_i gz_k, kept per lane until the row ends.
        T e[D2];
        CG<A, Bd, C>::evec(gz, x, e);
#pragma unroll
        for (int j = 0; j < D2; ++j) gyc[(it_.y_off + j) * 32 + lane] += wp * e[j];
      });
    }
    __syncthreads();
    const long long next = row + 2LL * gridDim.x;
    if (next < B) cw_load<T, true>(v, s, b, next, 1);
    // Fixed-order reductions over warps (and lanes for dY).
    const T* wbase = reinterpret_cast<const T*>(s.warps);
    T* gxrow = a.out0 + row * a.L1dim;
    if (v.chunk_mode) {
      // Warp w holds chunk (w % nch) of every X irrep at xirr.poff + (u % 32) * dim + i.
      const int nch = v.nch_all;
      for (int r = 0; r < v.nxirr; ++r) {
        const CwXIrrep xr = s.xirr[r];
        const int n = xr.nch * 32 * xr.dim;
        for (int e = threadIdx.x; e < n; e += blockDim.x) {
          const int c = e / (32 * xr.dim), q = e - c * 32 * xr.dim;
          T acc = T(0);
          for (int w = c; w < NW; w += nch)
            acc += wbase[static_cast<size_t>(w) * v.ws_elems + xr.poff + q];
          gxrow[xr.off + e] = acc;
        }
      }
    } else {
      for (int e = threadIdx.x; e < a.L1dim; e += blockDim.x) {
        T acc = T(0);
        for (int w = 0; w < NW; ++w) acc += wbase[static_cast<size_t>(w) * v.ws_elems + e];
        gxrow[e] = acc;
      }
    }
    T* gyrow = a.out1 + row * a.L2dim;
    for (int j = wid; j < a.L2dim; j += NW) {
      T acc = T(0);
      for (int w = 0; w < NW; ++w)
        acc += wbase[static_cast<size_t>(w) * v.ws_elems + v.dxn + j * 32 + lane];
      acc = group_sum(acc, 5);
      if (lane == 0) gyrow[j] = acc;
    }
    __syncthreads();
  }
}

}  // namespace oeqb
