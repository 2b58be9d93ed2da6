// Backward of shared-weight "uvw" tensor products (NequIP shape: every instruction
// 32 x 1 -> 32 channels, l <= 3, one weight matrix per instruction shared by all rows).
//
// With G_n[b, u, k] = sum_w W'_n[u, w] dZ[b, w, k] (W' = pw W, reference templates/
// loop_unroll_tp.cuh:184-216 uvw branch) the gradients are
//     dX[b, u, i] += sum_k P_n[b][i][k] G_n[b, u, k]             (P = sum_j C_ijk y_j)
//     dY[b, j]    += sum_(u, i, k) C_ijk X[b, u, i] G_n[b, u, k]
//     dW_n[u, w]  += pw sum_(b, k) T_n[b, u, k] dZ[b, w, k]      (T = sum_(i,j) C_ijk x_i y_j)
// The generic kernels add each row's dW with global atomics (one per weight per row); here
// the row-parallel gradients and the weight gradient are separate kernels:
//
//  * tp_uvw_sw_dxy: CTA = 32 rows x 8 channel groups of 4.  Per input irrep the thread keeps
//    its 4 x d1 dX values and x in registers; per instruction it forms G for its 4 channels
//    from 4 x 4 register blocks of W'^T (prepared once per call, [n][w][u]) and dZ, both
//    staged in shared memory by cp.async one instruction ahead, then adds hvec (dX) and evec
//    (dY) of the unrolled CG tables.  dY is folded over the 8 channel groups with shuffles and summed per row in
//    shared memory.  No atomics; every dX / dY element is written once.
//  * tp_uvw_sw_dw: split-K over row chunks.  CTA = 4 instructions (same l3) x 64 threads, each
//    thread a 4 x 4 (u, w) block of dW_n accumulated over the chunk's rows from shared-memory
//    tiles of T (computed per 8-row batch) and dZ; one atomic add per weight per CTA.
#pragma once

#include "tp_core.cuh"

namespace oeqb {

constexpr int kSwRows = 32;      // rows per tile (tp_uvw_sw_dxy)
constexpr int kSwThreads = 256;
constexpr int kSwYMax = 16;
constexpr int kSwBatch = 8;      // rows per shared-memory batch (tp_uvw_sw_dw)
constexpr int kSwDwSlots = 4;    // instructions per CTA (tp_uvw_sw_dw)

struct SwGroup {  // one input irrep and the instructions reading it
  int x_off, l1, ins_begin, ins_end;
};
struct SwIns {
  int l2, l3, y_off, z_off, wblk, pad0, pad1, pad2;
};
struct SwDw {  // weight-gradient instruction (ordered by l3)
  int l1, l2, l3, x_off, y_off, z_off, woff, pad;
  double pw;
};

template <class T>
struct ArgsSw {
  const T* X;
  const T* Y;
  const T* Wt;  // [nins][32 w][32 u], pw folded
  const T* dZ;
  T* dX;
  T* dY;
  T* dW;
  long long B;
  int L1dim, L2dim, L3dim;
  int ngroups, ndw;
  const SwGroup* groups;
  const SwIns* ins;
  const SwDw* dw;
  long long rows_per_chunk;  // tp_uvw_sw_dw
};

// Wt[n][w][u] = pw_n * W[woff_n + u * 32 + w] (oeq order of a 32 x 1 x 32 block).
template <class T>
__global__ void tp_uvw_sw_prep(const T* __restrict__ W, T* __restrict__ Wt,
                               const int* __restrict__ woff, const T* __restrict__ pw, int nins) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= nins * 1024) return;
  const int n = t >> 10, e = t & 1023, w = e >> 5, u = e & 31;
  Wt[t] = W[woff[n] + u * 32 + w] * pw[n];
}

// 4 consecutive values (16- or 32-byte aligned) into v[0..3].
template <class T>
__device__ __forceinline__ void ld4(T* v, const T* p) {
  if constexpr (sizeof(T) == 4) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = t.x;
    v[1] = t.y;
    v[2] = t.z;
    v[3] = t.w;
  } else {
    const double2 a = __ldg(reinterpret_cast<const double2*>(p));
    const double2 b = __ldg(reinterpret_cast<const double2*>(p) + 1);
    v[0] = a.x;
    v[1] = a.y;
    v[2] = b.x;
    v[3] = b.y;
  }
}

template <class T>
__device__ __forceinline__ void st4(T* p, const T* v) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  } else {
    reinterpret_cast<double2*>(p)[0] = make_double2(v[0], v[1]);
    reinterpret_cast<double2*>(p)[1] = make_double2(v[2], v[3]);
  }
}

// ------------------------------------------------------------------ dX and dY
//
// Per instruction the CTA's dZ tile (32 rows x the output block, 32 d3 values, row pitch
// padded by 4) and W'^T block (32 x 32) are copied into shared memory with cp.async, one
// instruction ahead of the compute (double buffer), so the FMA loop reads shared memory only.

constexpr int kSwZPitchMax = 32 * 7 + 4;

template <class T>
constexpr size_t sw_dxy_smem() {
  return sizeof(T) * (2 * static_cast<size_t>(kSwRows) * kSwZPitchMax + 2 * 1024 +
                      kSwRows * (kSwYMax + 1));
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(static_cast<unsigned>(__cvta_generic_to_shared(dst))), "l"(src),
               "r"(pred ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Issues the copies of instruction `in` into buffer b: dZ rows (invalid rows zero-filled) and
// the W'^T block.
template <class T>
__device__ __forceinline__ void sw_dxy_prefetch(const ArgsSw<T>& a, const SwIns& in,
                                                long long row0, T* zbuf, T* wbuf) {
  constexpr int V = 16 / sizeof(T);
  const int d3 = 2 * in.l3 + 1;
  const int pitch = 32 * d3 + 4;
  const int per_row = 32 * d3 / V;  // 16-byte granules per row
  for (int q = threadIdx.x; q < kSwRows * per_row; q += kSwThreads) {
    const int rr = q / per_row, e = q - rr * per_row;
    const long long row = row0 + rr;
    const bool ok = row < a.B;
    const T* src = a.dZ + (ok ? row : 0) * a.L3dim + in.z_off + e * V;
    cp_async16(zbuf + rr * pitch + e * V, src, ok);
  }
  const T* wsrc = a.Wt + static_cast<size_t>(in.wblk) * 1024;
  for (int q = threadIdx.x; q < 1024 / V; q += kSwThreads) cp_async16(wbuf + q * V, wsrc + q * V, true);
}

template <class T, int L1, int L2, int L3>
__device__ __forceinline__ void sw_dxy_ins(const ArgsSw<T>& a, const SwIns& in, long long row,
                                           bool valid, int g, int r, const T (&x)[4][2 * L1 + 1],
                                           T (&dx)[4][2 * L1 + 1], T* dys_row, const T* zbuf,
                                           const T* wbuf) {
  constexpr int D1 = 2 * L1 + 1, D2 = 2 * L2 + 1, D3 = 2 * L3 + 1;
  constexpr int PITCH = 32 * D3 + 4;
  T G[4][D3];
#pragma unroll
  for (int uu = 0; uu < 4; ++uu)
#pragma unroll
    for (int k = 0; k < D3; ++k) G[uu][k] = T(0);
  const T* zrow = zbuf + r * PITCH;
  const T* wt = wbuf + 4 * g;
#pragma unroll 2
  for (int w0 = 0; w0 < 32; w0 += 4) {
    T z[4 * D3];
#pragma unroll
    for (int e = 0; e < D3; ++e) {
      if constexpr (sizeof(T) == 4) {
        const float4 t = *reinterpret_cast<const float4*>(zrow + w0 * D3 + 4 * e);
        z[4 * e] = t.x;
        z[4 * e + 1] = t.y;
        z[4 * e + 2] = t.z;
        z[4 * e + 3] = t.w;
      } else {
        const double2 t0 = *reinterpret_cast<const double2*>(zrow + w0 * D3 + 4 * e);
        const double2 t1 = *reinterpret_cast<const double2*>(zrow + w0 * D3 + 4 * e + 2);
        z[4 * e] = t0.x;
        z[4 * e + 1] = t0.y;
        z[4 * e + 2] = t1.x;
        z[4 * e + 3] = t1.y;
      }
    }
#pragma unroll
    for (int ww = 0; ww < 4; ++ww) {
      T wv[4];
      if constexpr (sizeof(T) == 4) {
        const float4 t = *reinterpret_cast<const float4*>(wt + (w0 + ww) * 32);
        wv[0] = t.x;
        wv[1] = t.y;
        wv[2] = t.z;
        wv[3] = t.w;
      } else {
        const double2 t0 = *reinterpret_cast<const double2*>(wt + (w0 + ww) * 32);
        const double2 t1 = *reinterpret_cast<const double2*>(wt + (w0 + ww) * 32 + 2);
        wv[0] = t0.x;
        wv[1] = t0.y;
        wv[2] = t1.x;
        wv[3] = t1.y;
      }
#pragma unroll
      for (int uu = 0; uu < 4; ++uu)
#pragma unroll
        for (int k = 0; k < D3; ++k) G[uu][k] = fma(wv[uu], z[ww * D3 + k], G[uu][k]);
    }
  }
  T y[D2];
  const T* yrow = a.Y + row * a.L2dim + in.y_off;
#pragma unroll
  for (int j = 0; j < D2; ++j) y[j] = valid ? yrow[j] : T(0);
  T es[D2];
#pragma unroll
  for (int j = 0; j < D2; ++j) es[j] = T(0);
#pragma unroll
  for (int uu = 0; uu < 4; ++uu) {
    T h[D1], e[D2];
    CG<L1, L2, L3>::hvec(G[uu], y, h);
    CG<L1, L2, L3>::evec(G[uu], x[uu], e);
#pragma unroll
    for (int i = 0; i < D1; ++i) dx[uu][i] += h[i];
#pragma unroll
    for (int j = 0; j < D2; ++j) es[j] += e[j];
  }
  // Sum over the 8 channel groups of this row (lanes g, g ^ 1, ..., within 8 lanes).
#pragma unroll
  for (int j = 0; j < D2; ++j) {
    T v = es[j];
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    es[j] = v;
  }
  if (g == 0) {
#pragma unroll
    for (int j = 0; j < D2; ++j) dys_row[in.y_off + j] += es[j];
  }
}

template <class T>
__global__ void __launch_bounds__(kSwThreads) tp_uvw_sw_dxy(const ArgsSw<T> a) {
  extern __shared__ __align__(16) unsigned char sw_dxy_raw[];
  T* zb = reinterpret_cast<T*>(sw_dxy_raw);                    // [2][32][pitch]
  T* wb = zb + 2 * kSwRows * kSwZPitchMax;                     // [2][1024]
  T* dys = wb + 2 * 1024;                                      // [32][kSwYMax + 1]
  const int g = threadIdx.x & 7, r = threadIdx.x >> 3;
  const long long ntiles = (a.B + kSwRows - 1) / kSwRows;
  const int nins = a.ngroups > 0 ? a.groups[a.ngroups - 1].ins_end : 0;
  for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const long long row0 = tile * kSwRows;
    for (int i = threadIdx.x; i < kSwRows * (kSwYMax + 1); i += blockDim.x) dys[i] = T(0);
    if (nins > 0) sw_dxy_prefetch(a, a.ins[0], row0, zb, wb);
    cp_async_commit();
    const long long row = row0 + r;
    const bool valid = row < a.B;
    int ni = 0;  // running instruction index (buffer ni & 1)
    for (int gi = 0; gi < a.ngroups; ++gi) {
      const SwGroup gp = a.groups[gi];
      dispatch_l(gp.l1, [&]<int L1>() {
        constexpr int D1 = 2 * L1 + 1;
        T x[4][D1], dx[4][D1];
        const T* xp = a.X + row * a.L1dim + gp.x_off + 4 * g * D1;
#pragma unroll
        for (int uu = 0; uu < 4; ++uu)
#pragma unroll
          for (int i = 0; i < D1; ++i) {
            x[uu][i] = valid ? xp[uu * D1 + i] : T(0);
            dx[uu][i] = T(0);
          }
        for (; ni < gp.ins_end; ++ni) {
          const int b = ni & 1;
          if (ni + 1 < nins)
            sw_dxy_prefetch(a, a.ins[ni + 1], row0, zb + (b ^ 1) * kSwRows * kSwZPitchMax,
                            wb + (b ^ 1) * 1024);
          cp_async_commit();
          cp_async_wait<1>();
          __syncthreads();
          const SwIns in = a.ins[ni];
          dispatch_bc<L1>(pair_code(in.l2, in.l3), [&]<int L2, int L3>() {
            sw_dxy_ins<T, L1, L2, L3>(a, in, row, valid, g, r, x, dx, dys + r * (kSwYMax + 1),
                                      zb + b * kSwRows * kSwZPitchMax, wb + b * 1024);
          });
          __syncthreads();  // buffer b is refilled by the prefetch two instructions on
        }
        if (valid) {
          T* dp = a.dX + row * a.L1dim + gp.x_off + 4 * g * D1;
#pragma unroll
          for (int uu = 0; uu < 4; ++uu)
#pragma unroll
            for (int i = 0; i < D1; ++i) dp[uu * D1 + i] = dx[uu][i];
        }
      });
    }
    cp_async_wait<0>();
    __syncthreads();
    const long long left = a.B - row0;
    const int nr = left < kSwRows ? static_cast<int>(left) : kSwRows;
    for (int i = threadIdx.x; i < nr * a.L2dim; i += blockDim.x) {
      const int rr = i / a.L2dim, j = i - rr * a.L2dim;
      a.dY[(row0 + rr) * a.L2dim + j] = dys[rr * (kSwYMax + 1) + j];
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ forward (CUDA cores)
//
// Used for float64 (float32 runs on the tensor cores, tp_kernels_uvw_tc.cuh).  CTA = 32 rows x
// 8 groups of 4 output channels.  Per output irrep the thread accumulates Z[w][k] for its 4
// channels over the paths into it: per path the CTA computes T[u][k] = pw sum_i P[i][k] x[u][i]
// for its rows into shared memory (each thread 4 channels u), the path's 32 x 32 weight block
// is staged by cp.async (one path ahead), then Z[w][k] += sum_u W[u][w] T[u][k].

struct SwOut {  // one output irrep and the paths into it
  int z_off, l3, ins_begin, ins_end;
};
struct SwFIns {
  int l1, l2, x_off, y_off, woff, pad0, pad1, pad2;
  double pw;
};

constexpr int kSwTPitch = 32 * 7 + 1;  // T tile row pitch (odd: conflict-free row reads)

template <class T>
__host__ __device__ constexpr size_t sw_fwd_smem() {
  return sizeof(T) * (static_cast<size_t>(kSwRows) * kSwTPitch + 2 * 1024);
}

template <class T>
struct ArgsSwF {
  const T* X;
  const T* Y;
  const T* W;
  T* Z;
  long long B;
  int L1dim, L2dim, L3dim, nout;
  const SwOut* outs;
  const SwFIns* ins;
};

template <class T, int L1, int L2, int L3>
__device__ __forceinline__ void sw_fwd_t(const ArgsSwF<T>& a, const SwFIns& in, long long row,
                                         bool valid, int g, int r, T* ts) {
  constexpr int D1 = 2 * L1 + 1, D2 = 2 * L2 + 1, D3 = 2 * L3 + 1;
  T P[D1 * D3];
#pragma unroll
  for (int e = 0; e < D1 * D3; ++e) P[e] = T(0);
  T x[4][D1];
  if (valid) {
    T y[D2];
    const T* yrow = a.Y + row * a.L2dim + in.y_off;
#pragma unroll
    for (int j = 0; j < D2; ++j) y[j] = yrow[j] * T(in.pw);
    CG<L1, L2, L3>::pmat(y, P);
    const T* xp = a.X + row * a.L1dim + in.x_off + 4 * g * D1;
#pragma unroll
    for (int uu = 0; uu < 4; ++uu)
#pragma unroll
      for (int i = 0; i < D1; ++i) x[uu][i] = xp[uu * D1 + i];
  } else {
#pragma unroll
    for (int uu = 0; uu < 4; ++uu)
#pragma unroll
      for (int i = 0; i < D1; ++i) x[uu][i] = T(0);
  }
  T* tr = ts + r * kSwTPitch + 4 * g * D3;
#pragma unroll
  for (int uu = 0; uu < 4; ++uu)
#pragma unroll
    for (int k = 0; k < D3; ++k) {
      T t = T(0);
#pragma unroll
      for (int i = 0; i < D1; ++i) t = fma(P[i * D3 + k], x[uu][i], t);
      tr[uu * D3 + k] = t;
    }
}

template <class T, int L3>
__device__ __forceinline__ void sw_fwd_acc(const T* ts, const T* wb, int g, int r,
                                           T (&z)[4][2 * L3 + 1]) {
  constexpr int D3 = 2 * L3 + 1;
  const T* tr = ts + r * kSwTPitch;
#pragma unroll 4
  for (int u = 0; u < 32; ++u) {
    T t[D3], wv[4];
#pragma unroll
    for (int k = 0; k < D3; ++k) t[k] = tr[u * D3 + k];
    if constexpr (sizeof(T) == 4) {
      const float4 q = *reinterpret_cast<const float4*>(wb + u * 32 + 4 * g);
      wv[0] = q.x;
      wv[1] = q.y;
      wv[2] = q.z;
      wv[3] = q.w;
    } else {
      const double2 q0 = *reinterpret_cast<const double2*>(wb + u * 32 + 4 * g);
      const double2 q1 = *reinterpret_cast<const double2*>(wb + u * 32 + 4 * g + 2);
      wv[0] = q0.x;
      wv[1] = q0.y;
      wv[2] = q1.x;
      wv[3] = q1.y;
    }
#pragma unroll
    for (int ww = 0; ww < 4; ++ww)
#pragma unroll
      for (int k = 0; k < D3; ++k) z[ww][k] = fma(wv[ww], t[k], z[ww][k]);
  }
}

template <class T>
__device__ __forceinline__ void sw_fwd_prefetch_w(const ArgsSwF<T>& a, const SwFIns& in, T* wbuf) {
  constexpr int V = 16 / sizeof(T);
  for (int q = threadIdx.x; q < 1024 / V; q += kSwThreads) cp_async16(wbuf + q * V, a.W + in.woff + q * V, true);
}

template <class T>
__global__ void __launch_bounds__(kSwThreads) tp_uvw_sw_fwd(const ArgsSwF<T> a) {
  extern __shared__ __align__(16) unsigned char sw_fwd_raw[];
  T* ts = reinterpret_cast<T*>(sw_fwd_raw);  // [32 rows][pitch]
  T* wb = ts + kSwRows * kSwTPitch;           // [2][1024]
  const int g = threadIdx.x & 7, r = threadIdx.x >> 3;
  const long long ntiles = (a.B + kSwRows - 1) / kSwRows;
  const int nins = a.nout > 0 ? a.outs[a.nout - 1].ins_end : 0;
  for (long long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const long long row = tile * kSwRows + r;
    const bool valid = row < a.B;
    if (nins > 0) sw_fwd_prefetch_w(a, a.ins[0], wb);
    cp_async_commit();
    int ni = 0;
    for (int oi = 0; oi < a.nout; ++oi) {
      const SwOut o = a.outs[oi];
      dispatch_l(o.l3, [&]<int L3>() {
        constexpr int D3 = 2 * L3 + 1;
        T z[4][D3];
#pragma unroll
        for (int ww = 0; ww < 4; ++ww)
#pragma unroll
          for (int k = 0; k < D3; ++k) z[ww][k] = T(0);
        for (; ni < o.ins_end; ++ni) {
          const int b = ni & 1;
          const SwFIns in = a.ins[ni];
          dispatch_l(in.l1, [&]<int L1>() {
            dispatch_bc<L1>(pair_code(in.l2, L3), [&]<int L2, int C>() {
              if constexpr (C == L3) sw_fwd_t<T, L1, L2, L3>(a, in, row, valid, g, r, ts);
            });
          });
          if (ni + 1 < nins) sw_fwd_prefetch_w(a, a.ins[ni + 1], wb + (b ^ 1) * 1024);
          cp_async_commit();
          cp_async_wait<1>();
          __syncthreads();
          sw_fwd_acc<T, L3>(ts, wb + b * 1024, g, r, z);
          __syncthreads();
        }
        if (valid) {
          T* zp = a.Z + row * a.L3dim + o.z_off + 4 * g * D3;
#pragma unroll
          for (int ww = 0; ww < 4; ++ww)
#pragma unroll
            for (int k = 0; k < D3; ++k) zp[ww * D3 + k] = z[ww][k];
        }
      });
    }
    cp_async_wait<0>();
    __syncthreads();
  }
}

// ------------------------------------------------------------------ dW

template <class T, int L1, int L2, int L3>
__device__ __forceinline__ void sw_dw_fill(const ArgsSw<T>& a, const SwDw& d, long long row,
                                           bool valid, int t, T* ts, T* zs) {
  constexpr int D1 = 2 * L1 + 1, D2 = 2 * L2 + 1, D3 = 2 * L3 + 1;
  const int b = t >> 3, c4 = 4 * (t & 7);  // batch row, first channel (u for T, w for dZ)
  T tv[4][D3], zv[4 * D3];
#pragma unroll
  for (int uu = 0; uu < 4; ++uu)
#pragma unroll
    for (int k = 0; k < D3; ++k) tv[uu][k] = T(0);
#pragma unroll
  for (int e = 0; e < 4 * D3; ++e) zv[e] = T(0);
  if (valid) {
    T y[D2];
    const T* yrow = a.Y + row * a.L2dim + d.y_off;
#pragma unroll
    for (int j = 0; j < D2; ++j) y[j] = yrow[j];
    const T* xp = a.X + row * a.L1dim + d.x_off + c4 * D1;
#pragma unroll
    for (int uu = 0; uu < 4; ++uu) {
      T x[D1];
#pragma unroll
      for (int i = 0; i < D1; ++i) x[i] = xp[uu * D1 + i];
      CG<L1, L2, L3>::fwd(x, y, tv[uu]);
    }
    const T* zp = a.dZ + row * a.L3dim + d.z_off + c4 * D3;
#pragma unroll
    for (int e = 0; e < D3; ++e) ld4(zv + 4 * e, zp + 4 * e);
  }
  // ts / zs: [batch row][k][32 channels]
#pragma unroll
  for (int k = 0; k < D3; ++k) {
    T tt[4] = {tv[0][k], tv[1][k], tv[2][k], tv[3][k]};
    T zz[4] = {zv[k], zv[D3 + k], zv[2 * D3 + k], zv[3 * D3 + k]};
    st4(ts + (b * 7 + k) * 32 + c4, tt);
    st4(zs + (b * 7 + k) * 32 + c4, zz);
  }
}

// Dynamic shared memory of tp_uvw_sw_dw: T and dZ tiles [slot][batch row][k (<= 7)][32].
constexpr int kSwDwTile = kSwBatch * 7 * 32;
template <class T>
constexpr size_t sw_dw_smem() {
  return sizeof(T) * 2 * kSwDwSlots * kSwDwTile;
}

template <class T>
__global__ void __launch_bounds__(kSwThreads) tp_uvw_sw_dw(const ArgsSw<T> a) {
  extern __shared__ __align__(16) unsigned char sw_smem[];
  T* tsm = reinterpret_cast<T*>(sw_smem);
  T* zsm = tsm + kSwDwSlots * kSwDwTile;
  const int slot = threadIdx.x >> 6, t = threadIdx.x & 63;
  const int n = blockIdx.x * kSwDwSlots + slot;
  const bool active = n < a.ndw;
  SwDw d{};
  if (active) d = a.dw[n];
  const int d3 = 2 * d.l3 + 1;
  const int u0 = 4 * (t >> 3), w0 = 4 * (t & 7);
  T acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = T(0);
  const long long r0 = blockIdx.y * a.rows_per_chunk;
  const long long r1 = a.B < r0 + a.rows_per_chunk ? a.B : r0 + a.rows_per_chunk;
  T* ts = tsm + slot * kSwDwTile;
  T* zs = zsm + slot * kSwDwTile;
  for (long long rb = r0; rb < r1; rb += kSwBatch) {
    if (active) {
      const long long row = rb + (t >> 3);
      const bool valid = row < r1;
      dispatch_l(d.l1, [&]<int L1>() {
        dispatch_bc<L1>(pair_code(d.l2, d.l3), [&]<int L2, int L3>() {
          sw_dw_fill<T, L1, L2, L3>(a, d, row, valid, t, ts, zs);
        });
      });
    }
    __syncthreads();
    if (active) {
      for (int b = 0; b < kSwBatch; ++b)
        for (int k = 0; k < d3; ++k) {
          T tv[4], zv[4];
          const T* tp = ts + (b * 7 + k) * 32;
          const T* zp = zs + (b * 7 + k) * 32;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            tv[i] = tp[u0 + i];
            zv[i] = zp[w0 + i];
          }
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = fma(tv[i], zv[j], acc[i][j]);
        }
    }
    __syncthreads();
  }
  if (active) {
    const T pw = T(d.pw);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) atomicAdd(a.dW + d.woff + (u0 + i) * 32 + (w0 + j), acc[i][j] * pw);
  }
}

}  // namespace oeqb
