// Row-staged batch kernels for uvu problems with wide multiplicities (sm_100a).
//
// One CTA processes one batch row at a time.  The whole row -- X | Y | W (and dZ for the
// backward pass) -- is brought into shared memory by TMA bulk copies
// (cp.async.bulk ... mbarrier::complete_tx) into one of two row buffers, so the next row
// streams in while the current one is computed.  The row's work is split into items
// (forward: output irrep x chunk range; backward: instruction x chunk range) that are
// assigned to warps once per launch with a longest-processing-time schedule; every row
// reuses the same assignment.  The CG contractions read shared memory only.
//
// Forward: each warp stages a 32-lane output chunk per item and writes it with a bulk
// store (cp.async.bulk.global.shared::cta), double-buffered per warp.
// Backward: each warp accumulates dX and dY into private shared-memory partial rows; after
// a CTA barrier the partials are summed in fixed warp order, so dX/dY are bitwise
// reproducible.  dW is written directly (or atomically added when weights are shared).
// Each backward degree triple is a separate noinline function (one call per item), which
// keeps register allocation per triple instead of the union over all triples.
//
// Every mbarrier wait is bounded; on expiry the kernel raises the plan's status flag and
// continues (results are then invalid, but the GPU is never left spinning).
#pragma once

#include "tp_core.cuh"

namespace oeqb {

struct RowItem {
  int key;    // forward: group index; backward: instruction index
  int c0;     // first 32-lane chunk
  int nc;     // number of chunks
  int pad;
};

template <class T>
struct ArgsRow {
  Args<T> a;
  const RowItem* items;
  const int* witems;   // item indices, warp-major
  const int* wofs;     // [nwarps + 1] offsets into witems
  int nitems, nwitems;
  int nwarps;
  int offY, offW, offG, row_elems;  // row-buffer layout (elements of T), 16-byte aligned
  int use_tma;                      // 1: bulk copies; 0: cooperative loads
  int off_stage, off_dxp, off_dyp, ws_elems;  // per-warp scratch layout
};

// Bounded barrier waits: a wait gives up after kWaitNs of device time (never reached in
// normal operation, where a wait lasts microseconds) and raises status flag 3.  Once the flag
// is 3, later waits give up at once, so a kernel whose pipeline lost a phase runs to its end
// in milliseconds instead of timing out wait by wait.
constexpr unsigned long long kWaitNs = 2000000000ull;

__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(unsigned long long* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(unsigned long long* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(unsigned long long* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(unsigned long long* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}

// Bounded wait: returns false (and raises the status flag) if the phase never completes.
__device__ __forceinline__ bool mbar_wait(unsigned long long* bar, unsigned parity, int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (;;) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (status && *reinterpret_cast<volatile int*>(status) == 3) return false;
    if (global_ns() - t0 > kWaitNs) {
      if (status) atomicCAS(status, 0, 3);
      return false;
    }
  }
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes,
                                         unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, unsigned bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n" ::"l"(dst),
               "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;\n" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;\n" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group %0;\n" ::"n"(N) : "memory");
}

struct SmemRow {
  SmemDesc d;
  RowItem* items;
  int* witems;
  int* wofs;
  unsigned long long* bars;  // [2]
  unsigned char* rowbuf;     // 2 row buffers
  unsigned char* warps;      // per-warp scratch
};

template <class T>
__device__ __forceinline__ SmemRow stage_desc_row(const ArgsRow<T>& v, unsigned char* sm) {
  SmemRow s;
  s.d = stage_desc(v.a, sm);
  unsigned char* p = s.d.end;
  s.items = reinterpret_cast<RowItem*>(p);
  p += sizeof(RowItem) * v.nitems;
  s.witems = reinterpret_cast<int*>(p);
  p += sizeof(int) * v.nwitems;
  s.wofs = reinterpret_cast<int*>(p);
  p += sizeof(int) * (v.nwarps + 1);
  p = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t(15));
  s.bars = reinterpret_cast<unsigned long long*>(p);
  p += 16;
  s.rowbuf = p;
  p += 2 * sizeof(T) * static_cast<size_t>(v.row_elems);
  s.warps = p;
  auto copy = [&](void* dst, const void* src, int bytes) {
    const int* a = reinterpret_cast<const int*>(src);
    int* t = reinterpret_cast<int*>(dst);
    for (int i = threadIdx.x; i < bytes / 4; i += blockDim.x) t[i] = a[i];
  };
  copy(s.items, v.items, sizeof(RowItem) * v.nitems);
  copy(s.witems, v.witems, sizeof(int) * v.nwitems);
  copy(s.wofs, v.wofs, sizeof(int) * (v.nwarps + 1));
  if (threadIdx.x == 0) {
    mbar_init(&s.bars[0], 1);
    mbar_init(&s.bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  return s;
}

// Starts loading row `row` into buffer b (thread 0 only for TMA; all threads otherwise,
// synchronously, followed by the caller's barrier).
template <class T, bool BWD>
__device__ __forceinline__ void load_row(const ArgsRow<T>& v, const SmemRow& s, int b,
                                         long long row) {
  const Args<T>& a = v.a;
  T* buf = reinterpret_cast<T*>(s.rowbuf) + static_cast<size_t>(b) * v.row_elems;
  const T* srcs[4] = {a.X + row * a.L1dim, a.Y + row * a.L2dim,
                      a.shared_w ? nullptr : a.W + row * a.wnumel,
                      BWD ? a.Gz + row * a.L3dim : nullptr};
  const int lens[4] = {a.L1dim, a.L2dim, a.shared_w ? 0 : a.wnumel, BWD ? a.L3dim : 0};
  const int offs[4] = {0, v.offY, v.offW, v.offG};
  if (v.use_tma) {
    if (threadIdx.x == 0) {
      unsigned bytes = 0;
      for (int q = 0; q < 4; ++q) bytes += lens[q] * sizeof(T);
      mbar_expect_tx(&s.bars[b], bytes);
      for (int q = 0; q < 4; ++q)
        if (lens[q]) bulk_g2s(buf + offs[q], srcs[q], lens[q] * sizeof(T), &s.bars[b]);
    }
  } else {
    for (int q = 0; q < 4; ++q)
      for (int e = threadIdx.x; e < lens[q]; e += blockDim.x) buf[offs[q] + e] = srcs[q][e];
  }
}

// Writes one staged chunk (ul lanes of irrep r, chunk start c0) into a global row.
template <class T>
__device__ __forceinline__ void put_chunk(T* grow, const IrrepD& r, int c0, int ul, T* stage,
                                          int lane, bool bulk_ok) {
  if (r.si == 1) {
    T* dst = grow + r.off + c0 * r.dim;
    const unsigned bytes = ul * r.dim * sizeof(T);
    if (bulk_ok && ((reinterpret_cast<uintptr_t>(dst) | bytes) & 15) == 0) {
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        bulk_s2g(dst, stage, bytes);
        bulk_commit();
      }
      return;
    }
    __syncwarp();
    for (int e = lane; e < ul * r.dim; e += 32) dst[e] = stage[e];
  } else {
    __syncwarp();
    for (int k = 0; k < r.dim; ++k)
      if (lane < ul) grow[r.off + k * r.si + c0 + lane] = stage[k * ul + lane];
  }
}

// ---------------------------------------------------------------------------------------

template <class T, int NW>
__global__ void __launch_bounds__(NW * 32, (NW == 8 ? 2 : 1)) tp_fwd_row(const ArgsRow<T> v) {
  extern __shared__ __align__(16) unsigned char smem[];
  const SmemRow s = stage_desc_row(v, smem);
  const Args<T>& a = v.a;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  T* stage0 = reinterpret_cast<T*>(s.warps) + static_cast<size_t>(wid) * v.ws_elems + v.off_stage;
  int sb = 0;  // per-warp stage buffer toggle (2 x 32*kDMax)
  const long long B = a.nitems;
  if (blockIdx.x < B) load_row<T, false>(v, s, 0, blockIdx.x);
  if (blockIdx.x + gridDim.x < B) load_row<T, false>(v, s, 1, blockIdx.x + gridDim.x);
  if (!v.use_tma) __syncthreads();
  const T* Ws = a.shared_w ? a.W : nullptr;
  int it = 0;
  for (long long row = blockIdx.x; row < B; row += gridDim.x, ++it) {
    const int b = it & 1;
    if (v.use_tma) mbar_wait(&s.bars[b], (it >> 1) & 1, a.status);
    const T* buf = reinterpret_cast<const T*>(s.rowbuf) + static_cast<size_t>(b) * v.row_elems;
    RowPtrs<T> rp;
    rp.x = buf;
    rp.y = buf + v.offY;
    const T* wrow = a.shared_w ? Ws : buf + v.offW;
    T* zrow = a.out0 + row * a.L3dim;
    for (int wi = s.wofs[wid]; wi < s.wofs[wid + 1]; ++wi) {
      const RowItem item = s.items[s.witems[wi]];
      const GroupD gd = s.d.grp[item.key];
      const IrrepD r3 = s.d.ir3[gd.irrep];
      dispatch_l(r3.l, [&]<int L3>() {
        constexpr int D3 = 2 * L3 + 1;
        for (int c = item.c0; c < item.c0 + item.nc; ++c) {
          const int c0 = c * 32;
          const int ul = min(32, r3.mul - c0);
          const int u = c0 + lane;
          const bool act = u < r3.mul;
          T z[D3];
          zero(z);
          if (act) {
            for (int ii = gd.first; ii < gd.first + gd.count; ++ii) {
              const InstrD& in = s.d.ins[ii];
              const IrrepD r1 = s.d.ir1[in.i1];
              const IrrepD r2 = s.d.ir2[in.i2];
              dispatch_triple(in.code, [&]<int A, int Bd, int C>() {
                if constexpr (C == L3)
                  uvu_fwd<T, A, Bd, C, false>(in, r1, r2, rp, wrow + in.woff + c0 * in.m2, u, z);
              });
            }
          }
          T* stage = stage0 + sb * (32 * kDMax);
          sb ^= 1;
          if (lane == 0) bulk_wait_read<1>();  // the store issued 2 chunks ago has read its buffer
          __syncwarp();
          if (act) {
#pragma unroll
            for (int kk = 0; kk < D3; ++kk) stage[stage_index(r3, ul, lane, kk)] = z[kk];
          }
          put_chunk(zrow, r3, c0, ul, stage, lane, true);
        }
      });
    }
    if (wid == 0) {
      for (int zb = 0; zb < a.nzero; ++zb) {
        const IrrepD r3 = s.d.ir3[s.d.zb[zb]];
        for (int e = lane; e < r3.mul * r3.dim; e += 32) zrow[block_addr(r3, 0, r3.mul, e)] = T(0);
      }
    }
    __syncthreads();  // every warp is done with buffer b
    const long long next = row + 2LL * gridDim.x;
    if (next < B) load_row<T, false>(v, s, b, next);
    if (!v.use_tma) __syncthreads();
  }
  if (lane == 0) bulk_wait_all<0>();
}

// One backward item (instruction x chunk range) of one row, per degree triple.
template <class T, int A, int B, int C>
__device__ __noinline__ void row_bwd_item(const InstrD in, const IrrepD r1, const IrrepD r2,
                                          const IrrepD r3, const T* xs, const T* ys, const T* ws,
                                          const T* gs, int c_begin, int c_end, T* dxp, T* dyp,
                                          T* dw, bool shared_w, int lane) {
  constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1, D3 = 2 * C + 1;
  const T pw = T(in.pw);
  for (int v = 0; v < in.m2; ++v) {
    T y[D2];
    ldv(y, ys, r2, v);
    T gy[D2];
    zero(gy);
    for (int c = c_begin; c < c_end; ++c) {
      const int u = c * 32 + lane;
      if (u < in.m1) {
        const int u0 = c * 32, ul = min(32, in.m1 - u0);
        T x[D1], gz[D3];
        ldv(x, xs, r1, u);
        ldv(gz, gs, r3, u);
        const int wi = in.woff + u0 * in.m2 + v * ul + (u - u0);
        const T wp = ws[wi] * pw;
        T h[D1];
        CG<A, B, C>::hvec(gz, y, h);
        T sdot = T(0);
        T* gxr = dxp + r1.off + u * r1.su;
#pragma unroll
        for (int i = 0; i < D1; ++i) {
          gxr[i * r1.si] += wp * h[i];
          sdot += x[i] * h[i];
        }
        if (shared_w)
          atomic_add(dw + wi, sdot * pw);
        else
          dw[wi] = sdot * pw;
        T e[D2];
        CG<A, B, C>::evec(gz, x, e);
#pragma unroll
        for (int j = 0; j < D2; ++j) gy[j] += wp * e[j];
      }
    }
#pragma unroll
    for (int j = 0; j < D2; ++j) {
      const T t = group_sum(gy[j], 5);
      if (lane == 0) dyp[r2.off + v * r2.su + j * r2.si] += t;
    }
  }
}

template <class T, int NW>
__global__ void __launch_bounds__(NW * 32, (NW == 8 ? 2 : 1)) tp_bwd_row(const ArgsRow<T> v) {
  extern __shared__ __align__(16) unsigned char smem[];
  const SmemRow s = stage_desc_row(v, smem);
  const Args<T>& a = v.a;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  T* wsp = reinterpret_cast<T*>(s.warps) + static_cast<size_t>(wid) * v.ws_elems;
  T* dxp = wsp + v.off_dxp;
  T* dyp = wsp + v.off_dyp;
  const long long B = a.nitems;
  if (blockIdx.x < B) load_row<T, true>(v, s, 0, blockIdx.x);
  if (blockIdx.x + gridDim.x < B) load_row<T, true>(v, s, 1, blockIdx.x + gridDim.x);
  if (!v.use_tma) __syncthreads();
  int it = 0;
  for (long long row = blockIdx.x; row < B; row += gridDim.x, ++it) {
    const int b = it & 1;
    for (int e = lane; e < a.L1dim; e += 32) dxp[e] = T(0);
    for (int e = lane; e < a.L2dim; e += 32) dyp[e] = T(0);
    if (v.use_tma) mbar_wait(&s.bars[b], (it >> 1) & 1, a.status);
    __syncwarp();
    const T* buf = reinterpret_cast<const T*>(s.rowbuf) + static_cast<size_t>(b) * v.row_elems;
    const T* xs = buf;
    const T* ys = buf + v.offY;
    const T* ws = a.shared_w ? a.W : buf + v.offW;
    const T* gs = buf + v.offG;
    T* dwrow = a.shared_w ? a.out2 : a.out2 + row * a.wnumel;
    for (int wi = s.wofs[wid]; wi < s.wofs[wid + 1]; ++wi) {
      const RowItem item = s.items[s.witems[wi]];
      const InstrD& in = s.d.ins[item.key];
      const IrrepD r1 = s.d.ir1[in.i1];
      const IrrepD r2 = s.d.ir2[in.i2];
      const IrrepD r3 = s.d.ir3[in.i3];
      dispatch_triple(in.code, [&]<int A, int Bd, int C>() {
        row_bwd_item<T, A, Bd, C>(in, r1, r2, r3, xs, ys, ws, gs, item.c0, item.c0 + item.nc,
                                  dxp, dyp, dwrow, a.shared_w != 0, lane);
      });
      __syncwarp();
    }
    __syncthreads();  // partials complete; every warp is done with buffer b
    const long long next = row + 2LL * gridDim.x;
    if (next < B) load_row<T, true>(v, s, b, next);
    // Sum the per-warp partials in fixed warp order (bitwise reproducible).
    const T* wbase = reinterpret_cast<const T*>(s.warps);
    T* gxrow = a.out0 + row * a.L1dim;
    for (int e = threadIdx.x; e < a.L1dim; e += blockDim.x) {
      T acc = T(0);
      for (int w = 0; w < NW; ++w) acc += wbase[static_cast<size_t>(w) * v.ws_elems + v.off_dxp + e];
      gxrow[e] = acc;
    }
    T* gyrow = a.out1 + row * a.L2dim;
    for (int e = threadIdx.x; e < a.L2dim; e += blockDim.x) {
      T acc = T(0);
      for (int w = 0; w < NW; ++w) acc += wbase[static_cast<size_t>(w) * v.ws_elems + v.off_dyp + e];
      gyrow[e] = acc;
    }
    __syncthreads();  // partials consumed before the next row zeroes them
  }
}

}  // namespace oeqb
