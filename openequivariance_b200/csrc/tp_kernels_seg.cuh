// Channelwise-uvu batch kernels: the MACE / NequIP interaction class (BASELINE C2).
//
// Eligible problems: uvu, mul_ir layout, one copy of each instruction's Y irrep (m2 == 1),
// multiplicities that are multiples of 32, one instruction per output irrep, degrees in the
// unrolled range.  Reference semantics: templates/loop_unroll_tp.cuh (uvu branch) with the
// weight order of ComputationSchedule.py:653-714 (for m2 == 1 the weight of channel u of an
// instruction sits at weight_offset + u).
//
// Per row the Y operand is shared by every channel, so each instruction's contraction with
// Y is a small dense matrix
//     P[i][k] = pw * sum_j c_ijk y_j                       (D1 x D3, path weight folded in)
// computed once per row by the whole CTA from a term table (no per-channel recomputation).
// Then for channel u:
//     forward   z[u][k] = w[u] * sum_i x[u][i] P[i][k]
//     backward  h_i = sum_k P[i][k] gz[u][k];  dX[u][i] += w[u] h_i;  dW[u] = sum_i x[u][i] h_i
//               dY[j] += w[u] pw sum_(i,k) c_ijk x[u][i] gz[u][k]      (unrolled CG, per lane)
// Instructions are sorted by X irrep and cut into contiguous groups of similar cost.  A warp
// owns a unit (row, group, chunk block): for each instruction of its group it handles up to
// CPL 32-channel chunks at once (lane = channel within the chunk), so the instruction's
// dispatch, P load and output store are shared by CPL x 32 channels.  x and the dX
// accumulator stay in registers across each run of instructions with the same X irrep.
//
// Row staging (TMA bulk copies, mbarrier double buffering) is that of tp_kernels_row.cuh.
// Outputs leave through per-warp shared-memory stages and bulk stores; leader-only bulk
// operations are predicated instead of branched.  Backward sums are taken in a fixed order
// (runs, warps, lanes), so results are bitwise reproducible.
#pragma once

#include "tp_kernels_row.cuh"

namespace oeqb {

constexpr int kSegD = 2 * kLMaxUnrolled + 1;  // largest unrolled irrep dimension
// Chunks per lane and instruction (forward, backward); halved for double to stay in registers.
__host__ __device__ constexpr int seg_fwd_cpl(int elem) { return elem == 8 ? 1 : 4; }
__host__ __device__ constexpr int seg_bwd_cpl(int elem) { return elem == 8 ? 1 : 1; }
constexpr int kSegFwdCPLMax = 4;
constexpr int kSegStages = 2;                 // forward output staging slots per warp

struct SegInstr {  // 40 bytes
  int l1, l3, bc;  // degrees of X and output; pair_code(l2, l3) for dispatch_bc
  int y_off;       // Y row offset of the Y irrep
  int w_off;       // weight offset of channel 0 (chunk c adds 32 c)
  int z_off;       // output irrep offset (chunk c adds 32 c d3)
  int p_off;       // offset of the instruction's P matrix in the row's P block
  int pad;
  double pw;       // path weight
};

struct SegRun {  // instructions [n0, n1) share the X irrep at x_off
  int x_off, l1, nch, n0, n1;
  int poff;        // backward: this run's dX partial slot ([nch * 32][d1] elements)
  int pad0, pad1;
};

struct SegX {  // backward dX reduction: X irrep row range; runs [run0, run1) wrote it
  int off, n, run0, run1;
};

struct SegPEnt {  // one non-zero P entry: P[dst] = sum of nt terms starting at t0
  int dst, t0nt;  // t0nt = t0 << 8 | nt
};

template <class T>
struct SegTerm {
  T c;  // pw * c_ijk
  int j;
};

template <class T>
struct ArgsSeg {
  Args<T> a;
  const unsigned char* tables;  // SegInstr | SegRun | int grp[G+1] | SegX | SegPEnt | SegTerm
  int table_bytes;              // multiple of 16
  int off_run, off_grp, off_x, off_pent, off_term;  // byte offsets (instructions at 0)
  int ngroups, nsplit, cbs;     // units per row = ngroups x nsplit; chunks per block
  int nx, npent, psize;
  int offY, offW, offG, row_elems, rows_per_buf;
  int use_tma;
  int scratch_off;              // element offset of the scratch area after the P block
  int gyc_off;                  // backward: element offset of the dY columns in the scratch
};

template <class T>
struct SmemSeg {
  const SegInstr* ins;
  const SegRun* runs;
  const int* grp;
  const SegX* xs;
  const SegPEnt* pent;
  const SegTerm<T>* term;
  unsigned long long* bars;
  T* rowbuf;
  T* P;
  T* scratch;
};

template <class T>
__device__ __forceinline__ SmemSeg<T> stage_seg(const ArgsSeg<T>& v, unsigned char* sm) {
  SmemSeg<T> s;
  const uint4* src = reinterpret_cast<const uint4*>(v.tables);
  uint4* dst = reinterpret_cast<uint4*>(sm);
  for (int i = threadIdx.x; i < v.table_bytes / 16; i += blockDim.x) dst[i] = src[i];
  s.ins = reinterpret_cast<const SegInstr*>(sm);
  s.runs = reinterpret_cast<const SegRun*>(sm + v.off_run);
  s.grp = reinterpret_cast<const int*>(sm + v.off_grp);
  s.xs = reinterpret_cast<const SegX*>(sm + v.off_x);
  s.pent = reinterpret_cast<const SegPEnt*>(sm + v.off_pent);
  s.term = reinterpret_cast<const SegTerm<T>*>(sm + v.off_term);
  unsigned char* p = sm + v.table_bytes;
  s.bars = reinterpret_cast<unsigned long long*>(p);
  p += 16;
  s.rowbuf = reinterpret_cast<T*>(p);
  p += 2 * sizeof(T) * static_cast<size_t>(v.row_elems) * v.rows_per_buf;
  s.P = reinterpret_cast<T*>(p);
  s.scratch = s.P + v.scratch_off;
  // Entries of P that no term writes (structural zeros, padding) stay zero for good.
  for (int i = threadIdx.x; i < v.scratch_off; i += blockDim.x) s.P[i] = T(0);
  if (threadIdx.x == 0) {
    mbar_init(&s.bars[0], 1);
    mbar_init(&s.bars[1], 1);
    fence_mbar_init();
  }
  __syncthreads();
  return s;
}

// Loads rows [row0, row0 + n) into buffer b: row r holds X | Y | W (| dZ) at r * row_elems.
template <class T, bool BWD>
__device__ __forceinline__ void seg_load(const ArgsSeg<T>& v, const SmemSeg<T>& s, int b,
                                         long long row0, int n) {
  const Args<T>& a = v.a;
  T* buf = s.rowbuf + static_cast<size_t>(b) * v.row_elems * v.rows_per_buf;
  if (v.use_tma) {
    if (threadIdx.x == 0) {
      const int per_row = a.L1dim + a.L2dim + (a.shared_w ? 0 : a.wnumel) + (BWD ? a.L3dim : 0);
      mbar_expect_tx(&s.bars[b], static_cast<unsigned>(per_row * n * sizeof(T)));
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

// P blocks of the nr rows in a buffer (P block r at r * psize), cooperatively.
template <class T>
__device__ __forceinline__ void seg_pmat(const ArgsSeg<T>& v, const SmemSeg<T>& s, const T* buf,
                                         int nr) {
  const int total = v.npent * nr;
  for (int e = threadIdx.x; e < total; e += blockDim.x) {
    const int r = e / v.npent, q = e - r * v.npent;
    const SegPEnt pe = s.pent[q];
    const T* y = buf + static_cast<size_t>(r) * v.row_elems + v.offY;
    const int t0 = pe.t0nt >> 8, nt = pe.t0nt & 255;
    T acc = T(0);
    for (int t = t0; t < t0 + nt; ++t) acc += s.term[t].c * y[s.term[t].j];
    s.P[r * v.psize + pe.dst] = acc;
  }
}

// Broadcast load of N (multiple of 16 bytes) values from 16-byte aligned shared memory.
template <class T, int N>
__device__ __forceinline__ void lds_vec(T (&d)[N], const T* src) {
  if constexpr (sizeof(T) == 4) {
    static_assert(N % 4 == 0, "float vector length");
#pragma unroll
    for (int q = 0; q < N / 4; ++q) {
      const float4 t = reinterpret_cast<const float4*>(src)[q];
      d[4 * q] = t.x;
      d[4 * q + 1] = t.y;
      d[4 * q + 2] = t.z;
      d[4 * q + 3] = t.w;
    }
  } else {
    static_assert(N % 2 == 0, "double vector length");
#pragma unroll
    for (int q = 0; q < N / 2; ++q) {
      const double2 t = reinterpret_cast<const double2*>(src)[q];
      d[2 * q] = t.x;
      d[2 * q + 1] = t.y;
    }
  }
}

template <class T>
__host__ __device__ constexpr int seg_vpad(int n) {
  return sizeof(T) == 4 ? (n + 3) / 4 * 4 : (n + 1) / 2 * 2;
}

// Bulk store of a staged shared-memory block, issued by the lane where `leader` holds (the
// operation is predicated, so the warp does not diverge).  Followed by a commit.
__device__ __forceinline__ void bulk_store_leader(bool leader, void* dst, const void* src,
                                                  unsigned bytes) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %3, 0;\n"
      "@p cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n"
      "@p cp.async.bulk.commit_group;\n}\n" ::"l"(dst),
      "r"(smem_u32(src)), "r"(bytes), "r"(static_cast<int>(leader))
      : "memory");
}

// ---------------------------------------------------------------------------------------
// Forward: 8 warps, rows_per_buf rows per buffer; unit = (row of the buffer, group, block of
// cbs <= seg_fwd_cpl chunks).

template <class T>
__global__ void __launch_bounds__(256, sizeof(T) == 8 ? 1 : 2) tp_fwd_seg(const ArgsSeg<T> v) {
  extern __shared__ __align__(16) unsigned char smem[];
  const SmemSeg<T> s = stage_seg(v, smem);
  const Args<T>& a = v.a;
  constexpr int NW = 8, CPL = seg_fwd_cpl(sizeof(T)), SLOT = CPL * 32 * kSegD;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  T* stage0 = s.scratch + static_cast<size_t>(wid) * (kSegStages * SLOT);
  int sb = 0;
  const int R = v.rows_per_buf;
  const int upr = v.ngroups * v.nsplit;  // units per row
  const long long B = a.nitems;
  const long long nblk = (B + R - 1) / R;
  auto rows_in = [&](long long blk) { return static_cast<int>(min(static_cast<long long>(R), B - blk * R)); };
  if (blockIdx.x < nblk) seg_load<T, false>(v, s, 0, blockIdx.x * R, rows_in(blockIdx.x));
  if (blockIdx.x + gridDim.x < nblk)
    seg_load<T, false>(v, s, 1, (blockIdx.x + gridDim.x) * R, rows_in(blockIdx.x + gridDim.x));
  if (!v.use_tma) __syncthreads();
  int it = 0;
  for (long long blk = blockIdx.x; blk < nblk; blk += gridDim.x, ++it) {
    const int b = it & 1;
    const int nr = rows_in(blk);
    if (v.use_tma) mbar_wait(&s.bars[b], (it >> 1) & 1, a.status);
    const T* buf = s.rowbuf + static_cast<size_t>(b) * v.row_elems * R;
    seg_pmat(v, s, buf, nr);
    __syncthreads();
    for (int u = wid; u < nr * upr; u += NW) {
      const int r = u / upr, g = (u - r * upr) / v.nsplit, sp = u - r * upr - g * v.nsplit;
      const T* rb = buf + static_cast<size_t>(r) * v.row_elems;
      const T* Pr = s.P + r * v.psize;
      T* zrow = a.out0 + (blk * R + r) * a.L3dim;
      const int c0 = sp * v.cbs;
      for (int q = s.grp[g]; q < s.grp[g + 1]; ++q) {
        const SegRun run = s.runs[q];
        const int nc = min(v.cbs, run.nch - c0);
        if (nc <= 0) continue;
        dispatch_l(run.l1, [&]<int A>() {
          constexpr int D1 = 2 * A + 1;
          T x[CPL][D1];
#pragma unroll
          for (int cq = 0; cq < CPL; ++cq) {
            const T* xs = rb + run.x_off + ((c0 + cq) * 32 + lane) * D1;
#pragma unroll
            for (int i = 0; i < D1; ++i) x[cq][i] = cq < nc ? xs[i] : T(0);
          }
          for (int n = run.n0; n < run.n1; ++n) {
            const SegInstr in = s.ins[n];
            dispatch_l(in.l3, [&]<int C>() {
              constexpr int D3 = 2 * C + 1;
              T P[seg_vpad<T>(D1 * D3)];
              lds_vec(P, Pr + in.p_off);
              T* stage = stage0 + sb * SLOT;
              sb ^= 1;
              bulk_wait_read<kSegStages - 1>();  // the store that last used this slot has read it
              __syncwarp();
#pragma unroll
              for (int cq = 0; cq < CPL; ++cq) {
                if (cq < nc) {
                  const int ch = (c0 + cq) * 32 + lane;
                  const T w = a.shared_w ? a.W[in.w_off + ch] : rb[v.offW + in.w_off + ch];
#pragma unroll
                  for (int k = 0; k < D3; ++k) {
                    T acc = T(0);
#pragma unroll
                    for (int i = 0; i < D1; ++i) acc += x[cq][i] * P[i * D3 + k];
                    stage[(cq * 32 + lane) * D3 + k] = acc * w;
                  }
                }
              }
              T* dst = zrow + in.z_off + c0 * 32 * D3;
              const unsigned bytes = nc * 32 * D3 * sizeof(T);
              if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
                fence_async_smem();
                __syncwarp();
                bulk_store_leader(lane == 0, dst, stage, bytes);
              } else {
                __syncwarp();
                for (int e = lane; e < nc * 32 * D3; e += 32) dst[e] = stage[e];
              }
            });
          }
        });
      }
    }
    __syncthreads();
    const long long next = blk + 2LL * gridDim.x;
    if (next < nblk) seg_load<T, false>(v, s, b, next * R, rows_in(next));
    if (!v.use_tma) __syncthreads();
  }
  bulk_wait_all<0>();
}

// ---------------------------------------------------------------------------------------
// Backward: NW warps, one row per buffer; unit = (group, block of cbs <= seg_bwd_cpl chunks).
// Scratch: per-run dX partials, then per-warp dY lane columns [L2dim][32].

template <class T, int NW>
__global__ void __launch_bounds__(NW * 32, 1) tp_bwd_seg(const ArgsSeg<T> v) {
  extern __shared__ __align__(16) unsigned char smem[];
  const SmemSeg<T> s = stage_seg(v, smem);
  const Args<T>& a = v.a;
  constexpr int CPL = seg_bwd_cpl(sizeof(T));
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  T* part = s.scratch;
  T* gyc_all = part + v.gyc_off;
  T* gyc = gyc_all + static_cast<size_t>(wid) * a.L2dim * 32;
  const long long B = a.nitems;
  if (blockIdx.x < B) seg_load<T, true>(v, s, 0, blockIdx.x, 1);
  if (blockIdx.x + gridDim.x < B) seg_load<T, true>(v, s, 1, blockIdx.x + gridDim.x, 1);
  if (!v.use_tma) __syncthreads();
  int it = 0;
  for (long long row = blockIdx.x; row < B; row += gridDim.x, ++it) {
    const int b = it & 1;
    if (v.use_tma) mbar_wait(&s.bars[b], (it >> 1) & 1, a.status);
    const T* rb = s.rowbuf + static_cast<size_t>(b) * v.row_elems;
    seg_pmat(v, s, rb, 1);
    __syncthreads();
    for (int e = lane; e < a.L2dim * 32; e += 32) gyc[e] = T(0);
    __syncwarp();
    T* dwrow = a.shared_w ? a.out2 : a.out2 + row * a.wnumel;
    for (int u = wid; u < v.ngroups * v.nsplit; u += NW) {
      const int g = u / v.nsplit, sp = u - g * v.nsplit;
      const int c0 = sp * v.cbs;
      for (int q = s.grp[g]; q < s.grp[g + 1]; ++q) {
        const SegRun run = s.runs[q];
        const int nc = min(v.cbs, run.nch - c0);
        if (nc <= 0) continue;
        dispatch_l(run.l1, [&]<int A>() {
          constexpr int D1 = 2 * A + 1;
          T x[CPL][D1], gx[CPL][D1];
#pragma unroll
          for (int cq = 0; cq < CPL; ++cq) {
            const T* xs = rb + run.x_off + ((c0 + cq) * 32 + lane) * D1;
#pragma unroll
            for (int i = 0; i < D1; ++i) {
              x[cq][i] = cq < nc ? xs[i] : T(0);
              gx[cq][i] = T(0);
            }
          }
          for (int n = run.n0; n < run.n1; ++n) {
            const SegInstr in = s.ins[n];
            dispatch_bc<A>(in.bc, [&]<int Bd, int C>() {
              constexpr int D2 = 2 * Bd + 1, D3 = 2 * C + 1;
              T P[seg_vpad<T>(D1 * D3)];
              lds_vec(P, s.P + in.p_off);
              T ey[D2];
#pragma unroll
              for (int j = 0; j < D2; ++j) ey[j] = T(0);
#pragma unroll
              for (int cq = 0; cq < CPL; ++cq) {
                if (cq < nc) {
                  const int ch = (c0 + cq) * 32 + lane;
                  T gz[D3];
                  const T* gs = rb + v.offG + in.z_off + ch * D3;
#pragma unroll
                  for (int k = 0; k < D3; ++k) gz[k] = gs[k];
                  const T w = a.shared_w ? a.W[in.w_off + ch] : rb[v.offW + in.w_off + ch];
                  T sdot = T(0);
#pragma unroll
                  for (int i = 0; i < D1; ++i) {
                    T h = T(0);
#pragma unroll
                    for (int k = 0; k < D3; ++k) h += P[i * D3 + k] * gz[k];
                    gx[cq][i] += w * h;
                    sdot += x[cq][i] * h;
                  }
                  if (a.shared_w)
                    atomic_add(dwrow + in.w_off + ch, sdot);
                  else
                    dwrow[in.w_off + ch] = sdot;
                  T e[D2];
                  CG<A, Bd, C>::evec(gz, x[cq], e);
#pragma unroll
                  for (int j = 0; j < D2; ++j) ey[j] += w * e[j];
                }
              }
              const T pw = T(in.pw);
#pragma unroll
              for (int j = 0; j < D2; ++j) gyc[(in.y_off + j) * 32 + lane] += pw * ey[j];
            });
          }
#pragma unroll
          for (int cq = 0; cq < CPL; ++cq) {
            if (cq < nc) {
              T* gp = part + run.poff + ((c0 + cq) * 32 + lane) * D1;
#pragma unroll
              for (int i = 0; i < D1; ++i) gp[i] = gx[cq][i];
            }
          }
        });
      }
    }
    __syncthreads();
    const long long next = row + 2LL * gridDim.x;
    if (next < B) seg_load<T, true>(v, s, b, next, 1);
    // dX: sum the partial slots of the runs that wrote each X irrep, in run order.
    T* gxrow = a.out0 + row * a.L1dim;
    for (int r = 0; r < v.nx; ++r) {
      const SegX xr = s.xs[r];
      for (int e = threadIdx.x; e < xr.n; e += blockDim.x) {
        T acc = T(0);
        for (int q = xr.run0; q < xr.run1; ++q) acc += part[s.runs[q].poff + e];
        gxrow[xr.off + e] = acc;
      }
    }
    // dY: warps in order, then a lane butterfly.
    T* gyrow = a.out1 + row * a.L2dim;
    for (int j = wid; j < a.L2dim; j += NW) {
      T acc = T(0);
      for (int w = 0; w < NW; ++w) acc += gyc_all[(static_cast<size_t>(w) * a.L2dim + j) * 32 + lane];
      acc = group_sum(acc, 5);
      if (lane == 0) gyrow[j] = acc;
    }
  }
}

}  // namespace oeqb
