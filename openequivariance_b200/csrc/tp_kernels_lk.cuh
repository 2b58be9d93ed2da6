// Lockstep channelwise-uvu backward (BASELINE C2 shape, uniform multiplicities).
//
// Same mathematics as tp_bwd_seg (tp_kernels_seg.cuh): per row, P[i][k] = pw sum_j c_ijk y_j
// is built once in shared memory (each row i padded to a multiple of 4 values), and for
// channel u of instruction n
//     h_i = sum_k P[i][k] gz[u][k];  dX[u][i] += w[u] h_i;  dW[u] = sum_i x[u][i] h_i;
//     dY[j] += w[u] pw sum_(i,k) c_ijk x[u][i] gz[u][k].
// Work mapping: a CTA takes RB rows at a time and its NW consumer warps (16; 12 with CPL = 2)
// are (row, chunk) pairs, a chunk being 32 x CPL channels (lane l owns channels l, l + 32,
// ...; RB x NCH / CPL = NW).  Every warp walks the whole instruction list in the same order,
// so all warps run the same code at the same time (one instruction-cache footprint, equal
// work, no barrier imbalance), and each warp owns complete dX rows of its chunk (no
// partials).  With CPL = 2 one P block load, barrier wait and instruction decode serve two
// channels.
//
// Data movement (warp-specialised): a 17th warp is the producer.  X and Y of the RB rows are
// double-buffered at row-block granularity.  dZ and W are streamed per instruction through a
// ring of NS slots: slot t % NS holds the instruction's dZ segment (NCH x 32 x d3 contiguous
// values per row) and W segment (NCH x 32 values per row) for every row of the block.  Each
// buffer has a full barrier (TMA transaction count) and an empty barrier (one arrival per
// consumer warp); the producer refills a buffer as soon as its empty barrier completes, so
// consumers never carry copy work.  Consumers synchronise among themselves on named barrier 1.
//
// Y must be the spherical-harmonic layout (one irrep per degree l = 0..L in order), so the Y
// offset of degree l is l^2 at compile time and each lane keeps its dY partial sums in
// registers; a transposed butterfly folds them across lanes once per row block.
//
// Waits on barriers are bounded (status flag 3 on expiry); every warp passes every ring step,
// active or not, so each slot is always released.
#pragma once

#include "tp_kernels_seg.cuh"

namespace oeqb {

constexpr int kLkWarps = 16;  // largest consumer warp count; one producer warp more
// Consumer warps for CPL channels per lane.  Registers are split per SM sub-partition, so 17
// warps (5 on one quarter) cap a thread at 96 registers; two channels per lane need more, and
// 12 + 1 warps (at most 4 per quarter) allow 128.
__host__ __device__ constexpr int lk_warps(int cpl) { return cpl == 2 ? 12 : 16; }
constexpr int kLkMaxSlots = 12;
constexpr int kLkGy = (kLMaxUnrolled + 1) * (kLMaxUnrolled + 1);  // dY registers per lane

template <class T>
struct ArgsLk {
  Args<T> a;
  const unsigned char* tables;  // SegInstr | SegRun | grp | SegX | SegPEnt | SegTerm (one group)
  int table_bytes;
  int off_run, off_grp, off_x, off_pent, off_term;
  int ninstr, nrun, npent, psize;
  int nch, rb;                  // 32-channel chunks per instruction, rows per block
                                // (nch / CPL * rb = NW)
  int nslots;                   // ring slots
  int offY, xy_elems;           // X | Y row layout in the row buffer
  int slot_elems, slot_w_off;   // ring slot size; W part offset inside a slot
};

template <int NW>
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;\n" ::"n"(NW * 32) : "memory");
}

template <class T>
struct SmemLk {
  const SegInstr* ins;
  const SegRun* runs;
  const SegPEnt* pent;
  const SegTerm<T>* term;
  unsigned long long* row_bar;   // [2] full
  unsigned long long* row_emp;   // [2] empty
  unsigned long long* slot_bar;  // [kLkMaxSlots] full
  unsigned long long* slot_emp;  // [kLkMaxSlots] empty
  T* rowbuf;                     // [2][rb][xy_elems]
  T* ring;                       // [nslots][slot_elems]
  T* P;                          // [rb][psize]
  T* gys;                        // [16][kLkGy] per-warp dY sums
};

// Issues the ring slot of instruction n for rows [row0, row0 + nr): lane 0 posts the expected
// bytes, then lanes r < nr copy row r's dZ segment and lanes 16 + r its W segment (the
// producer warp issues the copies of one slot in parallel).
template <class T>
__device__ __forceinline__ void lk_fill(const ArgsLk<T>& v, const SmemLk<T>& s, int n, int slot,
                                        long long row0, int nr, int lane) {
  const Args<T>& a = v.a;
  const SegInstr in = s.ins[n];
  const int d3 = 2 * in.l3 + 1;
  const unsigned zb = static_cast<unsigned>(v.nch * 32 * d3 * sizeof(T));
  const unsigned wb = a.shared_w ? 0u : static_cast<unsigned>(v.nch * 32 * sizeof(T));
  if (lane == 0) mbar_expect_tx(&s.slot_bar[slot], nr * (zb + wb));
  __syncwarp();
  T* dst = s.ring + static_cast<size_t>(slot) * v.slot_elems;
  if (lane < nr) {
    const long long row = row0 + lane;
    bulk_g2s(dst + lane * v.nch * 32 * kSegD, a.Gz + row * a.L3dim + in.z_off, zb, &s.slot_bar[slot]);
  } else if (lane >= 16 && lane < 16 + nr && !a.shared_w) {
    const int r = lane - 16;
    const long long row = row0 + r;
    bulk_g2s(dst + v.slot_w_off + r * v.nch * 32, a.W + row * a.wnumel + in.w_off, wb,
             &s.slot_bar[slot]);
  }
}

// X and Y rows of a row block into row buffer b (lane r copies row r).
template <class T>
__device__ __forceinline__ void lk_load_rows(const ArgsLk<T>& v, const SmemLk<T>& s, int b,
                                             long long row0, int nr, int lane) {
  const Args<T>& a = v.a;
  if (lane == 0)
    mbar_expect_tx(&s.row_bar[b], static_cast<unsigned>(nr * (a.L1dim + a.L2dim) * sizeof(T)));
  __syncwarp();
  T* buf = s.rowbuf + static_cast<size_t>(b) * v.rb * v.xy_elems;
  if (lane < nr) {
    const long long row = row0 + lane;
    bulk_g2s(buf + lane * v.xy_elems, a.X + row * a.L1dim, a.L1dim * sizeof(T), &s.row_bar[b]);
    bulk_g2s(buf + lane * v.xy_elems + v.offY, a.Y + row * a.L2dim, a.L2dim * sizeof(T),
             &s.row_bar[b]);
  }
}

template <class T, int CPL>
__global__ void __launch_bounds__((lk_warps(CPL) + 1) * 32, 1) tp_bwd_lk(const ArgsLk<T> v) {
  constexpr int NW = lk_warps(CPL);
  extern __shared__ __align__(16) unsigned char smem[];
  const Args<T>& a = v.a;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  SmemLk<T> s;
  {
    const uint4* src = reinterpret_cast<const uint4*>(v.tables);
    uint4* dst = reinterpret_cast<uint4*>(smem);
    for (int i = threadIdx.x; i < v.table_bytes / 16; i += blockDim.x) dst[i] = src[i];
    s.ins = reinterpret_cast<const SegInstr*>(smem);
    s.runs = reinterpret_cast<const SegRun*>(smem + v.off_run);
    s.pent = reinterpret_cast<const SegPEnt*>(smem + v.off_pent);
    s.term = reinterpret_cast<const SegTerm<T>*>(smem + v.off_term);
    unsigned char* p = smem + v.table_bytes;
    s.row_bar = reinterpret_cast<unsigned long long*>(p);
    s.row_emp = s.row_bar + 2;
    s.slot_bar = s.row_emp + 2;
    s.slot_emp = s.slot_bar + kLkMaxSlots;
    p += 8 * (4 + 2 * kLkMaxSlots);
    s.rowbuf = reinterpret_cast<T*>(p);
    s.ring = s.rowbuf + static_cast<size_t>(2) * v.rb * v.xy_elems;
    s.P = s.ring + static_cast<size_t>(v.nslots) * v.slot_elems;
    s.gys = s.P + static_cast<size_t>(v.rb) * v.psize;
    for (int i = threadIdx.x; i < v.rb * v.psize; i += blockDim.x) s.P[i] = T(0);
    if (threadIdx.x == 0) {
      for (int i = 0; i < 2; ++i) {
        mbar_init(&s.row_bar[i], 1);
        mbar_init(&s.row_emp[i], NW);
      }
      for (int i = 0; i < kLkMaxSlots; ++i) {
        mbar_init(&s.slot_bar[i], 1);
        mbar_init(&s.slot_emp[i], NW);
      }
      fence_mbar_init();
    }
    __syncthreads();
  }
  const long long B = a.nitems;
  const long long nblk = (B + v.rb - 1) / v.rb;
  if (wid == NW) {
    // Producer warp: row blocks and ring slots in consumption order.
    if (blockIdx.x < nblk) {
      const int myblk = static_cast<int>((nblk - blockIdx.x + gridDim.x - 1) / gridDim.x);
      auto rows_of = [&](int kb, long long* row0) {
        *row0 = (blockIdx.x + static_cast<long long>(kb) * gridDim.x) * v.rb;
        return static_cast<int>(min(static_cast<long long>(v.rb), B - *row0));
      };
      long long row0;
      int nr = rows_of(0, &row0);
      lk_load_rows(v, s, 0, row0, nr, lane);
      if (myblk > 1) {
        long long r1;
        const int n1 = rows_of(1, &r1);
        lk_load_rows(v, s, 1, r1, n1, lane);
      }
      int slot = 0, wrap = 0;
      for (int kb = 0; kb < myblk; ++kb) {
        nr = rows_of(kb, &row0);
        if (kb >= 2) {
          // Row block kb reuses the row buffer of block kb - 2.
          mbar_wait(&s.row_emp[kb & 1], ((kb >> 1) - 1) & 1, a.status);
          lk_load_rows(v, s, kb & 1, row0, nr, lane);
        }
        for (int n = 0; n < v.ninstr; ++n) {
          if (wrap > 0) mbar_wait(&s.slot_emp[slot], (wrap - 1) & 1, a.status);
          lk_fill(v, s, n, slot, row0, nr, lane);
          if (++slot == v.nslots) {
            slot = 0;
            ++wrap;
          }
        }
      }
    }
    return;
  }
  const int nchw = v.nch / CPL;                       // warps per row
  const int r = wid / nchw, c = wid - r * nchw;       // this warp's row in the block and chunk
  const int ch = c * 32 * CPL + lane;                 // first channel; then + 32, ...
  // Loop invariants in registers: after the barrier waits (asm with memory clobbers) the
  // compiler would otherwise reload these kernel parameters from the constant bank per path.
  const int nslots = v.nslots;
  const size_t slot_elems = static_cast<size_t>(v.slot_elems);
  const int gz_base = r * v.nch * 32 * kSegD;           // this warp's dZ rows in a slot
  const int w_base = v.slot_w_off + r * v.nch * 32 + ch;  // this lane's weight in a slot
  const bool shared_w = a.shared_w != 0;
  const T* __restrict__ Wg = a.W;
  int* status = a.status;
  const T* ring = s.ring;
  unsigned long long* slot_bar = s.slot_bar;
  unsigned long long* slot_emp = s.slot_emp;
  const SegInstr* insv = s.ins;
  int t = 0;          // ring sequence number
  int slot = 0;       // t % nslots
  unsigned par = 0;   // (t / nslots) & 1
  int k = 0;
  for (long long blk = blockIdx.x; blk < nblk; blk += gridDim.x, ++k) {
    const int b = k & 1;
    const long long row0 = blk * v.rb;
    const int nr = static_cast<int>(min(static_cast<long long>(v.rb), B - row0));
    mbar_wait(&s.row_bar[b], (k >> 1) & 1, a.status);
    const T* xyb = s.rowbuf + static_cast<size_t>(b) * v.rb * v.xy_elems;
    // P blocks of the block's rows.
    for (int e = threadIdx.x; e < v.npent * nr; e += NW * 32) {
      const int rr = e / v.npent, q = e - rr * v.npent;
      const SegPEnt pe = s.pent[q];
      const T* y = xyb + rr * v.xy_elems + v.offY;
      const int t0 = pe.t0nt >> 8, nt = pe.t0nt & 255;
      T acc = T(0);
      for (int tt = t0; tt < t0 + nt; ++tt) acc += s.term[tt].c * y[s.term[tt].j];
      s.P[rr * v.psize + pe.dst] = acc;
    }
    consumer_sync<NW>();
    T gy[kLkGy];
#pragma unroll
    for (int j = 0; j < kLkGy; ++j) gy[j] = T(0);
    const bool active = r < nr;
    const long long row = row0 + r;
    const T* xr = xyb + r * v.xy_elems;
    const T* Pr = s.P + r * v.psize;
    T* dwrow = a.shared_w ? a.out2 : a.out2 + row * a.wnumel;
    for (int q = 0; q < v.nrun; ++q) {
      const SegRun run = s.runs[q];
      dispatch_l(run.l1, [&]<int A>() {
        constexpr int D1 = 2 * A + 1;
        T x[CPL][D1], gx[CPL][D1];
        const T* xs = xr + run.x_off + ch * D1;
#pragma unroll
        for (int q = 0; q < CPL; ++q)
#pragma unroll
          for (int i = 0; i < D1; ++i) {
            x[q][i] = active ? xs[q * 32 * D1 + i] : T(0);
            gx[q][i] = T(0);
          }
        for (int n = run.n0; n < run.n1; ++n) {
          mbar_wait(&slot_bar[slot], par, status);
          const SegInstr in = insv[n];
          const T* sl = ring + static_cast<size_t>(slot) * slot_elems;
          if (active) {
            dispatch_bc<A>(in.bc, [&]<int Bd, int C>() {
              constexpr int D2 = 2 * Bd + 1, D3 = 2 * C + 1;
              T gz[CPL][D3], w[CPL];
              const T* gs = sl + gz_base + ch * D3;
#pragma unroll
              for (int q = 0; q < CPL; ++q) {
#pragma unroll
                for (int kk = 0; kk < D3; ++kk) gz[q][kk] = gs[q * 32 * D3 + kk];
                w[q] = shared_w ? Wg[in.w_off + ch + 32 * q] : sl[w_base + 32 * q];
              }
              // P rows are padded to R3 values (16-byte aligned): one row live at a time.
              constexpr int R3 = seg_vpad<T>(D3);
              T sdot[CPL];
#pragma unroll
              for (int q = 0; q < CPL; ++q) sdot[q] = T(0);
#pragma unroll
              for (int i = 0; i < D1; ++i) {
                T Pi[R3];
                lds_vec(Pi, Pr + in.p_off + i * R3);
#pragma unroll
                for (int q = 0; q < CPL; ++q) {
                  T h = T(0);
#pragma unroll
                  for (int kk = 0; kk < D3; ++kk) h += Pi[kk] * gz[q][kk];
                  gx[q][i] += w[q] * h;
                  sdot[q] += x[q][i] * h;
                }
              }
#pragma unroll
              for (int q = 0; q < CPL; ++q) {
                if (shared_w)
                  atomic_add(dwrow + in.w_off + ch + 32 * q, sdot[q]);
                else
                  dwrow[in.w_off + ch + 32 * q] = sdot[q];
              }
#pragma unroll
              for (int q = 0; q < CPL; ++q) {
                T e[D2];
                CG<A, Bd, C>::evec(gz[q], x[q], e);
                const T wp = w[q] * T(in.pw);
#pragma unroll
                for (int j = 0; j < D2; ++j) gy[Bd * Bd + j] += wp * e[j];
              }
            });
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&slot_emp[slot]);
          ++t;
          if (++slot == nslots) {
            slot = 0;
            par ^= 1u;
          }
        }
        // This warp's chunk of the X irrep is complete.
        if (active) {
          T* dst = a.out0 + row * a.L1dim + run.x_off + ch * D1;
#pragma unroll
          for (int q = 0; q < CPL; ++q)
#pragma unroll
            for (int i = 0; i < D1; ++i) dst[q * 32 * D1 + i] = gx[q][i];
        }
      });
    }
    // Fold the lanes' dY sums: after the butterfly, lanes 2m and 2m+1 hold entry m summed
    // over the warp (steps keep the lower or upper half of the values by lane bit).
    {
      T h8[8], h4[4], h2[2], h1;
      const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const T send = b4 ? gy[m] : gy[8 + m];
        h8[m] = (b4 ? gy[8 + m] : gy[m]) + __shfl_xor_sync(0xffffffffu, send, 16);
      }
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const T send = b3 ? h8[m] : h8[4 + m];
        h4[m] = (b3 ? h8[4 + m] : h8[m]) + __shfl_xor_sync(0xffffffffu, send, 8);
      }
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        const T send = b2 ? h4[m] : h4[2 + m];
        h2[m] = (b2 ? h4[2 + m] : h4[m]) + __shfl_xor_sync(0xffffffffu, send, 4);
      }
      {
        const T send = b1 ? h2[0] : h2[1];
        h1 = (b1 ? h2[1] : h2[0]) + __shfl_xor_sync(0xffffffffu, send, 2);
      }
      h1 += __shfl_xor_sync(0xffffffffu, h1, 1);
      if ((lane & 1) == 0) s.gys[wid * kLkGy + (lane >> 1)] = h1;
    }
    consumer_sync<NW>();
    // Row buffer b and P are free (the producer refills b for the block after next).
    if (lane == 0) mbar_arrive(&s.row_emp[b]);
    // dY of the block's rows: the row's chunk warps in order.
    for (int task = threadIdx.x; task < nr * a.L2dim; task += NW * 32) {
      const int rr = task / a.L2dim, j = task - rr * a.L2dim;
      T acc = T(0);
      for (int cc = 0; cc < nchw; ++cc) acc += s.gys[(rr * nchw + cc) * kLkGy + j];
      a.out1[(row0 + rr) * a.L2dim + j] = acc;
    }
  }
}


// ---------------------------------------------------------------------------------------
// Lockstep channelwise-uvu forward (same problem class, every output irrep written by exactly
// one instruction).  Per row and instruction n, for channel u:
//     Z[u][k] = w[u] sum_i x[u][i] P[i][k],  P[i][k] = pw sum_j c_ijk y_j.
// Work mapping as in tp_bwd_lk: 16 consumer warps are (row, chunk of 32 x CPL channels)
// pairs walking the instruction list in the same order; a 17th warp is the producer.  X and Y
// are double-buffered per row block, the instruction's W segment of every row of the block
// streams through a ring of slots.  A warp's Z segment (32 x CPL channels x d3, contiguous in
// the row) is staged in shared memory (two buffers per warp) and written by one bulk store.
constexpr int kLfWarps = 16;

template <class T>
__device__ __forceinline__ void lf_fill(const ArgsLk<T>& v, const SmemLk<T>& s, int n, int slot,
                                        long long row0, int nr, int lane) {
  const Args<T>& a = v.a;
  const unsigned wb = a.shared_w ? 0u : static_cast<unsigned>(v.nch * 32 * sizeof(T));
  if (lane == 0) mbar_expect_tx(&s.slot_bar[slot], nr * wb);
  __syncwarp();
  if (wb != 0 && lane < nr) {
    const long long row = row0 + lane;
    bulk_g2s(s.ring + static_cast<size_t>(slot) * v.slot_elems + lane * v.nch * 32,
             a.W + row * a.wnumel + s.ins[n].w_off, wb, &s.slot_bar[slot]);
  }
}

template <class T, int CPL>
__global__ void __launch_bounds__((kLfWarps + 1) * 32, 1) tp_fwd_lk(const ArgsLk<T> v) {
  constexpr int NW = kLfWarps, ZSLOT = CPL * 32 * kSegD;
  extern __shared__ __align__(16) unsigned char smem[];
  const Args<T>& a = v.a;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  SmemLk<T> s;
  T* zst;  // [NW][2][ZSLOT] Z staging
  {
    const uint4* src = reinterpret_cast<const uint4*>(v.tables);
    uint4* dst = reinterpret_cast<uint4*>(smem);
    for (int i = threadIdx.x; i < v.table_bytes / 16; i += blockDim.x) dst[i] = src[i];
    s.ins = reinterpret_cast<const SegInstr*>(smem);
    s.runs = reinterpret_cast<const SegRun*>(smem + v.off_run);
    s.pent = reinterpret_cast<const SegPEnt*>(smem + v.off_pent);
    s.term = reinterpret_cast<const SegTerm<T>*>(smem + v.off_term);
    unsigned char* p = smem + v.table_bytes;
    s.row_bar = reinterpret_cast<unsigned long long*>(p);
    s.row_emp = s.row_bar + 2;
    s.slot_bar = s.row_emp + 2;
    s.slot_emp = s.slot_bar + kLkMaxSlots;
    p += 8 * (4 + 2 * kLkMaxSlots);
    s.rowbuf = reinterpret_cast<T*>(p);
    s.ring = s.rowbuf + static_cast<size_t>(2) * v.rb * v.xy_elems;
    s.P = s.ring + static_cast<size_t>(v.nslots) * v.slot_elems;
    s.gys = nullptr;
    zst = s.P + static_cast<size_t>(v.rb) * v.psize;
    for (int i = threadIdx.x; i < v.rb * v.psize; i += blockDim.x) s.P[i] = T(0);
    if (threadIdx.x == 0) {
      for (int i = 0; i < 2; ++i) {
        mbar_init(&s.row_bar[i], 1);
        mbar_init(&s.row_emp[i], NW);
      }
      for (int i = 0; i < kLkMaxSlots; ++i) {
        mbar_init(&s.slot_bar[i], 1);
        mbar_init(&s.slot_emp[i], NW);
      }
      fence_mbar_init();
    }
    __syncthreads();
  }
  const long long B = a.nitems;
  const long long nblk = (B + v.rb - 1) / v.rb;
  if (wid == NW) {
    // Producer warp: row blocks and W slots in consumption order.
    if (blockIdx.x < nblk) {
      const int myblk = static_cast<int>((nblk - blockIdx.x + gridDim.x - 1) / gridDim.x);
      auto rows_of = [&](int kb, long long* row0) {
        *row0 = (blockIdx.x + static_cast<long long>(kb) * gridDim.x) * v.rb;
        return static_cast<int>(min(static_cast<long long>(v.rb), B - *row0));
      };
      long long row0;
      int nr = rows_of(0, &row0);
      lk_load_rows(v, s, 0, row0, nr, lane);
      if (myblk > 1) {
        long long r1;
        const int n1 = rows_of(1, &r1);
        lk_load_rows(v, s, 1, r1, n1, lane);
      }
      int slot = 0, wrap = 0;
      for (int kb = 0; kb < myblk; ++kb) {
        nr = rows_of(kb, &row0);
        if (kb >= 2) {
          mbar_wait(&s.row_emp[kb & 1], ((kb >> 1) - 1) & 1, a.status);
          lk_load_rows(v, s, kb & 1, row0, nr, lane);
        }
        for (int n = 0; n < v.ninstr; ++n) {
          if (wrap > 0) mbar_wait(&s.slot_emp[slot], (wrap - 1) & 1, a.status);
          lf_fill(v, s, n, slot, row0, nr, lane);
          if (++slot == v.nslots) {
            slot = 0;
            ++wrap;
          }
        }
      }
    }
    return;
  }
  const int nchw = v.nch / CPL;                   // warps per row
  const int r = wid / nchw, c = wid - r * nchw;   // this warp's row in the block and chunk
  const int ch = c * 32 * CPL + lane;             // first channel; then + 32, ...
  const int nslots = v.nslots;
  const size_t slot_elems = static_cast<size_t>(v.slot_elems);
  const int w_base = r * v.nch * 32 + ch;         // this lane's weight in a slot
  const bool shared_w = a.shared_w != 0;
  const T* __restrict__ Wg = a.W;
  int* status = a.status;
  const T* ring = s.ring;
  unsigned long long* slot_bar = s.slot_bar;
  unsigned long long* slot_emp = s.slot_emp;
  const SegInstr* insv = s.ins;
  T* const zst0 = zst + static_cast<size_t>(wid) * 2 * ZSLOT;
  int sb = 0;
  int slot = 0;
  unsigned par = 0;
  int k = 0;
  for (long long blk = blockIdx.x; blk < nblk; blk += gridDim.x, ++k) {
    const int b = k & 1;
    const long long row0 = blk * v.rb;
    const int nr = static_cast<int>(min(static_cast<long long>(v.rb), B - row0));
    mbar_wait(&s.row_bar[b], (k >> 1) & 1, a.status);
    const T* xyb = s.rowbuf + static_cast<size_t>(b) * v.rb * v.xy_elems;
    for (int e = threadIdx.x; e < v.npent * nr; e += NW * 32) {
      const int rr = e / v.npent, q = e - rr * v.npent;
      const SegPEnt pe = s.pent[q];
      const T* y = xyb + rr * v.xy_elems + v.offY;
      const int t0 = pe.t0nt >> 8, nt = pe.t0nt & 255;
      T acc = T(0);
      for (int tt = t0; tt < t0 + nt; ++tt) acc += s.term[tt].c * y[s.term[tt].j];
      s.P[rr * v.psize + pe.dst] = acc;
    }
    consumer_sync<NW>();
    const bool active = r < nr;
    const long long row = row0 + r;
    const T* xr = xyb + r * v.xy_elems;
    const T* Pr = s.P + r * v.psize;
    T* zrow = a.out0 + row * a.L3dim;
    for (int q = 0; q < v.nrun; ++q) {
      const SegRun run = s.runs[q];
      dispatch_l(run.l1, [&]<int A>() {
        constexpr int D1 = 2 * A + 1;
        T x[CPL][D1];
        const T* xs = xr + run.x_off + ch * D1;
#pragma unroll
        for (int cq = 0; cq < CPL; ++cq)
#pragma unroll
          for (int i = 0; i < D1; ++i) x[cq][i] = active ? xs[cq * 32 * D1 + i] : T(0);
        for (int n = run.n0; n < run.n1; ++n) {
          mbar_wait(&slot_bar[slot], par, status);
          const SegInstr in = insv[n];
          const T* sl = ring + static_cast<size_t>(slot) * slot_elems;
          if (active) {
            dispatch_l(in.l3, [&]<int C>() {
              constexpr int D3 = 2 * C + 1, R3 = seg_vpad<T>(D3);
              T w[CPL], z[CPL][D3];
#pragma unroll
              for (int cq = 0; cq < CPL; ++cq) {
                w[cq] = shared_w ? Wg[in.w_off + ch + 32 * cq] : sl[w_base + 32 * cq];
#pragma unroll
                for (int kk = 0; kk < D3; ++kk) z[cq][kk] = T(0);
              }
#pragma unroll
              for (int i = 0; i < D1; ++i) {
                T Pi[R3];
                lds_vec(Pi, Pr + in.p_off + i * R3);
#pragma unroll
                for (int cq = 0; cq < CPL; ++cq)
#pragma unroll
                  for (int kk = 0; kk < D3; ++kk) z[cq][kk] += x[cq][i] * Pi[kk];
              }
              T* stage = zst0 + sb * ZSLOT;
              sb ^= 1;
              bulk_wait_read<1>();  // the store that last used this buffer has read it
              __syncwarp();
#pragma unroll
              for (int cq = 0; cq < CPL; ++cq)
#pragma unroll
                for (int kk = 0; kk < D3; ++kk)
                  stage[(cq * 32 + lane) * D3 + kk] = z[cq][kk] * w[cq];
              fence_async_smem();
              __syncwarp();
              bulk_store_leader(lane == 0, zrow + in.z_off + c * 32 * CPL * D3, stage,
                                CPL * 32 * D3 * sizeof(T));
            });
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&slot_emp[slot]);
          if (++slot == nslots) {
            slot = 0;
            par ^= 1u;
          }
        }
      });
    }
    // P is rebuilt for the next block only after every warp has finished with it.
    consumer_sync<NW>();
    if (lane == 0) mbar_arrive(&s.row_emp[b]);
  }
  bulk_wait_all<0>();  // every Z store has completed before the CTA exits
}

}  // namespace oeqb
