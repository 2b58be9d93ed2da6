// Tensor-core (tcgen05) forward of shared-weight "uvw" tensor products, float32.
//
// Problem class (NequIP-style fully connected paths): every instruction
// has mul1 = mul3 = 32, mul2 = 1, degrees l1, l3 <= 2 (l2 <= 3), weights shared by all rows.
// Per row b and instruction n (i1, i2 -> i3) the reference computes (templates/
// loop_unroll_tp.cuh:47-85, uvw branch)
//     Z[b, w, k] += pw_n sum_u W_n[u, w] T_n,k[b, u],   T_n,k[b, u] = sum_(i,j) C_ijk X[b,u,i] Y[b,j].
// For a tile of 128 rows and a fixed output component k this is a GEMM
//     D_(i3,k)[128 x 32] += A_n,k[128 x 32] * B_n[32 x 32],   A = T (rows x u), B = pw W (u x w),
// accumulated over every instruction into i3.  Mapping on sm_100a:
//
//  * A is produced by CUDA cores: 16 compute warps, warp (q, c) owns TMEM lane quarter q (rows
//    32q..32q+31, one row per thread) and channels u = 8c..8c+7.  A thread contracts its row's
//    X segment (staged in shared memory) with P[i][k] = sum_j C_ijk y_j (compile-time sparse CG
//    per degree triple) and writes T into a TMEM A slot with tcgen05.st.
//  * Float32 accuracy on the TF32 tensor pipe by the 3xTF32 split (A = Ah + Al, B = Bh + Bl,
//    D += Ah Bh + Ah Bl + Al Bh; error-compensated TF32 GEMM as published by Ootomo & Yokota,
//    2022).  B = pw W is split once per call by tp_uvw_tc_prep into the canonical no-swizzle
//    K-major layout (8 x 16-byte core matrices), so one bulk copy stages an instruction's
//    operand (hi | lo, 8 KiB) in a shared-memory ring.
//  * One thread of the MMA warp issues tcgen05.mma (kind::tf32, A from TMEM, B from shared
//    memory, D in TMEM, M = 128, N = 32, K = 8) and releases A slots / W slots / the
//    accumulator with tcgen05.commit on mbarriers.
//  * A producer warp stages X per input irrep with 2D TMA tensor copies (boxes of 128 rows x
//    32 floats, 128-byte swizzle so the row-per-thread reads are bank-conflict free,
//    double-buffered); a second producer warp streams the W ring with cp.async.bulk.
//  * Work unit = 128-row tile x output group (a run of output irreps whose 32 * (2 l3 + 1)
//    accumulator columns fit 160).  TMEM: two 160-column accumulator buffers (unit i uses
//    buffer i & 1, so the epilogue of unit i - 1 overlaps the MMAs of unit i) + 3 A slots of
//    64 columns (hi | lo).  The epilogue reads D with tcgen05.ld (each thread its row,
//    8 channels x d3 components = one contiguous piece of the Z row).
//
// Every mbarrier wait is bounded (status flag 3 on expiry); the producer drains its own
// copies and the MMA thread's work is complete before TMEM is released.
#pragma once

#include <cuda.h>

#include "tp_kernels_row.cuh"

namespace oeqb {

constexpr int kTcRows = 128;
constexpr int kTcComputeWarps = 16;
constexpr int kTcMmaWarp = 16;
constexpr int kTcProdWarp = 17;   // X stages (TMA tensor copies)
constexpr int kTcWProdWarp = 18;  // W ring (bulk copies)
constexpr int kTcThreads = 19 * 32;
constexpr int kTcDCols = 160;              // per accumulator buffer (two buffers)
constexpr int kTcASlots = 3;
constexpr int kTcACol0 = 2 * kTcDCols;      // A slot s: columns kTcACol0 + 64 s (+32 for lo)
constexpr int kTcWSlots = 4;
constexpr int kTcYMax = 16;
constexpr int kTcYStride = 17;
constexpr int kTcMaxD = 5;
constexpr int kTcXBox = kTcRows * 32;            // floats per TMA box (128 rows x 32 floats)
constexpr int kTcWBlock = 2 * 32 * 32;            // floats per instruction: hi | lo
constexpr int kTcTmemCols = 512;

struct TcStage {
  int x_off, l1, ins_begin, ins_end;
};
struct TcIns {
  int l2, l3, y_off, wblk, dcol, first, pad0, pad1;
};
struct TcOut {
  int z_off, d3, dcol, has;
};
struct TcPass {
  int stage_begin, stage_end, out_begin, out_end;
};

struct ArgsTc {
  const float* X;
  const float* Y;
  const float* Wsplit;  // [nins][hi 1024 | lo 1024], canonical core-matrix layout
  float* Z;
  long long B;
  int L1dim, L2dim, L3dim;
  int npass, nstage, nins, nout;  // output groups (work unit = 128-row tile x group), ...
  const TcPass* passes;
  const TcStage* stages;
  const TcIns* ins;
  const TcOut* outs;
  int* status;
};

// Schedule tables held in shared memory.
constexpr int kTcMaxGroups = 16, kTcMaxStages = 64, kTcMaxIns = 64, kTcMaxOuts = 48;

// Shared-memory image (dynamic; the no-swizzle operand layout needs 16-byte alignment only).
constexpr int kTcSmemBars = 0;                                   // 23 mbarriers + TMEM base
constexpr int kTcSmemTab = 256;                                  // schedule tables
constexpr int kTcSmemY = kTcSmemTab + 16 * kTcMaxGroups + 16 * kTcMaxStages + 32 * kTcMaxIns +
                         16 * kTcMaxOuts;                        // [2][128][17] floats
constexpr int kTcSmemW = (kTcSmemY + 2 * kTcRows * kTcYStride * 4 + 1023) / 1024 * 1024;
constexpr int kTcSmemX = kTcSmemW + kTcWSlots * kTcWBlock * 4;   // [2][kTcMaxD boxes]
constexpr int kTcSmemBytes = kTcSmemX + 2 * kTcMaxD * kTcXBox * 4 + 1024;  // + base alignment
static_assert(kTcSmemW % 1024 == 0 && kTcSmemX % 1024 == 0, "1024-byte aligned regions");
static_assert(kTcSmemBytes <= 227 * 1024, "shared memory image too large");

// ------------------------------------------------------------------ tcgen05 wrappers

__device__ __forceinline__ unsigned tf32_bits(float x) {
  unsigned r;
  asm("cvt.rna.tf32.f32 %0, %1;\n" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}

__device__ __forceinline__ void tmem_st8(unsigned taddr, const unsigned (&v)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};\n" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_ld8(unsigned taddr, unsigned (&v)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}
// Makes later uses of v data-dependent on a point after tcgen05.wait::ld.
__device__ __forceinline__ void reg_pin8(unsigned (&v)[8]) {
  asm volatile("" : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]),
               "+r"(v[6]), "+r"(v[7]));
}

// D[tmem] (+)= A[tmem] * B[smem desc]; kind::tf32, cta_group::1.
__device__ __forceinline__ void tc_mma_tf32(unsigned d_tmem, unsigned a_tmem,
                                            unsigned long long b_desc, unsigned idesc,
                                            unsigned accumulate) {
  const unsigned z = 0;
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(z), "r"(z), "r"(z), "r"(z)
      : "memory");
}

__device__ __forceinline__ void tc_commit(unsigned long long* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 2D tiled TMA load of box (x, y) of `map` into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            unsigned long long* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<unsigned long long>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Instruction descriptor: D f32, A/B tf32, both K-major, N = 32, M = 128.
constexpr unsigned kTcIdesc = (1u << 4) | (2u << 7) | (2u << 10) | ((32u >> 3) << 17) |
                              ((128u >> 4) << 24);

// Shared-memory descriptor of a no-swizzle K-major operand: core matrices of 8 rows x 16 B,
// K-adjacent core matrices 128 B apart (LBO), 8-row groups 1024 B apart (SBO), version 1.
__device__ __forceinline__ unsigned long long tc_bdesc(unsigned saddr) {
  return static_cast<unsigned long long>((saddr >> 4) & 0x3FFF) |
         (static_cast<unsigned long long>(128 >> 4) << 16) |
         (static_cast<unsigned long long>(1024 >> 4) << 32) | (1ull << 46);
}

// Float offset of element (k = u, n = w) of a 32 x 32 K-major operand block.
__host__ __device__ __forceinline__ int tc_bofs(int u, int w) {
  return (w >> 3) * 256 + (u >> 2) * 32 + (w & 7) * 4 + (u & 3);
}

// ------------------------------------------------------------------ weight split (per call)

// Wsplit[n] = (hi, lo) of pw_n * W_n[u][w] (oeq order for mul2 = 1: u * 32 + w) in the
// operand layout.  One thread per weight.
struct ArgsTcPrep {
  const float* W;
  float* Wsplit;
  const int* woff;     // [nins] weight offsets
  const float* pw;     // [nins] path weights
  int nins;
};

template <class T>
__global__ void tp_uvw_tc_prep(const ArgsTcPrep v) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= v.nins * 1024) return;
  const int n = t >> 10, e = t & 1023, u = e >> 5, w = e & 31;
  const float x = v.W[v.woff[n] + e] * v.pw[n];
  const float hi = __uint_as_float(tf32_bits(x));
  const float lo = __uint_as_float(tf32_bits(x - hi));
  float* dst = v.Wsplit + static_cast<size_t>(n) * kTcWBlock;
  dst[tc_bofs(u, w)] = hi;
  dst[1024 + tc_bofs(u, w)] = lo;
}

// ------------------------------------------------------------------ compute-warp pieces

struct TcBars {
  unsigned long long *x_full, *x_empty, *w_full, *w_empty, *a_full, *a_empty, *d_full, *d_empty,
      *mma_done;
  unsigned* tmem_slot;
};

__device__ __forceinline__ TcBars tc_bars(unsigned char* smem) {
  TcBars b;
  unsigned long long* p = reinterpret_cast<unsigned long long*>(smem + kTcSmemBars);
  b.x_full = p;
  b.x_empty = p + 2;
  b.w_full = p + 4;
  b.w_empty = p + 4 + kTcWSlots;
  b.a_full = p + 4 + 2 * kTcWSlots;
  b.a_empty = b.a_full + kTcASlots;
  b.d_full = b.a_empty + kTcASlots;
  b.d_empty = b.d_full + 2;
  b.mma_done = b.d_empty + 2;
  b.tmem_slot = reinterpret_cast<unsigned*>(b.mma_done + 1);
  return b;
}

// Barrier wait that lets the thread sleep until the phase completes (suspend-time hint), so
// waiting warps do not compete for issue slots; bounded like mbar_wait.
__device__ __forceinline__ bool tc_try_wait(unsigned long long* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(20000u)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool tc_wait(unsigned long long* bar, unsigned parity, int* status) {
  if (tc_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (;;) {
    if (tc_try_wait(bar, parity)) return true;
    if (status && *reinterpret_cast<volatile int*>(status) == 3) return false;
    if (global_ns() - t0 > kWaitNs) {
      if (status) atomicCAS(status, 0, 3);
      return false;
    }
  }
}

__device__ __forceinline__ bool tc_wait_ring(unsigned long long* bar, unsigned it, unsigned n,
                                            int* status) {
  if (it < n) return true;
  return tc_wait(bar, ((it / n) - 1) & 1, status);
}

// One stage (an input irrep of degree L1): the thread's X values x[8][D1] are in registers;
// runs every instruction of the stage, producing A slots.
template <int L1>
__device__ __forceinline__ void tc_stage_compute(const ArgsTc& a, const TcIns* insv,
                                                 const TcBars& bars,
                                                 const TcStage& st, const float* yrow,
                                                 const float (&x)[8 * (2 * L1 + 1)],
                                                 unsigned tbase_lane, int c, unsigned& a_it,
                                                 int lane) {
  constexpr int D1 = 2 * L1 + 1;
  for (int ni = st.ins_begin; ni < st.ins_end; ++ni) {
    const TcIns in = insv[ni];
    dispatch_bc<L1>(pair_code(in.l2, in.l3), [&]<int L2, int L3>() {
      constexpr int D3 = 2 * L3 + 1;
      float P[D1 * D3];
#pragma unroll
      for (int e = 0; e < D1 * D3; ++e) P[e] = 0.f;
      CG<L1, L2, L3>::pmat(yrow + in.y_off, P);
#pragma unroll
      for (int k = 0; k < D3; ++k) {
        unsigned hi[8], lo[8];
#pragma unroll
        for (int uu = 0; uu < 8; ++uu) {
          float t = 0.f;
#pragma unroll
          for (int i = 0; i < D1; ++i) t = fmaf(P[i * D3 + k], x[uu * D1 + i], t);
          hi[uu] = tf32_bits(t);
          lo[uu] = tf32_bits(t - __uint_as_float(hi[uu]));
        }
        const unsigned s = a_it % kTcASlots;
        tc_wait_ring(&bars.a_empty[s], a_it, kTcASlots, a.status);
        tc_fence_after();
        const unsigned col = tbase_lane + kTcACol0 + 64 * s + 8 * c;
        tmem_st8(col, hi);
        tmem_st8(col + 32, lo);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.a_full[s]);
        ++a_it;
      }
    });
  }
}

// Epilogue of one output irrep: 8 channels x D3 components of this thread's row.
template <int D3>
__device__ __forceinline__ void tc_store_out(const ArgsTc& a, const TcOut& o, unsigned tbase_lane,
                                             int c, long long row, bool valid) {
  float out[8 * D3];
  if (o.has) {
#pragma unroll
    for (int k = 0; k < D3; ++k) {
      unsigned v[8];
      tmem_ld8(tbase_lane + o.dcol + 32 * k + 8 * c, v);
      tmem_wait_ld();
      reg_pin8(v);
#pragma unroll
      for (int j = 0; j < 8; ++j) out[j * D3 + k] = __uint_as_float(v[j]);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8 * D3; ++e) out[e] = 0.f;
  }
  if (valid) {
    float4* dst = reinterpret_cast<float4*>(a.Z + row * a.L3dim + o.z_off + 8 * c * D3);
#pragma unroll
    for (int e = 0; e < 2 * D3; ++e)
      dst[e] = make_float4(out[4 * e], out[4 * e + 1], out[4 * e + 2], out[4 * e + 3]);
  }
}

// ------------------------------------------------------------------ the kernel

template <class T>
__global__ void __launch_bounds__(kTcThreads, 1)
    tp_uvw_tc_fwd(const __grid_constant__ ArgsTc a, const __grid_constant__ CUtensorMap xmap) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // 128-byte swizzled TMA boxes need a 1024-byte aligned destination.
  unsigned char* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const TcBars bars = tc_bars(smem);
  float* ybuf = reinterpret_cast<float*>(smem + kTcSmemY);
  float* wring = reinterpret_cast<float*>(smem + kTcSmemW);
  float* xbuf = reinterpret_cast<float*>(smem + kTcSmemX);
  TcPass* groups = reinterpret_cast<TcPass*>(smem + kTcSmemTab);
  TcStage* stages = reinterpret_cast<TcStage*>(groups + kTcMaxGroups);
  TcIns* insv = reinterpret_cast<TcIns*>(stages + kTcMaxStages);
  TcOut* outs = reinterpret_cast<TcOut*>(insv + kTcMaxIns);
  const long long ntiles = (a.B + kTcRows - 1) / kTcRows;
  const int ng = a.npass;
  const long long nunits = ntiles * ng;

  for (int i = threadIdx.x; i < a.npass; i += blockDim.x) groups[i] = a.passes[i];
  for (int i = threadIdx.x; i < a.nstage; i += blockDim.x) stages[i] = a.stages[i];
  for (int i = threadIdx.x; i < a.nins; i += blockDim.x) insv[i] = a.ins[i];
  for (int i = threadIdx.x; i < a.nout; i += blockDim.x) outs[i] = a.outs[i];
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars.x_full[i], 1);
      mbar_init(&bars.x_empty[i], kTcComputeWarps);
      mbar_init(&bars.d_full[i], 1);
      mbar_init(&bars.d_empty[i], kTcComputeWarps);
    }
    for (int i = 0; i < kTcWSlots; ++i) {
      mbar_init(&bars.w_full[i], 1);
      mbar_init(&bars.w_empty[i], 1);
    }
    for (int i = 0; i < kTcASlots; ++i) {
      mbar_init(&bars.a_full[i], kTcComputeWarps);
      mbar_init(&bars.a_empty[i], 1);
    }
    mbar_init(bars.mma_done, 1);
    fence_mbar_init();
  }
  if (wid == kTcMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
                     smem_u32(bars.tmem_slot)),
                 "n"(kTcTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = *bars.tmem_slot;

  if (wid == kTcProdWarp) {
    // ---------------- X producer: one TMA box per 32 floats of the stage's input block
    if (lane == 0) {
      unsigned xs_it = 0;
      for (long long u = blockIdx.x; u < nunits; u += gridDim.x) {
        const int row0 = static_cast<int>((u / ng) * kTcRows);
        const TcPass gp = groups[u % ng];
        for (int si = gp.stage_begin; si < gp.stage_end; ++si) {
          const TcStage st = stages[si];
          const int nbox = 2 * st.l1 + 1;
          const unsigned b = xs_it & 1;
          tc_wait_ring(&bars.x_empty[b], xs_it, 2, a.status);
          mbar_expect_tx(&bars.x_full[b], static_cast<unsigned>(nbox * kTcXBox * 4));
          float* dst = xbuf + static_cast<size_t>(b) * kTcMaxD * kTcXBox;
          for (int j = 0; j < nbox; ++j)
            tma_load_2d(dst + j * kTcXBox, &xmap, st.x_off + 32 * j, row0, &bars.x_full[b]);
          ++xs_it;
        }
      }
      // Drain (also after a timed-out wait): the last phase issued on each buffer has landed.
      for (unsigned i = xs_it > 2 ? xs_it - 2 : 0; i < xs_it; ++i)
        mbar_wait(&bars.x_full[i & 1], (i >> 1) & 1, nullptr);
    }
    __syncwarp();
  } else if (wid == kTcWProdWarp) {
    // ---------------- W producer: one 8 KiB operand image per instruction
    if (lane == 0) {
      unsigned w_it = 0;
      for (long long u = blockIdx.x; u < nunits; u += gridDim.x) {
        const TcPass gp = groups[u % ng];
        for (int si = gp.stage_begin; si < gp.stage_end; ++si) {
          const TcStage st = stages[si];
          for (int ni = st.ins_begin; ni < st.ins_end; ++ni) {
            const unsigned ws = w_it % kTcWSlots;
            tc_wait_ring(&bars.w_empty[ws], w_it, kTcWSlots, a.status);
            mbar_expect_tx(&bars.w_full[ws], kTcWBlock * 4);
            bulk_g2s(wring + ws * kTcWBlock,
                     a.Wsplit + static_cast<size_t>(insv[ni].wblk) * kTcWBlock, kTcWBlock * 4,
                     &bars.w_full[ws]);
            ++w_it;
          }
        }
      }
      for (unsigned i = w_it > kTcWSlots ? w_it - kTcWSlots : 0; i < w_it; ++i)  // drain
        mbar_wait(&bars.w_full[i % kTcWSlots], (i / kTcWSlots) & 1, nullptr);
    }
    __syncwarp();
  } else if (wid == kTcMmaWarp) {
    // ---------------- MMA issuer (one thread); unit i accumulates into D buffer i & 1
    if (lane == 0) {
      unsigned a_it = 0, w_it = 0, it = 0;
      const unsigned long long wdesc0 = tc_bdesc(smem_u32(wring));
      for (long long u = blockIdx.x; u < nunits; u += gridDim.x, ++it) {
        const TcPass gp = groups[u % ng];
        const unsigned db = it & 1;
        if (it >= 2) tc_wait(&bars.d_empty[db], ((it >> 1) - 1) & 1, a.status);
        tc_fence_after();
        for (int si = gp.stage_begin; si < gp.stage_end; ++si) {
          const TcStage st = stages[si];
          for (int ni = st.ins_begin; ni < st.ins_end; ++ni) {
            const TcIns in = insv[ni];
            const unsigned ws = w_it % kTcWSlots;
            tc_wait(&bars.w_full[ws], (w_it / kTcWSlots) & 1, a.status);
            // Start-address field advances in 16-byte units: slot ws at ws * 8 KiB, lo half at
            // +4 KiB, K step ks at +256 B.
            const unsigned long long dh = wdesc0 + ws * (kTcWBlock * 4 / 16);
            const unsigned long long dl = dh + 4096 / 16;
            const int d3 = 2 * in.l3 + 1;
            const unsigned dcol0 = tmem + db * kTcDCols + in.dcol;
            for (int k = 0; k < d3; ++k) {
              const unsigned s = a_it % kTcASlots;
              tc_wait(&bars.a_full[s], (a_it / kTcASlots) & 1, a.status);
              tc_fence_after();
              const unsigned dcol = dcol0 + 32 * k;
              const unsigned acol = tmem + kTcACol0 + 64 * s;
              tc_mma_tf32(dcol, acol, dh, kTcIdesc, in.first ? 0u : 1u);
              tc_mma_tf32(dcol, acol, dl, kTcIdesc, 1u);
              tc_mma_tf32(dcol, acol + 32, dh, kTcIdesc, 1u);
#pragma unroll
              for (int ks = 1; ks < 4; ++ks) {
                tc_mma_tf32(dcol, acol + 8 * ks, dh + 16 * ks, kTcIdesc, 1u);
                tc_mma_tf32(dcol, acol + 8 * ks, dl + 16 * ks, kTcIdesc, 1u);
                tc_mma_tf32(dcol, acol + 32 + 8 * ks, dh + 16 * ks, kTcIdesc, 1u);
              }
              tc_commit(&bars.a_empty[s]);
              ++a_it;
            }
            tc_commit(&bars.w_empty[ws]);
            ++w_it;
          }
        }
        tc_commit(&bars.d_full[db]);
      }
      // Every MMA of this thread has completed before TMEM is released (also when a wait
      // timed out and the pipeline ran on without its handshakes).
      tc_commit(bars.mma_done);
      mbar_wait(bars.mma_done, 0, nullptr);
    }
    __syncwarp();
  } else {
    // ---------------- compute warps: A slots of unit i, then the epilogue of unit i - 1
    const int q = wid & 3, c = wid >> 2;
    const int rl = 32 * q + lane;  // row within the tile
    const unsigned tbase_lane = tmem + (static_cast<unsigned>(32 * q) << 16);
    unsigned a_it = 0, xs_it = 0, it = 0;
    long long prev_row = 0;
    int prev_g = 0;
    auto epilogue = [&](unsigned pit, int g, long long row) {
      const unsigned db = pit & 1;
      tc_wait(&bars.d_full[db], (pit >> 1) & 1, a.status);
      tc_fence_after();
      const TcPass gp = groups[g];
      const unsigned dbase = tbase_lane + db * kTcDCols;
      const bool valid = row < a.B;
      for (int oi = gp.out_begin; oi < gp.out_end; ++oi) {
        const TcOut o = outs[oi];
        if (o.d3 == 1)
          tc_store_out<1>(a, o, dbase, c, row, valid);
        else if (o.d3 == 3)
          tc_store_out<3>(a, o, dbase, c, row, valid);
        else
          tc_store_out<5>(a, o, dbase, c, row, valid);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars.d_empty[db]);
    };
    for (long long u = blockIdx.x; u < nunits; u += gridDim.x, ++it) {
      const long long row = (u / ng) * kTcRows + rl;
      const int g = static_cast<int>(u % ng);
      const TcPass gp = groups[g];
      float* yb = ybuf + (it & 1) * kTcRows * kTcYStride;
      if (c == 0) {
        const bool valid = row < a.B;
        for (int j = 0; j < kTcYMax; ++j)
          yb[rl * kTcYStride + j] = (valid && j < a.L2dim) ? a.Y[row * a.L2dim + j] : 0.f;
      }
      asm volatile("bar.sync 1, %0;\n" ::"n"(kTcComputeWarps * 32) : "memory");
      const float* yrow = yb + rl * kTcYStride;
      for (int si = gp.stage_begin; si < gp.stage_end; ++si) {
        const TcStage st = stages[si];
        const unsigned b = xs_it & 1;
        tc_wait(&bars.x_full[b], (xs_it >> 1) & 1, a.status);
        // Row rl of box j: 32 floats, 16-byte chunk q stored at chunk q ^ (rl & 7).
        const float* xs = xbuf + static_cast<size_t>(b) * kTcMaxD * kTcXBox + rl * 32;
        dispatch_l(st.l1, [&]<int L1>() {
          if constexpr (L1 <= 2) {
            constexpr int D1 = 2 * L1 + 1;
            float x[8 * D1];
#pragma unroll
            for (int e = 0; e < 2 * D1; ++e) {
              const int f = 8 * c * D1 + 4 * e;  // float index inside the input block
              const float4 t = *reinterpret_cast<const float4*>(
                  xs + (f >> 5) * kTcXBox + ((((f & 31) >> 2) ^ (rl & 7)) << 2));
              x[4 * e] = t.x;
              x[4 * e + 1] = t.y;
              x[4 * e + 2] = t.z;
              x[4 * e + 3] = t.w;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars.x_empty[b]);
            tc_stage_compute<L1>(a, insv, bars, st, yrow, x, tbase_lane, c, a_it, lane);
          }
        });
        ++xs_it;
      }
      if (it > 0) epilogue(it - 1, prev_g, prev_row);
      prev_g = g;
      prev_row = row;
    }
    if (it > 0) epilogue(it - 1, prev_g, prev_row);
  }
  tc_fence_before();
  __syncthreads();
  if (wid == kTcMmaWarp) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem),
                 "n"(kTcTmemCols)
                 : "memory");
  }
}

}  // namespace oeqb
