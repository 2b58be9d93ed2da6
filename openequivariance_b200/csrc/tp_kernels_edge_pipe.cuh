// Software-pipelined single-path convolution kernels (atomic mode) for the C3 class: one uvu
// instruction whose irreps are the whole X, Y, Z rows, all of multiplicity 1, with one weight
// per edge (BASELINE C3: 1x2e x 1x3e -> 1x2e).
//
// Same work mapping as conv_fwd_edge1 / conv_bwd_edge1 (a warp owns 32 consecutive
// receiver-sorted edges per step, one edge per lane), but each warp keeps three 32-edge blocks
// in flight instead of one:
//   * the streamed per-edge data (rows, cols, W, Y: 48 bytes per edge in float32) of block k+2
//     is copied into a per-warp shared-memory ring with cp.async (16-byte chunks, no register
//     round trip), two blocks ahead of the compute;
//   * the gathers of block k+1 (X[col], and dZ[row] in the backward) are issued as soon as its
//     indices have landed, one block ahead, into registers that are first read when block k+1
//     is computed;
//   * block k is contracted, segment-summed over equal receivers (forward) and reduced into
//     global memory with vector reductions.
// The kernels this replaces waited on the index loads, then on the dependent gathers, once
// per 32 edges, with nothing else in flight (long-scoreboard stalls of ~11 per issue).
//
// Node arrays (X, dZ, and the dX accumulator) are read and written in a padded layout of
// 32-byte rows (workspace, filled by conv_pad_rows / emptied by conv_unpad_rows), so every
// gather and every reduction touches one aligned sector.
//
// Requirements (checked by the host): float32; rows/cols/W/Y/dY/dW pointers 16-byte aligned;
// per-edge weights with weight_numel == 1; D1, D3 <= 8.  Bad indices are dropped and raise
// status 1.
#pragma once

#include "tp_kernels_edge.cuh"

namespace oeqb {

// cp.async of one 16-byte chunk global -> shared (L2 only, bypassing L1).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// One warp's stage of the ring: the per-edge data of a 32-edge block.
template <int D2>
struct PipeStage {
  long long rows[32];
  long long cols[32];
  float w[32];
  float y[32 * D2];
};

// Copies block [base, base + 32) of rows / cols / W / Y into stage `st`.  Full blocks go as
// 16-byte cp.async chunks (the caller commits the group); the tail block of the edge list is
// copied with plain loads (entries past the end get row -1).
template <int D2>
__device__ __forceinline__ void pipe_stage_in(PipeStage<D2>& st, const long long* rows,
                                              const long long* cols, const float* W,
                                              const float* Y, long long base, long long n,
                                              int lane) {
  if (base >= n) return;
  if (base + 32 <= n) {
    constexpr int kIdx = 32 * 8 / 16;           // chunks of rows (and of cols)
    constexpr int kW = 32 * 4 / 16;
    constexpr int kY = 32 * D2 * 4 / 16;
    constexpr int kAll = 2 * kIdx + kW + kY;
    const char* src_r = reinterpret_cast<const char*>(rows + base);
    const char* src_c = reinterpret_cast<const char*>(cols + base);
    const char* src_w = reinterpret_cast<const char*>(W + base);
    const char* src_y = reinterpret_cast<const char*>(Y + base * D2);
    char* dst = reinterpret_cast<char*>(&st);
#pragma unroll
    for (int q0 = 0; q0 < kAll; q0 += 32) {
      const int q = q0 + lane;
      if (q < kAll) {
        const char* s;
        if (q < kIdx)
          s = src_r + 16 * q;
        else if (q < 2 * kIdx)
          s = src_c + 16 * (q - kIdx);
        else if (q < 2 * kIdx + kW)
          s = src_w + 16 * (q - 2 * kIdx);
        else
          s = src_y + 16 * (q - 2 * kIdx - kW);
        cp_async16(dst + 16 * q, s);
      }
    }
    return;
  }
  const int r = static_cast<int>(n - base);
  const long long e = base + lane;
  st.rows[lane] = lane < r ? rows[e] : -1;
  st.cols[lane] = lane < r ? cols[e] : 0;
  st.w[lane] = lane < r ? W[e] : 0.f;
#pragma unroll 1
  for (int i = lane; i < 32 * D2; i += 32) st.y[i] = i < r * D2 ? Y[base * D2 + i] : 0.f;
}

// Node rows in the padded layout of these kernels: row n of a [nodes, D] tensor (D <= 8) at
// n * 8 floats, 32-byte aligned, so a gather is one load of one sector: a 16-byte load for
// D <= 4, a 32-byte load (ld.global.v8, sm_100) above, with no alignment arithmetic on the lane.
constexpr int kPadRow = 8;

template <int D>
__device__ __forceinline__ void load_row8(float (&v)[D], const float* src, long long node) {
  static_assert(D <= kPadRow, "row wider than the padded layout");
  const float* r = src + node * kPadRow;
  if constexpr (D > 4) {
    float t[8];
    ldg_v8(t, r);
#pragma unroll
    for (int i = 0; i < D; ++i) v[i] = t[i];
  } else {
    const float4 t = __ldg(reinterpret_cast<const float4*>(r));
    const float u[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
    for (int i = 0; i < D; ++i) v[i] = u[i];
  }
}

template <int D>
__device__ __forceinline__ void zero_row(float (&v)[D]) {
#pragma unroll
  for (int i = 0; i < D; ++i) v[i] = 0.f;
}

// Copies [nodes, D] rows into the padded layout (zero tails).  The backward pads X and dZ and
// clears the padded dX accumulator in one launch.
__global__ void conv_pad_rows(const float* __restrict__ a, int da, float* __restrict__ pa,
                              const float* __restrict__ b, int db, float* __restrict__ pb,
                              float* __restrict__ zero, long long nodes) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
       t < nodes * kPadRow; t += stride) {
    const long long n = t / kPadRow;
    const int i = static_cast<int>(t - n * kPadRow);
    pa[t] = i < da ? a[n * da + i] : 0.f;
    if (pb) pb[t] = i < db ? b[n * db + i] : 0.f;
    if (zero) zero[t] = 0.f;
  }
}

// dX [nodes, D] from the padded accumulator.
__global__ void conv_unpad_rows(const float* __restrict__ src, float* __restrict__ dst, int d,
                                long long nodes) {
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long t = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
       t < nodes * d; t += stride) {
    const long long n = t / d;
    dst[t] = src[n * kPadRow + (t - n * d)];
  }
}

// Adds D values into a padded (32-byte aligned) row: one 16-byte vector reduction and the
// rest in the same sector.
template <int D>
__device__ __forceinline__ void red_row8(float* dst, const float (&v)[D]) {
  if constexpr (D >= 4) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"l"(dst), "f"(v[0]),
                 "f"(v[1]), "f"(v[2]), "f"(v[3])
                 : "memory");
    if constexpr (D >= 6) {
      asm volatile("red.global.add.v2.f32 [%0], {%1, %2};\n" ::"l"(dst + 4), "f"(v[4]), "f"(v[5])
                   : "memory");
      if constexpr (D == 7) atomic_add(dst + 6, v[6]);
    } else if constexpr (D == 5) {
      atomic_add(dst + 4, v[4]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < D; ++i) atomic_add(dst + i, v[i]);
  }
}

constexpr int kPipeStages = 3;

template <int D2>
__host__ __device__ constexpr size_t pipe_warp_bytes() {
  return sizeof(PipeStage<D2>) * kPipeStages;
}

// Validity of a staged edge: in_range = its position is before the end of the edge list (the
// tail stage pads with row -1); an in-range edge with an index outside [0, nodes) raises
// status 1 and is dropped.  One unsigned compare per index covers both bounds.
__device__ __forceinline__ bool pipe_valid(long long row, long long col, long long nodes,
                                           int* status, bool in_range) {
  const bool ok = static_cast<unsigned long long>(row) < static_cast<unsigned long long>(nodes) &&
                  static_cast<unsigned long long>(col) < static_cast<unsigned long long>(nodes);
  if (in_range && !ok) flag(status, 1);
  return in_range && ok;
}

// Coalesced 16-byte stores of a staged full block [32, D] (base + 32 <= n; base a multiple of
// 32, dst 16-byte aligned, src 16-byte aligned shared memory).
template <int D>
__device__ __forceinline__ void stage_out_full(float* dst, const float* src, long long base,
                                               int lane) {
  constexpr int NV = 32 * D / 4;
  float4* g = reinterpret_cast<float4*>(dst + base * D);
  const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
  for (int q0 = 0; q0 < NV; q0 += 32) {
    const int q = q0 + lane;
    if (NV % 32 == 0 || q < NV) g[q] = s4[q];
  }
}

// Backward: per edge dY = w evec(g, x), dW = x . hvec(g, y), dX[col] += w hvec(g, y), with
// g = pw dZ[row].  xp, gp: X and dZ in the padded layout; dxp: the padded dX accumulator
// (zeroed by the caller).  dY and dW leave through a per-warp staging buffer as coalesced
// 16-byte stores; dX is one vector reduction into a 32-byte row per edge.  The X and dZ rows
// of a block are gathered one block ahead.
template <int D2>
__host__ __device__ constexpr size_t pipe_bwd_warp_bytes() {
  return pipe_warp_bytes<D2>() + sizeof(float) * 32 * (D2 + 1);
}

// REC = false: atomic mode, dX reduced into the padded accumulator `out`.  REC = true: pass A
// of the deterministic backward, each edge's message to its sender (D1 values and the
// sender's index in the last of 8 slots: kE1Rec) written to `out` as one 32-byte record, in
// edge order; pass B (conv_bwd_edge1_band and its fix-up) sums them per sender in
// transpose_perm order.
template <int D2, bool REC>
__host__ __device__ constexpr size_t pipe_bwd_warp_bytes_m() {
  return pipe_bwd_warp_bytes<D2>() + (REC ? sizeof(float) * 32 * kE1Rec : 0);
}

template <int A, int B, int C, bool REC>
__global__ void __launch_bounds__(kEdgeWarps * 32) conv_bwd_edge1_pipe(const Args<float> a, const Edge1 p,
                                                                       const float* __restrict__ xp,
                                                                       const float* __restrict__ gp,
                                                                       float* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x & 31;
  const long long nw = static_cast<long long>(gridDim.x) * kEdgeWarps;
  const long long n = a.nitems;
  const float pw = static_cast<float>(p.pw);
  {
    constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1, D3 = 2 * C + 1;
    unsigned char* wbase = smem + (threadIdx.x >> 5) * pipe_bwd_warp_bytes_m<D2, REC>();
    auto* ring = reinterpret_cast<PipeStage<D2>*>(wbase);
    float* yo = reinterpret_cast<float*>(wbase + pipe_warp_bytes<D2>());  // [32 * D2] dY
    float* wo = yo + 32 * D2;                                              // [32] dW
    float* ho = wo + 32;                                                   // [32 * 8] records
    const long long step = nw * 32;
    long long base = (static_cast<long long>(blockIdx.x) * kEdgeWarps + (threadIdx.x >> 5)) * 32;
    if (base >= n) return;
    pipe_stage_in<D2>(ring[0], a.rows, a.cols, a.W, a.Y, base, n, lane);
    cp_async_commit();
    pipe_stage_in<D2>(ring[1], a.rows, a.cols, a.W, a.Y, base + step, n, lane);
    cp_async_commit();
    cp_async_wait<1>();
    __syncwarp();
    bool vc = pipe_valid(ring[0].rows[lane], ring[0].cols[lane], a.nnodes, a.status, base + lane < n);
    float xc[D1], gc[D3];
    if (vc) {
      load_row8<D1>(xc, xp, ring[0].cols[lane]);
      load_row8<D3>(gc, gp, ring[0].rows[lane]);
    } else {
      zero_row(xc);
      zero_row(gc);
    }
    int s = 0;
    for (; base < n; base += step) {
      const int s1 = s == kPipeStages - 1 ? 0 : s + 1;
      const int s2 = s1 == kPipeStages - 1 ? 0 : s1 + 1;
      pipe_stage_in<D2>(ring[s2], a.rows, a.cols, a.W, a.Y, base + 2 * step, n, lane);
      cp_async_commit();
      cp_async_wait<1>();
      __syncwarp();
      // The next block's X and dZ rows are gathered now, a block ahead of their use.
      const PipeStage<D2>& st = ring[s];
      const bool vn = pipe_valid(ring[s1].rows[lane], ring[s1].cols[lane], a.nnodes, a.status,
                                 base + step + lane < n);
      float xn[D1], gn[D3];
      if (vn) {
        load_row8<D1>(xn, xp, ring[s1].cols[lane]);
        load_row8<D3>(gn, gp, ring[s1].rows[lane]);
      } else {
        zero_row(xn);
        zero_row(gn);
      }
      float g[D3];
#pragma unroll
      for (int k = 0; k < D3; ++k) g[k] = gc[k];
      // Block k.  The contraction runs on every lane: a dropped edge has g = x = 0 (and the
      // tail stage pads Y and W with zeros), so its h, dY and dW are zero.
      const long long col = st.cols[lane];
      float h[D1], ev[D2], y[D2];
#pragma unroll
      for (int k = 0; k < D3; ++k) g[k] *= pw;
#pragma unroll
      for (int j = 0; j < D2; ++j) y[j] = st.y[lane * D2 + j];
      CG<A, B, C>::hvec(g, y, h);
      CG<A, B, C>::evec(g, xc, ev);
      const float w = st.w[lane];
      float sdot = 0.f;
#pragma unroll
      for (int i = 0; i < D1; ++i) {
        sdot += xc[i] * h[i];
        h[i] *= w;
      }
#pragma unroll
      for (int j = 0; j < D2; ++j) yo[lane * D2 + j] = ev[j] * w;
      wo[lane] = sdot;
      if constexpr (REC) {
        float r8[kE1Rec];
#pragma unroll
        for (int i = 0; i < kE1Rec - 1; ++i) r8[i] = i < D1 ? h[i] : 0.f;
        r8[kE1Rec - 1] = e1_key_bits<float>(vc ? col : -1);
        float4* hr = reinterpret_cast<float4*>(ho + lane * kE1Rec);
        hr[0] = make_float4(r8[0], r8[1], r8[2], r8[3]);
        hr[1] = make_float4(r8[4], r8[5], r8[6], r8[7]);
      }
      __syncwarp();
      if (base + 32 <= n) {
        stage_out_full<D2>(a.out1, yo, base, lane);
        stage_out_full<1>(a.out2, wo, base, lane);
        if constexpr (REC) stage_out_full<kE1Rec>(out, ho, base, lane);
      } else {
        e1_stage_out<float, D2>(a.out1, yo, base, n, lane);
        e1_stage_out<float, 1>(a.out2, wo, base, n, lane);
        if constexpr (REC) e1_stage_out<float, kE1Rec>(out, ho, base, n, lane);
      }
      if constexpr (!REC)
        if (vc) red_row8<D1>(out + col * kPadRow, h);
      __syncwarp();  // stage s and the output buffers are free again
#pragma unroll
      for (int i = 0; i < D1; ++i) xc[i] = xn[i];
#pragma unroll
      for (int k = 0; k < D3; ++k) gc[k] = gn[k];
      vc = vn;
      s = s1;
    }
    cp_async_wait<0>();
  }
}

// Atomic forward with two edges per lane: a warp takes 64 consecutive edges per step, lane l
// edges 2l and 2l+1, which nearly always share a receiver.  The lane adds its two messages
// when they do, so one segmented shuffle sum serves 64 edges (it is a third of the one-edge
// kernel's instructions); where the pair straddles a receiver boundary the first message goes
// to its receiver with its own vector reduction.  The stage ring, the padded X gathers one
// step ahead and the tail handling are as in conv_bwd_edge1_pipe, with 64-edge stages.
template <int D2>
struct PipeStage2 {
  long long rows[64];
  long long cols[64];
  float w[64];
  float y[64 * D2];
};

template <int D2>
__host__ __device__ constexpr size_t pipe2_warp_bytes() {
  return sizeof(PipeStage2<D2>) * kPipeStages;
}

template <int D2>
__device__ __forceinline__ void pipe2_stage_in(PipeStage2<D2>& st, const long long* rows,
                                               const long long* cols, const float* W,
                                               const float* Y, long long base, long long n,
                                               int lane) {
  if (base >= n) return;
  if (base + 64 <= n) {
    constexpr int kIdx = 64 * 8 / 16;
    constexpr int kW = 64 * 4 / 16;
    constexpr int kY = 64 * D2 * 4 / 16;
    constexpr int kAll = 2 * kIdx + kW + kY;
    const char* src_r = reinterpret_cast<const char*>(rows + base);
    const char* src_c = reinterpret_cast<const char*>(cols + base);
    const char* src_w = reinterpret_cast<const char*>(W + base);
    const char* src_y = reinterpret_cast<const char*>(Y + base * D2);
    char* dst = reinterpret_cast<char*>(&st);
#pragma unroll
    for (int q0 = 0; q0 < kAll; q0 += 32) {
      const int q = q0 + lane;
      if (q < kAll) {
        const char* s;
        if (q < kIdx)
          s = src_r + 16 * q;
        else if (q < 2 * kIdx)
          s = src_c + 16 * (q - kIdx);
        else if (q < 2 * kIdx + kW)
          s = src_w + 16 * (q - 2 * kIdx);
        else
          s = src_y + 16 * (q - 2 * kIdx - kW);
        cp_async16(dst + 16 * q, s);
      }
    }
    return;
  }
  const int r = static_cast<int>(n - base);
  for (int i = lane; i < 64; i += 32) {
    st.rows[i] = i < r ? rows[base + i] : -1;
    st.cols[i] = i < r ? cols[base + i] : 0;
    st.w[i] = i < r ? W[base + i] : 0.f;
  }
#pragma unroll 1
  for (int i = lane; i < 64 * D2; i += 32) st.y[i] = i < r * D2 ? Y[base * D2 + i] : 0.f;
}

template <int A, int B, int C>
__global__ void __launch_bounds__(kEdgeWarps * 32) conv_fwd_edge1_pipe2(const Args<float> a, const Edge1 p,
                                                                        const float* __restrict__ xp) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x & 31;
  const long long nw = static_cast<long long>(gridDim.x) * kEdgeWarps;
  const long long n = a.nitems;
  const float pw = static_cast<float>(p.pw);
  constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1, D3 = 2 * C + 1;
  auto* ring = reinterpret_cast<PipeStage2<D2>*>(smem + (threadIdx.x >> 5) * pipe2_warp_bytes<D2>());
  const long long step = nw * 64;
  long long base = (static_cast<long long>(blockIdx.x) * kEdgeWarps + (threadIdx.x >> 5)) * 64;
  if (base >= n) return;
  const int e0 = 2 * lane, e1 = 2 * lane + 1;
  pipe2_stage_in<D2>(ring[0], a.rows, a.cols, a.W, a.Y, base, n, lane);
  cp_async_commit();
  pipe2_stage_in<D2>(ring[1], a.rows, a.cols, a.W, a.Y, base + step, n, lane);
  cp_async_commit();
  cp_async_wait<1>();
  __syncwarp();
  bool v0c = pipe_valid(ring[0].rows[e0], ring[0].cols[e0], a.nnodes, a.status, base + e0 < n);
  bool v1c = pipe_valid(ring[0].rows[e1], ring[0].cols[e1], a.nnodes, a.status, base + e1 < n);
  float x0c[D1], x1c[D1];
  if (v0c) load_row8<D1>(x0c, xp, ring[0].cols[e0]); else zero_row(x0c);
  if (v1c) load_row8<D1>(x1c, xp, ring[0].cols[e1]); else zero_row(x1c);
  int s = 0;
  for (; base < n; base += step) {
    const int s1 = s == kPipeStages - 1 ? 0 : s + 1;
    const int s2 = s1 == kPipeStages - 1 ? 0 : s1 + 1;
    pipe2_stage_in<D2>(ring[s2], a.rows, a.cols, a.W, a.Y, base + 2 * step, n, lane);
    cp_async_commit();
    cp_async_wait<1>();
    __syncwarp();
    const bool v0n = pipe_valid(ring[s1].rows[e0], ring[s1].cols[e0], a.nnodes, a.status,
                                base + step + e0 < n);
    const bool v1n = pipe_valid(ring[s1].rows[e1], ring[s1].cols[e1], a.nnodes, a.status,
                                base + step + e1 < n);
    float x0n[D1], x1n[D1];
    if (v0n) load_row8<D1>(x0n, xp, ring[s1].cols[e0]); else zero_row(x0n);
    if (v1n) load_row8<D1>(x1n, xp, ring[s1].cols[e1]); else zero_row(x1n);
    const PipeStage2<D2>& st = ring[s];
    const long long r0 = v0c ? st.rows[e0] : -1, r1 = v1c ? st.rows[e1] : -1;
    // Both contractions run on every lane: a dropped edge has x = 0 (and the tail stage pads Y
    // and W with zeros), so its message is zero.
    float z0[D3], z1[D3];
#pragma unroll
    for (int k = 0; k < D3; ++k) z0[k] = z1[k] = 0.f;
    {
      float x[D1], y[D2];
      const float w = st.w[e0] * pw;
#pragma unroll
      for (int i = 0; i < D1; ++i) x[i] = x0c[i] * w;
#pragma unroll
      for (int j = 0; j < D2; ++j) y[j] = st.y[e0 * D2 + j];
      CG<A, B, C>::fwd(x, y, z0);
    }
    {
      float x[D1], y[D2];
      const float w = st.w[e1] * pw;
#pragma unroll
      for (int i = 0; i < D1; ++i) x[i] = x1c[i] * w;
#pragma unroll
      for (int j = 0; j < D2; ++j) y[j] = st.y[e1 * D2 + j];
      CG<A, B, C>::fwd(x, y, z1);
    }
    // The pair shares a receiver: one message.  Otherwise the first edge ends its receiver's
    // run inside this lane and is reduced on its own.
    if (r0 >= 0 && r0 == r1) {
#pragma unroll
      for (int k = 0; k < D3; ++k) z1[k] += z0[k];
    } else if (r0 >= 0) {
      red_vec(a.out0 + r0 * D3, z0);
    }
    const int k32 = static_cast<int>(r1);
    const int prev = __shfl_up_sync(0xffffffffu, k32, 1);
    const bool head = r1 >= 0 && (lane == 0 || prev != k32);
    e1_seg_sum<float, D3>(z1, k32, lane);
    if (head) red_vec(a.out0 + r1 * D3, z1);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < D1; ++i) {
      x0c[i] = x0n[i];
      x1c[i] = x1n[i];
    }
    v0c = v0n;
    v1c = v1n;
    s = s1;
  }
  cp_async_wait<0>();
}

// Deterministic forward, two edges per lane.  Warp w owns the edges of whole receivers: its
// nominal range [w E / W, (w+1) E / W) moved forward to receiver boundaries, walked in 64-edge
// blocks from the 4-aligned edge at or below the range start (so Y rows start 16-byte aligned;
// edges outside the range are masked).  Lane l holds edges 2l and 2l+1 (keys a <= b, the
// receivers).  When a == b the lane sums its pair.  Otherwise edge 2l ends run a inside the
// lane: its message goes to lane l-1 when that lane's second edge is in the same run (added
// to that lane's value, so the run's shuffle-tree sum includes it), and is stored as a
// complete row when the run has no other edge in this block (or, on lane 0, added to the
// sum carried from the previous block).  The lanes' second-edge runs are then summed as in
// conv_fwd_edge1_det: a segmented shuffle tree per block, sums of runs that continue into the
// next block carried in registers, and every receiver row written once with plain stores, in
// an order fixed by the partition (the grid is the device's resident CTAs), not by timing.
template <int A, int B, int C>
__global__ void __launch_bounds__(kEdgeWarps * 32) conv_fwd_edge1_det_pipe2(const Args<float> a, const Edge1 p,
                                                                            const float* __restrict__ xp) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x & 31;
  const long long nwarps = static_cast<long long>(gridDim.x) * kEdgeWarps;
  const long long wg = static_cast<long long>(blockIdx.x) * kEdgeWarps + (threadIdx.x >> 5);
  const long long n = a.nitems;
  const float pw = static_cast<float>(p.pw);
  auto key = [&](long long e) { return a.rows[e]; };
  const long long p0 = e1_snap(static_cast<long long>((static_cast<__int128>(n) * wg) / nwarps), n, key, lane);
  const long long p1 = e1_snap(static_cast<long long>((static_cast<__int128>(n) * (wg + 1)) / nwarps), n, key, lane);
  if (p0 >= p1) return;
  constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1, D3 = 2 * C + 1;
  auto* ring = reinterpret_cast<PipeStage2<D2>*>(smem + (threadIdx.x >> 5) * pipe2_warp_bytes<D2>());
  const int e0 = 2 * lane, e1 = 2 * lane + 1;
  // Validity of edge e of the block at `base`: inside [p0, p1) with good indices.
  auto valid = [&](const PipeStage2<D2>& st, long long base, int e) {
    const long long t = base + e;
    if (t < p0 || t >= p1) return false;
    return pipe_valid(st.rows[e], st.cols[e], a.nnodes, a.status, true);
  };
  long long base = p0 & ~3LL;
  pipe2_stage_in<D2>(ring[0], a.rows, a.cols, a.W, a.Y, base, p1, lane);
  cp_async_commit();
  pipe2_stage_in<D2>(ring[1], a.rows, a.cols, a.W, a.Y, base + 64, p1, lane);
  cp_async_commit();
  cp_async_wait<1>();
  __syncwarp();
  bool v0c = valid(ring[0], base, e0), v1c = valid(ring[0], base, e1);
  float x0c[D1], x1c[D1];
  if (v0c) load_row8<D1>(x0c, xp, ring[0].cols[e0]); else zero_row(x0c);
  if (v1c) load_row8<D1>(x1c, xp, ring[0].cols[e1]); else zero_row(x1c);
  float carry[D3];
  long long carry_key = -2;
  int s = 0;
  for (; base < p1; base += 64) {
    const int s1 = s == kPipeStages - 1 ? 0 : s + 1;
    const int s2 = s1 == kPipeStages - 1 ? 0 : s1 + 1;
    pipe2_stage_in<D2>(ring[s2], a.rows, a.cols, a.W, a.Y, base + 128, p1, lane);
    cp_async_commit();
    cp_async_wait<1>();
    __syncwarp();
    const bool more = base + 64 < p1;
    const bool v0n = more && valid(ring[s1], base + 64, e0);
    const bool v1n = more && valid(ring[s1], base + 64, e1);
    float x0n[D1], x1n[D1];
    if (v0n) load_row8<D1>(x0n, xp, ring[s1].cols[e0]); else zero_row(x0n);
    if (v1n) load_row8<D1>(x1n, xp, ring[s1].cols[e1]); else zero_row(x1n);
    const PipeStage2<D2>& st = ring[s];
    // Both contractions run on every lane: a masked or dropped edge has x = 0 (and the tail
    // stage pads Y and W with zeros), so its message is zero.
    float z0[D3], z1[D3];
#pragma unroll
    for (int k = 0; k < D3; ++k) z0[k] = z1[k] = 0.f;
    {
      float x[D1], y[D2];
      const float w = st.w[e0] * pw;
#pragma unroll
      for (int i = 0; i < D1; ++i) x[i] = x0c[i] * w;
#pragma unroll
      for (int j = 0; j < D2; ++j) y[j] = st.y[e0 * D2 + j];
      CG<A, B, C>::fwd(x, y, z0);
    }
    {
      float x[D1], y[D2];
      const float w = st.w[e1] * pw;
#pragma unroll
      for (int i = 0; i < D1; ++i) x[i] = x1c[i] * w;
#pragma unroll
      for (int j = 0; j < D2; ++j) y[j] = st.y[e1 * D2 + j];
      CG<A, B, C>::fwd(x, y, z1);
    }
    const long long ka = v0c ? st.rows[e0] : -1, kb = v1c ? st.rows[e1] : -1;
    if (ka >= 0 && ka == kb) {
#pragma unroll
      for (int k = 0; k < D3; ++k) z1[k] += z0[k];
    }
    // Edge 2l ending run ka inside the lane: to lane l-1 if its second edge is in the run.
    const bool endp = ka >= 0 && ka != kb;
    int prev_b = __shfl_up_sync(0xffffffffu, static_cast<int>(kb), 1);
    if (lane == 0) prev_b = -3;
    const bool push = endp && prev_b == static_cast<int>(ka);
    const bool recv = __shfl_down_sync(0xffffffffu, push ? 1 : 0, 1) != 0 && lane < 31;
#pragma unroll
    for (int k = 0; k < D3; ++k) {
      const float t = __shfl_down_sync(0xffffffffu, z0[k], 1);
      if (recv) z1[k] += t;
    }
    if (endp && !push) {
      // Run ka has no other edge in this block: complete, unless lane 0 continues the carry.
      if (lane == 0 && ka == carry_key) {
#pragma unroll
        for (int k = 0; k < D3; ++k) z0[k] = carry[k] + z0[k];
      }
      e1_store_row(a.out0 + ka * D3, z0);
    }
    // First receiver of the next block (edge 0 of its stage), to tell whether the last run
    // continues.
    const long long nk = more ? ring[s1].rows[0] : -3;
    e1_seg_block<float, D3>(z1, kb, nk, more, carry, carry_key, a.out0, lane);
    __syncwarp();
#pragma unroll
    for (int i = 0; i < D1; ++i) {
      x0c[i] = x0n[i];
      x1c[i] = x1n[i];
    }
    v0c = v0n;
    v1c = v1n;
    s = s1;
  }
  cp_async_wait<0>();
}

}  // namespace oeqb
