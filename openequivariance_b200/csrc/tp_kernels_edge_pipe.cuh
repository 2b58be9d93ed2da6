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
// Requirements (checked by the host): float32 rows/cols/W/Y/dY/dW pointers 16-byte aligned;
// per-edge weights with weight_numel == 1.  Bad indices are dropped and raise status 1.
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
  for (int i = lane; i < r * D2; i += 32) st.y[i] = Y[base * D2 + i];
}

// Register image of a gathered D-value row: the 16-byte aligned window that holds it
// (NW float4 loads) and the row's offset in it.  Rows whose window would pass the end of the
// tensor are loaded element by element at offset 0.
template <int D>
struct GatherWin {
  static constexpr int NW = (D + 6) / 4;
  float w[4 * NW];
  int o;

  __device__ __forceinline__ void load(const float* src, long long node, long long nodes, bool valid) {
    o = 0;
    if (!valid) {
#pragma unroll
      for (int i = 0; i < 4 * NW; ++i) w[i] = 0.f;
      return;
    }
    const long long f = node * D;
    const int off = static_cast<int>(f & 3);
    const long long b4 = f - off;
    if (b4 + 4 * NW <= nodes * D) {
      o = off;
#pragma unroll
      for (int q = 0; q < NW; ++q) {
        const float4 t = __ldg(reinterpret_cast<const float4*>(src + b4) + q);
        w[4 * q] = t.x;
        w[4 * q + 1] = t.y;
        w[4 * q + 2] = t.z;
        w[4 * q + 3] = t.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < D; ++i) w[i] = src[f + i];
#pragma unroll
      for (int i = D; i < 4 * NW; ++i) w[i] = 0.f;
    }
  }

  __device__ __forceinline__ void get(float (&v)[D]) const {
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
  }
};

constexpr int kPipeStages = 3;

template <int D2>
__host__ __device__ constexpr size_t pipe_warp_bytes() {
  return sizeof(PipeStage<D2>) * kPipeStages;
}

// Range check of a staged edge (bad indices raise status 1 and drop the edge).
__device__ __forceinline__ bool pipe_valid(long long row, long long col, long long nodes,
                                           int* status) {
  if (row == -1) return false;  // past the end of the edge list
  if (row < 0 || row >= nodes || col < 0 || col >= nodes) {
    flag(status, 1);
    return false;
  }
  return true;
}

template <class T>
__global__ void __launch_bounds__(kEdgeWarps * 32) conv_fwd_edge1_pipe(const Args<T> a, const Edge1 p) {
  static_assert(sizeof(T) == 4, "float32 only");
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x & 31;
  const long long nw = static_cast<long long>(gridDim.x) * kEdgeWarps;
  const long long n = a.nitems;
  const float pw = static_cast<float>(p.pw);
  dispatch_triple(p.code, [&]<int A, int B, int C>() {
    constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1, D3 = 2 * C + 1;
    auto* ring = reinterpret_cast<PipeStage<D2>*>(smem + (threadIdx.x >> 5) * pipe_warp_bytes<D2>());
    const long long step = nw * 32;
    long long base = (static_cast<long long>(blockIdx.x) * kEdgeWarps + (threadIdx.x >> 5)) * 32;
    if (base >= n) return;
    // Prologue: blocks 0 and 1 in flight, block 0's gathers issued.
    pipe_stage_in<D2>(ring[0], a.rows, a.cols, a.W, a.Y, base, n, lane);
    cp_async_commit();
    pipe_stage_in<D2>(ring[1], a.rows, a.cols, a.W, a.Y, base + step, n, lane);
    cp_async_commit();
    cp_async_wait<1>();
    __syncwarp();
    bool vc = pipe_valid(ring[0].rows[lane], ring[0].cols[lane], a.nnodes, a.status);
    GatherWin<D1> xc;
    xc.load(a.X, ring[0].cols[lane], a.nnodes, vc);
    int s = 0;
    for (; base < n; base += step) {
      const int s1 = s == kPipeStages - 1 ? 0 : s + 1;
      const int s2 = s1 == kPipeStages - 1 ? 0 : s1 + 1;
      // Block k+2 into the stage block k-1 used; block k+1 has landed after this wait.
      pipe_stage_in<D2>(ring[s2], a.rows, a.cols, a.W, a.Y, base + 2 * step, n, lane);
      cp_async_commit();
      cp_async_wait<1>();
      __syncwarp();
      const bool more = base + step < n;
      bool vn = false;
      GatherWin<D1> xn;
      if (more) vn = pipe_valid(ring[s1].rows[lane], ring[s1].cols[lane], a.nnodes, a.status);
      xn.load(a.X, more ? ring[s1].cols[lane] : 0, a.nnodes, vn);
      // Block k.
      const PipeStage<D2>& st = ring[s];
      const long long row = vc ? st.rows[lane] : -1;
      float z[D3];
#pragma unroll
      for (int k = 0; k < D3; ++k) z[k] = 0.f;
      if (vc) {
        float x[D1], y[D2];
        xc.get(x);
        const float w = st.w[lane] * pw;
#pragma unroll
        for (int i = 0; i < D1; ++i) x[i] *= w;
#pragma unroll
        for (int j = 0; j < D2; ++j) y[j] = st.y[lane * D2 + j];
        CG<A, B, C>::fwd(x, y, z);
      }
      const int r32 = static_cast<int>(row);
      const int prev = __shfl_up_sync(0xffffffffu, r32, 1);
      const bool head = row >= 0 && (lane == 0 || prev != r32);
      e1_seg_sum<float, D3>(z, r32, lane);
      if (head) red_vec(a.out0 + row * D3, z);
      __syncwarp();  // every lane is done with stage s before it is refilled
      xc = xn;
      vc = vn;
      s = s1;
    }
    cp_async_wait<0>();
  });
}

// Backward: per edge dY = w evec(g, x), dW = x . hvec(g, y), dX[col] += w hvec(g, y), with
// g = pw dZ[row].  dY and dW leave through a per-warp staging buffer as coalesced 16-byte
// stores; dX is one vector reduction per edge.
template <int D2>
__host__ __device__ constexpr size_t pipe_bwd_warp_bytes() {
  return pipe_warp_bytes<D2>() + sizeof(float) * 32 * (D2 + 1);
}

template <class T>
__global__ void __launch_bounds__(kEdgeWarps * 32) conv_bwd_edge1_pipe(const Args<T> a, const Edge1 p) {
  static_assert(sizeof(T) == 4, "float32 only");
  extern __shared__ __align__(16) unsigned char smem[];
  const int lane = threadIdx.x & 31;
  const long long nw = static_cast<long long>(gridDim.x) * kEdgeWarps;
  const long long n = a.nitems;
  const float pw = static_cast<float>(p.pw);
  dispatch_triple(p.code, [&]<int A, int B, int C>() {
    constexpr int D1 = 2 * A + 1, D2 = 2 * B + 1, D3 = 2 * C + 1;
    unsigned char* wbase = smem + (threadIdx.x >> 5) * pipe_bwd_warp_bytes<D2>();
    auto* ring = reinterpret_cast<PipeStage<D2>*>(wbase);
    float* yo = reinterpret_cast<float*>(wbase + pipe_warp_bytes<D2>());  // [32 * D2] dY
    float* wo = yo + 32 * D2;                                              // [32] dW
    const long long step = nw * 32;
    long long base = (static_cast<long long>(blockIdx.x) * kEdgeWarps + (threadIdx.x >> 5)) * 32;
    if (base >= n) return;
    pipe_stage_in<D2>(ring[0], a.rows, a.cols, a.W, a.Y, base, n, lane);
    cp_async_commit();
    pipe_stage_in<D2>(ring[1], a.rows, a.cols, a.W, a.Y, base + step, n, lane);
    cp_async_commit();
    cp_async_wait<1>();
    __syncwarp();
    bool vc = pipe_valid(ring[0].rows[lane], ring[0].cols[lane], a.nnodes, a.status);
    GatherWin<D1> xc;
    GatherWin<D3> gc;
    xc.load(a.X, ring[0].cols[lane], a.nnodes, vc);
    gc.load(a.Gz, ring[0].rows[lane], a.nnodes, vc);
    int s = 0;
    for (; base < n; base += step) {
      const int s1 = s == kPipeStages - 1 ? 0 : s + 1;
      const int s2 = s1 == kPipeStages - 1 ? 0 : s1 + 1;
      pipe_stage_in<D2>(ring[s2], a.rows, a.cols, a.W, a.Y, base + 2 * step, n, lane);
      cp_async_commit();
      cp_async_wait<1>();
      __syncwarp();
      const bool more = base + step < n;
      bool vn = false;
      if (more) vn = pipe_valid(ring[s1].rows[lane], ring[s1].cols[lane], a.nnodes, a.status);
      GatherWin<D1> xn;
      GatherWin<D3> gn;
      xn.load(a.X, more ? ring[s1].cols[lane] : 0, a.nnodes, vn);
      gn.load(a.Gz, more ? ring[s1].rows[lane] : 0, a.nnodes, vn);
      // Block k.
      const PipeStage<D2>& st = ring[s];
      float h[D1], ev[D2];
      float sdot = 0.f;
#pragma unroll
      for (int i = 0; i < D1; ++i) h[i] = 0.f;
#pragma unroll
      for (int j = 0; j < D2; ++j) ev[j] = 0.f;
      const long long col = st.cols[lane];
      if (vc) {
        float x[D1], y[D2], g[D3];
        xc.get(x);
        gc.get(g);
#pragma unroll
        for (int k = 0; k < D3; ++k) g[k] *= pw;
#pragma unroll
        for (int j = 0; j < D2; ++j) y[j] = st.y[lane * D2 + j];
        CG<A, B, C>::hvec(g, y, h);
        CG<A, B, C>::evec(g, x, ev);
        const float w = st.w[lane];
#pragma unroll
        for (int i = 0; i < D1; ++i) {
          sdot += x[i] * h[i];
          h[i] *= w;
        }
#pragma unroll
        for (int j = 0; j < D2; ++j) ev[j] *= w;
      }
#pragma unroll
      for (int j = 0; j < D2; ++j) yo[lane * D2 + j] = ev[j];
      wo[lane] = sdot;
      __syncwarp();
      e1_stage_out<float, D2>(a.out1, yo, base, n, lane);
      e1_stage_out<float, 1>(a.out2, wo, base, n, lane);
      if (vc) red_vec(a.out0 + col * D1, h);
      __syncwarp();  // stage s and the output buffer are free again
      xc = xn;
      gc = gn;
      vc = vn;
      s = s1;
    }
    cp_async_wait<0>();
  });
}

}  // namespace oeqb
