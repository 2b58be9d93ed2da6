// Host runtime behind the C ABI in include/oeqb200.h: descriptor parsing, plan tables,
// launch configuration and the kernel sequences of every pass.
//
// Kernel sequences follow the reference's JIT wrappers (extension/tensorproducts.hpp:77-116,
// extension/convolution.hpp:79-186): one launch per pass for the batch forward/backward,
// two for the double backward (part A = three forward terms into L3_dgrad, part B = two
// backward terms into the input gradients).  The reference's deterministic convolution
// needs an extra fixup launch per pass; this build snaps each warp's edge range to row
// boundaries instead, so every pass is a single launch.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <set>
#include <type_traits>
#include <string>
#include <unordered_map>
#include <vector>

#include "oeqb200.h"
#include "tp_core.cuh"
#include "tp_kernels_edge.cuh"
#include "tp_kernels_lk.cuh"
#include "tp_kernels_uvw_sw.cuh"
#include "tp_kernels_uvw_tc.cuh"

namespace oeqb {
template <class T>
const void* batch_kernel_ptr(int kind, bool uvw, bool db, int policy);
template <class T>
const void* det_kernel_ptr(int kind, bool uvw, bool db, bool kahan);
template <class T>
const void* row_kernel_ptr(int kind, int nwarps);
template <class T>
const void* seg_kernel_ptr(int kind);
template <class T>
const void* edge1_band_kernel(int l1, bool fix);
template <class T>
const void* lk_kernel_ptr(int cpl);
template <class T>
const void* lkf_kernel_ptr(int cpl);
template <class T>
const void* edge_kernel_ptr(int kind);
const void* uvw_tc_kernel_ptr(int kind);
template <class T>
const void* uvw_sw_kernel_ptr(int kind);
int set_error(int code, const std::string& msg);
// kern_edge_pipe.cu: 0 / 1 = pipelined atomic forward / backward of triple `code`, 2 = pad
// rows, 3 = unpad rows
const void* edge1_pipe_kernel(int kind, int code);
}  // namespace oeqb

using namespace oeqb;


namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

}  // namespace

// Error reporting shared with the other translation units of the library (kern_sc.cu).
int oeqb::set_error(int code, const std::string& msg) { return fail(code, msg); }

namespace {

#define OEQB_CUDA(expr)                                                                  \
  do {                                                                                   \
    cudaError_t e_ = (expr);                                                             \
    if (e_ != cudaSuccess)                                                               \
      return fail(OEQB_ERR_CUDA, std::string(#expr " failed: ") + cudaGetErrorString(e_)); \
  } while (0)

constexpr int64_t kMagic = 0x4251454F;

struct DevArrays {
  size_t ir1, ir2, ir3, ins_f, grp_f, zb_f, ins_b, grp_b, zb_b, cg, total;
};

struct KernelCfg {
  int blocks_per_sm = 0;
};

}  // namespace

struct oeqb_plan {
  int device = 0;
  int dtype = 1;
  int layout = 0;
  int uvw = 0;
  int shared_w = 0;
  int det = 0;
  int kahan = 0;
  int n1 = 0, n2 = 0, n3 = 0, nins = 0;
  int L1dim = 0, L2dim = 0, L3dim = 0, wnumel = 0;
  int lgG = 0;
  std::vector<IrrepD> ir1, ir2, ir3;
  std::vector<InstrD> ins_f, ins_b;
  std::vector<GroupD> grp_f, grp_b;
  std::vector<int> zb_f, zb_b;
  std::vector<CGEntry> cg;
  // Row-staged wide-uvu batch kernels (tp_kernels_row.cuh): items, per-warp lists.
  struct RowTable {
    std::vector<RowItem> items;
    std::vector<int> witems, wofs;
    int nwarps = 8;
    size_t off_items = 0, off_witems = 0, off_wofs = 0;
  } rowf, rowb;
  bool row_ok = false;
  // Channelwise-uvu segment kernels (tp_kernels_seg.cuh): one table image per pass.
  struct SegTable {
    bool ok = false;
    std::vector<unsigned char> blob;  // SegInstr | SegRun | grp | SegX | SegPEnt | SegTerm
    int off_run = 0, off_grp = 0, off_x = 0, off_pent = 0, off_term = 0;
    int ngroups = 1, nsplit = 1, cbs = 1, nx = 0, npent = 0, psize = 0, rows_per_buf = 1, nrun = 0;
    int scratch_off = 0, gyc_off = 0;
    int offY = 0, offW = 0, offG = 0, row_elems = 0;
    size_t smem = 0, dev_off = 0;
  } segf, segb, segl;
  // Lockstep backward (tp_kernels_lk.cuh) over the tables of segl.
  struct LkCfg {
    bool ok = false;
    int nch = 0, cpl = 1, rb = 0, nslots = 0, offY = 0, xy_elems = 0, slot_elems = 0,
        slot_w_off = 0;
    size_t smem = 0;
  } lk, lkf;  // backward, forward
  // Edge-per-lane convolution (tp_kernels_edge.cuh) for multiplicity-1 problems; edge1 = the
  // single-path variant (one instruction whose irreps are the whole rows).
  bool edge_ok = false;
  EdgeLayout edge{};
  bool edge1_ok = false;
  Edge1 edge1{};
  // Tensor-core shared-weight uvw forward (tp_kernels_uvw_tc.cuh).
  struct TcTable {
    bool ok = false;
    std::vector<TcPass> passes;
    std::vector<TcStage> stages;
    std::vector<TcIns> ins;
    std::vector<TcOut> outs;
    std::vector<int> woff;
    std::vector<float> pw;
    size_t off_passes = 0, off_stages = 0, off_ins = 0, off_outs = 0, off_woff = 0, off_pw = 0;
    float* wsplit = nullptr;  // plan-owned operand image of the weights (rewritten per call)
  } tc;
  // Shared-weight uvw backward (tp_kernels_uvw_sw.cuh).
  struct SwTable {
    bool ok = false;
    std::vector<SwGroup> groups;
    std::vector<SwIns> ins;
    std::vector<SwDw> dw;
    std::vector<SwOut> fouts;  // forward (float64): paths grouped by output irrep
    std::vector<SwFIns> fins;
    size_t off_fouts = 0, off_fins = 0;
    std::vector<int> woff;
    std::vector<float> pw_f;
    std::vector<double> pw_d;
    size_t off_groups = 0, off_ins = 0, off_dw = 0, off_woff = 0, off_pw = 0;
    void* wt = nullptr;  // plan-owned W'^T image [nins][32][32] (rewritten per call)
  } sw;

  DevArrays off{};
  unsigned char* dmem = nullptr;
  int* d_status = nullptr;
  int ws_elems = 0, off_t = 0, off_t2 = 0, off_gz = 0, off_dy = 0;
  size_t desc_f = 0, desc_b = 0;
  int sm_count = 148;
  std::mutex mu;
  std::unordered_map<const void*, int> occ;  // kernel -> resident blocks per SM
  size_t elem() const { return dtype == 2 ? 8 : 4; }
};

namespace {

size_t align16(size_t x) { return (x + 15) & ~size_t(15); }

size_t desc_bytes(const oeqb_plan& p, size_t ngrp, size_t nzero) {
  return align16(sizeof(InstrD) * p.nins + sizeof(IrrepD) * (p.n1 + p.n2 + p.n3) +
                 sizeof(GroupD) * ngrp + sizeof(int) * nzero);
}

// Group instructions by the irrep whose output/gradient they produce (stable order).
void make_groups(const std::vector<InstrD>& ins, bool by_out, int nirreps,
                 const std::vector<IrrepD>& irreps, std::vector<InstrD>& out_ins,
                 std::vector<GroupD>& groups, std::vector<int>& zero_blocks) {
  std::vector<InstrD> sorted = ins;
  std::stable_sort(sorted.begin(), sorted.end(), [&](const InstrD& a, const InstrD& b) {
    return by_out ? a.i3 < b.i3 : a.i1 < b.i1;
  });
  out_ins = sorted;
  groups.clear();
  std::vector<char> used(nirreps, 0);
  for (size_t i = 0; i < sorted.size();) {
    const int key = by_out ? sorted[i].i3 : sorted[i].i1;
    size_t j = i;
    while (j < sorted.size() && (by_out ? sorted[j].i3 : sorted[j].i1) == key) ++j;
    GroupD g{key, static_cast<int>(i), static_cast<int>(j - i), 0};
    groups.push_back(g);
    used[key] = 1;
    i = j;
  }
  zero_blocks.clear();
  for (int r = 0; r < nirreps; ++r)
    if (!used[r] && irreps[r].mul > 0) zero_blocks.push_back(r);
}

// Lockstep assignment: every item is one 32-lane chunk, items keep their instruction order
// and are dealt round-robin, so at any moment the warps of a CTA execute the code of the
// same one or two degree triples (the unrolled kernels are large; warps running different
// triples at once thrash the instruction cache).
void schedule_items(oeqb_plan::RowTable& t, const std::vector<double>& /*cost*/) {
  std::vector<RowItem> single;
  for (const RowItem& it : t.items)
    for (int c = it.c0; c < it.c0 + it.nc; ++c) single.push_back(RowItem{it.key, c, 1, 0});
  t.items = single;
  const int nw = t.nwarps;
  t.witems.clear();
  t.wofs.assign(1, 0);
  for (int w = 0; w < nw; ++w) {
    for (size_t i = w; i < t.items.size(); i += nw) t.witems.push_back(static_cast<int>(i));
    t.wofs.push_back(static_cast<int>(t.witems.size()));
  }
}

size_t round_elems(size_t n, size_t elem) {
  const size_t q = 16 / elem;
  return (n + q - 1) / q * q;
}

// Shared-memory bytes of a row kernel launch (must match stage_desc_row / the kernels).
size_t row_smem(const oeqb_plan& p, int kind, int nwarps, size_t elem, int* row_elems,
                int* offY, int* offW, int* offG, int* ws_elems) {
  const auto& t = kind == 0 ? p.rowf : p.rowb;
  const size_t desc = p.desc_f;  // both row kernels stage the forward-order tables
  const size_t tabs = align16(sizeof(RowItem) * t.items.size() + sizeof(int) * t.witems.size() +
                              sizeof(int) * (nwarps + 1));
  *offY = static_cast<int>(round_elems(p.L1dim, elem));
  *offW = *offY + static_cast<int>(round_elems(p.L2dim, elem));
  *offG = *offW + static_cast<int>(p.shared_w ? 0 : round_elems(p.wnumel, elem));
  *row_elems = *offG + static_cast<int>(kind == 1 ? round_elems(p.L3dim, elem) : 0);
  if (kind == 0)
    *ws_elems = 2 * 32 * kDMax;
  else
    *ws_elems = static_cast<int>(round_elems(p.L1dim, elem) + round_elems(p.L2dim, elem));
  return desc + tabs + 16 + 2 * elem * size_t(*row_elems) + size_t(nwarps) * (*ws_elems) * elem;
}

// The row kernels cover uvu problems with a 32-lane group whose degrees are all in the
// unrolled range and whose rows fit in shared memory; everything else runs on the v1
// kernels.
void build_row(oeqb_plan& p) {
  p.row_ok = false;
  if (p.uvw || p.lgG != 5) return;
  for (const InstrD& in : p.ins_f)
    if (in.code < 0) return;
  for (const IrrepD& r : p.ir3)
    if (r.l > kLMaxUnrolled) return;
  auto nnz = [&](const InstrD& in) { return static_cast<double>(in.cg_nnz); };
  p.rowf = {};
  p.rowb = {};
  std::vector<double> cf, cb;
  for (size_t g = 0; g < p.grp_f.size(); ++g) {
    const GroupD& gd = p.grp_f[g];
    const IrrepD& r3 = p.ir3[gd.irrep];
    double c = 2.0 * r3.dim;
    for (int i = gd.first; i < gd.first + gd.count; ++i)
      c += p.ins_f[i].m2 * (2.0 * nnz(p.ins_f[i]) + p.ir2[p.ins_f[i].i2].dim) + p.ir1[p.ins_f[i].i1].dim;
    p.rowf.items.push_back(RowItem{static_cast<int>(g), 0, (r3.mul + 31) / 32, 0});
    cf.push_back(c);
  }
  for (size_t i = 0; i < p.ins_f.size(); ++i) {
    const InstrD& in = p.ins_f[i];
    const double c = in.m2 * (4.0 * nnz(in) + 3.0 * p.ir1[in.i1].dim + p.ir2[in.i2].dim) +
                     p.ir3[in.i3].dim;
    p.rowb.items.push_back(RowItem{static_cast<int>(i), 0, (in.m1 + 31) / 32, 0});
    cb.push_back(c);
  }
  const size_t elem = p.dtype == 2 ? 8 : 4;
  const size_t budget = 220 * 1024;
  int re, oy, ow, og, we;
  p.rowf.nwarps = 8;
  schedule_items(p.rowf, cf);
  if (row_smem(p, 0, 8, elem, &re, &oy, &ow, &og, &we) > budget) return;
  p.rowb.nwarps = 16;
  if (row_smem(p, 1, 16, elem, &re, &oy, &ow, &og, &we) > budget) p.rowb.nwarps = 8;
  schedule_items(p.rowb, cb);
  if (row_smem(p, 1, p.rowb.nwarps, elem, &re, &oy, &ow, &og, &we) > budget) return;
  p.row_ok = true;
}

constexpr int kSegBwdWarps = 16;

template <class V>
int blob_put(std::vector<unsigned char>& blob, const std::vector<V>& v) {
  const size_t at = align16(blob.size());
  blob.resize(at + sizeof(V) * v.size());
  if (!v.empty()) std::memcpy(blob.data() + at, v.data(), sizeof(V) * v.size());
  return static_cast<int>(at);
}

// Builds the table image of one segment-kernel pass.  `order` lists the instructions sorted
// by X irrep; `bounds` splits it into contiguous groups (backward units; one group forward).
// P block of an instruction: D1 x D3 packed (row_pad false) or with each row padded to a
// multiple of 4 values, so that every row starts 16-byte aligned (row_pad true).
template <class T>
void seg_tables(const oeqb_plan& p, const std::vector<int>& order, const std::vector<int>& bounds,
                oeqb_plan::SegTable& t, bool row_pad = false) {
  std::vector<SegInstr> ins;
  std::vector<SegRun> runs;
  std::vector<int> grp;
  std::vector<SegX> xs;
  std::vector<SegPEnt> pent;
  std::vector<SegTerm<T>> term;
  int poff = 0;
  for (int idx : order) {
    const InstrD& in = p.ins_f[idx];
    const IrrepD& r1 = p.ir1[in.i1];
    const IrrepD& r3 = p.ir3[in.i3];
    SegInstr si{};
    si.l1 = in.l1;
    si.l3 = in.l3;
    si.bc = pair_code(in.l2, in.l3);
    si.y_off = p.ir2[in.i2].off;
    si.w_off = in.woff;
    si.z_off = r3.off;
    si.p_off = poff;
    si.pw = in.pw;
    ins.push_back(si);
    // Non-zero P entries: P[i][k] = sum_j (pw c_ijk) y_j, terms grouped by (i, k).
    std::vector<std::vector<std::pair<int, double>>> cell(size_t(r1.dim) * r3.dim);
    for (int e = in.cg_off; e < in.cg_off + in.cg_nnz; ++e) {
      const CGEntry& c = p.cg[e];
      cell[size_t(c.i) * r3.dim + c.k].push_back({si.y_off + c.j, in.pw * c.c});
    }
    const int rstride = row_pad ? (r3.dim + 3) / 4 * 4 : r3.dim;
    for (size_t q = 0; q < cell.size(); ++q) {
      if (cell[q].empty()) continue;
      const int i = static_cast<int>(q) / r3.dim, k = static_cast<int>(q) % r3.dim;
      pent.push_back(SegPEnt{poff + i * rstride + k,
                             (static_cast<int>(term.size()) << 8) | static_cast<int>(cell[q].size())});
      for (auto& tj : cell[q]) term.push_back(SegTerm<T>{T(tj.second), tj.first});
    }
    poff += (r1.dim * rstride + 3) / 4 * 4;
  }
  // Runs: maximal pieces of a group with one X irrep.  Groups are contiguous pieces of the
  // X-sorted list, so the runs of one X irrep are consecutive in the run table.
  std::vector<int> run_irrep;
  int pslot = 0;
  for (size_t g = 0; g + 1 < bounds.size(); ++g) {
    grp.push_back(static_cast<int>(runs.size()));
    for (int n = bounds[g]; n < bounds[g + 1]; ++n) {
      const InstrD& in = p.ins_f[order[n]];
      if (static_cast<int>(runs.size()) == grp.back() || run_irrep.back() != in.i1) {
        const IrrepD& r1 = p.ir1[in.i1];
        runs.push_back(SegRun{r1.off, r1.l, r1.mul / 32, n, n + 1, pslot, 0, 0});
        run_irrep.push_back(in.i1);
        pslot += (r1.mul * r1.dim + 3) / 4 * 4;
      } else {
        runs.back().n1 = n + 1;
      }
    }
  }
  grp.push_back(static_cast<int>(runs.size()));
  for (size_t r = 0; r < p.ir1.size(); ++r) {
    int r0 = 0, r1 = 0;
    for (size_t q = 0; q < runs.size(); ++q)
      if (run_irrep[q] == static_cast<int>(r)) {
        if (r1 == 0) r0 = static_cast<int>(q);
        r1 = static_cast<int>(q) + 1;
      }
    xs.push_back(SegX{p.ir1[r].off, p.ir1[r].mul * p.ir1[r].dim, r0, r1});
  }
  t.gyc_off = pslot;
  t.blob.clear();
  blob_put(t.blob, ins);
  t.off_run = blob_put(t.blob, runs);
  t.off_grp = blob_put(t.blob, grp);
  t.off_x = blob_put(t.blob, xs);
  t.off_pent = blob_put(t.blob, pent);
  t.off_term = blob_put(t.blob, term);
  t.blob.resize(align16(t.blob.size()));
  t.ngroups = static_cast<int>(bounds.size()) - 1;
  t.nrun = static_cast<int>(runs.size());
  t.nx = static_cast<int>(xs.size());
  t.npent = static_cast<int>(pent.size());
  t.psize = poff;
}

// Row layout and shared-memory bytes of a segment pass (must match stage_seg).
void seg_layout(const oeqb_plan& p, int kind, size_t elem, oeqb_plan::SegTable& t) {
  t.offY = static_cast<int>(round_elems(p.L1dim, elem));
  t.offW = t.offY + static_cast<int>(round_elems(p.L2dim, elem));
  t.offG = t.offW + static_cast<int>(p.shared_w ? 0 : round_elems(p.wnumel, elem));
  t.row_elems = t.offG + static_cast<int>(kind == 1 ? round_elems(p.L3dim, elem) : 0);
  t.scratch_off = static_cast<int>(round_elems(size_t(t.rows_per_buf) * t.psize, elem));
  size_t scratch;
  if (kind == 0)
    scratch = size_t(8) * kSegStages * seg_fwd_cpl(static_cast<int>(elem)) * 32 * kSegD;
  else
    scratch = size_t(t.gyc_off) + size_t(kSegBwdWarps) * p.L2dim * 32;
  t.smem = t.blob.size() + 16 + 2 * elem * size_t(t.row_elems) * t.rows_per_buf +
           elem * (size_t(t.scratch_off) + scratch);
}

// Channelwise uvu (MACE / NequIP interaction shape): mul_ir, one Y copy per instruction,
// multiplicities in whole 32-lane chunks, one instruction per output irrep, unrolled degrees.
void build_seg(oeqb_plan& p) {
  p.segf = {};
  p.segb = {};
  if (p.uvw || p.layout != 0 || !p.zb_f.empty() || p.ins_f.empty()) return;
  for (const GroupD& g : p.grp_f)
    if (g.count != 1) return;
  int nchmax = 0;
  for (const InstrD& in : p.ins_f) {
    if (in.code < 0 || in.m2 != 1 || in.m1 % 32 != 0 || in.m1 == 0) return;
    if (in.l1 > kLMaxUnrolled || in.l2 > kLMaxUnrolled || in.l3 > kLMaxUnrolled) return;
    nchmax = std::max(nchmax, in.m1 / 32);
  }
  std::vector<int> order(p.ins_f.size());
  for (size_t i = 0; i < order.size(); ++i) order[i] = static_cast<int>(i);
  std::stable_sort(order.begin(), order.end(), [&](int x, int y) {
    const InstrD &a = p.ins_f[x], &b = p.ins_f[y];
    return a.i1 != b.i1 ? a.i1 < b.i1 : a.i2 < b.i2;
  });
  const int n = static_cast<int>(order.size());
  const size_t elem = p.dtype == 2 ? 8 : 4;
  // Splits the X-sorted list into G contiguous groups of similar cost.
  auto split = [&](int G, bool bwd) {
    std::vector<double> cost(n);
    double total = 0;
    for (int q = 0; q < n; ++q) {
      const InstrD& in = p.ins_f[order[q]];
      const int d1 = 2 * in.l1 + 1, d2 = 2 * in.l2 + 1, d3 = 2 * in.l3 + 1;
      cost[q] = bwd ? 2.0 * d1 * d3 + 2.0 * in.cg_nnz + 2.0 * d2 + d3 + 12.0 : d1 * d3 + 2.0 * d3 + 10.0;
      total += cost[q];
    }
    std::vector<int> bounds{0};
    double acc = 0;
    for (int q = 0; q < n; ++q) {
      acc += cost[q];
      const int g = static_cast<int>(bounds.size());
      if (g < G && q + 1 < n && acc >= total * g / G) bounds.push_back(q + 1);
    }
    bounds.push_back(n);
    return bounds;
  };
  auto tables = [&](const std::vector<int>& bounds, oeqb_plan::SegTable& t) {
    if (p.dtype == 2)
      seg_tables<double>(p, order, bounds, t);
    else
      seg_tables<float>(p, order, bounds, t);
  };
  // Forward: 8 warps, units = groups x chunk blocks of up to seg_fwd_cpl chunks, one row per
  // buffer, two units per warp (C2, 50,000 rows: 848 us against 885 us with one unit per warp
  // and more with any count that is not a multiple of the warps).
  {
    oeqb_plan::SegTable& t = p.segf;
    t.cbs = std::min(seg_fwd_cpl(static_cast<int>(elem)), nchmax);
    t.nsplit = (nchmax + t.cbs - 1) / t.cbs;
    tables(split(std::max(1, std::min(n, 16 / std::min(16, t.nsplit))), false), t);
    t.rows_per_buf = 1;
    seg_layout(p, 0, elem, t);
    t.ok = t.smem <= 220 * 1024;
  }
  // Backward: 16 warps = groups x chunk blocks of up to seg_bwd_cpl chunks.
  {
    oeqb_plan::SegTable& t = p.segb;
    t.cbs = std::min(seg_bwd_cpl(static_cast<int>(elem)), nchmax);
    t.nsplit = (nchmax + t.cbs - 1) / t.cbs;
    tables(split(std::max(1, std::min(n, kSegBwdWarps / std::min(kSegBwdWarps, t.nsplit))), true), t);
    t.rows_per_buf = 1;
    seg_layout(p, 1, elem, t);
    t.ok = t.smem <= 220 * 1024;
  }
}

// Lockstep backward: segment-eligible problems whose instructions all span the same number
// of 32-channel chunks (dividing 16), that use every X irrep, and whose Y is the spherical-
// harmonic layout (one irrep of each degree 0..L in order).  An even chunk count runs two
// channels per lane (a warp covers 64 channels) on 12 consumer warps where they divide.
void build_lk(oeqb_plan& p) {
  p.lk = {};
  p.lkf = {};
  p.segl = {};
  if (!p.segb.ok || p.dtype != 1) return;  // fp64 operands do not fit the register budget
  if (p.ir2.size() > static_cast<size_t>(kLMaxUnrolled) + 1) return;
  for (size_t i = 0; i < p.ir2.size(); ++i)
    if (p.ir2[i].mul != 1 || p.ir2[i].l != static_cast<int>(i)) return;
  int nch = -1;
  std::vector<char> used(p.ir1.size(), 0);
  for (const InstrD& in : p.ins_f) {
    const int c = in.m1 / 32;
    if (nch >= 0 && c != nch) return;
    nch = c;
    used[in.i1] = 1;
  }
  if (nch <= 0) return;
  for (size_t r = 0; r < p.ir1.size(); ++r)
    if (!used[r] || p.ir1[r].mul != nch * 32) return;
  std::vector<int> order(p.ins_f.size());
  for (size_t i = 0; i < order.size(); ++i) order[i] = static_cast<int>(i);
  std::stable_sort(order.begin(), order.end(), [&](int x, int y) {
    const InstrD &a = p.ins_f[x], &b = p.ins_f[y];
    return a.i1 != b.i1 ? a.i1 < b.i1 : a.i2 < b.i2;
  });
  const int n = static_cast<int>(order.size());
  if (p.dtype == 2)
    seg_tables<double>(p, order, {0, n}, p.segl, true);
  else
    seg_tables<float>(p, order, {0, n}, p.segl, true);
  const size_t elem = p.dtype == 2 ? 8 : 4;
  oeqb_plan::LkCfg& c = p.lk;
  c.nch = nch;
  c.offY = static_cast<int>(round_elems(p.L1dim, elem));
  c.xy_elems = c.offY + static_cast<int>(round_elems(p.L2dim, elem));
  // Two channels per lane when the chunk count is even, the row-block mapping divides and at
  // least 3 ring slots still fit beside the larger row block; otherwise one.
  for (c.cpl = nch % 2 == 0 ? 2 : 1; c.cpl >= 1; --c.cpl) {
    c.nslots = 0;
    if (lk_warps(c.cpl) % (nch / c.cpl) != 0) continue;
    c.rb = lk_warps(c.cpl) / (nch / c.cpl);
    c.slot_w_off = c.rb * nch * 32 * kSegD;
    c.slot_elems = c.slot_w_off + (p.shared_w ? 0 : c.rb * nch * 32);
    const size_t fixed = p.segl.blob.size() + 8 * (4 + 2 * kLkMaxSlots) +
                         elem * (size_t(2) * c.rb * c.xy_elems + size_t(c.rb) * p.segl.psize +
                                 size_t(kLkWarps) * kLkGy);
    for (c.nslots = kLkMaxSlots; c.nslots >= 3; --c.nslots) {
      c.smem = fixed + elem * size_t(c.nslots) * c.slot_elems;
      if (c.smem <= 220 * 1024) break;
    }
    if (c.nslots >= 3) break;
  }
  c.ok = c.cpl >= 1 && c.nslots >= 3;
  // Lockstep forward (every output irrep written by one instruction: the segment forward's
  // condition): 16 consumer warps, a ring of W segments, two Z staging buffers per warp.
  if (!p.segf.ok) return;
  oeqb_plan::LkCfg& f = p.lkf;
  f = {};
  f.nch = nch;
  f.offY = c.offY;
  f.xy_elems = c.xy_elems;
  f.cpl = nch % 2 == 0 && kLfWarps % (nch / 2) == 0 ? 2 : 1;
  if (kLfWarps % (nch / f.cpl) != 0) return;
  f.rb = kLfWarps / (nch / f.cpl);
  f.slot_w_off = 0;
  f.slot_elems = p.shared_w ? 0 : f.rb * nch * 32;
  const size_t ffixed = p.segl.blob.size() + 8 * (4 + 2 * kLkMaxSlots) +
                        elem * (size_t(2) * f.rb * f.xy_elems + size_t(f.rb) * p.segl.psize +
                                size_t(kLfWarps) * 2 * f.cpl * 32 * kSegD);
  for (f.nslots = kLkMaxSlots; f.nslots >= 3; --f.nslots) {
    f.smem = ffixed + elem * size_t(f.nslots) * f.slot_elems;
    if (f.smem <= 220 * 1024) break;
  }
  f.ok = f.nslots >= 3;
}

// Convolutions whose instructions all have multiplicity 1 run one edge per lane.
void build_edge(oeqb_plan& p) {
  p.edge_ok = false;
  if (p.ins_f.empty()) return;
  for (const InstrD& in : p.ins_f)
    if (in.code < 0 || in.m1 != 1 || in.m2 != 1 || in.m3 != 1) return;
  p.edge = EdgeLayout{edge_pad(p.L1dim), edge_pad(p.L2dim), edge_pad(p.L3dim),
                      edge_pad(std::max(1, p.wnumel))};
  const size_t elem = p.dtype == 2 ? 8 : 4;
  p.edge_ok = edge_warp_elems(p.edge, true) * elem <= 12 * 1024;
  p.edge1_ok = p.edge_ok && p.ins_f.size() == 1 && p.n1 == 1 && p.n2 == 1 && p.n3 == 1 &&
               p.ir1[0].off == 0 && p.ir2[0].off == 0 && p.ir3[0].off == 0;
  if (p.edge1_ok) p.edge1 = Edge1{p.ins_f[0].code, p.ins_f[0].woff, p.ins_f[0].pw};
}

// Shared-weight float32 uvw problems of the NequIP shape run on the tensor cores: every
// instruction 32 x 1 -> 32 channels, l1, l3 <= 2, every output irrep 32 channels of l <= 2.
// Schedule: output groups = runs of output irreps whose accumulators fit one kTcDCols-column
// TMEM buffer (a work unit is a 128-row tile x a group); inside a group, one stage per input
// irrep (its X block staged once), instructions in output order; the first instruction into
// an output irrep overwrites its accumulator.
void build_uvw_tc(oeqb_plan& p) {
  auto& t = p.tc;
  t = oeqb_plan::TcTable{};
  if (p.dtype != 1 || !p.uvw || p.layout != 0 || !p.shared_w || p.ins_f.empty()) return;
  if (p.L1dim % 4 || p.L3dim % 4 || p.L2dim > kTcYMax) return;
  for (const IrrepD& r : p.ir1)
    if (r.off % 4 || r.l > 2) return;
  for (const IrrepD& r : p.ir3)
    if (r.off % 4 || r.l > 2 || r.mul != 32) return;
  std::vector<InstrD> ins;  // original order (weight blocks by instruction index)
  ins.resize(p.nins);
  for (const InstrD& in : p.ins_f) {
    if (in.code < 0 || in.m1 != 32 || in.m2 != 1 || in.m3 != 32 || in.l1 > 2 || in.l3 > 2)
      return;
    if (p.ir2[in.i2].off + 2 * in.l2 + 1 > p.L2dim) return;
  }
  // ins_f is a stable sort of the descriptor order by output; recover each instruction's
  // index from its weight offset (distinct per instruction).
  std::vector<std::pair<int, int>> by_woff;
  for (int n = 0; n < static_cast<int>(p.ins_f.size()); ++n)
    by_woff.push_back({p.ins_f[n].woff, n});
  std::sort(by_woff.begin(), by_woff.end());
  std::vector<int> blk(p.ins_f.size());
  for (size_t r = 0; r < by_woff.size(); ++r) blk[by_woff[r].second] = static_cast<int>(r);
  t.woff.resize(p.ins_f.size());
  t.pw.resize(p.ins_f.size());
  for (size_t n = 0; n < p.ins_f.size(); ++n) {
    t.woff[blk[n]] = p.ins_f[n].woff;
    t.pw[blk[n]] = static_cast<float>(p.ins_f[n].pw);
  }
  int o = 0;
  while (o < p.n3) {
    TcPass ps{};
    ps.stage_begin = static_cast<int>(t.stages.size());
    ps.out_begin = static_cast<int>(t.outs.size());
    int cols = 0, o_end = o;
    while (o_end < p.n3 && cols + 32 * p.ir3[o_end].dim <= kTcDCols) cols += 32 * p.ir3[o_end++].dim;
    std::vector<int> dcol(p.n3, -1);
    cols = 0;
    for (int r = o; r < o_end; ++r) {
      dcol[r] = cols;
      t.outs.push_back(TcOut{p.ir3[r].off, p.ir3[r].dim, cols, 0});
      cols += 32 * p.ir3[r].dim;
    }
    std::vector<char> seen(p.n3, 0);
    for (int i1 = 0; i1 < p.n1; ++i1) {
      TcStage st{p.ir1[i1].off, p.ir1[i1].l, static_cast<int>(t.ins.size()), 0};
      for (size_t n = 0; n < p.ins_f.size(); ++n) {
        const InstrD& in = p.ins_f[n];
        if (in.i1 != i1 || in.i3 < o || in.i3 >= o_end) continue;
        TcIns ti{};
        ti.l2 = in.l2;
        ti.l3 = in.l3;
        ti.y_off = p.ir2[in.i2].off;
        ti.wblk = blk[n];
        ti.dcol = dcol[in.i3];
        ti.first = seen[in.i3] ? 0 : 1;
        seen[in.i3] = 1;
        t.outs[ps.out_begin + (in.i3 - o)].has = 1;
        t.ins.push_back(ti);
      }
      st.ins_end = static_cast<int>(t.ins.size());
      if (st.ins_end > st.ins_begin) t.stages.push_back(st);
    }
    ps.stage_end = static_cast<int>(t.stages.size());
    ps.out_end = static_cast<int>(t.outs.size());
    t.passes.push_back(ps);
    o = o_end;
  }
  t.ok = t.passes.size() <= kTcMaxGroups && t.stages.size() <= kTcMaxStages &&
         t.ins.size() <= kTcMaxIns && t.outs.size() <= kTcMaxOuts;
}

// Shared-weight uvw problems with every instruction 32 x 1 -> 32 channels (l <= 3) use the
// dedicated backward: row-parallel dX / dY and a split-K weight gradient.
void build_uvw_sw(oeqb_plan& p) {
  auto& t = p.sw;
  t = oeqb_plan::SwTable{};
  if (!p.uvw || p.layout != 0 || !p.shared_w || p.ins_b.empty()) return;
  if (p.L1dim % 4 || p.L3dim % 4 || p.L2dim > kSwYMax) return;
  for (const IrrepD& r : p.ir1)
    if (r.off % 4) return;
  for (const IrrepD& r : p.ir3)
    if (r.off % 4) return;
  for (const InstrD& in : p.ins_b)
    if (in.code < 0 || in.m1 != 32 || in.m2 != 1 || in.m3 != 32) return;
  std::vector<std::pair<int, int>> by_woff;
  for (int n = 0; n < static_cast<int>(p.ins_b.size()); ++n)
    by_woff.push_back({p.ins_b[n].woff, n});
  std::sort(by_woff.begin(), by_woff.end());
  std::vector<int> blk(p.ins_b.size());
  for (size_t r = 0; r < by_woff.size(); ++r) blk[by_woff[r].second] = static_cast<int>(r);
  t.woff.resize(p.ins_b.size());
  t.pw_f.resize(p.ins_b.size());
  t.pw_d.resize(p.ins_b.size());
  for (size_t n = 0; n < p.ins_b.size(); ++n) {
    t.woff[blk[n]] = p.ins_b[n].woff;
    t.pw_f[blk[n]] = static_cast<float>(p.ins_b[n].pw);
    t.pw_d[blk[n]] = p.ins_b[n].pw;
  }
  for (int i1 = 0; i1 < p.n1; ++i1) {  // every input irrep: dX is written (zeros if unused)
    SwGroup g{p.ir1[i1].off, p.ir1[i1].l, static_cast<int>(t.ins.size()), 0};
    if (p.ir1[i1].mul != 32 && p.ir1[i1].mul != 0) return;
    for (size_t n = 0; n < p.ins_b.size(); ++n) {
      const InstrD& in = p.ins_b[n];
      if (in.i1 != i1) continue;
      t.ins.push_back(SwIns{in.l2, in.l3, p.ir2[in.i2].off, p.ir3[in.i3].off, blk[n], 0, 0, 0});
    }
    g.ins_end = static_cast<int>(t.ins.size());
    t.groups.push_back(g);
  }
  for (int i3 = 0; i3 < p.n3; ++i3) {  // forward tables (every output irrep is written)
    if (p.ir3[i3].mul != 32 && p.ir3[i3].mul != 0) return;
    SwOut o{p.ir3[i3].off, p.ir3[i3].l, static_cast<int>(t.fins.size()), 0};
    for (const InstrD& in : p.ins_f)
      if (in.i3 == i3)
        t.fins.push_back(SwFIns{in.l1, in.l2, p.ir1[in.i1].off, p.ir2[in.i2].off, in.woff, 0, 0,
                                0, in.pw});
    o.ins_end = static_cast<int>(t.fins.size());
    t.fouts.push_back(o);
  }
  std::vector<int> order(p.ins_b.size());
  for (size_t n = 0; n < order.size(); ++n) order[n] = static_cast<int>(n);
  std::stable_sort(order.begin(), order.end(),
                   [&](int a, int b) { return p.ins_b[a].l3 < p.ins_b[b].l3; });
  for (int n : order) {
    const InstrD& in = p.ins_b[n];
    t.dw.push_back(SwDw{in.l1, in.l2, in.l3, p.ir1[in.i1].off, p.ir2[in.i2].off,
                        p.ir3[in.i3].off, in.woff, 0, in.pw});
  }
  t.ok = true;
}

int parse_descriptor(const void* data, size_t n, oeqb_plan& p) {
  const unsigned char* b = static_cast<const unsigned char*>(data);
  if (n < 16 * 8) return fail(OEQB_ERR_INVALID, "descriptor too short");
  int64_t h[16];
  std::memcpy(h, b, sizeof(h));
  if (h[0] != kMagic || h[1] != 1) return fail(OEQB_ERR_INVALID, "bad descriptor magic/version");
  p.dtype = static_cast<int>(h[2]);
  p.layout = static_cast<int>(h[3]);
  p.uvw = static_cast<int>(h[4]);
  p.shared_w = static_cast<int>(h[5]);
  p.n1 = static_cast<int>(h[6]);
  p.n2 = static_cast<int>(h[7]);
  p.n3 = static_cast<int>(h[8]);
  p.nins = static_cast<int>(h[9]);
  p.L1dim = static_cast<int>(h[10]);
  p.L2dim = static_cast<int>(h[11]);
  p.L3dim = static_cast<int>(h[12]);
  p.wnumel = static_cast<int>(h[13]);
  const int64_t ncg = h[14];
  p.det = static_cast<int>(h[15] & 1);
  p.kahan = static_cast<int>((h[15] >> 1) & 1);
  if (p.dtype != 1 && p.dtype != 2) return fail(OEQB_ERR_INVALID, "dtype must be f32 or f64");
  if (p.layout != 0 && p.layout != 1) return fail(OEQB_ERR_INVALID, "bad layout");
  if (p.uvw && p.layout == 1)
    return fail(OEQB_ERR_UNSUPPORTED, "layout='ir_mul' is only supported for pure 'uvu' problems");
  if (p.kahan && p.dtype != 1)
    return fail(OEQB_ERR_UNSUPPORTED, "Kahan summation requires float32");
  if (p.n1 < 0 || p.n2 < 0 || p.n3 < 0 || p.nins <= 0 || ncg < 0)
    return fail(OEQB_ERR_INVALID, "bad descriptor counts");
  const size_t need = 16 * 8 + size_t(p.n1 + p.n2 + p.n3) * 24 + size_t(p.nins) * 56 +
                      size_t(ncg) * 32;
  if (n < need) return fail(OEQB_ERR_INVALID, "descriptor truncated");
  size_t pos = 16 * 8;
  auto rd = [&](void* dst, size_t k) {
    std::memcpy(dst, b + pos, k);
    pos += k;
  };
  auto read_irreps = [&](int cnt, std::vector<IrrepD>& out, int total_dim) -> int {
    out.resize(cnt);
    for (int i = 0; i < cnt; ++i) {
      int64_t t[3];
      rd(t, sizeof(t));
      IrrepD r;
      r.mul = static_cast<int>(t[0]);
      r.l = static_cast<int>(t[1]);
      r.dim = 2 * r.l + 1;
      r.off = static_cast<int>(t[2]);
      if (r.mul < 0 || r.l < 0 || r.off < 0 || r.off + r.mul * r.dim > total_dim)
        return fail(OEQB_ERR_INVALID, "irrep out of range");
      if (r.dim > kDMax)
        return fail(OEQB_ERR_UNSUPPORTED, "irreps with l > 7 are not supported");
      if (p.layout == 0) {
        r.su = r.dim;
        r.si = 1;
      } else {
        r.su = 1;
        r.si = r.mul;
      }
      out[i] = r;
    }
    return 0;
  };
  if (int rc = read_irreps(p.n1, p.ir1, p.L1dim)) return rc;
  if (int rc = read_irreps(p.n2, p.ir2, p.L2dim)) return rc;
  if (int rc = read_irreps(p.n3, p.ir3, p.L3dim)) return rc;
  std::vector<InstrD> ins(p.nins);
  for (int i = 0; i < p.nins; ++i) {
    int64_t t[6];
    double pw;
    rd(t, sizeof(t));
    rd(&pw, sizeof(pw));
    InstrD in{};
    in.i1 = static_cast<int>(t[0]);
    in.i2 = static_cast<int>(t[1]);
    in.i3 = static_cast<int>(t[2]);
    if (in.i1 < 0 || in.i1 >= p.n1 || in.i2 < 0 || in.i2 >= p.n2 || in.i3 < 0 || in.i3 >= p.n3)
      return fail(OEQB_ERR_INVALID, "instruction irrep index out of range");
    in.woff = static_cast<int>(t[3]);
    in.cg_off = static_cast<int>(t[4]);
    in.cg_nnz = static_cast<int>(t[5]);
    in.pw = pw;
    in.m1 = p.ir1[in.i1].mul;
    in.m2 = p.ir2[in.i2].mul;
    in.m3 = p.ir3[in.i3].mul;
    in.l1 = p.ir1[in.i1].l;
    in.l2 = p.ir2[in.i2].l;
    in.l3 = p.ir3[in.i3].l;
    in.code = triple_code(in.l1, in.l2, in.l3);
    if (in.l1 > kLMaxUnrolled || in.l2 > kLMaxUnrolled || in.l3 > kLMaxUnrolled) in.code = -1;
    if (!p.uvw && in.m1 != in.m3)
      return fail(OEQB_ERR_INVALID, "uvu instruction needs equal input/output multiplicity");
    const int64_t wsize = p.uvw ? int64_t(in.m1) * in.m2 * in.m3 : int64_t(in.m1) * in.m2;
    if (in.woff < 0 || in.woff + wsize > p.wnumel)
      return fail(OEQB_ERR_INVALID, "instruction weights out of range");
    if (in.cg_off < 0 || in.cg_nnz < 0 || in.cg_off + in.cg_nnz > ncg)
      return fail(OEQB_ERR_INVALID, "instruction CG table out of range");
    ins[i] = in;
  }
  p.cg.resize(ncg);
  const int d1max = 15;
  for (int64_t i = 0; i < ncg; ++i) {
    int64_t t[3];
    double c;
    rd(t, sizeof(t));
    rd(&c, sizeof(c));
    if (t[0] < 0 || t[1] < 0 || t[2] < 0 || t[0] >= d1max || t[1] >= d1max || t[2] >= d1max)
      return fail(OEQB_ERR_INVALID, "CG entry out of range");
    p.cg[i] = CGEntry{static_cast<int>(t[0]), static_cast<int>(t[1]), static_cast<int>(t[2]), 0, c};
  }
  make_groups(ins, true, p.n3, p.ir3, p.ins_f, p.grp_f, p.zb_f);
  make_groups(ins, false, p.n1, p.ir1, p.ins_b, p.grp_b, p.zb_b);
  // Lane-group size: a power of two covering the largest multiplicity a lane indexes.
  int mmax = 1;
  for (const InstrD& in : ins) mmax = std::max(mmax, std::max(in.m1, in.m3));
  int lg = 0;
  while ((1 << lg) < std::min(mmax, 32)) ++lg;
  p.lgG = lg;
  const int rpw = 32 >> lg;
  // Per-warp scratch layout (elements of T).
  int off = 32 * kDMax;  // output staging
  p.off_t = p.off_t2 = p.off_gz = off;
  if (p.uvw) {
    p.off_t = off;
    off += 32 * kDMax;
    p.off_t2 = off;
    off += 32 * kDMax;
    int gz = 0;
    for (const InstrD& in : ins) gz = std::max(gz, in.m3 * (2 * in.l3 + 1));
    p.off_gz = off;
    off += rpw * gz;
  }
  p.off_dy = off;
  off += rpw * p.L2dim;
  p.ws_elems = (off + 3) & ~3;
  p.desc_f = desc_bytes(p, p.grp_f.size(), p.zb_f.size());
  p.desc_b = desc_bytes(p, p.grp_b.size(), p.zb_b.size());
  build_row(p);
  build_seg(p);
  build_lk(p);
  build_edge(p);
  build_uvw_tc(p);
  build_uvw_sw(p);
  return 0;
}

template <class V>
size_t put(std::vector<unsigned char>& buf, const std::vector<V>& v) {
  size_t at = align16(buf.size());
  buf.resize(at + sizeof(V) * v.size() + 16);
  if (!v.empty()) std::memcpy(buf.data() + at, v.data(), sizeof(V) * v.size());
  return at;
}

// Lays out every device table of a plan in one host image (offsets recorded in the plan).
void layout_tables(oeqb_plan& p, std::vector<unsigned char>& buf) {
  buf.clear();
  p.off.ir1 = put(buf, p.ir1);
  p.off.ir2 = put(buf, p.ir2);
  p.off.ir3 = put(buf, p.ir3);
  p.off.ins_f = put(buf, p.ins_f);
  p.off.grp_f = put(buf, p.grp_f);
  p.off.zb_f = put(buf, p.zb_f);
  p.off.ins_b = put(buf, p.ins_b);
  p.off.grp_b = put(buf, p.grp_b);
  p.off.zb_b = put(buf, p.zb_b);
  p.off.cg = put(buf, p.cg);
  for (auto* t : {&p.rowf, &p.rowb}) {
    t->off_items = put(buf, t->items);
    t->off_witems = put(buf, t->witems);
    t->off_wofs = put(buf, t->wofs);
  }
  for (auto* t : {&p.segf, &p.segb, &p.segl}) t->dev_off = put(buf, t->blob);
  p.tc.off_passes = put(buf, p.tc.passes);
  p.tc.off_stages = put(buf, p.tc.stages);
  p.tc.off_ins = put(buf, p.tc.ins);
  p.tc.off_outs = put(buf, p.tc.outs);
  p.tc.off_woff = put(buf, p.tc.woff);
  p.tc.off_pw = put(buf, p.tc.pw);
  p.sw.off_groups = put(buf, p.sw.groups);
  p.sw.off_ins = put(buf, p.sw.ins);
  p.sw.off_dw = put(buf, p.sw.dw);
  p.sw.off_fouts = put(buf, p.sw.fouts);
  p.sw.off_fins = put(buf, p.sw.fins);
  p.sw.off_woff = put(buf, p.sw.woff);
  p.sw.off_pw = p.dtype == 2 ? put(buf, p.sw.pw_d) : put(buf, p.sw.pw_f);
  p.off.total = align16(buf.size());
  buf.resize(p.off.total);
}

int upload(oeqb_plan& p) {
  std::vector<unsigned char> buf;
  layout_tables(p, buf);
  OEQB_CUDA(cudaMalloc(&p.dmem, p.off.total));
  OEQB_CUDA(cudaMemcpy(p.dmem, buf.data(), p.off.total, cudaMemcpyHostToDevice));
  OEQB_CUDA(cudaMalloc(&p.d_status, sizeof(int)));
  OEQB_CUDA(cudaMemset(p.d_status, 0, sizeof(int)));
  if (p.tc.ok)
    OEQB_CUDA(cudaMalloc(&p.tc.wsplit, sizeof(float) * kTcWBlock * p.tc.woff.size()));
  if (p.sw.ok) OEQB_CUDA(cudaMalloc(&p.sw.wt, p.elem() * 1024 * p.sw.woff.size()));
  return 0;
}

template <class T>
Args<T> base_args(const oeqb_plan& p, bool fwd_order) {
  Args<T> a{};
  a.ir1 = reinterpret_cast<const IrrepD*>(p.dmem + p.off.ir1);
  a.ir2 = reinterpret_cast<const IrrepD*>(p.dmem + p.off.ir2);
  a.ir3 = reinterpret_cast<const IrrepD*>(p.dmem + p.off.ir3);
  a.ins = reinterpret_cast<const InstrD*>(p.dmem + (fwd_order ? p.off.ins_f : p.off.ins_b));
  a.grp = reinterpret_cast<const GroupD*>(p.dmem + (fwd_order ? p.off.grp_f : p.off.grp_b));
  a.zero_blocks = reinterpret_cast<const int*>(p.dmem + (fwd_order ? p.off.zb_f : p.off.zb_b));
  a.cgtab = reinterpret_cast<const CGEntry*>(p.dmem + p.off.cg);
  a.n1 = p.n1;
  a.n2 = p.n2;
  a.n3 = p.n3;
  a.nins = p.nins;
  a.ngrp = static_cast<int>(fwd_order ? p.grp_f.size() : p.grp_b.size());
  a.nzero = static_cast<int>(fwd_order ? p.zb_f.size() : p.zb_b.size());
  a.L1dim = p.L1dim;
  a.L2dim = p.L2dim;
  a.L3dim = p.L3dim;
  a.wnumel = p.wnumel;
  a.shared_w = p.shared_w;
  a.lgG = p.lgG;
  a.ws_elems = p.ws_elems;
  a.off_t = p.off_t;
  a.off_t2 = p.off_t2;
  a.off_gz = p.off_gz;
  a.off_dy = p.off_dy;
  a.status = p.d_status;
  return a;
}

// Raises a kernel's dynamic shared-memory limit to the device maximum, once per
// (device, kernel), so plans of different sizes never lower each other's limit.
std::mutex g_attr_mu;
std::set<std::pair<int, const void*>> g_attr_done;

int allow_max_smem(int device, const void* kernel) {
  std::lock_guard<std::mutex> g(g_attr_mu);
  if (g_attr_done.count({device, kernel})) return 0;
  int optin = 0;
  OEQB_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
  int static_bytes = 0;
  cudaFuncAttributes fa{};
  OEQB_CUDA(cudaFuncGetAttributes(&fa, kernel));
  static_bytes = static_cast<int>(fa.sharedSizeBytes);
  OEQB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 optin - static_bytes));
  g_attr_done.insert({device, kernel});
  return 0;
}

// Launches `kernel` over `items` work items.  det = segmented kernels (range per warp).
template <class T>
int launch(oeqb_plan& p, const void* kernel, const Args<T>& a, bool fwd_order, bool det,
           cudaStream_t stream) {
  if (a.nitems <= 0) return 0;
  const size_t smem = (fwd_order ? p.desc_f : p.desc_b) + size_t(kWarps) * p.ws_elems * sizeof(T);
  int per_sm;
  {
    std::lock_guard<std::mutex> g(p.mu);
    auto it = p.occ.find(kernel);
    if (it == p.occ.end()) {
      if (int rc = allow_max_smem(p.device, kernel)) return rc;
      int n = 0;
      OEQB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kThreads, smem));
      if (n <= 0) return fail(OEQB_ERR_UNSUPPORTED, "kernel does not fit on the device");
      it = p.occ.emplace(kernel, n).first;
    }
    per_sm = it->second;
  }
  const long long rpw = 32 >> p.lgG;
  long long blocks;
  if (!det) {
    const long long warps = (a.nitems + rpw - 1) / rpw;
    blocks = (warps + kWarps - 1) / kWarps;
  } else {
    // Segmented kernels: at least ~64 positions per warp keeps the snapped ranges useful.
    blocks = (a.nitems + kWarps * 64 - 1) / (kWarps * 64);
  }
  blocks = std::max<long long>(1, std::min<long long>(blocks, (long long)p.sm_count * per_sm));
  void* params[] = {const_cast<Args<T>*>(&a)};
  OEQB_CUDA(cudaLaunchKernel(kernel, dim3(static_cast<unsigned>(blocks)), dim3(kThreads), params,
                             smem, stream));
  return 0;
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; }
bool aligned32(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 31) == 0; }

template <class T>
int launch_row(oeqb_plan& p, int kind, const Args<T>& a, cudaStream_t stream) {
  if (a.nitems <= 0) return 0;
  const auto& t = kind == 0 ? p.rowf : p.rowb;
  ArgsRow<T> v;
  v.a = a;
  // Row items index the forward-order instruction table (and the forward groups).
  v.a.ins = reinterpret_cast<const InstrD*>(p.dmem + p.off.ins_f);
  v.a.grp = reinterpret_cast<const GroupD*>(p.dmem + p.off.grp_f);
  v.a.zero_blocks = reinterpret_cast<const int*>(p.dmem + p.off.zb_f);
  v.a.ngrp = static_cast<int>(p.grp_f.size());
  v.a.nzero = static_cast<int>(p.zb_f.size());
  v.items = reinterpret_cast<const RowItem*>(p.dmem + t.off_items);
  v.witems = reinterpret_cast<const int*>(p.dmem + t.off_witems);
  v.wofs = reinterpret_cast<const int*>(p.dmem + t.off_wofs);
  v.nitems = static_cast<int>(t.items.size());
  v.nwitems = static_cast<int>(t.witems.size());
  v.nwarps = t.nwarps;
  const size_t elem = sizeof(T);
  const size_t smem = row_smem(p, kind, t.nwarps, elem, &v.row_elems, &v.offY, &v.offW, &v.offG,
                               &v.ws_elems);
  v.off_stage = 0;
  v.off_dxp = 0;
  v.off_dyp = static_cast<int>(round_elems(p.L1dim, elem));
  // Bulk (TMA) copies need 16-byte aligned rows: every base pointer and row length.
  bool tma = aligned16(a.X) && aligned16(a.Y) && (p.L1dim * elem) % 16 == 0 &&
             (p.L2dim * elem) % 16 == 0;
  if (!p.shared_w) tma = tma && aligned16(a.W) && (p.wnumel * elem) % 16 == 0;
  if (kind == 1) tma = tma && aligned16(a.Gz) && (p.L3dim * elem) % 16 == 0;
  v.use_tma = tma ? 1 : 0;
  const void* kernel = row_kernel_ptr<T>(kind, t.nwarps);
  const int threads = 32 * t.nwarps;
  int per_sm;
  {
    std::lock_guard<std::mutex> g(p.mu);
    auto it = p.occ.find(kernel);
    if (it == p.occ.end()) {
      if (int rc = allow_max_smem(p.device, kernel)) return rc;
      int n = 0;
      OEQB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, smem));
      if (n <= 0) return fail(OEQB_ERR_UNSUPPORTED, "row kernel does not fit on the device");
      it = p.occ.emplace(kernel, n).first;
    }
    per_sm = it->second;
  }
  long long blocks = std::min<long long>(a.nitems, (long long)p.sm_count * per_sm);
  blocks = std::max<long long>(1, blocks);
  void* params[] = {&v};
  OEQB_CUDA(cudaLaunchKernel(kernel, dim3(static_cast<unsigned>(blocks)), dim3(threads), params,
                             smem, stream));
  return 0;
}

template <class T>
int launch_seg(oeqb_plan& p, int kind, const Args<T>& a, cudaStream_t stream) {
  if (a.nitems <= 0) return 0;
  const oeqb_plan::SegTable& t = kind == 0 ? p.segf : p.segb;
  ArgsSeg<T> v;
  v.a = a;
  v.tables = p.dmem + t.dev_off;
  v.table_bytes = static_cast<int>(t.blob.size());
  v.off_run = t.off_run;
  v.off_grp = t.off_grp;
  v.off_x = t.off_x;
  v.off_pent = t.off_pent;
  v.off_term = t.off_term;
  v.ngroups = t.ngroups;
  v.nsplit = t.nsplit;
  v.cbs = t.cbs;
  v.gyc_off = t.gyc_off;
  v.nx = t.nx;
  v.npent = t.npent;
  v.psize = t.psize;
  v.offY = t.offY;
  v.offW = t.offW;
  v.offG = t.offG;
  v.row_elems = t.row_elems;
  v.rows_per_buf = t.rows_per_buf;
  v.scratch_off = t.scratch_off;
  const size_t elem = sizeof(T);
  bool tma = aligned16(a.X) && aligned16(a.Y) && (p.L1dim * elem) % 16 == 0 &&
             (p.L2dim * elem) % 16 == 0;
  if (!p.shared_w) tma = tma && aligned16(a.W) && (p.wnumel * elem) % 16 == 0;
  if (kind == 1) tma = tma && aligned16(a.Gz) && (p.L3dim * elem) % 16 == 0;
  v.use_tma = tma ? 1 : 0;
  const void* kernel = seg_kernel_ptr<T>(kind);
  const int threads = kind == 0 ? 256 : 32 * kSegBwdWarps;
  int per_sm;
  {
    std::lock_guard<std::mutex> g(p.mu);
    auto it = p.occ.find(kernel);
    if (it == p.occ.end()) {
      if (int rc = allow_max_smem(p.device, kernel)) return rc;
      int n = 0;
      OEQB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, t.smem));
      if (n <= 0) return fail(OEQB_ERR_UNSUPPORTED, "channelwise kernel does not fit on the device");
      it = p.occ.emplace(kernel, n).first;
    }
    per_sm = it->second;
  }
  const long long units = (a.nitems + t.rows_per_buf - 1) / t.rows_per_buf;
  long long blocks = std::min<long long>(units, (long long)p.sm_count * per_sm);
  blocks = std::max<long long>(1, blocks);
  void* params[] = {&v};
  OEQB_CUDA(cudaLaunchKernel(kernel, dim3(static_cast<unsigned>(blocks)), dim3(threads), params,
                             t.smem, stream));
  return 0;
}

// fwd = true: the lockstep forward (tp_fwd_lk), else the backward (tp_bwd_lk).
template <class T>
int launch_lk(oeqb_plan& p, const Args<T>& a, cudaStream_t stream, bool fwd = false) {
  const oeqb_plan::SegTable& t = p.segl;
  const oeqb_plan::LkCfg& c = fwd ? p.lkf : p.lk;
  const int nwarps = fwd ? kLfWarps : lk_warps(c.cpl);
  ArgsLk<T> v;
  v.a = a;
  v.tables = p.dmem + t.dev_off;
  v.table_bytes = static_cast<int>(t.blob.size());
  v.off_run = t.off_run;
  v.off_grp = t.off_grp;
  v.off_x = t.off_x;
  v.off_pent = t.off_pent;
  v.off_term = t.off_term;
  v.ninstr = static_cast<int>(p.ins_f.size());
  v.nrun = t.nrun;
  v.npent = t.npent;
  v.psize = t.psize;
  v.nch = c.nch;
  v.rb = c.rb;
  v.nslots = c.nslots;
  v.offY = c.offY;
  v.xy_elems = c.xy_elems;
  v.slot_elems = c.slot_elems;
  v.slot_w_off = c.slot_w_off;
  const void* kernel = fwd ? lkf_kernel_ptr<T>(c.cpl) : lk_kernel_ptr<T>(c.cpl);
  {
    std::lock_guard<std::mutex> g(p.mu);
    auto it = p.occ.find(kernel);
    if (it == p.occ.end()) {
      if (int rc = allow_max_smem(p.device, kernel)) return rc;
      int n = 0;
      OEQB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
          &n, kernel, 32 * (nwarps + 1), c.smem));
      if (n <= 0) return fail(OEQB_ERR_UNSUPPORTED, "lockstep kernel does not fit on the device");
      p.occ.emplace(kernel, n);
    }
  }
  const long long nblk = (a.nitems + c.rb - 1) / c.rb;
  const long long blocks = std::max<long long>(1, std::min<long long>(nblk, p.sm_count));
  void* params[] = {&v};
  OEQB_CUDA(cudaLaunchKernel(kernel, dim3(static_cast<unsigned>(blocks)),
                             dim3(32 * (nwarps + 1)), params, c.smem, stream));
  return 0;
}

// Every bulk copy of the lockstep backward is row-granular: rows and base pointers must be
// 16-byte aligned.
template <class T>
bool lk_aligned(const oeqb_plan& p, const Args<T>& a) {
  const size_t e = sizeof(T);
  bool ok = aligned16(a.X) && aligned16(a.Y) && aligned16(a.Gz) && aligned16(a.out0) &&
            (p.L1dim * e) % 16 == 0 && (p.L2dim * e) % 16 == 0 && (p.L3dim * e) % 16 == 0;
  if (!p.shared_w) ok = ok && aligned16(a.W) && (p.wnumel * e) % 16 == 0;
  return ok;
}

template <class T>
int launch_edge(oeqb_plan& p, int kind, const Args<T>& a, cudaStream_t stream) {
  if (a.nitems <= 0) return 0;
  const void* kernel = edge_kernel_ptr<T>(kind);
  const size_t smem = align16(sizeof(InstrD) * p.nins) +
                      sizeof(T) * size_t(kEdgeWarps) * edge_warp_elems(p.edge, kind == 1);
  int per_sm;
  {
    std::lock_guard<std::mutex> g(p.mu);
    auto it = p.occ.find(kernel);
    if (it == p.occ.end()) {
      if (int rc = allow_max_smem(p.device, kernel)) return rc;
      int n = 0;
      OEQB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kEdgeWarps * 32, smem));
      if (n <= 0) return fail(OEQB_ERR_UNSUPPORTED, "edge convolution kernel does not fit");
      it = p.occ.emplace(kernel, n).first;
    }
    per_sm = it->second;
  }
  const long long warps = (a.nitems + 31) / 32;
  long long blocks = std::min<long long>((warps + kEdgeWarps - 1) / kEdgeWarps,
                                         (long long)p.sm_count * per_sm);
  blocks = std::max<long long>(1, blocks);
  EdgeLayout L = p.edge;
  void* params[] = {const_cast<Args<T>*>(&a), &L};
  OEQB_CUDA(cudaLaunchKernel(kernel, dim3(static_cast<unsigned>(blocks)), dim3(kEdgeWarps * 32),
                             params, smem, stream));
  return 0;
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime (no link-time
// dependency on libcuda).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// Tensor-core uvw forward: split the weights into the operand image, then the persistent
// kernel (one CTA per SM over 128-row tile x output-group units).  The weight image is
// plan-owned, so forward calls of one plan on different streams must be ordered by the caller.
int launch_uvw_tc(oeqb_plan& p, const Args<float>& a, cudaStream_t stream) {
  if (a.nitems <= 0) return 0;
  auto encode = tensor_map_encoder();
  if (!encode) return fail(OEQB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  // X as a 2D tensor [rows, L1dim]; boxes of 128 rows x 32 floats, 128-byte swizzle.
  CUtensorMap xmap;
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(p.L1dim),
                                static_cast<cuuint64_t>(a.nitems)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(p.L1dim) * sizeof(float)};
    const cuuint32_t box[2] = {32, kTcRows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = encode(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(a.X),
                              dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
      return fail(OEQB_ERR_CUDA, "cuTensorMapEncodeTiled failed with code " + std::to_string(r));
  }
  const int nins = static_cast<int>(p.tc.woff.size());
  ArgsTcPrep pr{a.W, p.tc.wsplit, reinterpret_cast<const int*>(p.dmem + p.tc.off_woff),
                reinterpret_cast<const float*>(p.dmem + p.tc.off_pw), nins};
  {
    void* params[] = {&pr};
    OEQB_CUDA(cudaLaunchKernel(uvw_tc_kernel_ptr(1), dim3((nins * 1024 + 255) / 256), dim3(256),
                               params, 0, stream));
  }
  const void* kernel = uvw_tc_kernel_ptr(0);
  {
    std::lock_guard<std::mutex> g(p.mu);
    if (p.occ.find(kernel) == p.occ.end()) {
      if (int rc = allow_max_smem(p.device, kernel)) return rc;
      int n = 0;
      OEQB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kTcThreads, kTcSmemBytes));
      if (n <= 0) return fail(OEQB_ERR_UNSUPPORTED, "tensor-core uvw kernel does not fit");
      p.occ.emplace(kernel, n);
    }
  }
  ArgsTc t{};
  t.X = a.X;
  t.Y = a.Y;
  t.Wsplit = p.tc.wsplit;
  t.Z = a.out0;
  t.B = a.nitems;
  t.L1dim = p.L1dim;
  t.L2dim = p.L2dim;
  t.L3dim = p.L3dim;
  t.npass = static_cast<int>(p.tc.passes.size());
  t.nstage = static_cast<int>(p.tc.stages.size());
  t.nins = static_cast<int>(p.tc.ins.size());
  t.nout = static_cast<int>(p.tc.outs.size());
  t.passes = reinterpret_cast<const TcPass*>(p.dmem + p.tc.off_passes);
  t.stages = reinterpret_cast<const TcStage*>(p.dmem + p.tc.off_stages);
  t.ins = reinterpret_cast<const TcIns*>(p.dmem + p.tc.off_ins);
  t.outs = reinterpret_cast<const TcOut*>(p.dmem + p.tc.off_outs);
  t.status = p.d_status;
  const long long units = (a.nitems + kTcRows - 1) / kTcRows * t.npass;
  const long long blocks = std::min<long long>(units, p.sm_count);
  void* params[] = {&t, &xmap};
  OEQB_CUDA(cudaLaunchKernel(kernel, dim3(static_cast<unsigned>(blocks)), dim3(kTcThreads), params,
                             kTcSmemBytes, stream));
  return 0;
}

// Shared-weight uvw backward: W'^T image, row-parallel dX / dY, split-K dW (dW was zeroed).
template <class T>
int launch_uvw_sw(oeqb_plan& p, const Args<T>& a, cudaStream_t stream) {
  if (a.nitems <= 0) return 0;
  const int nins = static_cast<int>(p.sw.woff.size());
  {
    const T* W = a.W;
    T* Wt = static_cast<T*>(p.sw.wt);
    const int* woff = reinterpret_cast<const int*>(p.dmem + p.sw.off_woff);
    const T* pw = reinterpret_cast<const T*>(p.dmem + p.sw.off_pw);
    void* params[] = {&W, &Wt, &woff, &pw, const_cast<int*>(&nins)};
    OEQB_CUDA(cudaLaunchKernel(uvw_sw_kernel_ptr<T>(2), dim3((nins * 1024 + 255) / 256), dim3(256),
                               params, 0, stream));
  }
  ArgsSw<T> v{};
  v.X = a.X;
  v.Y = a.Y;
  v.Wt = static_cast<const T*>(p.sw.wt);
  v.dZ = a.Gz;
  v.dX = a.out0;
  v.dY = a.out1;
  v.dW = a.out2;
  v.B = a.nitems;
  v.L1dim = p.L1dim;
  v.L2dim = p.L2dim;
  v.L3dim = p.L3dim;
  v.ngroups = static_cast<int>(p.sw.groups.size());
  v.ndw = static_cast<int>(p.sw.dw.size());
  v.groups = reinterpret_cast<const SwGroup*>(p.dmem + p.sw.off_groups);
  v.ins = reinterpret_cast<const SwIns*>(p.dmem + p.sw.off_ins);
  v.dw = reinterpret_cast<const SwDw*>(p.dmem + p.sw.off_dw);
  const void* kxy = uvw_sw_kernel_ptr<T>(0);
  int per_sm;
  {
    std::lock_guard<std::mutex> g(p.mu);
    auto it = p.occ.find(kxy);
    if (it == p.occ.end()) {
      if (int rc = allow_max_smem(p.device, kxy)) return rc;
      int n = 0;
      OEQB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kxy, kSwThreads, sw_dxy_smem<T>()));
      if (n <= 0) return fail(OEQB_ERR_UNSUPPORTED, "uvw backward kernel does not fit");
      it = p.occ.emplace(kxy, n).first;
    }
    per_sm = it->second;
  }
  const long long tiles = (a.nitems + kSwRows - 1) / kSwRows;
  const long long bxy = std::max<long long>(1, std::min<long long>(tiles, (long long)p.sm_count * per_sm));
  // Weight gradient: instruction groups x row chunks, about four CTAs per SM.
  const int ngrp = (v.ndw + kSwDwSlots - 1) / kSwDwSlots;
  long long chunks = std::max<long long>(1, (4LL * p.sm_count + ngrp - 1) / ngrp);
  v.rows_per_chunk = std::max<long long>(kSwBatch, (a.nitems + chunks - 1) / chunks);
  v.rows_per_chunk = (v.rows_per_chunk + kSwBatch - 1) / kSwBatch * kSwBatch;
  chunks = (a.nitems + v.rows_per_chunk - 1) / v.rows_per_chunk;
  const void* kdw = uvw_sw_kernel_ptr<T>(1);
  if (int rc = allow_max_smem(p.device, kdw)) return rc;
  void* params[] = {&v};
  OEQB_CUDA(cudaLaunchKernel(kxy, dim3(static_cast<unsigned>(bxy)), dim3(kSwThreads), params,
                             sw_dxy_smem<T>(), stream));
  OEQB_CUDA(cudaLaunchKernel(kdw, dim3(ngrp, static_cast<unsigned>(chunks)), dim3(kSwThreads),
                             params, sw_dw_smem<T>(), stream));
  return 0;
}

// Single-path edge kernels (tp_kernels_edge.cuh).  kind: 2 atomic forward, 3 atomic backward,
// 4 deterministic forward, 5 deterministic backward pass A, 6 pass B.  The deterministic
// kernels split the edges over a fixed number of warps (the device's resident capacity), so a
// plan on one device always sums in the same order.
template <class T>
int launch_edge1(oeqb_plan& p, int kind, const Args<T>& a, T* ws, cudaStream_t stream) {
  if (a.nitems <= 0) return 0;
  const void* kernel = edge_kernel_ptr<T>(kind);
  if (!kernel) return fail(OEQB_ERR_UNSUPPORTED, "no single-path edge kernel of this kind");
  const int d2 = 2 * ((p.edge1.code >> 4) & 15) + 1;
  const int per_warp = kind == 2 || kind == 4 ? 32 * d2 : kind == 3 ? 64 * d2
                       : kind == 5 ? 64 * d2 + 32 * kE1Rec : 0;
  const size_t smem = sizeof(T) * size_t(kEdgeWarps) * per_warp;
  int per_sm;
  {
    std::lock_guard<std::mutex> g(p.mu);
    auto it = p.occ.find(kernel);
    if (it == p.occ.end()) {
      int n = 0;
      OEQB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kEdgeWarps * 32, smem));
      if (n <= 0) return fail(OEQB_ERR_UNSUPPORTED, "edge convolution kernel does not fit");
      it = p.occ.emplace(kernel, n).first;
    }
    per_sm = it->second;
  }
  const long long cap = (long long)p.sm_count * per_sm;
  long long blocks;
  if (kind == 4) {
    blocks = cap;  // fixed partition (deterministic summation order)
  } else {
    const long long warps = (a.nitems + 31) / 32;
    blocks = std::max<long long>(1, std::min<long long>((warps + kEdgeWarps - 1) / kEdgeWarps, cap));
  }
  Edge1 e = p.edge1;
  void* params[] = {const_cast<Args<T>*>(&a), &e, &ws};
  OEQB_CUDA(cudaLaunchKernel(kernel, dim3(static_cast<unsigned>(blocks)), dim3(kEdgeWarps * 32),
                             params, smem, stream));
  return 0;
}

// Pipelined single-path kernels (tp_kernels_edge_pipe.cuh): float32, one weight per edge,
// 16-byte aligned streams.  OEQB_EDGE_PIPE=0 selects the unpipelined kernels instead.
bool edge1_pipe_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("OEQB_EDGE_PIPE");
    return !(e && std::string(e) == "0");
  }();
  return on;
}

// The plan class of the pipelined kernels, atomic or deterministic (without Kahan); pointer
// alignment is checked per call.
bool edge1_pipe_class(const oeqb_plan& p) {
  const int d1 = 2 * ((p.edge1.code >> 8) & 15) + 1, d3 = 2 * (p.edge1.code & 15) + 1;
  return edge1_pipe_enabled() && p.dtype == 1 && !p.kahan && p.edge1_ok && !p.shared_w &&
         p.wnumel == 1 && d1 <= 8 && d3 <= 8 && edge1_pipe_kernel(0, p.edge1.code) != nullptr;
}

// Workspace of the pipelined kernels, in 32-byte node rows: X | dZ | then the dX accumulator
// (atomic), or one 32-byte record per edge (deterministic backward pass A) followed by pass B's
// 64-byte side slots, one per 32-position block.
constexpr size_t kPadRowBytes = 32;
size_t edge1_pipe_ws_bytes(const oeqb_plan& p, int64_t nnz, int64_t nodes) {
  const size_t rows = 2 * kPadRowBytes * size_t(std::max<int64_t>(nodes, 0));
  const size_t e = size_t(std::max<int64_t>(nnz, 0));
  return rows + (p.det ? kPadRowBytes * e + sizeof(float) * kBandSlot * ((e + 31) / 32)
                       : kPadRowBytes * size_t(std::max<int64_t>(nodes, 0))) + 256;
}

template <class T>
bool edge1_pipe_ok(const oeqb_plan& p, const Args<T>& a, const void* ws, size_t ws_bytes) {
  if constexpr (!std::is_same_v<T, float>) {
    return false;
  } else {
    return edge1_pipe_class(p) && ws && aligned32(ws) &&
           ws_bytes >= edge1_pipe_ws_bytes(p, a.nitems, a.nnodes) && aligned16(a.rows) &&
           aligned16(a.cols) && aligned16(a.W) && aligned16(a.Y);
  }
}

// conv_pad_rows over `nodes` rows: a (width da) -> pa, optionally b (width db) -> pb, and
// optionally zero[] cleared.
int launch_pad(const oeqb_plan& p, const float* a, int da, float* pa, const float* b, int db,
               float* pb, float* zero, long long nodes, cudaStream_t stream) {
  if (nodes <= 0) return 0;
  const long long work = nodes * 8;
  const unsigned blocks = static_cast<unsigned>(
      std::min<long long>((work + 255) / 256, static_cast<long long>(p.sm_count) * 8));
  void* params[] = {&a, &da, &pa, &b, &db, &pb, &zero, &nodes};
  OEQB_CUDA(cudaLaunchKernel(edge1_pipe_kernel(2, 0), dim3(blocks), dim3(256), params, 0, stream));
  return 0;
}

int launch_unpad(const oeqb_plan& p, const float* src, float* dst, int d, long long nodes,
                 cudaStream_t stream) {
  if (nodes <= 0) return 0;
  const long long work = nodes * d;
  const unsigned blocks = static_cast<unsigned>(
      std::min<long long>((work + 255) / 256, static_cast<long long>(p.sm_count) * 8));
  void* params[] = {&src, &dst, &d, &nodes};
  OEQB_CUDA(cudaLaunchKernel(edge1_pipe_kernel(3, 0), dim3(blocks), dim3(256), params, 0, stream));
  return 0;
}

// Deterministic backward pass B of the single-path class: the banded per-block sums of the
// records `recs` (written by pass A in edge order), then the fix-up that joins runs across
// 32-position blocks through the side slots `side` (kBandSlot values per block).  The caller
// has cleared dX (a.out0): rows of nodes that send no edge are not written.
template <class T>
int launch_band(oeqb_plan& p, const Args<T>& a, const T* recs, T* side, cudaStream_t stream) {
  const int l1 = (p.edge1.code >> 8) & 15;
  const void* kb = edge1_band_kernel<T>(l1, false);
  const void* kf = edge1_band_kernel<T>(l1, true);
  if (!kb || !kf) return fail(OEQB_ERR_UNSUPPORTED, "no pass B kernel for this degree");
  int nb;
  {
    std::lock_guard<std::mutex> g(p.mu);
    auto it = p.occ.find(kb);
    if (it == p.occ.end()) {
      int m = 0;
      OEQB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&m, kb, kEdgeWarps * 32, 0));
      if (m <= 0) return fail(OEQB_ERR_UNSUPPORTED, "pass B kernel does not fit");
      it = p.occ.emplace(kb, m).first;
    }
    nb = it->second;
  }
  const long long blocks32 = (a.nitems + 31) / 32;
  const long long ctas = std::max<long long>(
      1, std::min<long long>((long long)p.sm_count * nb, (blocks32 + kEdgeWarps - 1) / kEdgeWarps));
  Edge1 e = p.edge1;
  void* pb[] = {const_cast<Args<T>*>(&a), &e, &recs, &side};
  OEQB_CUDA(cudaLaunchKernel(kb, dim3(static_cast<unsigned>(ctas)), dim3(kEdgeWarps * 32), pb, 0,
                             stream));
  const T* cside = side;
  void* pf[] = {const_cast<Args<T>*>(&a), &cside};
  const unsigned fblocks = static_cast<unsigned>(
      std::max<long long>(1, std::min<long long>((blocks32 + 255) / 256, (long long)p.sm_count * 8)));
  OEQB_CUDA(cudaLaunchKernel(kf, dim3(fblocks), dim3(256), pf, 0, stream));
  return 0;
}

// Forward (pads X into the workspace first): kind 0 atomic, 4 deterministic.  Backward (pads
// X and dZ): kind 1 atomic (clears the padded dX accumulator, then copies dX out), kind 5
// deterministic (pass A writes the per-edge records, pass B, conv_bwd_edge1_band and its
// fix-up, sums them per sender).
// Main kernel of the pipelined single-path pass `kind` on node arrays already in the padded
// layout (xp, gp, and out = the padded dX accumulator or the records).  sm_budget: 0 = CTAs
// for every SM, > 0 = for at most that many SMs, < 0 = for all but that many (so that work
// running beside the launch, e.g. a collective or another kernel, finds SMs free).
template <class T>
int launch_edge1_pipe_main(oeqb_plan& p, int kind, const Args<T>& a, const float* xp,
                           const float* gp, float* out, int sm_budget, cudaStream_t stream) {
  const bool bwd = kind == 1 || kind == 5;
  const void* kernel = edge1_pipe_kernel(kind, p.edge1.code);
  if (!kernel) return fail(OEQB_ERR_UNSUPPORTED, "no pipelined kernel for this degree triple");
  const int d2 = 2 * ((p.edge1.code >> 4) & 15) + 1;
  const int epw = kind == 0 || kind == 4 ? 64 : 32;  // edges per warp step (the forwards take two per lane)
  const size_t stage = 2 * epw * sizeof(long long) + epw * sizeof(float) * (1 + d2);
  const size_t per_warp = 3 * stage + (bwd ? 32 * sizeof(float) * (d2 + 1) : 0) +
                          (kind == 5 ? 32 * sizeof(float) * kE1Rec : 0);
  const size_t smem = size_t(kEdgeWarps) * per_warp;
  int per_sm;
  {
    std::lock_guard<std::mutex> g(p.mu);
    auto it = p.occ.find(kernel);
    if (it == p.occ.end()) {
      if (int rc = allow_max_smem(p.device, kernel)) return rc;
      int n = 0;
      OEQB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kEdgeWarps * 32, smem));
      if (n <= 0) return fail(OEQB_ERR_UNSUPPORTED, "pipelined edge kernel does not fit");
      it = p.occ.emplace(kernel, n).first;
    }
    per_sm = it->second;
  }
  const int sms = sm_budget > 0 ? std::min(sm_budget, p.sm_count)
                                 : std::max(1, p.sm_count + std::min(0, sm_budget));
  const long long cap = (long long)sms * per_sm;
  const long long warps = (a.nitems + epw - 1) / epw;
  const long long blocks =
      kind == 4 ? (long long)p.sm_count * per_sm
                : std::max<long long>(1, std::min<long long>((warps + kEdgeWarps - 1) / kEdgeWarps, cap));
  Edge1 e = p.edge1;
  void* params_f[] = {const_cast<Args<T>*>(&a), &e, &xp};
  void* params_b[] = {const_cast<Args<T>*>(&a), &e, &xp, &gp, &out};
  OEQB_CUDA(cudaLaunchKernel(kernel, dim3(static_cast<unsigned>(blocks)), dim3(kEdgeWarps * 32),
                             bwd ? params_b : params_f, smem, stream));
  return 0;
}

template <class T>
int launch_edge1_pipe(oeqb_plan& p, int kind, const Args<T>& a, void* ws, cudaStream_t stream) {
  const bool bwd = kind == 1 || kind == 5;
  if (a.nitems <= 0) {
    if (bwd) OEQB_CUDA(cudaMemsetAsync(a.out0, 0, sizeof(T) * size_t(a.nnodes) * p.L1dim, stream));
    return 0;
  }
  const void* kernel = edge1_pipe_kernel(kind, p.edge1.code);
  if (!kernel) return fail(OEQB_ERR_UNSUPPORTED, "no pipelined kernel for this degree triple");
  const int d1 = 2 * ((p.edge1.code >> 8) & 15) + 1, d3 = 2 * (p.edge1.code & 15) + 1;
  float* xp = static_cast<float*>(ws);
  float* gp = xp + 8 * size_t(a.nnodes);
  float* tail = gp + 8 * size_t(a.nnodes);  // dX accumulator (kind 1) or records (kind 5)
  if (!bwd) {
    if (int rc = launch_pad(p, reinterpret_cast<const float*>(a.X), d1, xp, nullptr, 0, nullptr,
                            nullptr, a.nnodes, stream))
      return rc;
  } else {
    if (int rc = launch_pad(p, reinterpret_cast<const float*>(a.X), d1, xp,
                            reinterpret_cast<const float*>(a.Gz), d3, gp,
                            kind == 1 ? tail : nullptr, a.nnodes, stream))
      return rc;
  }
  if (int rc = launch_edge1_pipe_main<T>(p, kind, a, xp, gp, tail, 0, stream)) return rc;
  if (kind == 1)
    return launch_unpad(p, tail, reinterpret_cast<float*>(a.out0), d1, a.nnodes, stream);
  if (kind == 5) {
    // Pass B writes plain dX rows; rows of nodes that send no edge stay at the cleared zero.
    OEQB_CUDA(cudaMemsetAsync(a.out0, 0, sizeof(T) * size_t(a.nnodes) * p.L1dim, stream));
    if constexpr (std::is_same_v<T, float>)
      return launch_band<float>(p, a, tail, tail + size_t(kE1Rec) * size_t(a.nitems), stream);
    else
      return fail(OEQB_ERR_UNSUPPORTED, "the pipelined kernels are float32 only");
  }
  return 0;
}

// Workspace of the unpipelined single-path deterministic backward: one record per edge, then
// pass B's side slots (kBandSlot values per 32 edges).
size_t edge1_det_ws_bytes(const oeqb_plan& p, int64_t nnz) {
  if (!(p.edge1_ok && p.det && !p.kahan) || nnz <= 0) return 0;
  return (size_t(nnz) * kE1Rec + size_t(kBandSlot) * ((size_t(nnz) + 31) / 32)) * p.elem();
}

// Shared-weight uvw forward on CUDA cores (float64).
template <class T>
int launch_uvw_sw_fwd(oeqb_plan& p, const Args<T>& a, cudaStream_t stream) {
  if (a.nitems <= 0) return 0;
  const void* kernel = uvw_sw_kernel_ptr<T>(3);
  int per_sm;
  {
    std::lock_guard<std::mutex> g(p.mu);
    auto it = p.occ.find(kernel);
    if (it == p.occ.end()) {
      if (int rc = allow_max_smem(p.device, kernel)) return rc;
      int n = 0;
      OEQB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kSwThreads, sw_fwd_smem<T>()));
      if (n <= 0) return fail(OEQB_ERR_UNSUPPORTED, "uvw forward kernel does not fit");
      it = p.occ.emplace(kernel, n).first;
    }
    per_sm = it->second;
  }
  ArgsSwF<T> v{};
  v.X = a.X;
  v.Y = a.Y;
  v.W = a.W;
  v.Z = a.out0;
  v.B = a.nitems;
  v.L1dim = p.L1dim;
  v.L2dim = p.L2dim;
  v.L3dim = p.L3dim;
  v.nout = static_cast<int>(p.sw.fouts.size());
  v.outs = reinterpret_cast<const SwOut*>(p.dmem + p.sw.off_fouts);
  v.ins = reinterpret_cast<const SwFIns*>(p.dmem + p.sw.off_fins);
  const long long tiles = (a.nitems + kSwRows - 1) / kSwRows;
  const long long blocks = std::max<long long>(1, std::min<long long>(tiles, (long long)p.sm_count * per_sm));
  void* params[] = {&v};
  OEQB_CUDA(cudaLaunchKernel(kernel, dim3(static_cast<unsigned>(blocks)), dim3(kSwThreads), params,
                             sw_fwd_smem<T>(), stream));
  return 0;
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

int check_plan(const oeqb_plan* p) {
  if (!p) return fail(OEQB_ERR_INVALID, "null plan");
  return 0;
}

template <class T>
int tp_forward_t(oeqb_plan* p, int64_t B, const void* X, const void* Y, const void* W, void* Z,
                 cudaStream_t s) {
  Args<T> a = base_args<T>(*p, true);
  a.nitems = B;
  a.X = static_cast<const T*>(X);
  a.Y = static_cast<const T*>(Y);
  a.W = static_cast<const T*>(W);
  a.out0 = static_cast<T*>(Z);
  if constexpr (std::is_same_v<T, float>) {
    if (p->tc.ok && aligned16(X) && aligned16(Z)) return launch_uvw_tc(*p, a, s);
  } else {
    if (p->sw.ok && aligned16(W)) return launch_uvw_sw_fwd(*p, a, s);
  }
  if (p->lkf.ok && lk_aligned(*p, a)) return launch_lk(*p, a, s, true);
  if (p->segf.ok) return launch_seg(*p, 0, a, s);
  if (p->row_ok) return launch_row(*p, 0, a, s);
  return launch(*p, batch_kernel_ptr<T>(0, p->uvw, false, kBatch), a, true, false, s);
}

template <class T>
int tp_backward_t(oeqb_plan* p, int64_t B, const void* X, void* dX, const void* Y, void* dY,
                  const void* W, void* dW, const void* dZ, cudaStream_t s) {
  if (p->shared_w) OEQB_CUDA(cudaMemsetAsync(dW, 0, sizeof(T) * p->wnumel, s));
  Args<T> a = base_args<T>(*p, false);
  a.nitems = B;
  a.X = static_cast<const T*>(X);
  a.Y = static_cast<const T*>(Y);
  a.W = static_cast<const T*>(W);
  a.Gz = static_cast<const T*>(dZ);
  a.out0 = static_cast<T*>(dX);
  a.out1 = static_cast<T*>(dY);
  a.out2 = static_cast<T*>(dW);
  if (p->sw.ok && aligned16(dZ)) return launch_uvw_sw(*p, a, s);
  if (p->lk.ok && lk_aligned(*p, a)) return launch_lk(*p, a, s);
  if (p->segb.ok) return launch_seg(*p, 1, a, s);
  if (p->row_ok) return launch_row(*p, 1, a, s);
  return launch(*p, batch_kernel_ptr<T>(1, p->uvw, false, kBatch), a, false, false, s);
}

template <class T>
int tp_double_backward_t(oeqb_plan* p, int64_t B, const void* X, const void* Y, const void* W,
                         const void* dZ, const void* ddX, const void* ddY, const void* ddW,
                         void* gX, void* gY, void* gW, void* gZ, cudaStream_t s) {
  Args<T> a = base_args<T>(*p, true);
  a.nitems = B;
  a.X = static_cast<const T*>(X);
  a.Y = static_cast<const T*>(Y);
  a.W = static_cast<const T*>(W);
  a.dA = static_cast<const T*>(ddX);
  a.dB = static_cast<const T*>(ddY);
  a.dC = static_cast<const T*>(ddW);
  a.out0 = static_cast<T*>(gZ);
  if (int rc = launch(*p, batch_kernel_ptr<T>(0, p->uvw, true, kBatch), a, true, false, s)) return rc;
  if (p->shared_w) OEQB_CUDA(cudaMemsetAsync(gW, 0, sizeof(T) * p->wnumel, s));
  Args<T> b = base_args<T>(*p, false);
  b.nitems = B;
  b.X = a.X;
  b.Y = a.Y;
  b.W = a.W;
  b.Gz = static_cast<const T*>(dZ);
  b.dA = a.dA;
  b.dB = a.dB;
  b.dC = a.dC;
  b.out0 = static_cast<T*>(gX);
  b.out1 = static_cast<T*>(gY);
  b.out2 = static_cast<T*>(gW);
  return launch(*p, batch_kernel_ptr<T>(1, p->uvw, true, kBatch), b, false, false, s);
}

template <class T>
int conv_fwd_t(oeqb_plan* p, bool db, const void* X, const void* Y, const void* W, const void* ddX,
               const void* ddY, const void* ddW, void* Z, const int64_t* rows, const int64_t* cols,
               int64_t nnz, int64_t nodes, void* ws, size_t ws_bytes, cudaStream_t s) {
  OEQB_CUDA(cudaMemsetAsync(Z, 0, sizeof(T) * size_t(nodes) * p->L3dim, s));
  Args<T> a = base_args<T>(*p, true);
  a.nitems = nnz;
  a.nnodes = nodes;
  a.X = static_cast<const T*>(X);
  a.Y = static_cast<const T*>(Y);
  a.W = static_cast<const T*>(W);
  a.dA = static_cast<const T*>(ddX);
  a.dB = static_cast<const T*>(ddY);
  a.dC = static_cast<const T*>(ddW);
  a.out0 = static_cast<T*>(Z);
  a.rows = reinterpret_cast<const long long*>(rows);
  a.cols = reinterpret_cast<const long long*>(cols);
  if (p->det) {
    if (!db && edge1_pipe_ok(*p, a, ws, ws_bytes)) return launch_edge1_pipe<T>(*p, 4, a, ws, s);
    if (!db && p->edge1_ok && !p->kahan && aligned16(Y))
      return launch_edge1<T>(*p, 4, a, nullptr, s);
    return launch(*p, det_kernel_ptr<T>(0, p->uvw, db, p->kahan), a, true, true, s);
  }
  if (!db && edge1_pipe_ok(*p, a, ws, ws_bytes)) return launch_edge1_pipe<T>(*p, 0, a, ws, s);
  if (!db && p->edge1_ok && aligned16(Y)) return launch_edge1<T>(*p, 2, a, nullptr, s);
  if (!db && p->edge_ok) return launch_edge(*p, 0, a, s);
  return launch(*p, batch_kernel_ptr<T>(0, p->uvw, db, kConvAtomic), a, true, false, s);
}

template <class T>
int conv_bwd_t(oeqb_plan* p, bool db, const void* X, const void* Y, const void* W, const void* dZ,
               const void* ddX, const void* ddY, const void* ddW, void* gX, void* gY, void* gW,
               const int64_t* rows, const int64_t* cols, const int64_t* perm, int64_t nnz,
               int64_t nodes, void* ws, size_t ws_bytes, cudaStream_t s) {
  Args<T> a = base_args<T>(*p, false);
  a.nitems = nnz;
  a.nnodes = nodes;
  a.X = static_cast<const T*>(X);
  a.Y = static_cast<const T*>(Y);
  a.W = static_cast<const T*>(W);
  a.Gz = static_cast<const T*>(dZ);
  a.dA = static_cast<const T*>(ddX);
  a.dB = static_cast<const T*>(ddY);
  a.dC = static_cast<const T*>(ddW);
  a.out0 = static_cast<T*>(gX);
  a.out1 = static_cast<T*>(gY);
  a.out2 = static_cast<T*>(gW);
  a.rows = reinterpret_cast<const long long*>(rows);
  a.cols = reinterpret_cast<const long long*>(cols);
  a.perm = reinterpret_cast<const long long*>(perm);
  // The pipelined backward writes every dX row itself (through its padded accumulator, or the
  // per-sender sums of pass B).
  if (!db && edge1_pipe_ok(*p, a, ws, ws_bytes) && aligned16(gY) && aligned16(gW)) {
    if (!p->det) return launch_edge1_pipe<T>(*p, 1, a, ws, s);
    if (!perm) return fail(OEQB_ERR_INVALID, "deterministic convolution needs transpose_perm");
    return launch_edge1_pipe<T>(*p, 5, a, ws, s);
  }
  OEQB_CUDA(cudaMemsetAsync(gX, 0, sizeof(T) * size_t(nodes) * p->L1dim, s));
  if (p->shared_w) OEQB_CUDA(cudaMemsetAsync(gW, 0, sizeof(T) * p->wnumel, s));
  if (p->det) {
    if (!perm) return fail(OEQB_ERR_INVALID, "deterministic convolution needs transpose_perm");
    const size_t need = edge1_det_ws_bytes(*p, nnz);
    // Records are read with 32-byte loads (float) or 16-byte loads (double).
    const bool ws_ok = ws && (sizeof(T) == 4 ? aligned32(ws) : aligned16(ws));
    if (!db && need && ws_ok && ws_bytes >= need && aligned16(Y) && aligned16(gY)) {
      T* recs = static_cast<T*>(ws);
      if (int rc = launch_edge1<T>(*p, 5, a, recs, s)) return rc;
      return launch_band<T>(*p, a, recs, recs + size_t(kE1Rec) * size_t(nnz), s);
    }
    OEQB_CUDA(cudaMemsetAsync(gY, 0, sizeof(T) * size_t(nnz) * p->L2dim, s));
    return launch(*p, det_kernel_ptr<T>(1, p->uvw, db, p->kahan), a, false, true, s);
  }
  if (!db && p->edge1_ok && aligned16(Y) && aligned16(gY))
    return launch_edge1<T>(*p, 3, a, nullptr, s);
  if (!db && p->edge_ok) return launch_edge(*p, 1, a, s);
  return launch(*p, batch_kernel_ptr<T>(1, p->uvw, db, kConvAtomic), a, false, false, s);
}

}  // namespace

// ---------------------------------------------------------------------------------------
// Graph validation (oeqb_conv_validate).  One thread per edge position; every defect found
// sets its bit in report[0] (bit k = defect code k), so the host can name the most basic
// one whatever the thread order.  seen[] is a bitmap over edge positions for the
// permutation test.  Reads only in-range addresses: a transpose_perm entry is used as an
// index only after its own range check.
__global__ void conv_validate_kernel(const long long* __restrict__ rows,
                                     const long long* __restrict__ cols,
                                     const long long* __restrict__ perm, long long nnz,
                                     long long nodes, int need_sorted, unsigned* report,
                                     unsigned* seen) {
  unsigned bits = 0;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long e = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; e < nnz;
       e += stride) {
    const long long r = rows[e], c = cols[e];
    if (r < 0 || r >= nodes || c < 0 || c >= nodes) bits |= 1u << 1;
    if (need_sorted && e + 1 < nnz && rows[e + 1] < r) bits |= 1u << 4;
    if (perm) {
      const long long q = perm[e];
      if (q < 0 || q >= nnz) {
        bits |= 1u << 2;
        continue;
      }
      const unsigned bit = 1u << (q & 31);
      if (atomicOr(seen + (q >> 5), bit) & bit) bits |= 1u << 5;
      if (e + 1 < nnz) {
        const long long q2 = perm[e + 1];
        if (q2 >= 0 && q2 < nnz && cols[q2] < cols[q]) bits |= 1u << 6;
      }
    }
  }
  bits |= __shfl_xor_sync(0xffffffffu, bits, 16);
  bits |= __shfl_xor_sync(0xffffffffu, bits, 8);
  bits |= __shfl_xor_sync(0xffffffffu, bits, 4);
  bits |= __shfl_xor_sync(0xffffffffu, bits, 2);
  bits |= __shfl_xor_sync(0xffffffffu, bits, 1);
  if (bits && (threadIdx.x & 31) == 0) atomicOr(report, bits);
}

namespace {
// Messages of the device status codes (plan status flags and validation defects).
const char* status_message(int code) {
  switch (code) {
    case 1: return "edge index out of range: every rows/cols entry must lie in [0, num_nodes)";
    case 2: return "transpose_perm entry out of range: entries must lie in [0, num_edges)";
    case 3: return "a kernel's pipeline wait expired; the outputs of that call are incomplete";
    case 4: return "rows are not sorted: the deterministic convolution needs receiver-sorted edges";
    case 5: return "transpose_perm is not a permutation: an edge position appears twice";
    case 6: return "transpose_perm does not list the edges in sender (cols) order";
    default: return "unknown device status";
  }
}
}  // namespace

// ---------------------------------------------------------------------------------------
// Allocation-free forward (oeqb_tp_forward_noalloc).  The problem tables live in this
// file-scope device array instead of plan memory, so the call needs no device allocation.  Every call on a device shares the array and leaves its contents
// behind; calls whose GPU work overlaps (e.g. on two streams) race on it.
constexpr size_t kNoAllocBytes = 64 * 1024;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

namespace {
std::mutex g_noalloc_mu;
constexpr int kMaxDevices = 64;
unsigned char* g_noalloc_addr[kMaxDevices] = {};

// Device address of the array on `device` (which must be current); resolved once per device.
int noalloc_base(int device, unsigned char** out) {
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  if (device < 0 || device >= kMaxDevices) return fail(OEQB_ERR_INVALID, "device index out of range");
  if (!g_noalloc_addr[device]) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr)
      return fail(OEQB_ERR_CUDA, std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
    g_noalloc_addr[device] = static_cast<unsigned char*>(ptr);
  }
  *out = g_noalloc_addr[device];
  return 0;
}
}  // namespace

extern "C" {

const char* oeqb_version(void) { return "oeqb200 0.1.0 (sm_100a)"; }

const char* oeqb_last_error(void) { return g_last_error.c_str(); }

int oeqb_plan_create(const void* descriptor, size_t nbytes, int device, oeqb_plan** out) {
  if (!descriptor || !out) return fail(OEQB_ERR_INVALID, "null argument");
  *out = nullptr;
  auto* p = new oeqb_plan();
  p->device = device;
  if (int rc = parse_descriptor(descriptor, nbytes, *p)) {
    delete p;
    return rc;
  }
  DeviceGuard g(device);
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) == cudaSuccess && sms > 0)
    p->sm_count = sms;
  if (int rc = upload(*p)) {
    if (p->dmem) cudaFree(p->dmem);
    if (p->d_status) cudaFree(p->d_status);
    if (p->tc.wsplit) cudaFree(p->tc.wsplit);
    if (p->sw.wt) cudaFree(p->sw.wt);
    delete p;
    return rc;
  }
  *out = p;
  return 0;
}

int oeqb_plan_destroy(oeqb_plan* p) {
  if (!p) return 0;
  {
    DeviceGuard g(p->device);
    if (p->dmem) cudaFree(p->dmem);
    if (p->d_status) cudaFree(p->d_status);
    if (p->tc.wsplit) cudaFree(p->tc.wsplit);
    if (p->sw.wt) cudaFree(p->sw.wt);
  }
  delete p;
  return 0;
}

size_t oeqb_conv_workspace_bytes(const oeqb_plan* p, int64_t nnz, int64_t node_count) {
  if (!p) return 0;
  if (edge1_pipe_class(*p)) return edge1_pipe_ws_bytes(*p, nnz, node_count);
  return edge1_det_ws_bytes(*p, nnz);
}

int oeqb_plan_check_status(oeqb_plan* p, int* status, void* stream) {
  if (int rc = check_plan(p)) return rc;
  DeviceGuard g(p->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int h = 0;
  OEQB_CUDA(cudaMemcpyAsync(&h, p->d_status, sizeof(int), cudaMemcpyDeviceToHost, s));
  OEQB_CUDA(cudaStreamSynchronize(s));
  OEQB_CUDA(cudaMemsetAsync(p->d_status, 0, sizeof(int), s));
  if (status) *status = h;
  return h ? fail(OEQB_ERR_DEVICE, status_message(h)) : 0;
}

size_t oeqb_conv_validate_scratch_bytes(int64_t nnz) {
  return nnz <= 0 ? 16 : 16 + 4 * static_cast<size_t>((nnz + 31) / 32);
}

int oeqb_conv_validate(const int64_t* rows, const int64_t* cols, const int64_t* transpose_perm,
                       int64_t nnz, int64_t node_count, int need_sorted_rows, void* scratch,
                       size_t scratch_bytes, void* stream) {
  if (nnz < 0 || node_count < 0) return fail(OEQB_ERR_INVALID, "negative size");
  if (nnz == 0) return 0;
  if (!rows || !cols) return fail(OEQB_ERR_INVALID, "null rows/cols");
  const size_t need = oeqb_conv_validate_scratch_bytes(nnz);
  if (!scratch || scratch_bytes < need || (reinterpret_cast<uintptr_t>(scratch) & 15))
    return fail(OEQB_ERR_INVALID, "validation scratch must be 16-byte aligned and hold " +
                                      std::to_string(need) + " bytes");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto* report = static_cast<unsigned*>(scratch);
  OEQB_CUDA(cudaMemsetAsync(scratch, 0, need, s));
  const long long blocks = std::min<long long>((nnz + 255) / 256, 148LL * 8);
  conv_validate_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(
      reinterpret_cast<const long long*>(rows), reinterpret_cast<const long long*>(cols),
      reinterpret_cast<const long long*>(transpose_perm), nnz, node_count, need_sorted_rows,
      report, report + 4);
  OEQB_CUDA(cudaGetLastError());
  unsigned h = 0;
  OEQB_CUDA(cudaMemcpyAsync(&h, report, sizeof(h), cudaMemcpyDeviceToHost, s));
  OEQB_CUDA(cudaStreamSynchronize(s));
  for (int code = 1; code < 32; ++code)
    if (h & (1u << code)) return fail(OEQB_ERR_INVALID, status_message(code));
  return 0;
}

int oeqb_tp_forward(oeqb_plan* p, int64_t batch, const void* L1_in, const void* L2_in,
                    const void* W, void* L3_out, void* stream) {
  if (batch < 0) return fail(OEQB_ERR_INVALID, "negative batch");
  if (int rc = check_plan(p)) return rc;
  DeviceGuard g(p->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return p->dtype == 1 ? tp_forward_t<float>(p, batch, L1_in, L2_in, W, L3_out, s)
                       : tp_forward_t<double>(p, batch, L1_in, L2_in, W, L3_out, s);
}

int oeqb_tp_backward(oeqb_plan* p, int64_t batch, const void* L1_in, void* L1_grad,
                     const void* L2_in, void* L2_grad, const void* W, void* W_grad,
                     const void* L3_grad, void* stream) {
  if (batch < 0) return fail(OEQB_ERR_INVALID, "negative batch");
  if (int rc = check_plan(p)) return rc;
  DeviceGuard g(p->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return p->dtype == 1
             ? tp_backward_t<float>(p, batch, L1_in, L1_grad, L2_in, L2_grad, W, W_grad, L3_grad, s)
             : tp_backward_t<double>(p, batch, L1_in, L1_grad, L2_in, L2_grad, W, W_grad, L3_grad, s);
}

int oeqb_tp_double_backward(oeqb_plan* p, int64_t batch, const void* L1_in, const void* L2_in,
                            const void* W, const void* L3_grad, const void* L1_dgrad,
                            const void* L2_dgrad, const void* W_dgrad, void* L1_grad,
                            void* L2_grad, void* W_grad, void* L3_dgrad, void* stream) {
  if (batch < 0) return fail(OEQB_ERR_INVALID, "negative batch");
  if (int rc = check_plan(p)) return rc;
  DeviceGuard g(p->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return p->dtype == 1
             ? tp_double_backward_t<float>(p, batch, L1_in, L2_in, W, L3_grad, L1_dgrad, L2_dgrad,
                                           W_dgrad, L1_grad, L2_grad, W_grad, L3_dgrad, s)
             : tp_double_backward_t<double>(p, batch, L1_in, L2_in, W, L3_grad, L1_dgrad, L2_dgrad,
                                            W_dgrad, L1_grad, L2_grad, W_grad, L3_dgrad, s);
}

int oeqb_conv_forward(oeqb_plan* p, const void* L1_in, const void* L2_in, const void* W,
                      void* L3_out, const int64_t* rows, const int64_t* cols, int64_t nnz,
                      int64_t node_count, void* workspace, size_t workspace_bytes, void* stream) {
  if (nnz < 0 || node_count < 0) return fail(OEQB_ERR_INVALID, "negative size");
  if (int rc = check_plan(p)) return rc;
  DeviceGuard g(p->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return p->dtype == 1 ? conv_fwd_t<float>(p, false, L1_in, L2_in, W, nullptr, nullptr, nullptr,
                                           L3_out, rows, cols, nnz, node_count, workspace,
                                           workspace_bytes, s)
                       : conv_fwd_t<double>(p, false, L1_in, L2_in, W, nullptr, nullptr, nullptr,
                                            L3_out, rows, cols, nnz, node_count, workspace,
                                            workspace_bytes, s);
}

int oeqb_conv_backward(oeqb_plan* p, const void* L1_in, void* L1_grad, const void* L2_in,
                       void* L2_grad, const void* W, void* W_grad, const void* L3_grad,
                       const int64_t* rows, const int64_t* cols, int64_t nnz, int64_t node_count,
                       void* workspace, size_t workspace_bytes, const int64_t* transpose_perm,
                       void* stream) {
  if (nnz < 0 || node_count < 0) return fail(OEQB_ERR_INVALID, "negative size");
  if (int rc = check_plan(p)) return rc;
  DeviceGuard g(p->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return p->dtype == 1
             ? conv_bwd_t<float>(p, false, L1_in, L2_in, W, L3_grad, nullptr, nullptr, nullptr,
                                 L1_grad, L2_grad, W_grad, rows, cols, transpose_perm, nnz,
                                 node_count, workspace, workspace_bytes, s)
             : conv_bwd_t<double>(p, false, L1_in, L2_in, W, L3_grad, nullptr, nullptr, nullptr,
                                  L1_grad, L2_grad, W_grad, rows, cols, transpose_perm, nnz,
                                  node_count, workspace, workspace_bytes, s);
}

int oeqb_conv_double_backward(oeqb_plan* p, const void* L1_in, const void* L2_in, const void* W,
                              const void* L3_grad, const void* L1_dgrad, const void* L2_dgrad,
                              const void* W_dgrad, void* L1_grad, void* L2_grad, void* W_grad,
                              void* L3_dgrad, const int64_t* rows, const int64_t* cols,
                              int64_t nnz, int64_t node_count, void* workspace,
                              size_t workspace_bytes, const int64_t* transpose_perm,
                              void* stream) {
  (void)workspace;  // the double backward runs the generic kernels, which need none
  (void)workspace_bytes;
  if (nnz < 0 || node_count < 0) return fail(OEQB_ERR_INVALID, "negative size");
  if (int rc = check_plan(p)) return rc;
  DeviceGuard g(p->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p->dtype == 1) {
    if (int rc = conv_fwd_t<float>(p, true, L1_in, L2_in, W, L1_dgrad, L2_dgrad, W_dgrad, L3_dgrad,
                                   rows, cols, nnz, node_count, nullptr, 0, s))
      return rc;
    return conv_bwd_t<float>(p, true, L1_in, L2_in, W, L3_grad, L1_dgrad, L2_dgrad, W_dgrad,
                             L1_grad, L2_grad, W_grad, rows, cols, transpose_perm, nnz, node_count,
                             nullptr, 0, s);
  }
  if (int rc = conv_fwd_t<double>(p, true, L1_in, L2_in, W, L1_dgrad, L2_dgrad, W_dgrad, L3_dgrad,
                                  rows, cols, nnz, node_count, nullptr, 0, s))
    return rc;
  return conv_bwd_t<double>(p, true, L1_in, L2_in, W, L3_grad, L1_dgrad, L2_dgrad, W_dgrad,
                            L1_grad, L2_grad, W_grad, rows, cols, transpose_perm, nnz, node_count,
                            nullptr, 0, s);
}

int oeqb_conv_rows8_ok(const oeqb_plan* p) {
  return p && !p->det && edge1_pipe_class(*p) ? 1 : 0;
}

namespace {
int rows8_check(const oeqb_plan* p, const void* xp, const float* Y, const float* W,
                const int64_t* rows, const int64_t* cols, int64_t nnz, int64_t nodes) {
  if (int rc = check_plan(p)) return rc;
  if (!oeqb_conv_rows8_ok(p))
    return fail(OEQB_ERR_UNSUPPORTED, "the padded-row entry points take float32 atomic "
                                      "single-path plans with one weight per edge");
  if (nnz < 0 || nodes < 0) return fail(OEQB_ERR_INVALID, "negative size");
  if (!aligned32(xp))
    return fail(OEQB_ERR_INVALID, "padded-row entry points need 32-byte aligned padded rows");
  if (!aligned16(Y) || !aligned16(W) || !aligned16(rows) || !aligned16(cols))
    return fail(OEQB_ERR_INVALID, "padded-row entry points need 16-byte aligned arrays");
  return 0;
}
}  // namespace

int oeqb_conv_forward_rows8(oeqb_plan* p, const float* xp, const float* Y, const float* W,
                            float* Z, const int64_t* rows, const int64_t* cols, int64_t nnz,
                            int64_t node_count, int accumulate, int sm_budget, void* stream) {
  if (int rc = rows8_check(p, xp, Y, W, rows, cols, nnz, node_count)) return rc;
  DeviceGuard g(p->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!accumulate) OEQB_CUDA(cudaMemsetAsync(Z, 0, sizeof(float) * size_t(node_count) * p->L3dim, s));
  if (nnz == 0) return 0;
  Args<float> a = base_args<float>(*p, true);
  a.nitems = nnz;
  a.nnodes = node_count;
  a.Y = Y;
  a.W = W;
  a.out0 = Z;
  a.rows = reinterpret_cast<const long long*>(rows);
  a.cols = reinterpret_cast<const long long*>(cols);
  return launch_edge1_pipe_main<float>(*p, 0, a, xp, nullptr, nullptr, sm_budget, s);
}

int oeqb_conv_backward_rows8(oeqb_plan* p, const float* xp, const float* gp, const float* Y,
                             const float* W, float* dY, float* dW, float* dxp,
                             const int64_t* rows, const int64_t* cols, int64_t nnz,
                             int64_t node_count, int sm_budget, void* stream) {
  if (int rc = rows8_check(p, xp, Y, W, rows, cols, nnz, node_count)) return rc;
  if (!aligned32(gp) || !aligned32(dxp))
    return fail(OEQB_ERR_INVALID, "padded-row entry points need 32-byte aligned padded rows");
  if (!aligned16(dY) || !aligned16(dW))
    return fail(OEQB_ERR_INVALID, "padded-row entry points need 16-byte aligned arrays");
  if (nnz == 0) return 0;
  DeviceGuard g(p->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Args<float> a = base_args<float>(*p, false);
  a.nitems = nnz;
  a.nnodes = node_count;
  a.Y = Y;
  a.W = W;
  a.out1 = dY;
  a.out2 = dW;
  a.rows = reinterpret_cast<const long long*>(rows);
  a.cols = reinterpret_cast<const long long*>(cols);
  return launch_edge1_pipe_main<float>(*p, 1, a, xp, gp, dxp, sm_budget, s);
}

int oeqb_tp_forward_noalloc(const void* descriptor, size_t nbytes, int device, int64_t batch,
                            const void* L1_in, const void* L2_in, const void* W, void* L3_out,
                            void* stream) {
  if (!descriptor) return fail(OEQB_ERR_INVALID, "null descriptor");
  if (batch < 0) return fail(OEQB_ERR_INVALID, "negative batch");
  oeqb_plan p;
  p.device = device;
  if (int rc = parse_descriptor(descriptor, nbytes, p)) return rc;
  // This entry point runs the table-driven forward kernel only.  Every specialised path is
  // switched off here, including the shared-weight uvw ones (tc, sw), whose weight images
  // only oeqb_plan_create allocates.
  p.row_ok = false;
  p.segf = {};
  p.segb = {};
  p.segl = {};
  p.lk = {};
  p.lkf = {};
  p.tc = {};
  p.sw = {};
  std::vector<unsigned char> img;
  layout_tables(p, img);
  const size_t need = img.size();
  if (need > kNoAllocBytes)
    return fail(OEQB_ERR_UNSUPPORTED,
                "problem tables need " + std::to_string(need) +
                    " bytes; the allocation-free entry point holds at most " +
                    std::to_string(kNoAllocBytes) + " bytes (use a plan instead)");
  DeviceGuard g(device);
  unsigned char* base = nullptr;
  if (int rc = noalloc_base(device, &base)) return rc;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) == cudaSuccess && sms > 0)
    p.sm_count = sms;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  p.dmem = base;
  // The table kernel of the batch forward raises no device status (it indexes only rows
  // below `batch` and its own tables), so no status word is kept: the returned code is the
  // whole error report of this call.
  p.d_status = nullptr;
  OEQB_CUDA(cudaMemcpyAsync(base, img.data(), img.size(), cudaMemcpyHostToDevice, s));
  const int rc = p.dtype == 1 ? tp_forward_t<float>(&p, batch, L1_in, L2_in, W, L3_out, s)
                              : tp_forward_t<double>(&p, batch, L1_in, L2_in, W, L3_out, s);
  p.dmem = nullptr;  // not owned
  return rc;
}

}  // extern "C"
