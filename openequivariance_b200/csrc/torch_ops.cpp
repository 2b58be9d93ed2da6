// Thin libtorch registration of the reference's operator schemas, forwarding to the C ABI
// of liboeqb200.so.
//
// The schemas, the per-argument validation and its error texts ("Shape mismatch for tensor
// ...", "... is not on the GPU.", "Dtype mismatch for tensor ...") and the output
// allocation rules follow openequivariance/extension/torch_core.hpp:114-139 and 300-722,
// so torch fakes, autograd registration, torch.compile and export keep working unchanged.
// The `json_bytes` argument carries this package's binary problem descriptor; `hash` keys
// the plan cache (one plan per (hash, device)), as in torch_core.hpp:185-296.
#include <cstring>
#include <ATen/ATen.h>
#include <ATen/Context.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <map>
#include <mutex>
#include <sstream>
#include <string>
#include <tuple>
#include <utility>
#include <vector>

#include "oeqb200.h"

namespace {

using at::Tensor;

struct PlanInfo {
  oeqb_plan* plan = nullptr;
  int64_t L1_dim = 0, L2_dim = 0, L3_dim = 0, weight_numel = 0;
  bool shared_weights = false;
  bool deterministic = false;
  at::ScalarType dtype = at::kFloat;
};

std::mutex g_mu;
std::map<std::pair<int64_t, int>, PlanInfo> g_plans;

std::string sizes_str(at::IntArrayRef s) {
  std::ostringstream o;
  o << "[";
  for (size_t i = 0; i < s.size(); ++i) o << (i ? ", " : "") << s[i];
  o << "]";
  return o.str();
}

void check_tensor(const Tensor& t, std::initializer_list<int64_t> shape, at::ScalarType dtype,
                  const char* name) {
  bool ok = t.dim() == static_cast<int64_t>(shape.size());
  if (ok) {
    int64_t i = 0;
    for (int64_t d : shape) {
      if (t.size(i++) != d) {
        ok = false;
        break;
      }
    }
  }
  TORCH_CHECK(ok, "Shape mismatch for tensor '", name, "'. Expected: ",
              sizes_str(std::vector<int64_t>(shape)), ". Got: ", sizes_str(t.sizes()));
  TORCH_CHECK(t.is_cuda(), "Tensor '", name, "' is not on the GPU.");
  TORCH_CHECK(t.scalar_type() == dtype, "Dtype mismatch for tensor '", name,
              "'. Expected: ", static_cast<int>(dtype), ". Got: ",
              static_cast<int>(t.scalar_type()));
}

const PlanInfo& get_plan(const Tensor& desc, int64_t hash, int device) {
  std::lock_guard<std::mutex> g(g_mu);
  auto key = std::make_pair(hash, device);
  auto it = g_plans.find(key);
  if (it != g_plans.end()) return it->second;
  TORCH_CHECK(desc.device().is_cpu() && desc.scalar_type() == at::kByte,
              "problem descriptor must be a CPU uint8 tensor");
  Tensor d = desc.contiguous();
  const auto* h = reinterpret_cast<const int64_t*>(d.data_ptr<uint8_t>());
  TORCH_CHECK(d.numel() >= 128, "problem descriptor too short");
  PlanInfo info;
  int rc = oeqb_plan_create(d.data_ptr<uint8_t>(), static_cast<size_t>(d.numel()), device,
                            &info.plan);
  TORCH_CHECK(rc == 0, "oeqb_plan_create failed: ", oeqb_last_error());
  info.dtype = h[2] == 2 ? at::kDouble : at::kFloat;
  info.shared_weights = h[5] != 0;
  info.L1_dim = h[10];
  info.L2_dim = h[11];
  info.L3_dim = h[12];
  info.weight_numel = h[13];
  info.deterministic = (h[15] & 1) != 0;
  return g_plans.emplace(key, info).first->second;
}

void check_rc(int rc) { TORCH_CHECK(rc == 0, "OpenEquivariance-B200 kernel error: ", oeqb_last_error()); }

void* stream_of(const Tensor& t) {
  return reinterpret_cast<void*>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

// Device checks.  The kernels never fault on bad indices: they skip them and raise the
// plan's status flag.  With checks on (OEQB_DEVICE_CHECKS=1 in the environment, or
// oeqb200::set_device_checks(True)), every convolution call first validates its graph on
// the device (oeqb_conv_validate) and raises before launching anything if it is bad, and
// every call reads the plan's status after its launches and raises if a kernel flagged
// something.  Both synchronise the stream, so they are skipped while the stream is being
// captured into a CUDA graph.  With checks off, oeqb200::check_device_status() reads the
// flags of every plan on demand.
std::atomic<bool> g_checks{[] {
  const char* e = std::getenv("OEQB_DEVICE_CHECKS");
  return e != nullptr && std::string(e) == "1";
}()};

bool checks_active(void* stream) {
  if (!g_checks.load(std::memory_order_relaxed)) return false;
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(static_cast<cudaStream_t>(stream), &st) != cudaSuccess) return false;
  return st == cudaStreamCaptureStatusNone;
}

void validate_graph(const Tensor& rows, const Tensor& cols, const Tensor* perm, int64_t nnz,
                    int64_t nodes, bool sorted_rows, void* stream) {
  const size_t need = oeqb_conv_validate_scratch_bytes(nnz);
  Tensor scratch = at::empty({static_cast<int64_t>(need)}, rows.options().dtype(at::kByte));
  const int rc = oeqb_conv_validate(rows.data_ptr<int64_t>(), cols.data_ptr<int64_t>(),
                                    perm ? perm->data_ptr<int64_t>() : nullptr, nnz, nodes,
                                    sorted_rows ? 1 : 0, scratch.data_ptr(), need, stream);
  TORCH_CHECK(rc == 0, "OpenEquivariance-B200 input check failed: ", oeqb_last_error());
}

void check_status(const PlanInfo& k, void* stream) {
  int st = 0;
  const int rc = oeqb_plan_check_status(k.plan, &st, stream);
  TORCH_CHECK(rc == 0, "OpenEquivariance-B200 device error: ", oeqb_last_error());
}

bool set_device_checks(bool enabled) { return g_checks.exchange(enabled); }

// Reads (and clears) the status flag of every plan of the current device; raises on the
// first that is set.
void check_device_status() {
  const int dev = c10::cuda::current_device();
  std::vector<oeqb_plan*> plans;
  {
    std::lock_guard<std::mutex> g(g_mu);
    for (auto& kv : g_plans)
      if (kv.first.second == dev) plans.push_back(kv.second.plan);
  }
  void* s = reinterpret_cast<void*>(c10::cuda::getCurrentCUDAStream(dev).stream());
  for (oeqb_plan* p : plans) {
    int st = 0;
    const int rc = oeqb_plan_check_status(p, &st, s);
    TORCH_CHECK(rc == 0, "OpenEquivariance-B200 device error: ", oeqb_last_error());
  }
}

int tensor_device(const Tensor& t) { return t.is_cuda() ? t.device().index() : 0; }

void check_weights(const PlanInfo& k, const Tensor& W, int64_t rows, const char* name) {
  if (k.shared_weights)
    check_tensor(W, {k.weight_numel}, k.dtype, name);
  else
    check_tensor(W, {rows, k.weight_numel}, k.dtype, name);
}

// ----------------------------- batch tensor product -----------------------------------

Tensor jit_tp_forward(Tensor json_bytes, int64_t hash, Tensor L1_in, Tensor L2_in, Tensor W,
                      int64_t L3_dim) {
  const PlanInfo& k = get_plan(json_bytes, hash, tensor_device(L1_in));
  const int64_t B = L1_in.size(0);
  check_tensor(L1_in, {B, k.L1_dim}, k.dtype, "L1_in");
  check_tensor(L2_in, {B, k.L2_dim}, k.dtype, "L2_in");
  check_weights(k, W, B, "W");
  (void)L3_dim;
  c10::cuda::CUDAGuard guard(L1_in.device());
  Tensor L3_out = at::empty({B, k.L3_dim}, L1_in.options());
  Tensor x = L1_in.contiguous(), y = L2_in.contiguous(), w = W.contiguous();
  void* st = stream_of(L1_in);
  check_rc(oeqb_tp_forward(k.plan, B, x.data_ptr(), y.data_ptr(), w.data_ptr(), L3_out.data_ptr(),
                           st));
  if (checks_active(st)) check_status(k, st);
  return L3_out;
}

std::tuple<Tensor, Tensor, Tensor> jit_tp_backward(Tensor json_bytes, int64_t hash, Tensor L1_in,
                                                   Tensor L2_in, Tensor W, Tensor L3_grad) {
  const PlanInfo& k = get_plan(json_bytes, hash, tensor_device(L1_in));
  const int64_t B = L1_in.size(0);
  check_tensor(L1_in, {B, k.L1_dim}, k.dtype, "L1_in");
  check_tensor(L2_in, {B, k.L2_dim}, k.dtype, "L2_in");
  check_tensor(L3_grad, {B, k.L3_dim}, k.dtype, "L3_grad");
  check_weights(k, W, B, "W");
  c10::cuda::CUDAGuard guard(L1_in.device());
  Tensor L1_grad = at::empty_like(L1_in, at::MemoryFormat::Contiguous);
  Tensor L2_grad = at::empty_like(L2_in, at::MemoryFormat::Contiguous);
  Tensor W_grad = at::empty_like(W, at::MemoryFormat::Contiguous);
  Tensor x = L1_in.contiguous(), y = L2_in.contiguous(), w = W.contiguous(),
         gz = L3_grad.contiguous();
  void* st = stream_of(L1_in);
  check_rc(oeqb_tp_backward(k.plan, B, x.data_ptr(), L1_grad.data_ptr(), y.data_ptr(),
                            L2_grad.data_ptr(), w.data_ptr(), W_grad.data_ptr(), gz.data_ptr(),
                            st));
  if (checks_active(st)) check_status(k, st);
  return {L1_grad, L2_grad, W_grad};
}

// Problem-descriptor flags (the int64 header of json_bytes, include/oeqb200.h): uvw and
// shared weights.
bool shared_weight_uvw(const Tensor& json_bytes) {
  if (json_bytes.numel() < 16 * 8 || !json_bytes.is_cpu()) return false;
  int64_t h[16];
  std::memcpy(h, json_bytes.contiguous().data_ptr<uint8_t>(), sizeof(h));
  return h[4] != 0 && h[5] != 0;
}

std::tuple<Tensor, Tensor, Tensor, Tensor> jit_tp_double_backward(
    Tensor json_bytes, int64_t hash, Tensor L1_in, Tensor L2_in, Tensor W, Tensor L3_grad,
    Tensor L1_dgrad, Tensor L2_dgrad, Tensor W_dgrad) {
  const PlanInfo& k = get_plan(json_bytes, hash, tensor_device(L1_in));
  const int64_t B = L1_in.size(0);
  check_tensor(L1_in, {B, k.L1_dim}, k.dtype, "L1_in");
  check_tensor(L2_in, {B, k.L2_dim}, k.dtype, "L2_in");
  check_tensor(L3_grad, {B, k.L3_dim}, k.dtype, "L3_grad");
  check_tensor(L1_dgrad, {B, k.L1_dim}, k.dtype, "L1_dgrad");
  check_tensor(L2_dgrad, {B, k.L2_dim}, k.dtype, "L2_dgrad");
  check_weights(k, W, B, "W");
  check_weights(k, W_dgrad, B, "W_dgrad");
  c10::cuda::CUDAGuard guard(L1_in.device());
  Tensor L1_grad = at::empty_like(L1_in, at::MemoryFormat::Contiguous);
  Tensor L2_grad = at::empty_like(L2_in, at::MemoryFormat::Contiguous);
  Tensor W_grad = at::empty_like(W, at::MemoryFormat::Contiguous);
  Tensor L3_dgrad = at::empty_like(L3_grad, at::MemoryFormat::Contiguous);
  Tensor x = L1_in.contiguous(), y = L2_in.contiguous(), w = W.contiguous(),
         gz = L3_grad.contiguous(), dx = L1_dgrad.contiguous(), dy = L2_dgrad.contiguous(),
         dw = W_dgrad.contiguous();
  if (shared_weight_uvw(json_bytes) && B > 0) {
    // Shared-weight uvw: the product is trilinear, so the double backward is three forwards
    // and three backwards with one operand swapped (the dedicated kernels of this class),
    // summed here; the generic double-backward kernels would add every row's weight gradient
    // with global atomics.
    const auto st = stream_of(L1_in);
    auto fwd = [&](const Tensor& a, const Tensor& b, const Tensor& c) {
      Tensor z = at::empty_like(L3_grad, at::MemoryFormat::Contiguous);
      check_rc(oeqb_tp_forward(k.plan, B, a.data_ptr(), b.data_ptr(), c.data_ptr(), z.data_ptr(), st));
      return z;
    };
    auto bwd = [&](const Tensor& a, const Tensor& b, const Tensor& c) {
      Tensor ga = at::empty_like(L1_in, at::MemoryFormat::Contiguous);
      Tensor gb = at::empty_like(L2_in, at::MemoryFormat::Contiguous);
      Tensor gc = at::empty_like(W, at::MemoryFormat::Contiguous);
      check_rc(oeqb_tp_backward(k.plan, B, a.data_ptr(), ga.data_ptr(), b.data_ptr(),
                                gb.data_ptr(), c.data_ptr(), gc.data_ptr(), gz.data_ptr(), st));
      return std::make_tuple(ga, gb, gc);
    };
    L3_dgrad = fwd(dx, y, w);
    L3_dgrad.add_(fwd(x, dy, w));
    L3_dgrad.add_(fwd(x, y, dw));
    auto [gx1, unused_y1, gw1] = bwd(x, dy, w);
    auto [unused_x2, gy2, gw2] = bwd(dx, y, w);
    auto [gx3, gy3, unused_w3] = bwd(x, y, dw);
    if (checks_active(st)) check_status(k, st);
    return {gx1.add_(gx3), gy2.add_(gy3), gw1.add_(gw2), L3_dgrad};
  }
  void* st = stream_of(L1_in);
  check_rc(oeqb_tp_double_backward(k.plan, B, x.data_ptr(), y.data_ptr(), w.data_ptr(),
                                   gz.data_ptr(), dx.data_ptr(), dy.data_ptr(), dw.data_ptr(),
                                   L1_grad.data_ptr(), L2_grad.data_ptr(), W_grad.data_ptr(),
                                   L3_dgrad.data_ptr(), st));
  if (checks_active(st)) check_status(k, st);
  return {L1_grad, L2_grad, W_grad, L3_dgrad};
}

// ----------------------------------- convolution ---------------------------------------

struct ConvIdx {
  int64_t nnz, nodes;
};

ConvIdx check_conv_common(const PlanInfo& k, const Tensor& L1_in, const Tensor& L2_in,
                          const Tensor& rows, const Tensor& cols, const Tensor& workspace,
                          const Tensor& transpose_perm, const char* what) {
  const int64_t nnz = rows.size(0);
  const int64_t nodes = L1_in.size(0);
  check_tensor(L1_in, {nodes, k.L1_dim}, k.dtype, "L1_in");
  check_tensor(L2_in, {nnz, k.L2_dim}, k.dtype, "L2_in");
  TORCH_CHECK(workspace.dim() == 1, "Shape mismatch for tensor 'workspace'. Expected a 1-D buffer.");
  TORCH_CHECK(workspace.is_cuda(), "Tensor 'workspace' is not on the GPU.");
  TORCH_CHECK(workspace.scalar_type() == at::kByte, "Dtype mismatch for tensor 'workspace'.");
  check_tensor(rows, {nnz}, at::kLong, "rows");
  check_tensor(cols, {nnz}, at::kLong, "cols");
  if (k.deterministic)
    check_tensor(transpose_perm, {nnz}, at::kLong, "transpose perm");
  else
    at::globalContext().alertNotDeterministic(what);
  return {nnz, nodes};
}

Tensor jit_conv_forward(Tensor json_bytes, int64_t hash, Tensor L1_in, Tensor L2_in, Tensor W,
                        int64_t L3_dim, Tensor rows, Tensor cols, Tensor workspace,
                        Tensor transpose_perm) {
  const PlanInfo& k = get_plan(json_bytes, hash, tensor_device(L1_in));
  (void)L3_dim;
  ConvIdx c = check_conv_common(k, L1_in, L2_in, rows, cols, workspace, transpose_perm,
                                "OpenEquivariance_conv_atomic_forward");
  check_weights(k, W, c.nnz, "W");
  c10::cuda::CUDAGuard guard(L1_in.device());
  Tensor L3_out = at::empty({c.nodes, k.L3_dim}, L1_in.options());
  Tensor x = L1_in.contiguous(), y = L2_in.contiguous(), w = W.contiguous(),
         r = rows.contiguous(), cl = cols.contiguous();
  void* st = stream_of(L1_in);
  const bool chk = checks_active(st);
  if (chk) validate_graph(r, cl, nullptr, c.nnz, c.nodes, k.deterministic, st);
  // Some kernels keep node rows in a padded layout in the workspace; a module's buffer that is
  // too small is replaced for this call (torch's caching allocator).
  Tensor ws = workspace;
  const size_t need = oeqb_conv_workspace_bytes(k.plan, c.nnz, c.nodes);
  if (need > static_cast<size_t>(workspace.numel()))
    ws = at::empty({static_cast<int64_t>(need)}, workspace.options());
  check_rc(oeqb_conv_forward(k.plan, x.data_ptr(), y.data_ptr(), w.data_ptr(), L3_out.data_ptr(),
                             r.data_ptr<int64_t>(), cl.data_ptr<int64_t>(), c.nnz, c.nodes,
                             ws.data_ptr(), static_cast<size_t>(ws.numel()), st));
  if (chk) check_status(k, st);
  return L3_out;
}

// Convolution backward into caller-provided gradient tensors (contiguous; e.g. row slices
// of larger buffers).  Shared by jit_conv_backward and oeqb200::conv_backward_into.
void conv_backward_impl(const PlanInfo& k, const ConvIdx& c, Tensor L1_in, Tensor L2_in,
                        Tensor W, Tensor L3_grad, Tensor rows, Tensor cols, Tensor workspace,
                        Tensor transpose_perm, Tensor& L1_grad, Tensor& L2_grad, Tensor& W_grad);

std::tuple<Tensor, Tensor, Tensor> jit_conv_backward(Tensor json_bytes, int64_t hash,
                                                     Tensor L1_in, Tensor L2_in, Tensor W,
                                                     Tensor L3_grad, Tensor rows, Tensor cols,
                                                     Tensor workspace, Tensor transpose_perm) {
  const PlanInfo& k = get_plan(json_bytes, hash, tensor_device(L1_in));
  ConvIdx c = check_conv_common(k, L1_in, L2_in, rows, cols, workspace, transpose_perm,
                                "OpenEquivariance_conv_atomic_backward");
  check_tensor(L3_grad, {c.nodes, k.L3_dim}, k.dtype, "L3_grad");
  check_weights(k, W, c.nnz, "W");
  c10::cuda::CUDAGuard guard(L1_in.device());
  Tensor L1_grad = at::empty_like(L1_in, at::MemoryFormat::Contiguous);
  Tensor L2_grad = at::empty_like(L2_in, at::MemoryFormat::Contiguous);
  Tensor W_grad = at::empty_like(W, at::MemoryFormat::Contiguous);
  conv_backward_impl(k, c, L1_in, L2_in, W, L3_grad, rows, cols, workspace, transpose_perm,
                     L1_grad, L2_grad, W_grad);
  return {L1_grad, L2_grad, W_grad};
}

void conv_backward_into(Tensor json_bytes, int64_t hash, Tensor L1_in, Tensor L2_in, Tensor W,
                        Tensor L3_grad, Tensor rows, Tensor cols, Tensor workspace,
                        Tensor transpose_perm, Tensor L1_grad, Tensor L2_grad, Tensor W_grad) {
  const PlanInfo& k = get_plan(json_bytes, hash, tensor_device(L1_in));
  ConvIdx c = check_conv_common(k, L1_in, L2_in, rows, cols, workspace, transpose_perm,
                                "OpenEquivariance_conv_atomic_backward");
  check_tensor(L3_grad, {c.nodes, k.L3_dim}, k.dtype, "L3_grad");
  check_weights(k, W, c.nnz, "W");
  check_tensor(L1_grad, {c.nodes, k.L1_dim}, k.dtype, "L1_grad");
  check_tensor(L2_grad, {c.nnz, k.L2_dim}, k.dtype, "L2_grad");
  check_weights(k, W_grad, c.nnz, "W_grad");
  TORCH_CHECK(L1_grad.is_contiguous() && L2_grad.is_contiguous() && W_grad.is_contiguous(),
              "conv_backward_into: gradient outputs must be contiguous");
  c10::cuda::CUDAGuard guard(L1_in.device());
  conv_backward_impl(k, c, L1_in, L2_in, W, L3_grad, rows, cols, workspace, transpose_perm,
                     L1_grad, L2_grad, W_grad);
}

void conv_backward_impl(const PlanInfo& k, const ConvIdx& c, Tensor L1_in, Tensor L2_in,
                        Tensor W, Tensor L3_grad, Tensor rows, Tensor cols, Tensor workspace,
                        Tensor transpose_perm, Tensor& L1_grad, Tensor& L2_grad, Tensor& W_grad) {
  Tensor x = L1_in.contiguous(), y = L2_in.contiguous(), w = W.contiguous(),
         gz = L3_grad.contiguous(), r = rows.contiguous(), cl = cols.contiguous();
  Tensor tp = k.deterministic ? transpose_perm.contiguous() : Tensor();
  // The single-path kernels keep one record per edge (deterministic) or padded node rows
  // (atomic) in the workspace; a module's buffer that is too small is replaced for this call
  // (torch's caching allocator).
  Tensor ws = workspace;
  const size_t need = oeqb_conv_workspace_bytes(k.plan, c.nnz, c.nodes);
  if (need > static_cast<size_t>(workspace.numel()))
    ws = at::empty({static_cast<int64_t>(need)}, workspace.options());
  void* st = stream_of(L1_in);
  const bool chk = checks_active(st);
  if (chk) validate_graph(r, cl, k.deterministic ? &tp : nullptr, c.nnz, c.nodes, k.deterministic, st);
  check_rc(oeqb_conv_backward(
      k.plan, x.data_ptr(), L1_grad.data_ptr(), y.data_ptr(), L2_grad.data_ptr(), w.data_ptr(),
      W_grad.data_ptr(), gz.data_ptr(), r.data_ptr<int64_t>(), cl.data_ptr<int64_t>(), c.nnz,
      c.nodes, ws.data_ptr(), static_cast<size_t>(ws.numel()),
      k.deterministic ? tp.data_ptr<int64_t>() : nullptr, st));
  if (chk) check_status(k, st);
}

std::tuple<Tensor, Tensor, Tensor, Tensor> jit_conv_double_backward(
    Tensor json_bytes, int64_t hash, Tensor L1_in, Tensor L2_in, Tensor W, Tensor L3_grad,
    Tensor L1_dgrad, Tensor L2_dgrad, Tensor W_dgrad, Tensor rows, Tensor cols, Tensor workspace,
    Tensor transpose_perm) {
  const PlanInfo& k = get_plan(json_bytes, hash, tensor_device(L1_in));
  ConvIdx c = check_conv_common(k, L1_in, L2_in, rows, cols, workspace, transpose_perm,
                                "OpenEquivariance_conv_atomic_double_backward");
  check_tensor(L3_grad, {c.nodes, k.L3_dim}, k.dtype, "L3_grad");
  check_tensor(L1_dgrad, {c.nodes, k.L1_dim}, k.dtype, "L1_dgrad");
  check_tensor(L2_dgrad, {c.nnz, k.L2_dim}, k.dtype, "L2_dgrad");
  check_weights(k, W, c.nnz, "W");
  check_weights(k, W_dgrad, c.nnz, "W_dgrad");
  c10::cuda::CUDAGuard guard(L1_in.device());
  Tensor L1_grad = at::empty_like(L1_in, at::MemoryFormat::Contiguous);
  Tensor L2_grad = at::empty_like(L2_in, at::MemoryFormat::Contiguous);
  Tensor W_grad = at::empty_like(W, at::MemoryFormat::Contiguous);
  Tensor L3_dgrad = at::empty_like(L3_grad, at::MemoryFormat::Contiguous);
  Tensor x = L1_in.contiguous(), y = L2_in.contiguous(), w = W.contiguous(),
         gz = L3_grad.contiguous(), dx = L1_dgrad.contiguous(), dy = L2_dgrad.contiguous(),
         dw = W_dgrad.contiguous(), r = rows.contiguous(), cl = cols.contiguous();
  Tensor tp = k.deterministic ? transpose_perm.contiguous() : Tensor();
  void* st = stream_of(L1_in);
  const bool chk = checks_active(st);
  if (chk) validate_graph(r, cl, k.deterministic ? &tp : nullptr, c.nnz, c.nodes, k.deterministic, st);
  check_rc(oeqb_conv_double_backward(
      k.plan, x.data_ptr(), y.data_ptr(), w.data_ptr(), gz.data_ptr(), dx.data_ptr(),
      dy.data_ptr(), dw.data_ptr(), L1_grad.data_ptr(), L2_grad.data_ptr(), W_grad.data_ptr(),
      L3_dgrad.data_ptr(), r.data_ptr<int64_t>(), cl.data_ptr<int64_t>(), c.nnz, c.nodes,
      workspace.data_ptr(), static_cast<size_t>(workspace.numel()),
      k.deterministic ? tp.data_ptr<int64_t>() : nullptr, st));
  if (chk) check_status(k, st);
  return {L1_grad, L2_grad, W_grad, L3_dgrad};
}

// Padded-row convolution (this package's ops; the multi-GPU partition's layout).
bool conv_rows8_ok(Tensor json_bytes, int64_t hash, int64_t device) {
  const PlanInfo& k = get_plan(json_bytes, hash, static_cast<int>(device));
  return oeqb_conv_rows8_ok(k.plan) != 0;
}

void check_rows8(const Tensor& t, int64_t rows, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kFloat && t.dim() == 2 && t.size(0) == rows &&
                  t.size(1) == 8 && t.is_contiguous(),
              "Tensor '", name, "' must be a contiguous float32 [", rows, ", 8] GPU tensor");
}

void conv_forward_rows8(Tensor json_bytes, int64_t hash, Tensor xp, Tensor Y, Tensor W, Tensor Z,
                        Tensor rows, Tensor cols, bool accumulate, int64_t sm_budget) {
  const PlanInfo& k = get_plan(json_bytes, hash, tensor_device(xp));
  const int64_t nodes = xp.size(0), nnz = rows.size(0);
  check_rows8(xp, nodes, "xp");
  check_tensor(Y, {nnz, k.L2_dim}, k.dtype, "L2_in");
  check_weights(k, W, nnz, "W");
  check_tensor(Z, {nodes, k.L3_dim}, k.dtype, "L3_out");
  check_tensor(rows, {nnz}, at::kLong, "rows");
  check_tensor(cols, {nnz}, at::kLong, "cols");
  TORCH_CHECK(Y.is_contiguous() && W.is_contiguous() && Z.is_contiguous() && rows.is_contiguous() &&
                  cols.is_contiguous(), "conv_forward_rows8: tensors must be contiguous");
  c10::cuda::CUDAGuard guard(xp.device());
  void* st = stream_of(xp);
  const bool chk = checks_active(st);
  if (chk) validate_graph(rows, cols, nullptr, nnz, nodes, false, st);
  check_rc(oeqb_conv_forward_rows8(k.plan, xp.data_ptr<float>(), Y.data_ptr<float>(),
                                   W.data_ptr<float>(), Z.data_ptr<float>(), rows.data_ptr<int64_t>(),
                                   cols.data_ptr<int64_t>(), nnz, nodes, accumulate ? 1 : 0,
                                   static_cast<int>(sm_budget), st));
  if (chk) check_status(k, st);
}

void conv_backward_rows8(Tensor json_bytes, int64_t hash, Tensor xp, Tensor gp, Tensor Y, Tensor W,
                         Tensor dY, Tensor dW, Tensor dxp, Tensor rows, Tensor cols,
                         int64_t sm_budget) {
  const PlanInfo& k = get_plan(json_bytes, hash, tensor_device(xp));
  const int64_t nodes = xp.size(0), nnz = rows.size(0);
  check_rows8(xp, nodes, "xp");
  check_rows8(gp, nodes, "gp");
  check_rows8(dxp, nodes, "dxp");
  check_tensor(Y, {nnz, k.L2_dim}, k.dtype, "L2_in");
  check_weights(k, W, nnz, "W");
  check_tensor(dY, {nnz, k.L2_dim}, k.dtype, "L2_grad");
  check_weights(k, dW, nnz, "W_grad");
  check_tensor(rows, {nnz}, at::kLong, "rows");
  check_tensor(cols, {nnz}, at::kLong, "cols");
  TORCH_CHECK(Y.is_contiguous() && W.is_contiguous() && dY.is_contiguous() && dW.is_contiguous() &&
                  rows.is_contiguous() && cols.is_contiguous(),
              "conv_backward_rows8: tensors must be contiguous");
  c10::cuda::CUDAGuard guard(xp.device());
  void* st = stream_of(xp);
  const bool chk = checks_active(st);
  if (chk) validate_graph(rows, cols, nullptr, nnz, nodes, false, st);
  check_rc(oeqb_conv_backward_rows8(k.plan, xp.data_ptr<float>(), gp.data_ptr<float>(),
                                    Y.data_ptr<float>(), W.data_ptr<float>(), dY.data_ptr<float>(),
                                    dW.data_ptr<float>(), dxp.data_ptr<float>(),
                                    rows.data_ptr<int64_t>(), cols.data_ptr<int64_t>(), nnz, nodes,
                                    static_cast<int>(sm_budget), st));
  if (chk) check_status(k, st);
}

// ----------------------------- symmetric contraction ----------------------------------

int dtype_code(const Tensor& t) {
  TORCH_CHECK(t.scalar_type() == at::kFloat || t.scalar_type() == at::kDouble,
              "expected float32 or float64, got ", t.scalar_type());
  return t.scalar_type() == at::kDouble ? 2 : 1;
}

// group_gemm (torch_core.hpp:653-684): same checks and output shapes; ragged_counts may live
// on the host (as the reference's bincount does) or on the device.
Tensor group_gemm(Tensor A, Tensor B, Tensor ragged_counts, int64_t num_W, int64_t batch_size,
                  int64_t m, int64_t k, int64_t ragged_inner) {
  TORCH_CHECK(A.scalar_type() == B.scalar_type(), "group_gemm: A and B must have the same dtype");
  TORCH_CHECK(ragged_counts.scalar_type() == at::kLong, "group_gemm: ragged_counts must be int64");
  TORCH_CHECK(A.is_cuda() && B.is_cuda(), "group_gemm: A and B must be on the GPU");
  const c10::cuda::CUDAGuard guard(A.device());
  Tensor Ac = A.contiguous(), Bc = B.contiguous();
  Tensor counts = ragged_counts.to(A.device(), /*non_blocking=*/false).contiguous();
  Tensor offsets = at::zeros({num_W + 1}, counts.options());
  if (num_W > 0) offsets.narrow(0, 1, num_W).copy_(at::cumsum(counts.narrow(0, 0, num_W), 0));
  Tensor C;
  int64_t rows;
  if (ragged_inner == 0) {
    rows = B.size(0);
    C = at::empty({rows, batch_size, m}, A.options());
  } else {
    rows = A.size(0);
    C = at::empty({num_W, batch_size, m, k}, A.options());
  }
  check_rc(oeqb_group_gemm(dtype_code(A), Ac.data_ptr(), Bc.data_ptr(),
                           offsets.data_ptr<int64_t>(), static_cast<int>(num_W), rows,
                           static_cast<int>(batch_size), static_cast<int>(m), static_cast<int>(k),
                           static_cast<int>(ragged_inner), C.data_ptr(), stream_of(A)));
  return C;
}

std::vector<int> int_list(at::IntArrayRef v) { return std::vector<int>(v.begin(), v.end()); }

// Fused symmetric contraction (this package's op; no reference schema).  The float64
// kernels take at most 4 padded outputs per pass; wider float64 output sets run in chunks
// of 4 outputs, each pass writing its own columns of `out` (and its own coefficient
// columns of the gradient), with the x gradients of the chunks summed in chunk order.
constexpr int kF64Chunk = 4;

bool chunked(const Tensor& x, const Tensor& coef) {
  return x.scalar_type() == at::kDouble && coef.size(3) > kF64Chunk;
}

Tensor chunk_coef(const Tensor& coef, int64_t s, int64_t n) {
  Tensor c = at::zeros({coef.size(0), coef.size(1), coef.size(2), kF64Chunk}, coef.options());
  c.narrow(3, 0, n).copy_(coef.narrow(3, s, n));
  return c;
}

Tensor sc_forward(Tensor x, Tensor perm, Tensor elem_offsets, Tensor coef, at::IntArrayRef out_col,
                  at::IntArrayRef out_step, int64_t out_dim, int64_t degree) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 3, "sc_forward: x must be a [N, C, K] GPU tensor");
  TORCH_CHECK(coef.dim() == 4 && coef.scalar_type() == x.scalar_type(), "sc_forward: coef must be [E, C, M, DT] of x's dtype");
  const c10::cuda::CUDAGuard guard(x.device());
  Tensor xc = x.contiguous(), cc = coef.contiguous();
  Tensor out = at::empty({x.size(0), out_dim}, x.options());
  const auto col = int_list(out_col), step = int_list(out_step);
  TORCH_CHECK(col.size() == step.size(), "sc_forward: out_col / out_step length mismatch");
  const int nout = static_cast<int>(col.size());
  auto run = [&](const Tensor& cf, int dt, int s, int n) {
    check_rc(oeqb_sc_forward(dtype_code(x), x.size(0), static_cast<int>(x.size(1)),
                             static_cast<int>(x.size(2)), static_cast<int>(degree), dt, n,
                             col.data() + s, step.data() + s, out_dim,
                             static_cast<int>(coef.size(0)), xc.data_ptr(),
                             perm.data_ptr<int64_t>(), elem_offsets.data_ptr<int64_t>(),
                             cf.data_ptr(), out.data_ptr(), stream_of(x)));
  };
  if (!chunked(x, cc)) {
    run(cc, static_cast<int>(cc.size(3)), 0, nout);
    return out;
  }
  for (int s = 0; s < nout; s += kF64Chunk) {
    const int n = std::min(kF64Chunk, nout - s);
    run(chunk_coef(cc, s, n), kF64Chunk, s, n);
  }
  return out;
}

std::tuple<Tensor, Tensor> sc_backward(Tensor x, Tensor perm, Tensor elem_offsets,
                                       Tensor coef, Tensor grad_out,
                                       at::IntArrayRef out_col, at::IntArrayRef out_step,
                                       int64_t degree) {
  TORCH_CHECK(x.is_cuda() && x.dim() == 3, "sc_backward: x must be a [N, C, K] GPU tensor");
  const c10::cuda::CUDAGuard guard(x.device());
  Tensor xc = x.contiguous(), cc = coef.contiguous(), gc = grad_out.contiguous();
  const auto col = int_list(out_col), step = int_list(out_step);
  const int nout = static_cast<int>(col.size());
  auto run = [&](const Tensor& cf, int dt, int s, int n, Tensor& gx, Tensor& gcoef) {
    check_rc(oeqb_sc_backward(dtype_code(x), x.size(0), static_cast<int>(x.size(1)),
                              static_cast<int>(x.size(2)), static_cast<int>(degree), dt, n,
                              col.data() + s, step.data() + s, gc.size(1),
                              static_cast<int>(coef.size(0)), xc.data_ptr(),
                              perm.data_ptr<int64_t>(), elem_offsets.data_ptr<int64_t>(),
                              cf.data_ptr(), gc.data_ptr(), gx.data_ptr(), gcoef.data_ptr(),
                              stream_of(x)));
  };
  if (!chunked(x, cc)) {
    Tensor gx = at::empty_like(xc);
    Tensor gcoef = at::empty_like(cc);
    run(cc, static_cast<int>(cc.size(3)), 0, nout, gx, gcoef);
    return {gx, gcoef};
  }
  Tensor gx_sum = at::zeros_like(xc);
  Tensor gcoef = at::zeros_like(cc);
  for (int s = 0; s < nout; s += kF64Chunk) {
    const int n = std::min(kF64Chunk, nout - s);
    Tensor cf = chunk_coef(cc, s, n);
    Tensor gx = at::empty_like(xc);
    Tensor gcf = at::empty_like(cf);
    run(cf, kF64Chunk, s, n, gx, gcf);
    gx_sum.add_(gx);
    gcoef.narrow(3, s, n).copy_(gcf.narrow(3, 0, n));
  }
  return {gx_sum, gcoef};
}

}  // namespace

TORCH_LIBRARY(oeqb200, m) {
  m.def("set_device_checks(bool enabled) -> bool", &set_device_checks);
  m.def("check_device_status() -> ()", &check_device_status);
  m.def("conv_rows8_ok(Tensor json_bytes, int hash, int device) -> bool", &conv_rows8_ok);
  m.def("conv_forward_rows8(Tensor json_bytes, int hash, Tensor xp, Tensor Y, Tensor W, Tensor(a!) Z, Tensor rows, Tensor cols, bool accumulate, int sm_budget) -> ()");
  m.def("conv_backward_rows8(Tensor json_bytes, int hash, Tensor xp, Tensor gp, Tensor Y, Tensor W, Tensor(a!) dY, Tensor(b!) dW, Tensor(c!) dxp, Tensor rows, Tensor cols, int sm_budget) -> ()");
  m.def("conv_backward_into(Tensor json_bytes, int hash, Tensor L1_in, Tensor L2_in, Tensor W, Tensor L3_grad, Tensor rows, Tensor cols, Tensor workspace, Tensor transpose_perm, Tensor(a!) L1_grad, Tensor(b!) L2_grad, Tensor(c!) W_grad) -> ()");
  m.def("sc_forward(Tensor x, Tensor perm, Tensor elem_offsets, Tensor coef, int[] out_col, int[] out_step, int out_dim, int degree) -> Tensor");
  m.def("sc_backward(Tensor x, Tensor perm, Tensor elem_offsets, Tensor coef, Tensor grad_out, int[] out_col, int[] out_step, int degree) -> (Tensor, Tensor)");
}

TORCH_LIBRARY_IMPL(oeqb200, CUDA, m) {
  m.impl("sc_forward", &sc_forward);
  m.impl("conv_backward_into", &conv_backward_into);
  m.impl("conv_forward_rows8", &conv_forward_rows8);
  m.impl("conv_backward_rows8", &conv_backward_rows8);
  m.impl("sc_backward", &sc_backward);
}

TORCH_LIBRARY(libtorch_tp_jit, m) {
  m.def("jit_tp_forward(Tensor json_bytes, int hash, Tensor L1_in, Tensor L2_in, Tensor W, int L3_dim) -> Tensor");
  m.def("jit_tp_backward(Tensor json_bytes, int hash, Tensor L1_in, Tensor L2_in, Tensor W, Tensor L3_grad) -> (Tensor, Tensor, Tensor)");
  m.def("jit_tp_double_backward(Tensor json_bytes, int hash, Tensor L1_in, Tensor L2_in, Tensor W, Tensor L3_grad, Tensor L1_dgrad, Tensor L2_dgrad, Tensor W_dgrad) -> (Tensor, Tensor, Tensor, Tensor)");
  m.def("jit_conv_forward(Tensor json_bytes, int hash, Tensor L1_in, Tensor L2_in, Tensor W, int L3_dim, Tensor rows, Tensor cols, Tensor workspace, Tensor transpose_perm) -> Tensor");
  m.def("jit_conv_backward(Tensor json_bytes, int hash, Tensor L1_in, Tensor L2_in, Tensor W, Tensor L3_grad, Tensor rows, Tensor cols, Tensor workspace, Tensor transpose_perm) -> (Tensor, Tensor, Tensor)");
  m.def("jit_conv_double_backward(Tensor json_bytes, int hash, Tensor L1_in, Tensor L2_in, Tensor W, Tensor L3_grad, Tensor L1_dgrad, Tensor L2_dgrad, Tensor W_dgrad, Tensor rows, Tensor cols, Tensor workspace, Tensor transpose_perm) -> (Tensor, Tensor, Tensor, Tensor)");
  m.def("group_gemm(Tensor A, Tensor B, Tensor ragged_counts, int num_W, int batch_size, int m, int k, int ragged_inner) -> Tensor");
}

TORCH_LIBRARY_IMPL(libtorch_tp_jit, CUDA, m) {
  m.impl("jit_tp_forward", &jit_tp_forward);
  m.impl("jit_tp_backward", &jit_tp_backward);
  m.impl("jit_tp_double_backward", &jit_tp_double_backward);
  m.impl("jit_conv_forward", &jit_conv_forward);
  m.impl("jit_conv_backward", &jit_conv_backward);
  m.impl("jit_conv_double_backward", &jit_conv_double_backward);
  m.impl("group_gemm", &group_gemm);
}
