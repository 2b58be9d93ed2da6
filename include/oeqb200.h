/*
 * oeqb200.h -- C ABI of the B200-native Clebsch-Gordan tensor-product library
 * (liboeqb200.so).
 *
 * Every entry point takes plain pointers and sizes, returns 0 on success and a
 * non-zero OEQB_ERR_* code on failure (the message is available from
 * oeqb_last_error()), and never aborts the process.  Device pointers must live on the
 * device the plan was created for; `stream` is a cudaStream_t (NULL = legacy default
 * stream).  All launches are asynchronous on that stream.
 *
 * The entry points replace the reference's JIT runtime interfaces:
 *   plan create        <- JITTPImpl / JITConvImpl constructors + NVRTC compile
 *                         (openequivariance/extension/tensorproducts.hpp:22-49,
 *                          convolution.hpp:37-77, backend/backend_cuda.hpp:199-301)
 *   oeqb_tp_*          <- JITTPImpl::exec_tensor_product / backward / double_backward
 *                         (openequivariance/extension/tensorproducts.hpp:77-116)
 *   oeqb_conv_*        <- JITConvImpl::exec_conv / backward / double_backward
 *                         (openequivariance/extension/convolution.hpp:79-186)
 *   oeqb_sc_*          <- group_gemm + the torch glue of the MACE symmetric contraction
 *                         (openequivariance/extension/group_mm.hpp:38-141,
 *                          _torch/symmetric_contraction/SymmetricContraction.py:220-336)
 *
 * Problem descriptor (little-endian, produced by openequivariance_b200.plan.pack_descriptor):
 *   int64 header[16] = { magic 0x4251454F ("OEQB"), version 1, dtype (1=f32, 2=f64),
 *                        layout (0=mul_ir, 1=ir_mul), mode (0=uvu, 1=uvw), shared_weights,
 *                        n_irreps_in1, n_irreps_in2, n_irreps_out, n_instructions,
 *                        L1_dim, L2_dim, L3_dim, weight_numel, n_cg_entries,
 *                        flags (bit0 deterministic conv, bit1 Kahan summation) }
 *   int64 irreps[(n1+n2+n3)][3]         = { mul, l, offset } for in1, in2, out in order
 *   instructions[n_instructions]        = { int64 i_in1, i_in2, i_out, weight_offset,
 *                                           cg_offset, cg_nnz; double path_weight }
 *   cg[n_cg_entries]                    = { int64 i, j, k; double value }
 * Weights are in the reference's "oeq" order (multiplicities split in chunks of 32,
 * uvu blocks [v][u], uvw blocks [v][u][w]).
 */
#ifndef OEQB200_H_
#define OEQB200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OEQB_OK 0
#define OEQB_ERR_INVALID 1      /* bad argument or descriptor */
#define OEQB_ERR_UNSUPPORTED 2  /* problem outside the supported subset */
#define OEQB_ERR_CUDA 3         /* CUDA runtime error */
#define OEQB_ERR_DEVICE 4       /* a kernel flagged an out-of-range index */

typedef struct oeqb_plan oeqb_plan;

/* Library version string. */
const char* oeqb_version(void);

/* Message of the last failing call on this host thread ("" if none). */
const char* oeqb_last_error(void);

/* Builds a plan for `device` from a problem descriptor (see above).  Replaces the
 * reference's per-problem NVRTC compile: kernels are compiled ahead of time for
 * sm_100a and specialised per degree triple; the plan only uploads tables. */
int oeqb_plan_create(const void* descriptor, size_t nbytes, int device, oeqb_plan** out);
int oeqb_plan_destroy(oeqb_plan* plan);

/* Bytes of workspace oeqb_conv_forward / oeqb_conv_backward use for `nnz` edges and
 * `node_count` nodes (replaces the reference's workspace sizing,
 * core/LoopUnrollConv.py:138-170).  Nonzero only for single-path multiplicity-1 problems
 * (BASELINE C3's class).  Float32 plans with one weight per edge keep X and dZ in 32-byte
 * rows, then the dX accumulator (atomic: 3 x 32 x node_count bytes + 256) or one 32-byte
 * record per edge and 64 bytes per 32 edges for the backward's per-block sums (deterministic:
 * 2 x 32 x node_count + 32 x nnz + 64 x ceil(nnz / 32) + 256); other deterministic plans keep
 * one 8-value record per edge and 16 values per 32 edges for the backward's per-block sums.  With a smaller (or, for the float32 kernels, not 32-byte
 * aligned) workspace those plans run slower kernels that need none.  The double backward
 * needs none. */
size_t oeqb_conv_workspace_bytes(const oeqb_plan* plan, int64_t nnz, int64_t node_count);

/* Synchronises `stream` and reports (then clears) the plan's device error flag:
 * 0 = clean, 1 = an edge index was out of range, 2 = a permutation entry was out of
 * range, 3 = a pipeline wait inside a kernel expired (that call's outputs are incomplete).
 * Kernels skip bad entries instead of faulting.  Returns OEQB_ERR_DEVICE with the message
 * when the flag was set.  (The reference has no counterpart: its kernels index unchecked.) */
int oeqb_plan_check_status(oeqb_plan* plan, int* status, void* stream);

/* Checks a convolution graph on the device before it is used, synchronously on `stream`
 * (no counterpart in the reference, whose kernels trust their indices).  Reports, as
 * OEQB_ERR_INVALID with the message of the most basic defect found:
 *   rows/cols entries outside [0, node_count);
 *   transpose_perm (if not NULL) entries outside [0, nnz), repeated entries (not a
 *   permutation), or an order that does not sort the edges by cols (sender);
 *   rows not sorted, when need_sorted_rows is nonzero (deterministic plans).
 * `scratch` is device memory of at least oeqb_conv_validate_scratch_bytes(nnz) bytes,
 * 16-byte aligned; the call clears it itself. */
size_t oeqb_conv_validate_scratch_bytes(int64_t nnz);
int oeqb_conv_validate(const int64_t* rows, const int64_t* cols, const int64_t* transpose_perm,
                       int64_t nnz, int64_t node_count, int need_sorted_rows, void* scratch,
                       size_t scratch_bytes, void* stream);

/* ---- batch tensor product (replaces tensorproducts.hpp:77-88) ----
 * L1_in [batch, L1_dim], L2_in [batch, L2_dim], W [batch, weight_numel] or
 * [weight_numel] when the weights are shared, L3_out [batch, L3_dim]. */
int oeqb_tp_forward(oeqb_plan* plan, int64_t batch, const void* L1_in, const void* L2_in,
                    const void* W, void* L3_out, void* stream);

/* (tensorproducts.hpp:90-100) All gradients are outputs; shared-weight W_grad is
 * zeroed by the call before accumulation. */
int oeqb_tp_backward(oeqb_plan* plan, int64_t batch, const void* L1_in, void* L1_grad,
                     const void* L2_in, void* L2_grad, const void* W, void* W_grad,
                     const void* L3_grad, void* stream);

/* (tensorproducts.hpp:102-116) Inputs L1_in, L2_in, W, L3_grad and the upstream
 * gradients L1_dgrad, L2_dgrad, W_dgrad; outputs L1_grad, L2_grad, W_grad, L3_dgrad. */
int oeqb_tp_double_backward(oeqb_plan* plan, int64_t batch, const void* L1_in,
                            const void* L2_in, const void* W, const void* L3_grad,
                            const void* L1_dgrad, const void* L2_dgrad, const void* W_dgrad,
                            void* L1_grad, void* L2_grad, void* W_grad, void* L3_dgrad,
                            void* stream);

/* ---- fused graph convolution (replaces convolution.hpp:79-186) ----
 * z[rows[e]] += TP(x[cols[e]], y[e], W[e]).  rows/cols are int64 [nnz]; L1_in and L3_out
 * have node_count rows, L2_in and W (unless shared) have nnz rows.  In deterministic
 * mode rows must be sorted (receiver-major) and transpose_perm[p] is the index of the
 * p-th edge in sender-sorted order; results are bitwise reproducible.  Outputs are
 * zero-initialised by the call. */
int oeqb_conv_forward(oeqb_plan* plan, const void* L1_in, const void* L2_in, const void* W,
                      void* L3_out, const int64_t* rows, const int64_t* cols, int64_t nnz,
                      int64_t node_count, void* workspace, size_t workspace_bytes, void* stream);

int oeqb_conv_backward(oeqb_plan* plan, const void* L1_in, void* L1_grad, const void* L2_in,
                       void* L2_grad, const void* W, void* W_grad, const void* L3_grad,
                       const int64_t* rows, const int64_t* cols, int64_t nnz,
                       int64_t node_count, void* workspace, size_t workspace_bytes,
                       const int64_t* transpose_perm, void* stream);

int oeqb_conv_double_backward(oeqb_plan* plan, const void* L1_in, const void* L2_in,
                              const void* W, const void* L3_grad, const void* L1_dgrad,
                              const void* L2_dgrad, const void* W_dgrad, void* L1_grad,
                              void* L2_grad, void* W_grad, void* L3_dgrad, const int64_t* rows,
                              const int64_t* cols, int64_t nnz, int64_t node_count,
                              void* workspace, size_t workspace_bytes,
                              const int64_t* transpose_perm, void* stream);

/* ---- convolution on node arrays in padded rows (no counterpart in the reference) ----
 * For float32 atomic plans of the single-path multiplicity-1 class with one weight per edge
 * (oeqb_conv_rows8_ok returns 1).  Node arrays are [node_count, 8] floats: row n of X (or dZ,
 * dX) in the first L1 (L3) of its 8 slots, 32-byte aligned rows; the padding slots are never read.  This
 * is the kernels' own layout, so callers that keep node data in it for many calls (the
 * multi-GPU partition of openequivariance_b200.distributed, whose halo rows arrive from other
 * GPUs straight into such a buffer) skip the per-call layout copies of oeqb_conv_forward /
 * oeqb_conv_backward.  Y, W, dY, dW, rows and cols are as there.
 *   forward:  Z [node_count, L3_dim] (unpadded) = sum over edges (accumulate = 0), or += it
 *             (accumulate != 0);
 *   backward: dY, dW written; dX contributions added into the padded accumulator dxp (the
 *             caller clears it).
 * sm_budget bounds the SMs the launch puts CTAs on: 0 = all, > 0 = at most that many, < 0 =
 * all but that many (for work that runs beside it, e.g. a collective or the other edge block
 * on another stream).  The padded arrays (xp, gp, dxp) 32-byte aligned, the others 16-byte
 * aligned. */
int oeqb_conv_rows8_ok(const oeqb_plan* plan);
int oeqb_conv_forward_rows8(oeqb_plan* plan, const float* xp, const float* Y, const float* W,
                            float* Z, const int64_t* rows, const int64_t* cols, int64_t nnz,
                            int64_t node_count, int accumulate, int sm_budget, void* stream);
int oeqb_conv_backward_rows8(oeqb_plan* plan, const float* xp, const float* gp, const float* Y,
                             const float* W, float* dY, float* dW, float* dxp,
                             const int64_t* rows, const int64_t* cols, int64_t nnz,
                             int64_t node_count, int sm_budget, void* stream);

/* ---- MACE symmetric contraction (replaces the group_gemm + torch pipeline of
 * _torch/symmetric_contraction/SymmetricContraction.py:124-336 and extension/group_mm.hpp) ----
 * The contraction of correlation <= 3 is a polynomial of degree <= 3 in the k components of
 * each (node, channel) feature vector.  The caller passes its coefficients on the distinct
 * monomials: coef [num_elements, channels, m, dt] with m = k + k(k+1)/2 [+ k(k+1)(k+2)/6 for
 * degree 3], monomials ordered by degree, then lexicographically by (a <= b <= c), and dt
 * padded output components per (node, channel) (4 or 16; the first nout are used).  perm
 * [nodes] lists the nodes sorted by element and elem_offsets [num_elements + 1] gives each
 * element's range in it.  x is [nodes, channels, k]; output component o of channel c of node n is
 * written to out[n * out_dim + out_col[o] + c * out_step[o]].  Supported: k in {4, 9},
 * degree 1..3, float32 / float64 (dtype 1 / 2); dt = 16 for float32 only.  No host
 * synchronisation. */
int oeqb_sc_forward(int dtype, int64_t nodes, int channels, int k, int degree, int dt, int nout,
                    const int* out_col, const int* out_step, int64_t out_dim, int num_elements,
                    const void* x, const int64_t* perm, const int64_t* elem_offsets,
                    const void* coef, void* out, void* stream);

/* Gradients of oeqb_sc_forward for the upstream gradient grad_out (laid out like out):
 * grad_x [nodes, channels, k] (skipped if NULL) and grad_coef [num_elements, channels, m, dt]
 * (skipped if NULL; padding columns are written as zero-weighted sums).  Sums are taken in
 * a fixed order: results are bitwise reproducible. */
int oeqb_sc_backward(int dtype, int64_t nodes, int channels, int k, int degree, int dt, int nout,
                     const int* out_col, const int* out_step, int64_t out_dim, int num_elements,
                     const void* x, const int64_t* perm, const int64_t* elem_offsets,
                     const void* coef, const void* grad_out, void* grad_x, void* grad_coef,
                     void* stream);

/* Ragged grouped GEMM of the reference's group_gemm op (extension/group_mm.hpp:38-141),
 * row-major.  Rows are grouped contiguously: group g owns rows [offsets[g], offsets[g+1])
 * (offsets is a device array of num_groups + 1 entries).
 *   ragged_inner == 0: A [num_groups, batch, m, k], B [rows, batch, k] -> C [rows, batch, m],
 *                      C[r,b,:] = A[g(r),b] @ B[r,b,:]
 *   ragged_inner == 1: A [rows, batch, m], B [rows, batch, k] -> C [num_groups, batch, m, k],
 *                      C[g,b] = sum over rows r of g of A[r,b,:] (outer) B[r,b,:]  */
int oeqb_group_gemm(int dtype, const void* A, const void* B, const int64_t* offsets,
                    int num_groups, int64_t rows, int batch, int m, int k, int ragged_inner,
                    void* C, void* stream);

/* ---- allocation-free batch forward (no counterpart in the reference) ----
 * Same result as oeqb_plan_create + oeqb_tp_forward, for callers that must not allocate
 * device memory: code running inside another runtime's memory manager (an XLA/JAX custom
 * call, an inference server with a fixed arena) or a real-time loop where cudaMalloc's
 * implicit synchronisation and fragmentation are not acceptable.  The problem tables live
 * in a static device array of the library (OEQB_NOALLOC_BYTES, loaded on every device
 * the library is used on and kept until process exit); problems whose tables exceed it are
 * rejected with OEQB_ERR_UNSUPPORTED.  The first call on a device, with that device
 * current, resolves the array's device address (cudaGetSymbolAddress); make that first call
 * before any stream capture.  Every call parses the descriptor and copies its tables from a
 * host buffer of the call into the array with cudaMemcpyAsync on `stream`.  All calls on a
 * device share the array and leave their tables in it, so calls whose GPU work overlaps race;
 * serialise them (one stream).  The call runs the table-driven forward kernel whatever the
 * problem, and that kernel raises no device status: the returned code is the whole error
 * report.  Inputs and outputs are as for oeqb_tp_forward. */
#define OEQB_NOALLOC_BYTES 65536
int oeqb_tp_forward_noalloc(const void* descriptor, size_t nbytes, int device, int64_t batch,
                            const void* L1_in, const void* L2_in, const void* W, void* L3_out,
                            void* stream);

#ifdef __cplusplus
}
#endif

#endif /* OEQB200_H_ */
