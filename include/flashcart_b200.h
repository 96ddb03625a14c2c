/*
 * flashcart_b200 -- C ABI of the B200 (sm_100a) kernels behind FlashCart's o3 operators.
 *
 * Every entry point takes plain pointers to DEVICE memory (row-major, contiguous),
 * sizes, a POD descriptor and a cudaStream_t, and returns an int status
 * (FC_OK = 0, negative values below). No entry point frees caller memory or
 * synchronises the stream; outputs are owned by the caller. Device memory is allocated
 * only as stream-ordered workspace: fc_linear_fwd/bwd (the tf32 split of the weights,
 * from the library's memory pool) and fc_newton_schulz (see there); the *_presplit
 * linear entry points and every other entry point allocate nothing.
 * Accumulated outputs (scatter targets) are zero-filled inside the call with
 * cudaMemsetAsync on the given stream. Errors in the DATA (an index out of range,
 * an unsorted receiver list) are OR-ed into the optional device word `status`
 * (FC_DEV_* bits) instead of faulting; pass NULL to skip the check.
 *
 * Layouts follow the reference exactly (reference = inm-leibniz/flashcart,
 * paths relative to its src/flashcart/):
 *  - feature rows are rank blocks l = 0..l_max, each (2l+1, features), component axis
 *    outer and channels contiguous (o3/utils.py:206-262);
 *  - stored STF component order per rank (o3/_codegen_common.py:37-73);
 *  - tensor-product output rank block (2l+1, paths_l, F) or (2l+1, F) when paths are
 *    reduced, F = max(in1_features, in2_features) (o3/_tensor_product.py:1146-1149);
 *  - per-edge / per-row weights (rows, n_total_paths * F), path-major
 *    (o3/utils.py:127-154), path order of o3/utils.py:157-203.
 */
#ifndef FLASHCART_B200_H
#define FLASHCART_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef FC_HOST_EMU
typedef struct CUstream_st* fc_stream_t;
#else
typedef void* fc_stream_t;
#endif

/* status codes returned by every entry point */
#define FC_OK 0
#define FC_ERR_INVALID -1     /* bad argument (shape, rank, null pointer, dtype) */
#define FC_ERR_UNSUPPORTED -2 /* configuration outside the compiled kernels (rank > 3, ...) */
#define FC_ERR_LAUNCH -3      /* CUDA launch or runtime error; see fc_last_error() */
#define FC_ERR_CAPACITY -4    /* a size exceeds a fixed capacity of the entry point */

/* bits of the optional device status word */
#define FC_DEV_BAD_INDEX 1    /* an edge index pointed outside its node array */
#define FC_DEV_UNSORTED 2     /* receiver indices were not ascending */
#define FC_DEV_TIMEOUT 4      /* a bounded device-side wait expired (results invalid) */

/* dtypes */
#define FC_F32 0
#define FC_F64 1
#define FC_BF16 2  /* fc_newton_schulz input; fc_linear_fwd storage (x, weights, y in bf16) */

/* activation applied to a linear map's input (fc_linear_desc.act): the radial MLP's SiLU
 * between its layers (nn/layers.py:12-44) folded into the next layer's GEMM */
#define FC_ACT_NONE 0
#define FC_ACT_SILU 1

/* linear-map arithmetic */
#define FC_PREC_IEEE 0 /* fp32-accurate: fp64 FMA, or fp32 on tensor cores as 3xTF32 (hi*hi+hi*lo+lo*hi) */
#define FC_PREC_TF32 1 /* fp32 only: one tf32 tensor-core product, fp32 accumulation */

#define FC_MAX_L 3

/* Version string "flashcart_b200 <semver> (<build info>)". */
const char* fc_version(void);
/* Message of the last failing call on this host thread ("" if none). */
const char* fc_last_error(void);

/* ------------------------------------------------------------------------------
 * Receiver CSR.
 * Replaces torch.searchsorted(idx_i, arange(n_nodes + 1)) in the reference
 * tp_fwd/tp_bwd ops (o3/_tensor_product.py:396-405): rowptr[k] = number of edges
 * with idx_i < k, for k = 0..n_nodes. Also flags FC_DEV_UNSORTED when idx_i is not
 * ascending (the reference's torch._assert_async, o3/_tensor_product.py:397-401)
 * and FC_DEV_BAD_INDEX for idx_i outside [0, n_nodes).
 * ------------------------------------------------------------------------------ */
int fc_build_rowptr(const int64_t* idx_i, int64_t n_edges, int64_t n_nodes, int64_t* rowptr,
                    int32_t* status, fc_stream_t stream);

/* ------------------------------------------------------------------------------
 * Cartesian tensor product.
 * ------------------------------------------------------------------------------ */
typedef struct fc_tp_desc {
  int32_t in1_l_max, in2_l_max, out_l_max;
  int32_t in1_features, in2_features; /* equal, or one of them 1 (broadcast) */
  int32_t symmetric_product;          /* keep only l1 >= l2 paths (in1 == in2) */
  int32_t shared_weights;             /* weights: (n_total_paths*F) instead of (rows, ...) */
  int32_t reduce_paths;               /* sum the paths of each output rank */
  int32_t dtype;                      /* FC_F32 / FC_F64 */
} fc_tp_desc;

/* Number of paths (sum over output ranks) of a descriptor, or a negative status. */
int fc_tp_num_paths(const fc_tp_desc* desc);
/* Width of one output row in elements, or a negative status. */
int64_t fc_tp_out_dim(const fc_tp_desc* desc);

/* Forward. Replaces flashcart::tp_fwd (o3/_tensor_product.py:332-479).
 * Convolution when rowptr != NULL: out[i] = sum over edges e of receiver i of
 *   W[e] (.) TP(in1[idx_j[e]], in2[e]);  in2/weights have one row per edge,
 *   rowptr from fc_build_rowptr, n_out_rows = number of receivers, n_in1_rows =
 *   rows of in1 (idx_j range), n_in2_rows = edges (rows of in2 and weights).
 *   With no edges (n_in2_rows == 0) in2, weights and idx_j may be NULL and every
 *   output row is zero; the same holds for fc_tp_bwd / fc_tp_dbwd.
 * Dense when rowptr == NULL: row r of out from row r of in1, in2 and weights;
 *   n_out_rows = n_in1_rows = n_in2_rows = rows. */
int fc_tp_fwd(const fc_tp_desc* desc, const void* in1, const void* in2, const void* weights,
              const int64_t* rowptr, const int64_t* idx_j, int64_t n_out_rows, int64_t n_in1_rows,
              int64_t n_in2_rows, void* out, int32_t* status, fc_stream_t stream);

/* Allocation-free convolution forward. No counterpart in the reference: an extra
 * entry point for callers that cannot allocate device memory themselves, e.g. a
 * simulation engine plug-in (an MD code whose own memory manager owns every device
 * byte and hands out only pointers into its buffers), or a time-step loop that may not
 * call cudaMalloc because it can synchronise the device and stall the step.
 * Same result as fc_build_rowptr + fc_tp_fwd (convolution) with n_out_rows = n_nodes
 * and n_in1_rows = n_in1_rows: receivers (idx_i, rows of out) are the first n_nodes
 * atoms, senders (idx_j, rows of in1) may reach further, e.g. an MD plug-in whose
 * receivers are its nlocal owned atoms and whose senders include the ghosts
 * (n_in1_rows = nlocal + nghost). The receiver CSR is built into a fixed workspace
 * inside the library's own device memory (2 MiB per device, held until process exit),
 * so at most 262,144 receiver nodes are accepted; larger n_nodes returns
 * FC_ERR_CAPACITY without launching anything (the sender count is not limited). The
 * call itself never allocates or frees. The first call on a device looks the workspace
 * up (cudaGetSymbolAddress) with that device current: make it before any stream
 * capture. The looked-up address is kept for the life of the process and does not
 * survive cudaDeviceReset (do not reset a device between calls). All calls share the
 * one workspace: calls that can overlap on the GPU (different streams without
 * ordering) race and must be serialised by the caller. */
int fc_tp_conv_fwd_noalloc(const fc_tp_desc* desc, const void* in1, const void* in2,
                           const void* weights, const int64_t* idx_i, const int64_t* idx_j,
                           int64_t n_nodes, int64_t n_in1_rows, int64_t n_edges, void* out,
                           int32_t* status, fc_stream_t stream);

/* Newton-Schulz orthogonalisation of a batch of Muon updates on the tensor cores (bf16).
 * Replaces _batched_newtonschulz (training/muon.py:27-61). update: (batch, rows, cols),
 * row-major, dtype FC_F32 or FC_BF16; out: (batch, rows, cols) bf16. A tall matrix
 * (rows > cols) is iterated transposed, as in the reference. X <- X / max(||X||_F, eps),
 * then `steps` iterations with coeffs = (a, b, c) and `polish_steps` with polish = (a, b, c):
 * G = X X^T, U = b G + c G G, X = a X + U X, each product in fp32 and rounded to bf16.
 * min(rows, cols) and max(rows, cols) must be multiples of 8. Uses a stream-ordered
 * workspace of 2 bytes x batch x (2 rows cols + 2 min(rows, cols)^2). */
int fc_newton_schulz(const void* update, int dtype, int64_t batch, int rows, int cols, const float* coeffs,
                     int steps, const float* polish, int polish_steps, float eps, void* out, int32_t* status,
                     fc_stream_t stream);

/* Backward. Replaces flashcart::tp_bwd (o3/_tensor_product.py:588-787).
 * grad_in1 / grad_in2 / grad_weights may be NULL (not requested). n_in2_rows = rows
 * of in2 (edges for a convolution). Scatter targets are zero-filled here. */
int fc_tp_bwd(const fc_tp_desc* desc, const void* grad_out, const void* in1, const void* in2,
              const void* weights, const int64_t* rowptr, const int64_t* idx_j, int64_t n_out_rows,
              int64_t n_in1_rows, int64_t n_in2_rows, void* grad_in1, void* grad_in2,
              void* grad_weights, int32_t* status, fc_stream_t stream);
/* Backward of a dense product (no edges) with gradients from elsewhere added in the same
 * pass: grad_in1 = VJP_in1 + residual_in1 over the first residual_in1_comps components of
 * each in1 row (residual rows of residual_in1_ld elements; the rest of the row has no
 * residual), grad_in2 = VJP_in2 + residual_in2 (whole rows, may be grad_in2 itself). For
 * the node-level products of the product layers (o3/_tensor_product.py:588-787 with
 * rowptr == NULL), whose inputs also feed other terms of the layer's sum
 * (nn/layers.py:768-1018). float32, both inputs with 64 or 128 channels, paths kept, no
 * weight gradient, 8-byte aligned rows; otherwise FC_ERR_UNSUPPORTED. Either residual may
 * be NULL. residual_in1_comps must lie in [0, (in1_l_max + 1)^2] and residual_in1_ld be
 * even and at least residual_in1_comps x in1_features; otherwise FC_ERR_INVALID. */
int fc_tp_bwd_residual(const fc_tp_desc* desc, const void* grad_out, const void* in1, const void* in2,
                       const void* weights, int64_t n_rows, const void* residual_in1, int64_t residual_in1_ld,
                       int32_t residual_in1_comps, const void* residual_in2, void* grad_in1, void* grad_in2,
                       int32_t* status, fc_stream_t stream);

/* Double backward: VJP of fc_tp_bwd with tangents (v_in1, v_in2, v_weights) on its
 * three outputs (NULL = zero tangent). Replaces the autograd of flashcart::tp_bwd
 * (tp_dbwd, o3/_tensor_product.py:837-1093). Outputs may be NULL. */
int fc_tp_dbwd(const fc_tp_desc* desc, const void* grad_out, const void* in1, const void* in2,
               const void* weights, const void* v_in1, const void* v_in2, const void* v_weights,
               const int64_t* rowptr, const int64_t* idx_j, int64_t n_out_rows, int64_t n_in1_rows,
               int64_t n_in2_rows, void* d_grad_out, void* d_in1, void* d_in2, void* d_weights,
               int32_t* status, fc_stream_t stream);

/* ------------------------------------------------------------------------------
 * Direction tensors (edge attributes): stored STF components of T^l(x), l <= l_max,
 * for unit vectors x (n, 3) -> (n, (l_max+1)^2).
 * Replace flashcart::irreps_fwd / irreps_bwd / irreps_dbwd (o3/_irreps.py:84-186).
 * ------------------------------------------------------------------------------ */
int fc_irreps_fwd(const void* x, int64_t n, int32_t l_max, int32_t dtype, void* out, fc_stream_t stream);
int fc_irreps_bwd(const void* grad_out, const void* x, int64_t n, int32_t l_max, int32_t dtype,
                  void* grad_x, fc_stream_t stream);
int fc_irreps_dbwd(const void* grad_out, const void* x, const void* v, int64_t n, int32_t l_max,
                   int32_t dtype, void* d_grad_out, void* d_x, fc_stream_t stream);

/* ------------------------------------------------------------------------------
 * Equivariant linear map: for each active rank l (l <= min(in_l_max, out_l_max))
 *   y[n, m, :] = x[n, m, :] @ (scale[l] * W_l)^T,   m = 0..m_values[l]-1,
 *   W_l: (f_out_values[l], f_in_values[l]) row-major,
 * where rank l of a row starts at in_offsets[l] (x) / out_offsets[l] (y) and its
 * component m at + m * f_in (x) / + m * f_out (y). Output columns after the last
 * active rank are zero. The descriptor carries the same metadata as the reference
 * op flashcart::linear_fwd (in_offsets, out_offsets, m_values, f_in_values,
 * f_out_values; o3/_linear.py:113-166, 328-385) plus the row widths.
 * `weights` is a HOST array of per-rank DEVICE pointers, `scale` a DEVICE array with
 * one entry per active rank (dtype of x; float32 for FC_BF16).
 * dtype FC_BF16 (forward only): x, weights (f_out, f_in) and y in bf16, products on the
 * tensor cores (tcgen05 kind::f16) accumulated in fp32 and rounded once to bf16: the
 * bf16 storage path of the linear maps, half the bytes of the float32 maps. Rank blocks,
 * offsets and row widths must be multiples of 8 elements (16-byte TMA rows).
 * ------------------------------------------------------------------------------ */
typedef struct fc_linear_desc {
  int32_t n_active;                     /* active ranks, 0..FC_MAX_L+1 */
  int32_t dtype;                        /* FC_F32 / FC_F64, or FC_BF16 (fc_linear_fwd only) */
  int32_t precision;                    /* FC_PREC_IEEE or FC_PREC_TF32 (fp32 only) */
  int32_t act;                          /* FC_ACT_NONE, or FC_ACT_SILU (fp32 on the TMA path only):
                                           forward y = (sW) silu(x), backward grad_x = silu'(x) *
                                           ((sW)^T g); no weight gradients (frozen weights) */
  int64_t in_dim, out_dim;              /* row widths of x and y */
  int64_t in_offsets[FC_MAX_L + 1];
  int64_t out_offsets[FC_MAX_L + 1];
  int32_t m_values[FC_MAX_L + 1];
  int32_t f_in_values[FC_MAX_L + 1];
  int32_t f_out_values[FC_MAX_L + 1];
} fc_linear_desc;

/* Forward. Replaces flashcart::linear_fwd (o3/_linear.py:328-385). */
int fc_linear_fwd(const fc_linear_desc* desc, const void* x, const void* const* weights,
                  const void* scale, int64_t n, void* out, int32_t* status, fc_stream_t stream);
/* Backward. Replaces flashcart::linear_bwd (o3/_linear.py:457-538). grad_x may be
 * NULL; grad_weights may be NULL or a host array of per-rank device pointers (each
 * fully overwritten). Columns of grad_x outside the active ranks are zero. */
int fc_linear_bwd(const fc_linear_desc* desc, const void* grad_out, const void* x,
                  const void* const* weights, const void* scale, int64_t n, void* grad_x,
                  void* const* grad_weights, int32_t* status, fc_stream_t stream);
/* Double backward. Replaces flashcart::linear_dbwd (o3/_linear.py:571-778): the VJP of
 * fc_linear_bwd for tangents v_grad_x (like x) and v_grad_weights (like weights), with
 * gx = g (sW) and gW_l = s_l g^T x per rank:
 *   d_grad_out = v_grad_x (sW)^T + x (s v_grad_weights)^T,
 *   d_x = g (s v_grad_weights),  d_weights[l] = s_l g^T v_grad_x.
 * A NULL tangent counts as zero; each of d_grad_out, d_x and d_weights may be NULL (not
 * wanted) and is otherwise fully overwritten. With both tangents given, d_grad_out
 * needs one stream-ordered workspace of n * out_dim elements from the library's pool. */
int fc_linear_dbwd(const fc_linear_desc* desc, const void* grad_out, const void* x, const void* const* weights,
                   const void* v_grad_x, const void* const* v_grad_weights, const void* scale, int64_t n,
                   void* d_grad_out, void* d_x, void* const* d_weights, int32_t* status, fc_stream_t stream);

/* Weights split once. The float32 maps run on the tensor cores as 3xTF32, which needs every
 * weight matrix as tf32 hi and lo parts; fc_linear_fwd/bwd split them on every call.
 * fc_linear_presplit writes, per active rank l, the split of weights[l] into split[l]
 * (2 * N * kp floats, kp = (K + 3) & ~3; forward: K = f_in_values[l], N = f_out_values[l];
 * backward: K = f_out_values[l], N = f_in_values[l]); fc_linear_fwd_presplit /
 * fc_linear_bwd_presplit take those buffers next to the weights (which layouts outside
 * the TMA-fed kernel still read) and skip the split. The caller keeps the buffers valid
 * and re-splits after changing the weights. float32 only. Replace the same reference ops
 * as fc_linear_fwd / fc_linear_bwd. */
int fc_linear_presplit(const fc_linear_desc* desc, const void* const* weights, int32_t backward,
                       void* const* split, fc_stream_t stream);
int fc_linear_fwd_presplit(const fc_linear_desc* desc, const void* x, const void* const* weights,
                           const void* const* split, const void* scale, int64_t n, void* out, int32_t* status,
                           fc_stream_t stream);
int fc_linear_bwd_presplit(const fc_linear_desc* desc, const void* grad_out, const void* x,
                           const void* const* weights, const void* const* split, const void* scale, int64_t n,
                           void* grad_x, void* const* grad_weights, int32_t* status, fc_stream_t stream);

/* Residual forms of the float32 maps: out = (sW) x + residual and grad_x = (sW)^T grad_out
 * + residual, the residual laid out like the output row (out_dim, resp. in_dim floats per
 * row; it may be the output buffer itself, which then accumulates), added in the GEMM's
 * epilogue instead of by a separate pass over the rows. They carry the residual
 * connections of the node-level layers around the maps of o3/_linear.py:328-538 (the gate
 * layer's `node_feats + output_linear(...)`, nn/layers.py:609-635, the interaction's skip
 * sum, nn/layers.py:395-405, and the sums of their gradients). float32 on the TMA-fed
 * tensor-core path only: the active ranks must cover the whole row, their blocks must be
 * uniform with at most 128 output columns (node-level maps), act must be FC_ACT_NONE, and
 * rows must be 16-byte aligned; otherwise FC_ERR_UNSUPPORTED and nothing is written.
 * split: the lin_presplit buffers, or NULL (split per call). No weight gradients. */
int fc_linear_fwd_residual(const fc_linear_desc* desc, const void* x, const void* const* weights,
                           const void* const* split, const void* scale, int64_t n, const void* residual, void* out,
                           int32_t* status, fc_stream_t stream);
int fc_linear_bwd_residual(const fc_linear_desc* desc, const void* grad_out, const void* const* weights,
                           const void* const* split, const void* scale, int64_t n, const void* residual,
                           void* grad_x, int32_t* status, fc_stream_t stream);

/* ---------------------------------------------------------------- halo exchange
 * Row gather / scatter for ghost-atom exchange in a domain decomposition (owned rows
 * first, ghost rows after them). The transport between ranks is the caller's (NCCL, MPI,
 * an MD engine's communicator); these move rows between the feature array and the
 * contiguous send / receive buffers. Replace the device-side halves of
 * lammps_forward_exchange / lammps_reverse_exchange (utils/lammps.py:67-118): owner rows
 * copied into ghost rows, ghost-row gradients added into owner rows.
 * Rows hold row_elems elements of dtype (FC_F32 / FC_F64). An index outside
 * [0, n_rows) sets FC_DEV_BAD_INDEX in *status (if given) and its row is skipped. */
/* buf[k, :] = x[idx[k], :] for k < n_idx (rows of a bad index are written as zeros). */
int fc_halo_pack(const void* x, int64_t n_rows, int64_t row_elems, int32_t dtype, const int64_t* idx,
                 int64_t n_idx, void* buf, int32_t* status, fc_stream_t stream);
/* accumulate == 0: x[idx[k], :] = buf[k, :] (ghost rows receive their owners' features;
 * indices should be distinct). accumulate != 0: x[idx[k], :] += buf[k, :] with atomic
 * adds (ghost gradients added to their owners; repeated indices allowed, the order of
 * the additions is not fixed). */
int fc_halo_unpack(const void* buf, int64_t n_idx, int64_t row_elems, int32_t dtype, const int64_t* idx, void* x,
                   int64_t n_rows, int32_t accumulate, int32_t* status, fc_stream_t stream);

/* ---------------------------------------------------------------- RMS layer norm
 * Fused forward and first-order backward of RMSLayerNorm (nn/layers.py:413-540, affine,
 * without centering): per row, q_c = sum_l l_weights[l] * inv_l[c] with inv_l the
 * (l,l)->0 symmetric scalar tensor product of the row with itself (nn/layers.py:456-466,
 * 517), r = (mean_c q_c + eps)^(-1/2), y = x * r * gains[l, c]. x, y, grad_y, grad_x:
 * (n_rows, (l_max+1)^2 * features) rows; gains: (l_max+1, features); l_weights: l_max+1
 * values; rstd: n_rows values written by the forward and read by the backward.
 * dtype FC_F32 or FC_F64 for every array. The backward returns grad_x only (gains and
 * l_weights are constants of the call). */
int fc_rms_norm_fwd(int32_t l_max, int32_t features, int32_t dtype, const void* x, const void* gains,
                    const void* l_weights, double eps, int64_t n_rows, void* y, void* rstd,
                    fc_stream_t stream);
int fc_rms_norm_bwd(int32_t l_max, int32_t features, int32_t dtype, const void* grad_y, const void* x,
                    const void* gains, const void* l_weights, const void* rstd, int64_t n_rows,
                    void* grad_x, fc_stream_t stream);

/* ---------------------------------------------------------------- equivariant gate
 * The gating product of EquivariantGatedLayer.forward (nn/layers.py:609-635):
 * y[n, (l, m), c] = values[n, (l, m), c] * gates[n, l, c] for every rank block of a row
 * (the reference's per-rank multiply and concatenation), and its first-order backward.
 * values, y, grad_y, grad_values: (n_rows, (l_max+1)^2 * features) rows; gates,
 * grad_gates: (n_rows, l_max+1, features). grad_values or grad_gates may be NULL. */
int fc_gate_fwd(int32_t l_max, int32_t features, int32_t dtype, const void* values, const void* gates,
                int64_t n_rows, void* y, fc_stream_t stream);
int fc_gate_bwd(int32_t l_max, int32_t features, int32_t dtype, const void* grad_y, const void* values,
                const void* gates, int64_t n_rows, void* grad_values, void* grad_gates, fc_stream_t stream);

/* ---------------------------------------------------------------- edge expansion
 * Cartesian expansion of edge features: out[e, k, c] = moments[e, k] * h[e, r, c] over the
 * (l_max+1)^2 stored components k of the direction moments (rows of fc_irreps_fwd), laid
 * out as rank blocks (rank l at l^2 * features). per_rank = 0: h is (n_rows, features),
 * shared by all ranks -- the composition T^l(r^) (x) radial features of the reference's
 * pieces (o3/irreps.py:54-72, nn/radial.py, nn/layers.py:84-131), which it materialises
 * with broadcast products and a concatenation; per_rank = 1: h is (n_rows, l_max+1,
 * features) -- the factorised form T_l (x) (h W_l^T) of an equivariant linear map
 * (o3/linear.py:88-128) applied to that expansion. The backward returns grad_moments
 * (n_rows, (l_max+1)^2) and grad_h (h's shape); either may be NULL. */
int fc_edge_expand_fwd(int32_t l_max, int32_t features, int32_t per_rank, int32_t dtype, const void* moments,
                       const void* h, int64_t n_rows, void* out, fc_stream_t stream);
int fc_edge_expand_bwd(int32_t l_max, int32_t features, int32_t per_rank, int32_t dtype, const void* grad_out,
                       const void* moments, const void* h, int64_t n_rows, void* grad_moments, void* grad_h,
                       fc_stream_t stream);

/* ---------------------------------------------------------------- edge geometry
 * Fused edge geometry of the potential, one pass per edge. Replaces the chain that
 * FlashCartPotential.forward runs before its interaction layers (model/flashcart.py:
 * 264-286): get_edge_vectors (utils/geometry.py:25-53: v = r_j - r_i + S . cell[batch[i]],
 * row 0 of edge_index = receiver i, row 1 = sender j), distances and directions
 * v / max(|v|, 1e-4), Irreps(l_max).forward_normalized (o3/irreps.py:54-72), the
 * ChebyshevBasis (nn/radial.py:98-128) times the PolynomialCutoff envelope
 * (nn/radial.py:181-245) that InteractionLayer.forward multiplies into its radial-MLP
 * input (nn/layers.py:351-356). Outputs: edge_attrs (n_edges, (l_max+1)^2) and radial
 * (n_edges, n_radial) = basis * envelope, both row-major in the positions' dtype.
 * positions (n_nodes, 3); cells (n_cells, 3, 3), cell rows are lattice vectors; shifts
 * (n_edges, 3) int32 image counts (unused when use_shifts is 0); batch (n_nodes) graph of
 * each atom (read only when n_cells > 1). An edge index (or graph index) out of range sets
 * FC_DEV_BAD_INDEX; the edge's outputs are zero and it contributes no gradient. */
typedef struct fc_edge_geometry_desc {
  int32_t l_max;      /* rank of the edge attributes, 0..3 */
  int32_t n_radial;   /* Chebyshev functions, 1..64 */
  int32_t cosine;     /* 1: x = cos(pi t) ("cosine"), 0: x = 2t - 1 ("affine") */
  int32_t poly_order; /* polynomial cutoff order p >= 2 */
  int32_t use_shifts; /* 0: v = r_j - r_i (shifts and cells not read) */
  int32_t dtype;      /* FC_F32 or FC_F64 */
  double r_min;       /* Chebyshev range: t = (r - r_min) / (r_max - r_min) */
  double r_max;
  double r_cut;       /* envelope cutoff radius */
} fc_edge_geometry_desc;

int fc_edge_geometry_fwd(const fc_edge_geometry_desc* desc, const void* positions, int64_t n_nodes,
                         const void* cells, int64_t n_cells, const int32_t* shifts, const int64_t* edge_index,
                         const int64_t* batch, int64_t n_edges, void* edge_attrs, void* radial, int32_t* status,
                         fc_stream_t stream);
/* First derivative: grad_positions (n_nodes, 3) and grad_cells (n_cells, 3, 3; may be
 * NULL) are zeroed by the call and receive the vector-Jacobian products of edge_attrs and
 * radial with the given gradients (either may be NULL for zero). */
int fc_edge_geometry_bwd(const fc_edge_geometry_desc* desc, const void* positions, int64_t n_nodes,
                         const void* cells, int64_t n_cells, const int32_t* shifts, const int64_t* edge_index,
                         const int64_t* batch, int64_t n_edges, const void* grad_attrs, const void* grad_radial,
                         void* grad_positions, void* grad_cells, int32_t* status, fc_stream_t stream);

/* The same geometry from edge vectors given per edge (n_edges, 3) instead of positions:
 * the LAMMPS ML-IAP layout, where LAMMPS supplies rij with the periodic translation
 * applied (replaces the vectors branch of model/flashcart.py:264-286 for the graphs of
 * calculators/lammps_mliap.py:122-170). desc->use_shifts is ignored. The backward writes
 * grad_vectors (n_edges, 3) = the vector-Jacobian product per edge (dE/dv: the pair
 * forces of lammps_mliap.py:711-738), zeros when both gradients are NULL. */
int fc_edge_geometry_vec_fwd(const fc_edge_geometry_desc* desc, const void* vectors, int64_t n_edges,
                             void* edge_attrs, void* radial, int32_t* status, fc_stream_t stream);
int fc_edge_geometry_vec_bwd(const fc_edge_geometry_desc* desc, const void* vectors, int64_t n_edges,
                             const void* grad_attrs, const void* grad_radial, void* grad_vectors, int32_t* status,
                             fc_stream_t stream);

/* ---------------------------------------------------------------- neighbour list
 * Periodic cell list of an orthorhombic cell on the GPU. Replaces the host neighbour
 * search that feeds the model (data/neighbors.py:120-143, matscipy neighbour_list("ijS"):
 * pairs |r_j - r_i + S . cell| < r_max, self pair removed, row 0 = receiver i, row 1 =
 * sender j, receivers ascending) with the canonical order (i, j, S) of
 * flashcart_b200/data/neighbors.py and the same float64 arithmetic, so the two lists are
 * equal element for element. Two calls: fc_neighbor_count bins the atoms into the
 * caller's workspace (fc_neighbor_workspace_bytes) and writes the receiver CSR rowptr
 * (n_atoms + 1 int64, rowptr[n_atoms] = number of edges); after reading n_edges the
 * caller allocates edge_index (2, n_edges) int64 and shifts (n_edges, 3) int32 and calls
 * fc_neighbor_fill with the same workspace. */
typedef struct fc_nl_desc {
  double lengths[3];     /* cell edge lengths (diagonal of the cell matrix) */
  double inv_lengths[3]; /* diagonal of the inverse cell matrix (as the host list computes it) */
  double bin_widths[3];  /* lengths / bins, each >= r_max */
  double r_max_sq;       /* cutoff squared */
  int32_t bins[3];       /* cell-list bins per axis, each >= 3 */
  int32_t reserved;
} fc_nl_desc;
int64_t fc_neighbor_workspace_bytes(const fc_nl_desc* desc, int64_t n_atoms);
int fc_neighbor_count(const fc_nl_desc* desc, const double* positions, int64_t n_atoms, void* workspace,
                      int64_t* rowptr, int32_t* status, fc_stream_t stream);
int fc_neighbor_fill(const fc_nl_desc* desc, int64_t n_atoms, const void* workspace, const int64_t* rowptr,
                     int64_t n_edges, int64_t* edge_index, int32_t* shifts, int32_t* status,
                     fc_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASHCART_B200_H */
