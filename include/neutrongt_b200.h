/*
 * neutrongt_b200 — C ABI of the B200 (sm_100a) kernels for NeutronGT's hot path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t, launches
 * asynchronously on that stream, allocates nothing, and returns an int status
 * (NGT_OK = 0).  No exception crosses the ABI.  Pointers are device pointers unless a
 * parameter says "host".  Workspaces are caller-owned; their size comes from the
 * matching *_workspace_size query.  Entry points keep no state between calls, with two
 * exceptions: ngt_spattn_backward_noalloc uses one fixed scratch array per device (shared
 * by all its calls; see its comment), and ngt_linear_status reads a per-device counter of
 * the Linear kernels' bounded-wait timeouts.
 *
 * Element layout of attention tensors: row-major [n, heads, head_dim] (the reference's
 * [1, s, H, D] with b == 1, viewed as [s, H, D] at
 * NeutronGT/models/gt_dist_node_level_single_window.py:125-127).
 *
 * Edge convention (as the reference, :130-131): edge_index[0][e] = source = the K/V
 * row, edge_index[1][e] = destination = the Q row and the aggregation target.
 */
#ifndef NEUTRONGT_B200_H
#define NEUTRONGT_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define NGT_API __attribute__((visibility("default")))
#else
#define NGT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *ngt_stream_t; /* == cudaStream_t */

enum ngt_status {
    NGT_OK = 0,
    NGT_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad dtype */
    NGT_ERR_UNSUPPORTED = 2,      /* shape/dtype combination without a kernel */
    NGT_ERR_WORKSPACE = 3,        /* workspace smaller than the size query returned */
    NGT_ERR_CUDA = 4,             /* a CUDA launch or runtime call failed */
    NGT_ERR_MISALIGNED = 5,       /* a pointer is not 16-byte aligned where required */
    NGT_ERR_TOO_LARGE = 6         /* a size exceeds the 32-bit index range */
};

enum ngt_dtype { NGT_F32 = 0, NGT_BF16 = 1 };

/* ABI version (increments on any signature change) and status names. */
NGT_API int ngt_abi_version(void);
NGT_API const char *ngt_status_string(int status);

/* ------------------------------------------------------------------------------------
 * Window edge list -> CSR (destination-major and source-major, stable).
 *
 * Replaces the per-edge index/scatter bookkeeping of `CoreAttention.sparse_attention_bias`
 * (NeutronGT/models/gt_dist_node_level_single_window.py:130-131, 161-178: gathers by
 * edge_index[0]/[1] and torch_scatter by edge_index[1]) with two CSR views built once
 * per window.  Ties keep edge order.
 *
 *   edge_index      int64 [2, e] (row 0 = src, row 1 = dst), values must lie in [0, n)
 *   dst_rowptr      int32 [n+1]; dst_src int32 [e]: source of each dst-major slot
 *   src_rowptr      int32 [n+1]; src_dst int32 [e]: destination of each src-major slot
 *   src_to_dst_slot int32 [e] (nullable): dst-major slot of each src-major slot
 *   info            int32 [2]: info[0] = number of out-of-range indices (0 when valid),
 *                   info[1] = max destination index, or -1 when e == 0
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_edge_csr_workspace_size(int64_t n, int64_t e, size_t *bytes /* host */);
NGT_API int ngt_edge_csr_build(int64_t n, int64_t e, const int64_t *edge_index, int32_t *dst_rowptr,
                       int32_t *dst_src, int32_t *src_rowptr, int32_t *src_dst,
                       int32_t *src_to_dst_slot, int32_t *info, void *workspace,
                       size_t workspace_bytes, ngt_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Heavy-row segments of both CSR views (no counterpart in the reference: a scheduling table for
 * the kernels below).  In power-law windows a few hub rows hold hundreds of entries while most
 * rows hold one or two; one warp per row would make the hub's warp the whole kernel's critical
 * path.  A row of degree d > seg_edges is cut into ceil(d / seg_edges) segments of seg_edges
 * consecutive entries, each processed by its own warp; the partial sums are added in segment
 * order afterwards, so results do not depend on scheduling.
 *   seg_first  int32 [2n]: entries 0..n-1 for the destination view, n..2n-1 for the source view;
 *              the first segment number of a heavy row, -1 for other rows
 *   seg_row    int32 [2 * cap]: [0, cap) destination view, [cap, 2 cap) source view; the row
 *              of each segment; cap from ngt_edge_csr_segment_capacity(e, seg_edges)
 *   counts     int32 [2] (device): segments of the destination and of the source view
 * Segment numbers within a view are dense in [0, counts[view]).
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_edge_csr_segment_capacity(int64_t e, int32_t seg_edges, int64_t *cap /* host */);
NGT_API int ngt_edge_csr_segments(int64_t n, int64_t e, const int32_t *dst_rowptr, const int32_t *src_rowptr,
                                  int32_t seg_edges, int32_t *seg_first, int32_t *seg_row, int32_t *counts,
                                  ngt_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Graph-sparse window attention, forward.
 *
 * Replaces `CoreAttention.sparse_attention_bias` forward
 * (NeutronGT/models/gt_dist_node_level_single_window.py:112-179; same math in
 * NeutronGT/models/graphormer_dist_node_level.py:67-98) in one fused pass: per edge
 * score, clamp to [-5, 5], optional bias, exp, and the weighted sum, with no per-edge
 * tensor in HBM.
 *
 *   q, k, v, out    dtype [n, heads, head_dim]
 *   edge_bias       float [e, heads] in dst-major slot order (nullable) — the gathered
 *                   attn_bias[0, h, src, dst] of :142-152
 *   z               float [n, heads]: sum of exp(score) per row and head (saved for the
 *                   backward; may be null when no backward follows)
 *   node_scores     float [node_scores_len]: sum over in-edges of the head-mean of
 *                   exp(score) (:177-178); the reference's length is max(dst) + 1
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_spattn_forward(int dtype, int64_t n, int64_t e, int heads, int head_dim, const void *q,
                       const void *k, const void *v, const int32_t *dst_rowptr,
                       const int32_t *dst_src, const float *edge_bias, void *out, float *z,
                       float *node_scores, int64_t node_scores_len, ngt_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Graph-sparse window attention, backward (the autograd graph of :130-175 written out).
 * Atomic-free: dq from the dst-major CSR, dk/dv from the src-major CSR, in one launch
 * after a per-row delta = <dout, out> pass.
 *
 *   delta           float [n, heads] caller-provided scratch
 *   dq, dk, dv      dtype [n, heads, head_dim], every row written
 *   src_to_dst_slot required when edge_bias is given
 *   dedge_bias      float [e, heads] in dst-major slot order (nullable): gradient of the
 *                   per-edge bias
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_spattn_backward(int dtype, int64_t n, int64_t e, int heads, int head_dim, const void *q,
                        const void *k, const void *v, const void *out, const void *dout,
                        const float *z, const int32_t *dst_rowptr, const int32_t *dst_src,
                        const int32_t *src_rowptr, const int32_t *src_dst,
                        const int32_t *src_to_dst_slot, const float *edge_bias, float *delta,
                        void *dq, void *dk, void *dv, float *dedge_bias, ngt_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Sparse attention with heavy rows split into segments (tables from ngt_edge_csr_segments;
 * same results as ngt_spattn_forward / ngt_spattn_backward up to fp32 summation order).
 *   seg_edges, *_seg_first, *_seg_row, *_nseg: one view's tables (nseg == 0: none)
 *   seg_part   fp32 scratch, 16-byte aligned, ngt_spattn_seg_part_size(pass, ...) bytes
 *              (pass 0: forward, pass 1: backward)
 * Shapes outside the vector layout (see above) run unsegmented and ignore the tables.
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_spattn_seg_part_size(int pass, int heads, int head_dim, int64_t dst_nseg, int64_t src_nseg,
                                     size_t *bytes /* host */);
NGT_API int ngt_spattn_forward_seg(int dtype, int64_t n, int64_t e, int heads, int head_dim, const void *q,
                                   const void *k, const void *v, const int32_t *dst_rowptr,
                                   const int32_t *dst_src, const float *edge_bias, void *out, float *z,
                                   float *node_scores, int64_t node_scores_len, int32_t seg_edges,
                                   const int32_t *dst_seg_first, const int32_t *dst_seg_row, int64_t dst_nseg,
                                   float *seg_part, ngt_stream_t stream);
NGT_API int ngt_spattn_backward_seg(int dtype, int64_t n, int64_t e, int heads, int head_dim, const void *q,
                                    const void *k, const void *v, const void *out, const void *dout,
                                    const float *z, const int32_t *dst_rowptr, const int32_t *dst_src,
                                    const int32_t *src_rowptr, const int32_t *src_dst,
                                    const int32_t *src_to_dst_slot, const float *edge_bias, float *delta,
                                    void *dq, void *dk, void *dv, float *dedge_bias, int32_t seg_edges,
                                    const int32_t *dst_seg_first, const int32_t *dst_seg_row, int64_t dst_nseg,
                                    const int32_t *src_seg_first, const int32_t *src_seg_row, int64_t src_nseg,
                                    float *seg_part, ngt_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Graph-sparse window attention, backward, allocating nothing.  No counterpart in the
 * reference: an extra entry point of this library.
 *
 * Same arguments and results as ngt_spattn_backward minus `delta`: the n * heads floats of
 * per-row scratch come from a fixed array inside the library (NGT_NOALLOC_MAX_ROWS_X_HEADS
 * floats = 8 MiB, reserved on every GPU that loads the library until the process exits).
 * For callers that cannot allocate device memory where they run the backward — e.g. code
 * running inside a fixed memory budget with no allocator handle, or host runtimes that do
 * not own a CUDA allocator and may not call cudaMalloc mid-step.  The caller still passes
 * every input and output buffer.
 *
 *   - n * heads above NGT_NOALLOC_MAX_ROWS_X_HEADS returns NGT_ERR_TOO_LARGE, before any work.
 *   - The first call on a device looks up the array's device address with that device
 *     current (the current device must be the one the pointers live on); make that first
 *     call before any stream capture.
 *   - Every call shares the one array.  Each call writes all the scratch it reads, so no
 *     clearing is needed, but calls that overlap on the GPU (other streams, other threads)
 *     race on it: serialise them.
 * ---------------------------------------------------------------------------------- */
#define NGT_NOALLOC_MAX_ROWS_X_HEADS 2097152
NGT_API int ngt_spattn_backward_noalloc(int dtype, int64_t n, int64_t e, int heads, int head_dim,
                                        const void *q, const void *k, const void *v,
                                        const void *out, const void *dout, const float *z,
                                        const int32_t *dst_rowptr, const int32_t *dst_src,
                                        const int32_t *src_rowptr, const int32_t *src_dst,
                                        const int32_t *src_to_dst_slot, const float *edge_bias,
                                        void *dq, void *dk, void *dv, float *dedge_bias,
                                        ngt_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Dense full-attention window, forward, on the tcgen05 tensor cores.
 *
 * Replaces `CoreAttention.full_attention` (NeutronGT/models/gt_dist_node_level_single_window.py:56-109,
 * graphormer_dist_node_level.py:42-65) for attn_bias = mask = pruning_mask = None:
 *   S = scale * q k^T (the reference's scale is sqrt(head_dim), multiplied), P = softmax(S),
 *   dropout(P) with keep probability 1 - dropout_p, out = P v,
 *   node_scores[j] += score_scale * sum_i |S[i, j]|   (score_scale = 1 / total heads gives the
 *   reference's head mean; the caller zeroes node_scores once per call of all heads).
 *
 *   q, k, v, out    bf16 [s, heads, head_dim], head_dim a multiple of 8 and <= 64, 16-byte aligned
 *   lse             float [heads, s]: log-sum-exp of each row of S (for the backward)
 *   status          int32 [1] device flag, set to 1 if a bounded wait inside the kernel gave up
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_dense_attn_forward(int64_t s, int heads, int head_dim, float scale, float score_scale,
                                   float dropout_p, uint64_t seed, const void *q, const void *k,
                                   const void *v, void *out, float *lse, float *node_scores,
                                   int32_t *status, ngt_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Dense full-attention window, backward (the autograd graph of full_attention written out,
 * dropout mask regenerated from the same seed).
 *
 *   lse             float [heads, s] from ngt_dense_attn_forward
 *   delta           float [heads, s] caller scratch
 *   dq_accum        float [s, heads, head_dim] caller scratch (zeroed by this call)
 *   dq, dk, dv      bf16 [s, heads, head_dim]
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_dense_attn_backward(int64_t s, int heads, int head_dim, float scale, float dropout_p,
                                    uint64_t seed, const void *q, const void *k, const void *v,
                                    const void *out, const void *dout, const float *lse, float *delta,
                                    float *dq_accum, void *dq, void *dk, void *dv, int32_t *status,
                                    ngt_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Dense full-attention window with an additive bias: the attn_bias / pruning_mask / mask arguments
 * of `CoreAttention.full_attention` (NeutronGT/models/gt_dist_node_level_single_window.py:78-99).
 * Same arguments and results as ngt_dense_attn_forward / ngt_dense_attn_backward, plus
 *   bias              float: X = S + bias[h, i, j] before the softmax, element (h, i, j) at
 *                     h * bias_head_stride + i * s + j; bias_head_stride 0 (one [s, s] matrix for
 *                     every head) or s * s ([heads, s, s]).  -inf entries (masked keys) get no weight;
 *                     a row with no finite entry gets lse = -inf and an output of 0.
 *   dbias (backward)  float [heads, s, s] (nullable): dX = P (dP - delta), 0 at -inf entries.
 * Any head_dim <= 64 that is a multiple of 8 (single-role tcgen05 kernels, head_dim padded to 32
 * or 64); node scores are those of the raw S, as the reference computes them before the bias.
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_dense_attn_forward_bias(int64_t s, int heads, int head_dim, float scale, float score_scale,
                                        float dropout_p, uint64_t seed, const void *q, const void *k, const void *v,
                                        const float *bias, int64_t bias_head_stride, void *out, float *lse,
                                        float *node_scores, int32_t *status, ngt_stream_t stream);
NGT_API int ngt_dense_attn_backward_bias(int64_t s, int heads, int head_dim, float scale, float dropout_p,
                                         uint64_t seed, const void *q, const void *k, const void *v, const void *out,
                                         const void *dout, const float *lse, const float *bias,
                                         int64_t bias_head_stride, float *delta, float *dq_accum, void *dq, void *dk,
                                         void *dv, float *dbias, int32_t *status, ngt_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Window subgraph (the window's edge list from the global CSR).
 *
 * Replaces `_subgraph_from_csr` (NeutronGT/core/node_level_pipeline/window_state.py:92-119):
 * for each window node i in window order, its global neighbours in CSR order that are in
 * the window, relabelled to window positions.  Output edge_index [2, E_w] int64 with
 * row 0 = i (local source) and row 1 = local destination — the same order as the
 * reference.  Two calls: _count fills out_rowptr [w+1] (int64, out_rowptr[w] = E_w) and
 * leaves a node map in the workspace; _fill (same workspace, not modified in between)
 * writes the edges.  info[0] = count of window nodes that are out of range or repeated.
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_window_subgraph_workspace_size(int64_t num_global_nodes, int64_t window_nodes,
                                       size_t *bytes /* host */);
NGT_API int ngt_window_subgraph_count(int64_t num_global_nodes, const int64_t *rowptr, const int64_t *col,
                              const int64_t *nodes, int64_t window_nodes, int64_t *out_rowptr,
                              int32_t *info, void *workspace, size_t workspace_bytes,
                              ngt_stream_t stream);
NGT_API int ngt_window_subgraph_fill(int64_t num_global_nodes, const int64_t *rowptr, const int64_t *col,
                             const int64_t *nodes, int64_t window_nodes, const int64_t *out_rowptr,
                             int64_t *out_edge_index, int64_t num_edges, void *workspace,
                             size_t workspace_bytes, ngt_stream_t stream);

/* ------------------------------------------------------------------------------------
 * APPNP personalised PageRank with per-iteration top-k pruning.
 *
 * Replaces the propagation loop of `personal_pagerank_appnp`
 * (NeutronGT/core/ppr_backends/appnp_backend.py:259-305): the cuSPARSE SpGEMM of
 * `csr_spgemm` (NeutronGT/core/ppr_backends/csrc/cusparse_spgemm.cu:65-267, via
 * appnp_backend.py:165-200), the teleport merge (`_aggregate_sparse_entries`, :68-77) and
 * the per-row top-k (`_segment_topk_from_csr`, :102-140) become one kernel that keeps
 * each seed's row on chip.  Values in fp64 with a canonical order: contributions to a
 * column are added in ascending source column, ties rank by ascending column.
 *
 *   rowptr int64 [n+1], col int32 [rowptr[n]]: the graph (P = D^-1 A, D = max(outdeg,1));
 *                   pruned mode merges rows, so each row's columns must ascend (repeats allowed)
 *   in_rowptr/in_col the transpose (in-adjacency, sources ascending within a row); read only
 *                   in dense mode, nullable otherwise
 *   iter_topk       > 0: entries kept per iteration (1..32); <= 0: no pruning (dense mode)
 *   final_keep      entries kept at the end (1..32 in dense mode; <= 0 keeps all when pruned)
 *   out_col int64 / out_val float / out_val64 double (nullable): [num_seeds, keep_stride],
 *   out_cnt int32 [num_seeds]; entries of seed s in (value desc, column asc) order.
 *   info int32 [1]: set to 0 (kept for the ABI; every row now fits: large expansions are
 *                   processed in column windows).
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_ppr_workspace_size(int64_t n, int64_t max_degree, int64_t iter_topk, int64_t num_seeds,
                           size_t *bytes /* host */);
NGT_API int ngt_ppr_appnp_topk(int64_t n, const int64_t *rowptr, const int32_t *col,
                       const int64_t *in_rowptr, const int32_t *in_col, double alpha,
                       int64_t num_iterations, int64_t iter_topk, int64_t final_keep,
                       int64_t source_start, int64_t source_end, int64_t max_degree,
                       int64_t keep_stride, int64_t *out_col, float *out_val, double *out_val64,
                       int32_t *out_cnt, int32_t *info, void *workspace, size_t workspace_bytes,
                       ngt_stream_t stream);

/* ----------------------------------------------------------------------------------
 * Row-wise fp32 operators of the GT / Graphormer layers: LayerNorm forward / backward and the
 * column sum that is a Linear layer's bias gradient.  Replace torch's nn.LayerNorm kernels and
 * the `grad.sum(0)` of nn.Linear's backward in the models' layers
 * (NeutronGT/models/gt_dist_node_level_single_window.py:311-325, graphormer_dist_node_level.py:179,
 * 183, 286).  x, y, dy, dx are row-major [rows, cols] fp32 with cols % 4 == 0 and cols <= 1024,
 * 16-byte aligned; mean and rstd are [rows]; gamma, beta, dgamma, dbeta, out are [cols], 16-byte
 * aligned.  Column sums are added in a fixed order (no atomics).  workspace (16-byte aligned):
 * ngt_rowops_workspace_size bytes.
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_rowops_workspace_size(int64_t rows, int cols, size_t *bytes /* host */);
NGT_API int ngt_layernorm_forward(int64_t rows, int cols, const float *x, const float *gamma, const float *beta,
                                  float eps, float *y, float *mean, float *rstd, ngt_stream_t stream);
NGT_API int ngt_layernorm_backward(int64_t rows, int cols, const float *x, const float *dy, const float *gamma,
                                   const float *mean, const float *rstd, float *dx, float *dgamma, float *dbeta,
                                   void *workspace, size_t workspace_bytes, ngt_stream_t stream);
NGT_API int ngt_column_sum(int64_t rows, int cols, const float *x, float *out, void *workspace,
                           size_t workspace_bytes, ngt_stream_t stream);

/* ----------------------------------------------------------------------------------
 * fp32 Linear layers of the GT / Graphormer models (y = x W^T + b): replace the GEMMs torch
 * runs for nn.Linear's forward and backward (NeutronGT/models/gt_dist_node_level_single_window.py:
 * 235-237, 313-318, 361; graphormer_dist_node_level.py:179, 183, 286).  All tensors row-major fp32,
 * 16-byte aligned: x / dx [rows, in_features], y / dy [rows, out_features], weight / dweight
 * [out_features, in_features], bias / dbias [out_features] (bias and dbias may be NULL).
 * in_features and out_features are multiples of 4.  fp32 precision throughout: with both
 * dimensions <= 256 the forward and input grad run on the tcgen05 tensor cores with split TF32
 * operands (three TF32 products per pair: hi*hi + hi*lo + lo*hi, fp32 accumulation), otherwise
 * on CUDA-core FFMA; the weight grad runs on the same split-TF32 tensor-core kernel when
 * in_features <= 256 and rows >= 64 (row ranges of at most 512 rows, summed in a fixed order),
 * else on FFMA.
 *   ngt_linear_forward         y = x W^T + b          in_features  <= 256 (else NGT_ERR_UNSUPPORTED)
 *   ngt_linear_backward_input  dx = dy W              out_features <= 256 (else NGT_ERR_UNSUPPORTED)
 *   ngt_linear_backward_weight dW = dy^T x, db = column sums of dy; any size; summed in a fixed
 *                              order (bitwise reproducible); workspace from
 *                              ngt_linear_weight_workspace_size (depends on the current device's
 *                              SM count: query on the device that runs the call).
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_linear_forward(int64_t rows, int in_features, int out_features, const float *x,
                               const float *weight, const float *bias, float *y, ngt_stream_t stream);
NGT_API int ngt_linear_backward_input(int64_t rows, int in_features, int out_features, const float *dy,
                                      const float *weight, float *dx, ngt_stream_t stream);
NGT_API int ngt_linear_weight_workspace_size(int64_t rows, int in_features, int out_features,
                                             size_t *bytes /* host */);
NGT_API int ngt_linear_backward_weight(int64_t rows, int in_features, int out_features, const float *x,
                                       const float *dy, float *dweight, float *dbias, void *workspace,
                                       size_t workspace_bytes, ngt_stream_t stream);
/* ------------------------------------------------------------------------------------
 * bf16 Linear layers (the large model's projections) on the tcgen05 tensor cores.
 *
 * Replace torch's bf16 Linear GEMMs in GPH_Large's QKV, output and FFN projections
 * (NeutronGT/models/gt_dist_node_level_single_window.py:235-237, 313-318;
 * graphormer_dist_node_level.py:139, 179, 183) with the same contract as the fp32 entry points
 * above, on bf16 tensors: x / dx [rows, in_features], y / dy [rows, out_features], weight /
 * dweight [out_features, in_features], bias / dbias [out_features] (nullable), all bf16,
 * row-major, 16-byte aligned; in_features and out_features multiples of 8.  fp32 accumulation;
 * results rounded to bf16 once.
 *   ngt_linear_bf16_forward          y = x W^T + b
 *   ngt_linear_bf16_backward_input   dx = dy W
 *   ngt_linear_bf16_backward_weight  dW = dy^T x and db = column sums of dy, each summed in a
 *                                    fixed order (bitwise reproducible); fp32 workspace of
 *                                    ngt_linear_bf16_weight_workspace_size bytes (depends on the
 *                                    current device's SM count)
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_linear_bf16_forward(int64_t rows, int in_features, int out_features, const void *x,
                                    const void *weight, const void *bias, void *y, ngt_stream_t stream);
NGT_API int ngt_linear_bf16_backward_input(int64_t rows, int in_features, int out_features, const void *dy,
                                           const void *weight, void *dx, ngt_stream_t stream);
NGT_API int ngt_linear_bf16_weight_workspace_size(int64_t rows, int in_features, int out_features,
                                                  size_t *bytes /* host */);
NGT_API int ngt_linear_bf16_backward_weight(int64_t rows, int in_features, int out_features, const void *x,
                                            const void *dy, void *dweight, void *dbias, void *workspace,
                                            size_t workspace_bytes, ngt_stream_t stream);
/* Number of tensor-core Linear CTAs (fp32 and bf16 kernels) whose bounded waits ran out (they store
 * nothing) since the library was loaded; synchronous.  No counterpart in the reference (torch's
 * GEMMs do not wait). */
NGT_API int ngt_linear_status(int32_t *timeouts /* host */);

/* ------------------------------------------------------------------------------------
 * Push-based approximate personalised PageRank + per-seed top-k.
 *
 * Replaces the reference's default backend, personal_pagerank_torch_geometric
 * (NeutronGT/core/ppr_backends/torch_geometric_backend.py:5-30: PyG get_ppr(edge_index, alpha, eps),
 * then a per-source top-k loop).  Per seed s in [seed_start, seed_end): the push method with a LIFO
 * stack (p = {s: 0}, r = {s: alpha}; pop u: p[u] += r[u], r[u] = 0, r[v] += (1 - alpha) r[u] /
 * deg(u) for v in adj(u) in CSR order, push v when r[v] >= alpha * eps * deg(v) and v is not on the
 * stack), fp64, each operation one IEEE rounding.  Kept: p in insertion order when it has at most
 * topk entries, else the topk largest by (value desc, node asc).
 *   rowptr int64 [n+1], col int32 [E] (columns ascending within a row, as PyG sorts them)
 *   slots        concurrent seeds (one warp each); workspace from ngt_ppr_push_workspace_size(n, slots)
 *                (about 29 bytes x n per slot; its flags are cleared by the call)
 *   out_idx / out_val / out_val64 (nullable) [(seed_end - seed_start) * topk], out_cnt [seeds]
 *   info         int32 [1]: seeds stopped by the termination guard (0 in practice)
 * ngt_ppr_push_stats reads the last call's push and adjacency-read totals from its workspace
 * (synchronous).  alpha in (0, 1], eps > 0.
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_ppr_push_workspace_size(int64_t n, int64_t slots, size_t *bytes /* host */);
NGT_API int ngt_ppr_push_topk(int64_t n, const int64_t *rowptr, const int32_t *col, double alpha, double eps,
                              int64_t seed_start, int64_t seed_end, int64_t topk, int64_t slots, int64_t *out_idx,
                              float *out_val, double *out_val64, int32_t *out_cnt, int32_t *info, void *workspace,
                              size_t workspace_bytes, ngt_stream_t stream);
NGT_API int ngt_ppr_push_stats(const void *workspace, int64_t n, int64_t slots, int64_t *pushes_and_reads /* host [2] */,
                               ngt_stream_t stream);

/* ------------------------------------------------------------------------------------
 * CSR column check and narrowing for the PPR entry points (the reference's wrappers check the
 * graph with torch reductions and convert it to int32 for cuSPARSE, appnp_backend.py:36-58,
 * cusparse_ops.py:76-94; here one pass over the columns does both).
 *   rowptr int64 [n+1], a valid row pointer (starts at 0, non-decreasing, rowptr[n] = nnz)
 *   col    int64 [nnz] in, col32 int32 [nnz] out (the same values, narrowed)
 *   flags  int32 [1] device: set by the call, bit 0 = a column outside [0, n), bit 1 = a column
 *          below its predecessor within a row (rows not ascending)
 * nnz > 0 needs n > 0.  Asynchronous on `stream`.
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_csr_col32_checked(int64_t n, int64_t nnz, const int64_t *rowptr, const int64_t *col, int32_t *col32,
                                  int32_t *flags, ngt_stream_t stream);

/* ------------------------------------------------------------------------------------
 * Sparse x sparse product C = A B of fp32 CSR matrices.
 *
 * Replaces csr_spgemm (NeutronGT/core/ppr_backends/cusparse_ops.py:97-114; cuSPARSE SpGEMM in
 * csrc/cusparse_spgemm.cu:65-267): A [m x n], B [n x n], C [m x n] holding every structural entry
 * of the product (entries that cancel to 0 stay, as cuSPARSE keeps them), columns ascending per
 * row, each value the fp32 sum of its products in A's entry order.  Two calls on one workspace:
 *   ngt_csr_spgemm_symbolic  writes rowptr_c int64 [m+1] (rowptr_c[m] = nnz(C)); zeroes the workspace
 *   ngt_csr_spgemm_numeric   fills col_c int64 [nnz], val_c float [nnz] (after the symbolic call)
 *   rowptr_a / rowptr_b int64, col_a / col_b int32 (in [0, n)), val_a / val_b float
 *   slots    concurrent rows (one warp each); workspace from ngt_csr_spgemm_workspace_size
 *            (per slot: 5 bytes x n of accumulator and flags, plus two column buffers of
 *            4 bytes x the power of two >= n, the touched list and its merge partner)
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_csr_spgemm_workspace_size(int64_t m, int64_t n, int64_t slots, size_t *bytes /* host */);
NGT_API int ngt_csr_spgemm_symbolic(int64_t m, int64_t n, const int64_t *rowptr_a, const int32_t *col_a,
                                    const int64_t *rowptr_b, const int32_t *col_b, int64_t slots, int64_t *rowptr_c,
                                    void *workspace, size_t workspace_bytes, ngt_stream_t stream);
NGT_API int ngt_csr_spgemm_numeric(int64_t m, int64_t n, const int64_t *rowptr_a, const int32_t *col_a,
                                   const float *val_a, const int64_t *rowptr_b, const int32_t *col_b,
                                   const float *val_b, int64_t slots, const int64_t *rowptr_c, int64_t *col_c,
                                   float *val_c, void *workspace, size_t workspace_bytes, ngt_stream_t stream);

/* ----------------------------------------------------------------------------------
 * Window construction between PPR and the training windows.
 *
 * ngt_ppr_adjacency replaces build_adj_fromat (NeutronGT/core/ppr_preprocess.py:30-71): the PPR
 * list edge_index int64 [2, m] (row 0 seed, row 1 neighbour) with values fp32 [m] becomes the
 * symmetric weighted adjacency of n nodes (n = max index + 1 in the reference): each undirected
 * pair {u, v} once, weight int32(max(sum of its PPR values * 1000, 1)) with the values added in
 * entry order; xadj int32 [n+1], adjncy / eweights int32 [2m] capacity (2U used).  Rows list the
 * pairs with u < v first, then u > v, each in key order: the stable form of the reference's
 * argsort (which does not promise an order inside a row).  info int32 [2] (device): out-of-range
 * entries, U.
 *
 * ngt_halo_degree + ngt_halo_merge replace _merge_related_nodes
 * (NeutronGT/core/metisPartition.py:397-425): the window part int64 [p] (any order) gets the
 * topk_percent % (rounded down) of its distinct external neighbours with the largest summed edge
 * weight, ties in first-encounter order (window order, then CSR order); the result is sorted.
 * ngt_halo_degree writes the window's summed degree `total` (device int64) that sizes the merge:
 * workspace from ngt_halo_merge_workspace_size(n, p, total) (ngt_halo_degree needs the size for
 * total = 0); out int64 [p + total] capacity; counts int64 [3] (device): merged size, selected,
 * distinct external neighbours.
 *
 * ngt_duplicate_rerange replaces _find_duplicate_nodes_and_rerange
 * (NeutronGT/core/metisPartition.py:333-363; window_state.py:52-73 for a rank's windows): nodes
 * that occur in two or more of the `parts` windows (nodes int64, window k at
 * [offsets[k], offsets[k+1])) move to the front of every window that holds them, both groups in
 * window order; dup_counts int64 [parts] (device) = the length of each front group.  bad int32
 * (device): node ids outside [0, n).
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_ppr_adjacency_workspace_size(int64_t m, int64_t n, size_t *bytes /* host */);
NGT_API int ngt_ppr_adjacency(int64_t m, int64_t n, const int64_t *edge_index, const float *values, int32_t *xadj,
                              int32_t *adjncy, int32_t *eweights, int32_t *info, void *workspace,
                              size_t workspace_bytes, ngt_stream_t stream);
NGT_API int ngt_halo_degree(int64_t n, const int32_t *xadj, int64_t p, const int64_t *part, int64_t *total,
                            void *workspace, size_t workspace_bytes, ngt_stream_t stream);
NGT_API int ngt_halo_merge_workspace_size(int64_t n, int64_t p, int64_t total, size_t *bytes /* host */);
NGT_API int ngt_halo_merge(int64_t n, const int32_t *xadj, const int32_t *adjncy, const int32_t *eweights,
                           int64_t p, const int64_t *part, int64_t total, int32_t topk_percent, int64_t *out,
                           int64_t *counts, void *workspace, size_t workspace_bytes, ngt_stream_t stream);
NGT_API int ngt_duplicate_rerange_workspace_size(int64_t n, int64_t total, size_t *bytes /* host */);
NGT_API int ngt_duplicate_rerange(int64_t n, int32_t parts, const int64_t *offsets, const int64_t *nodes,
                                  int64_t total, int64_t *out_nodes, int64_t *dup_counts, int32_t *bad,
                                  void *workspace, size_t workspace_bytes, ngt_stream_t stream);

/* ----------------------------------------------------------------------------------
 * Random connections of isolated nodes: replaces add_isolated_connections
 * (NeutronGT/core/ppr_preprocess.py:94-132).  Nodes of [0, n) that appear in neither edge list
 * (isolated, ascending) are linked to each appearing node (ascending) with probability
 * connect_prob; new edges (isolated, appearing) in row-major order of that pair grid, as
 * torch.where on the reference's dense mask gives them.  The reference draws the mask with
 * torch.rand on an [isolated x appearing] tensor; here each pair's draw is a counter-based
 * SplitMix64 hash of (seed, isolated index, appearing index), computed twice (count, fill) and
 * never stored: same distribution, not the same bits.
 *   count: counts int64 [3] (device) = isolated, appearing, new edges; bad int32 (device) =
 *          entries outside [0, n)
 *   fill:  new_edge_index int64 [2, e_new], e_new = counts[2]; same workspace, untouched between
 *          the two calls
 * ---------------------------------------------------------------------------------- */
NGT_API int ngt_isolated_connections_workspace_size(int64_t n, size_t *bytes /* host */);
NGT_API int ngt_isolated_connections_count(int64_t n, int64_t m_ppr, const int64_t *ppr_edge_index, int64_t m_graph,
                                           const int64_t *graph_edge_index, double connect_prob, uint64_t seed,
                                           int64_t *counts, int32_t *bad, void *workspace, size_t workspace_bytes,
                                           ngt_stream_t stream);
NGT_API int ngt_isolated_connections_fill(int64_t n, double connect_prob, uint64_t seed, const int64_t *counts,
                                          int64_t e_new, int64_t *new_edge_index, void *workspace,
                                          size_t workspace_bytes, ngt_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* NEUTRONGT_B200_H */
