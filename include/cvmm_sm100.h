/*
 * cvmm_sm100.h — C ABI of the B200 (sm_100a) CVMM library (libcvmm_sm100.so).
 *
 * CVMM ("conditional vector-matrix multiplication") is the top-k
 * mixture-of-experts projection of RobertCsordas/cvmm_codex: every route r
 * (one token's choice of one expert) multiplies one input row by the weight
 * matrix keys[e] of the expert e it was routed to.
 *
 * Conventions shared by every entry point:
 *   - all pointers are device pointers; sizes are element counts;
 *   - every function is stream-ordered on `stream` (a cudaStream_t) and never
 *     synchronises the host;
 *   - no function allocates device memory. Scratch comes from the caller as
 *     `workspace` / `workspace_bytes`, sized by the matching *_workspace_size
 *     query;
 *   - the return value is a status code (CVMM_OK or a negative CVMM_ERR_*);
 *     cvmm_last_error() gives a message for the last failure on this thread;
 *   - dtype codes follow the reference's dtype_to_type_id (cvmm.py:36-44).
 *
 * "Sorted order" below means the expert-major stable order produced by
 * cvmm_sel_prepare: position p of the sorted arrays is the p-th route when
 * routes are ordered by (expert id, route id).
 */
#ifndef CVMM_SM100_H
#define CVMM_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* cvmm_stream_t; /* == cudaStream_t */

/* dtype codes */
#define CVMM_F32 0
#define CVMM_F16 1
#define CVMM_BF16 2
#define CVMM_I32 3
#define CVMM_I64 4

/* status codes */
#define CVMM_OK 0
#define CVMM_ERR_INVALID_ARG -1
#define CVMM_ERR_UNSUPPORTED_DTYPE -2
#define CVMM_ERR_LAUNCH -3
#define CVMM_ERR_WORKSPACE -4
#define CVMM_ERR_DEVICE -5
/* device status word codes (cvmm_device_status) */
#define CVMM_DEV_TIMEOUT 1
#define CVMM_DEV_BAD_INDEX 2

/* ABI version of this header; bumped on any signature change. */
int cvmm_abi_version(void);  /* 10 */

/* Caps the number of SMs the persistent tensor-core GEMMs launched from now on
 * may occupy (one CTA per SM, nearly all of its shared memory); 0 removes the
 * cap. Returns the previous cap. Process-wide. A data-parallel caller sets it
 * while an NCCL collective (the grad-W all-reduce) runs next to the grad-x
 * kernels, so the collective's CTAs find free SMs instead of waiting for the
 * GEMM to end. No reference counterpart (the reference is single-GPU). */
int cvmm_set_sm_limit(int n_sms);

/* Turns programmatic dependent launch on (1) or off (0) for the kernels
 * launched from now on; returns the previous setting. On by default unless the
 * environment sets CVMM_B200_PDL=0. With it on, each kernel's CTAs may be
 * scheduled while the previous kernel on the stream drains and wait on the
 * device for its completion, which hides launch latency and kernel prologues
 * between the back-to-back kernels of one CVMM call (and in captured graphs).
 * Results are identical either way. No reference counterpart. */
int cvmm_set_pdl(int enable);

/* Message for the last failed call on the calling host thread. */
const char* cvmm_last_error(void);

/* Reads (and with reset != 0 clears) the device status word that kernels set
 * instead of trapping. Synchronises `stream`. Returns the code (0 = clean);
 * where/aux receive the kernel tag and offending value when non-NULL. */
int cvmm_device_status(int reset, int* where, long long* aux, cvmm_stream_t stream);

/* Failure-path self-test: launches one thread that waits on a barrier nothing
 * arrives on, through the bounded wait all persistent kernels use, with a limit
 * of limit_ns (1 us .. 100 ms) instead of the kernels' 2 s. Afterwards
 * cvmm_device_status reports CVMM_DEV_TIMEOUT with where == 99, and the
 * context stays usable. No reference counterpart (the reference has no device
 * failure detection). */
int cvmm_selftest_wait_timeout(int64_t limit_ns, cvmm_stream_t stream);

/* ------------------------------------------------------------------------
 * Selector preparation.
 * Replaces cvmm_prepare_sel2 (cvmm.py:1786-1803) and cvmm_prepare_sel
 * (cvmm.py:24-27): fsel = int32(sel); (ssel, idx) = fsel.sort();
 *   route_input == 0: sel_index = idx // top_k, out_index = idx
 *   route_input != 0: sel_index = idx,          out_index unused (may be NULL)
 * The sort is a stable device radix sort, so ties keep route order; this is
 * bit-exact with torch.sort(stable=True).
 *   sel: [n_routes] int64 or int32 (sel_dtype CVMM_I64 / CVMM_I32)
 *   raw_sel, sorted_sel: [n_routes] int32; sel_index, out_index: [n_routes] int64
 * ------------------------------------------------------------------------ */
size_t cvmm_sel_prepare_workspace_size(int64_t n_routes);
int cvmm_sel_prepare(const void* sel, int sel_dtype, int64_t n_routes, int64_t top_k,
                     int route_input, int32_t* raw_sel, int32_t* sorted_sel,
                     int64_t* sel_index, int64_t* out_index, void* workspace,
                     size_t workspace_bytes, cvmm_stream_t stream);

/* Allocation-free cvmm_sel_prepare, for callers that cannot allocate device
 * memory on the call path (a host owning all device memory through its own
 * fixed plan, a serving loop that must not call cudaMalloc because it can
 * synchronise the device). It has no counterpart in the reference.
 * Same arguments and results as cvmm_sel_prepare minus the workspace: the
 * scratch is a static device array of about 1.5 MiB that every GPU loading
 * the library keeps until exit, so n_routes is limited to
 * CVMM_NOALLOC_MAX_ROUTES (larger inputs return CVMM_ERR_INVALID_ARG).
 * The first call on a device looks up that array's address with that device
 * current; make that first call before any stream capture. All calls share
 * the one array, so calls whose work overlaps on the GPU (different streams,
 * or different host threads) race and must be serialised by the caller. */
#define CVMM_NOALLOC_MAX_ROUTES 65536
int cvmm_sel_prepare_noalloc(const void* sel, int sel_dtype, int64_t n_routes, int64_t top_k,
                             int route_input, int32_t* raw_sel, int32_t* sorted_sel,
                             int64_t* sel_index, int64_t* out_index, cvmm_stream_t stream);

/* Inclusive end offset of every expert's segment in sorted order:
 * offsets[e] = #routes with expert <= e (missing experts repeat the previous
 * value). Replaces _cvmm_expert_offsets / cvmm_expert_offsets_kernel
 * (cvmm.py:68-78, 315-335, 1108-1120). */
int cvmm_expert_offsets(const int32_t* sorted_sel, int64_t n_routes, int64_t n_experts,
                        int64_t* offsets, cvmm_stream_t stream);

/* ------------------------------------------------------------------------
 * Forward gathered GEMM. Replaces torch op mylib::cvmm_triton / cvmm_triton
 * (cvmm.py:808-867) and cvmm_kernel (cvmm.py:121-243).
 * For every sorted position p with expert e (from offsets):
 *   out[row_p] = cast_out( op(x[sel_index[p]]) . op(keys[e]) )   fp32 accumulate
 *   row_p = out_index[p] if out_index != NULL else sel_index[p]
 * x: [x_rows, k_dim] row-major with leading dimension x_ld;
 * keys[e][k][n] at keys + e*ks_e + k*ks_k + n*ks_n (any strides);
 * out: [n_routes, n_dim] with leading dimension out_ld.
 * op_dtype selects the arithmetic: CVMM_BF16 / CVMM_F16 run on the tcgen05
 * tensor cores (operands rounded to op_dtype, fp32 accumulate), CVMM_F32 runs
 * an exact fp32 FFMA kernel (the reference's allow_tf32=False path).
 * ------------------------------------------------------------------------ */
/* Workspace bytes that suffice for cvmm_forward, cvmm_backward_x and
 * cvmm_backward_w on n_routes routes over n_experts experts with
 * keys[e] of shape [k_dim, n_dim] (pass k_dim = n_dim = 0 for the
 * forward / grad-input tile table alone). */
size_t cvmm_gemm_workspace_size(int64_t n_routes, int64_t n_experts, int64_t k_dim,
                                int64_t n_dim, int x_dtype, int keys_dtype, int op_dtype,
                                int64_t x_rows);
int cvmm_forward(const void* x, int x_dtype, int64_t x_rows, int64_t x_ld,
                 const int64_t* sel_index, const int64_t* out_index, const int64_t* offsets,
                 int64_t n_routes, const void* keys, int keys_dtype, int64_t n_experts,
                 int64_t k_dim, int64_t n_dim, int64_t ks_e, int64_t ks_k, int64_t ks_n,
                 void* out, int out_dtype, int64_t out_ld, int op_dtype,
                 const int32_t* x_pad_start, const int32_t* out_pad_start, void* x_copy,
                 void* workspace, size_t workspace_bytes, cvmm_stream_t stream);

/* Forward gathered GEMM with the sigma-MoE layer's activation fused into the
 * epilogue: for every route, pre_act[row_p] = op(acc) and
 * out[row_p] = gelu(op(acc)) = 0.5 z (1 + erf(z / sqrt 2)) in fp32 on the
 * rounded z, rounded once more (both [n_routes, n_dim] with out_ld).
 * Replaces cvmm(x, sel, w_up) followed by F.gelu in the reference's FFN layer
 * (benchmark_ffn_moe.py:93-94): the activation pass over the route outputs
 * disappears and pre_act is what the GELU backward reads. bf16/fp16 op_dtype
 * and out_dtype == op_dtype; x_copy as in cvmm_forward. */
int cvmm_forward_gelu(const void* x, int x_dtype, int64_t x_rows, int64_t x_ld,
                      const int64_t* sel_index, const int64_t* out_index, const int64_t* offsets,
                      int64_t n_routes, const void* keys, int keys_dtype, int64_t n_experts,
                      int64_t k_dim, int64_t n_dim, int64_t ks_e, int64_t ks_k, int64_t ks_n,
                      void* out, void* pre_act, int out_dtype, int64_t out_ld, int op_dtype,
                      void* x_copy, void* workspace, size_t workspace_bytes, cvmm_stream_t stream);

/* grad_pre_act[i] = grad[i] * gelu'(pre_act[i]) in fp32, rounded to dtype
 * (bf16/fp16); the backward of F.gelu (torch's GeluBackward, erf form). */
int cvmm_gelu_backward(const void* grad, const void* pre_act, void* grad_pre_act, int dtype, int64_t n,
                       cvmm_stream_t stream);

/* Router of the sigma-MoE layer (benchmark_ffn_moe.py:89-92) in one launch:
 * probs = softmax(float(logits)) over n_experts (<= 1024);
 * (weights, sel) = top_k(probs) in descending order (ties: lower expert id);
 * weights /= max(sum(weights), 1e-20) when renormalize != 0.
 * logits: [n_tokens, n_experts] fp32/bf16/fp16; sel: int64 [n_tokens, top_k];
 * weights: fp32 [n_tokens, top_k]; 1 <= top_k <= 32. */
int cvmm_router_topk(const void* logits, int logits_dtype, int64_t n_tokens, int64_t n_experts, int64_t top_k,
                     int renormalize, int64_t* sel, float* weights, cvmm_stream_t stream);
/* With x_pad_start != NULL, x is the expert-padded sorted layout made by
 * cvmm_sort_rows_padded: the x row of sorted position p is then
 * x_pad_start[e] + p - seg_begin(e), x_rows is ignored, and sel_index only
 * names the output rows (when out_index is NULL). bf16/fp16 op_dtype with
 * x_dtype == op_dtype only.
 * With out_pad_start != NULL, out is written in the expert-padded sorted
 * layout instead (row of sorted position p: out_pad_start[e] + p - seg_begin(e),
 * n_routes + n_experts * CVMM_PAD_ROWS rows, padding rows included) by dense
 * tensor-memory-to-TMA stores; out_index is then ignored. bf16/fp16 out_dtype
 * and op_dtype, 16-byte aligned rows. Read it back per route through
 * cvmm_padded_route_rows.
 * With x_copy != NULL (row-indexed x, bf16/fp16 op_dtype), the forward also
 * writes the op_dtype rows it gathers into x_copy in the expert-padded sorted
 * layout ([n_routes + n_experts * CVMM_PAD_ROWS, k_dim], padding rows zero),
 * exactly what cvmm_sort_rows_padded would produce; cvmm_pad_starts gives its
 * pad_start for the grad-W call. This replaces a separate copy pass (the
 * reference's grouped-x copy, cvmm.py:1123-1138). */

/* Weighted combine of the forward: out[t] = cast( sum_j cast_y(w[t,j]) * y[t*top_k+j] ),
 * fp32 accumulate. Replaces the bmm at cvmm.py:1543-1545. */
int cvmm_weighted_combine(const void* y, int y_dtype, const void* w, int w_dtype,
                          void* out, int out_dtype, int64_t n_tokens, int64_t top_k,
                          int64_t n_dim, const int32_t* y_rows, cvmm_stream_t stream);
/* y_rows != NULL: the y row of route r is y_rows[r] (e.g. an expert-padded
 * sorted forward output with the map of cvmm_padded_route_rows); NULL: r. */

/* ------------------------------------------------------------------------
 * Backward grad-input GEMM. Replaces cvmm_grouped_bwd_x_kernel
 * (cvmm.py:363-421) with its launcher (cvmm.py:1199-1223) and the fused
 * cvmm_weighted_route_bwd_x_kernel (cvmm.py:1008-1105, launcher 1386-1433).
 * For every sorted position p with expert e:
 *   a_p = op(g[g_index[p] / g_div]) . op(keys[e])^T          (fp32 acc)
 * With g_pad_start != NULL, g is the expert-padded sorted layout made by
 * cvmm_sort_rows_padded (pad 128): the g row of sorted position p is
 * g_pad_start[e] + p - seg_begin(e) and g_index / g_div are ignored
 * (bf16/fp16 op_dtype only).
 *   mode 0: out[out_index[p]] = cast_out(a_p)
 *   mode 1 (weighted, route-shaped x):
 *           out[out_index[p]]  = cast_out( op(op(a_p) * op(w[out_index[p]])) )
 *           gsel[out_index[p]] += sum_j op(a_p)_j * x[out_index[p] / x_div]_j   (fp32)
 *           (x_div = 1 for route-shaped x; x_div = r when r consecutive routes
 *           share one x row, e.g. the 2 routes of one SwitchHead head)
 * keys strides are those of keys[e][k_dim][n_dim] as in cvmm_forward; the
 * product contracts over n_dim and produces k_dim columns.
 * gsel must be zeroed by the caller (mode 1 accumulates into it).
 * ------------------------------------------------------------------------ */
int cvmm_backward_x(const void* g, int g_dtype, int64_t g_ld, const int64_t* g_index,
                    int64_t g_div, const int64_t* out_index, const int64_t* offsets,
                    int64_t n_routes, const void* keys, int keys_dtype, int64_t n_experts,
                    int64_t k_dim, int64_t n_dim, int64_t ks_e, int64_t ks_k, int64_t ks_n,
                    void* out, int out_dtype, int64_t out_ld, int mode, const void* w,
                    int w_dtype, const void* x, int x_dtype, int64_t x_ld, int64_t x_div,
                    float* gsel, int op_dtype, const int32_t* g_pad_start,
                    const int32_t* out_pad_start, void* workspace, size_t workspace_bytes,
                    cvmm_stream_t stream);
/* out_pad_start != NULL (mode 0 only): out is written in the expert-padded
 * sorted layout as in cvmm_forward, out_index is ignored. */

/* Backward grad-weight. Replaces cvmm_grouped_bwd_w_gather_x_kernel /
 * cvmm_grouped_bwd_w_kernel / cvmm_grouped_bwd_w_weighted_kernel
 * (cvmm.py:424-604, launchers 1141-1198, 1341-1383):
 *   grad_w[e][m][n] = sum_{p in seg(e)} op(x[x_index[p]/x_div][m]) * s_p * op(g[g_index[p]/g_div][n])
 *   s_p = 1, or with w != NULL: the g row is first multiplied by op(w[w_index[p]])
 *   and rounded to op_dtype (cvmm.py:591-599).
 * grad_w: [n_experts, m_dim, n_dim] fp32, fully written (empty experts get 0).
 * x_pad_start / g_pad_start != NULL: x / g is the expert-padded sorted
 * layout of cvmm_sort_rows_padded and x_index, x_div / g_index, g_div are
 * ignored (bf16/fp16 op_dtype, operand dtype == op_dtype). A padded g is
 * used as it is (a copy made with cvmm_sort_rows_padded's `scale` already
 * carries the route weights: pass w = NULL), or, with w != NULL, it is the
 * unscaled copy and the weights are applied in shared memory with the same
 * rounding, which lets one unscaled copy also feed cvmm_backward_x.
 * Long expert segments are split over several CTAs (split-K); their partial
 * sums live in the workspace (cvmm_gemm_workspace_size with k_dim = m_dim)
 * and are added in a fixed order, so results are deterministic. */
int cvmm_backward_w(const void* x, int x_dtype, int64_t x_ld, const int64_t* x_index,
                    int64_t x_div, const void* g, int g_dtype, int64_t g_ld,
                    const int64_t* g_index, int64_t g_div, const void* w, int w_dtype,
                    const int64_t* w_index, const int64_t* offsets, int64_t n_routes,
                    int64_t n_experts, int64_t m_dim, int64_t n_dim, float* grad_w,
                    int op_dtype, const int32_t* x_pad_start, const int32_t* g_pad_start,
                    void* workspace, size_t workspace_bytes, cvmm_stream_t stream);
/* Kernels one cvmm_backward_w call with these arguments launches (for launch
 * accounting): the unit-list build (unless the tensor-core GEMM builds it in
 * shared memory), the route-row resolve (unless both operands are padded and
 * unweighted), the GEMM and the split-K reduction. No reference counterpart. */
int cvmm_backward_w_launches(int64_t n_routes, int64_t n_experts, int64_t m_dim, int64_t n_dim, int op_dtype,
                             int both_padded, int weighted);

/* ------------------------------------------------------------------------
 * Expert-padded sorted copy of route rows. Replaces the reference's grouping
 * copy cvmm_group_routes / cvmm_group_routes_kernel (cvmm.py:338-360,
 * 1123-1138), with every expert's segment padded with zero rows to a multiple
 * of CVMM_PAD_ROWS rows so that the GEMMs read it as dense tensor-core tiles:
 *   dst[pad_start[e] + (p - seg_begin(e))] = op(src[index[p] / div])
 *       or, with scale != NULL, op( op(src[index[p] / div]) * op(scale[index[p]]) )
 * where op() rounds to dst_dtype (the weighted grad-W operand rounding of
 * cvmm.py:591-599). pad_start[e] (int32) = sum over e' < e of
 * round_up(count(e'), CVMM_PAD_ROWS); the padding rows of every segment are
 * zero. dst holds n_routes + n_experts * CVMM_PAD_ROWS rows of `cols`
 * elements (leading dimension cols); rows past the last segment are not
 * written. Pass dst / pad_start as x / x_pad_start or g / g_pad_start of
 * cvmm_forward, cvmm_backward_x and cvmm_backward_w.
 * ------------------------------------------------------------------------ */
#define CVMM_PAD_ROWS 128
/* pad_start[e] of the expert-padded sorted layout for these offsets. */
int cvmm_pad_starts(const int64_t* offsets, int64_t n_experts, int32_t* pad_start, cvmm_stream_t stream);
int cvmm_sort_rows_padded(const void* src, int src_dtype, int64_t src_ld, const int64_t* index,
                          int64_t div, const void* scale, int scale_dtype,
                          const int32_t* sorted_sel, const int64_t* offsets, int64_t n_routes,
                          int64_t n_experts, int64_t cols, void* dst, int dst_dtype,
                          int32_t* pad_start, cvmm_stream_t stream);
/* cvmm_sort_rows_padded with two additions, each saving a launch:
 * pad_start_ready != 0: pad_start already holds the pad starts of these
 * offsets (from cvmm_pad_starts or an earlier copy over the same selector)
 * and is only read; route_rows != NULL: also writes
 * route_rows[index[p]] = the padded row of sorted position p, the map
 * cvmm_padded_route_rows makes (the row map of the k-sum, cvmm.py:1199-1223).
 * Same copy as the reference's grouping copy (cvmm.py:338-360). */
int cvmm_sort_rows_padded_ex(const void* src, int src_dtype, int64_t src_ld, const int64_t* index, int64_t div,
                             const void* scale, int scale_dtype, const int32_t* sorted_sel, const int64_t* offsets,
                             int64_t n_routes, int64_t n_experts, int64_t cols, void* dst, int dst_dtype,
                             int32_t* pad_start, int pad_start_ready, int32_t* route_rows, cvmm_stream_t stream);

/* Sum over the top-k routes of each token: out[t] = cast( sum_j src[t*top_k+j] ),
 * fp32 accumulate. Replaces grouped_x.view(..., top_k, d).sum(-2) (cvmm.py:1223). */
int cvmm_sum_routes(const void* src, int src_dtype, void* out, int out_dtype,
                    int64_t n_tokens, int64_t top_k, int64_t d, const int32_t* src_rows,
                    cvmm_stream_t stream);
/* src_rows != NULL: the src row of route r is src_rows[r]; NULL: r. */

/* Route -> row map of the expert-padded sorted layout:
 *   rows[route[p]] = pad_start[e] + p - seg_begin(e)   for sorted p,
 * with route[p] the route id of sorted position p (out_index, or sel_index
 * for route-indexed selectors). Lets cvmm_sum_routes / cvmm_weighted_combine
 * read outputs written with out_pad_start. No reference counterpart: the
 * reference scatters outputs straight to route order (cvmm.py:213-218). */
int cvmm_padded_route_rows(const int64_t* route, const int32_t* sorted_sel, const int64_t* offsets,
                           const int32_t* pad_start, int64_t n_routes, int64_t n_experts,
                           int32_t* rows, cvmm_stream_t stream);

/* Token-input weighted backward tail (cvmm.py:1737-1746):
 *   grad_x[t]      = cast( sum_j cast_r(w[t,j]) * route_grad[t,j] )       (if grad_x)
 *   grad_sel[t,j]  = sum_d float(route_grad[t,j,d]) * float(x[t,d])        (if grad_sel, fp32)
 * route_grad: [n_tokens*top_k, d]; x: [n_tokens, d]. */
int cvmm_weighted_token_backward(const void* route_grad, int rg_dtype, const void* w,
                                 int w_dtype, const void* x, int x_dtype, void* grad_x,
                                 int gx_dtype, float* grad_sel, int64_t n_tokens,
                                 int64_t top_k, int64_t d, cvmm_stream_t stream);

/* Elementwise dtype conversion (round-to-nearest-even), e.g. fp32 expert
 * weights to a bf16 operand copy. Supports the float dtypes only. */
int cvmm_cast(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t n,
              cvmm_stream_t stream);
/* cvmm_cast that may start while the previous kernel on the stream is still
 * running (programmatic launch): it reads src at once, waits for that kernel,
 * and only then writes dst, so every later kernel still sees the usual stream
 * order. Use it only for a src that no kernel of this library enqueued
 * earlier on the stream writes (expert weights updated by the caller's own
 * kernels are fine: this library's kernels start only after those finish).
 * It overlaps the reads of the keys cast with the selector sort. Same result as cvmm_cast
 * (the reference's in-kernel weight cast, cvmm.py:202-204). */
int cvmm_cast_ahead(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t n, cvmm_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* CVMM_SM100_H */
