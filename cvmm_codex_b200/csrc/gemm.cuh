// Problem descriptions shared by the two GEMM engines (tcgen05 tensor-core
// kernels for bf16/fp16 arithmetic, exact-fp32 FFMA kernels for fp32
// arithmetic) and the expert-segment tile scheduler.
#pragma once

#include "common.cuh"

namespace cvmm {

// "Row-gathered" grouped GEMM: the forward pass and grad-input.
// For sorted position p of expert e:
//   acc_p[n] = sum_k op(A[a_row(p)][k]) * op(B_e[k][n]),   a_row(p) = a_index[p] / a_div
//   mode 0: C[c_index[p]][n] = cast(acc_p[n])
//   mode 1: C[c_index[p]][n] = cast(op(op(acc_p[n]) * op(w[c_index[p]])))
//           gsel[c_index[p]] += sum_n op(acc_p[n]) * x[c_index[p]][n]
struct RowGemm {
  const void* a; int a_dtype; int64_t a_ld; int64_t a_rows;  // a_rows: bound on indexed rows
  const int64_t* a_index; int64_t a_div;
  const void* b; int b_dtype; int64_t bs_e, bs_k, bs_n;
  void* c; int c_dtype; int64_t c_ld;
  const int64_t* c_index;
  const int64_t* offsets;
  int64_t n_routes, n_experts, K, N;
  int mode;
  const void* w; int w_dtype;
  const void* x; int x_dtype; int64_t x_ld;
  int64_t x_div;       // mode 1: route p's x row is c_index[p] / x_div (1, or the routes sharing one row)
  float* gsel;
  int op_dtype;
  const int4* tiles;   // (expert, first sorted position, rows, tile index) per M tile; with
                       // 128-row tiles, tile t covers rows 128 t .. 128 t + 127 of the
                       // expert-padded sorted layout
  void* a_copy;        // non-null: also write the op-dtype A tiles there (expert-padded sorted layout)
  const int* a_pad_start;  // non-null: A is the expert-padded sorted layout (row = pad_start[e] + p - seg_begin(e))
  const int* c_pad_start;  // non-null: C is the expert-padded sorted layout (16-bit, mode 0; c_index unused)
  const int* n_tiles;  // number of valid entries in `tiles`
  int act;             // mode 0 only, 0 = none; 1 = GELU: c2[row] = op(acc) (the pre-activation, kept for
  void* c2;            // the backward) and c[row] = cast(gelu(op(acc))), the up-projection + F.gelu of
                       // the sigma-MoE layer in one epilogue (erf form, fp32 math on the rounded value)
};

// GELU of the reference's F.gelu (approximate = 'none'): 0.5 x (1 + erf(x / sqrt 2)),
// evaluated in fp32 on an op-dtype value, in that operation order.
__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

// d gelu / dx = Phi(x) + x phi(x), Phi the normal CDF, phi its density.
__device__ __forceinline__ float gelu_erf_grad(float x) {
  const float cdf = 0.5f * (1.0f + erff(x * 0.70710678118654752f));
  const float pdf = expf(-0.5f * x * x) * 0.39894228040143268f;
  return cdf + x * pdf;
}

// Per-expert segment reduction: grad-weight.
//   out[e][m][n] = sum_{p in seg(e)} op(X[x_row(p)][m]) * G'_p[n]
//   G'_p[n] = op(G[g_row(p)][n])                       (w == nullptr)
//           = op(op(G[g_row(p)][n]) * op(w[w_index[p]])) (weighted)
struct SegGemm {
  const void* x; int x_dtype; int64_t x_ld; const int64_t* x_index; int64_t x_div;
  const void* g; int g_dtype; int64_t g_ld; const int64_t* g_index; int64_t g_div;
  const void* w; int w_dtype; const int64_t* w_index;
  const int64_t* offsets;
  int64_t n_routes, n_experts, M, N;
  float* out;
  int op_dtype;
  int64_t chunk;        // routes per work unit (split-K)
  const int4* units;    // (expert, first sorted position, partial slot or -1, end position);
                        // nullptr: the tensor-core kernel builds the list in shared memory
  const int* n_units;
  int2* expert_slots;   // written by CTA 0 when the kernel builds its own unit list
  float* partials;      // [slots][M][N] partial sums of split experts
  // Per sorted route, resolved before the GEMM (tensor-core path): x row,
  // grad row (int32) and op-rounded route weight (fp32); padded by
  // kRouteRowsPad entries so 16-byte-aligned bulk copies may run past the end.
  const int* x_pad_start;  // non-null: x is the expert-padded sorted layout
  const int* g_pad_start;  // non-null: g is the expert-padded sorted layout
  const int* xrow;
  const int* grow;
  const float* wsc;
};

constexpr int64_t kRouteRowsPad = 128;
// Rows each expert segment of the expert-padded sorted layout is padded to.
constexpr int64_t kPadRows = CVMM_PAD_ROWS;
// Experts up to which the tensor-core row GEMM builds its tile table in the
// kernel (RowGemm::tiles == nullptr) instead of reading one from build_tiles.
constexpr int64_t kRowPlanExperts = 1024;
// The tensor-core grad-W builds its unit list in shared memory (no
// build_units launch) for at most this many experts and units.
constexpr int64_t kOwnUnitExperts = 128;
constexpr int64_t kOwnUnits = 384;
int pad_starts(const int64_t* offsets, int64_t n_experts, int64_t pad, int* pad_start, cudaStream_t stream);
int sort_rows_padded(const void* src, int src_dtype, int64_t src_ld, const int64_t* index, int64_t div,
                     const void* scale, int scale_dtype, const int32_t* sorted_sel, const int64_t* offsets,
                     const int* pad_start, int64_t n_routes, int64_t n_experts, int64_t cols, void* dst,
                     int dst_dtype, cudaStream_t stream, int32_t* route_rows = nullptr);
int resolve_route_rows(const SegGemm& p, int* xrow, int* grow, float* wsc, cudaStream_t stream);

__device__ __forceinline__ int64_t seg_begin(const int64_t* offsets, int64_t e) {
  return e > 0 ? offsets[e - 1] : 0;
}

// Upper bound of the number of M tiles of height bm over all expert segments.
inline int64_t max_row_tiles(int64_t n_routes, int64_t n_experts, int bm) {
  return (n_routes + bm - 1) / bm + n_experts;
}

// Host launchers (return a CVMM status).
int build_tiles(const int64_t* offsets, int64_t n_experts, int bm, int4* tiles, int* n_tiles,
                cudaStream_t stream);
int build_units(const int64_t* offsets, int64_t n_experts, int64_t chunk, int4* units, int* n_units,
                int2* expert_slots, cudaStream_t stream);
int seg_reduce(const int2* expert_slots, const float* partials, float* out, int64_t n_experts, int64_t mn,
               cudaStream_t stream);
int launch_row_gemm_simt(const RowGemm& p, int64_t max_tiles, cudaStream_t stream);
int launch_seg_gemm_simt(const SegGemm& p, int64_t max_units, cudaStream_t stream);
int launch_row_gemm_umma(const RowGemm& p, int64_t max_tiles, cudaStream_t stream);
int launch_seg_gemm_umma(const SegGemm& p, int64_t max_units, cudaStream_t stream);

}  // namespace cvmm
