// extern "C" entry points of libcvmm_sm100.so (declared in include/cvmm_sm100.h),
// argument validation, engine selection and the small memory-bound kernels
// (weighted combine, top-k sums, token-input weighted backward tail, casts).
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "gemm.cuh"
#include "launch.h"
#include "ptx.cuh"

namespace cvmm {

static thread_local char t_err[512];

int fail(int code, const char* msg) {
  snprintf(t_err, sizeof(t_err), "%s", msg);
  return code;
}

int fail_cuda(const char* where) {
  cudaError_t e = cudaGetLastError();
  snprintf(t_err, sizeof(t_err), "%s: %s", where, cudaGetErrorString(e));
  return CVMM_ERR_LAUNCH;
}

static std::atomic<int> g_pdl{-1};  // -1: not read from the environment yet

bool pdl_enabled() {
  int v = g_pdl.load(std::memory_order_relaxed);
  if (v < 0) {
    const char* ev = getenv("CVMM_B200_PDL");
    int want = (ev && ev[0] == '0') ? 0 : 1;
    int expected = -1;
    g_pdl.compare_exchange_strong(expected, want);
    v = g_pdl.load(std::memory_order_relaxed);
  }
  return v != 0;
}

int check_launch(const char* where) {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return CVMM_OK;
  snprintf(t_err, sizeof(t_err), "%s: %s", where, cudaGetErrorString(e));
  return CVMM_ERR_LAUNCH;
}

// ------------------------------------------------------------------ small kernels
// out[t][n] = sum_j wj * src[row(t*k + j)][n], wj = round(w[t*k+j], src dtype)
// or 1, row(r) = rows[r] (expert-padded sorted source) or r. One thread per 8
// consecutive columns of one token; VEC: 16-bit rows read and written with
// 16-byte accesses, up to kCombineBatch route rows in flight per thread.
// Routes are added in ascending j (the reference's sum / bmm order).
constexpr int kCombineBatch = 4;

template <bool VEC>
__global__ void __launch_bounds__(256) combine_kernel(const void* __restrict__ src, int s_dtype,
                                                      const void* __restrict__ w, int w_dtype,
                                                      const int32_t* __restrict__ rows, void* __restrict__ out,
                                                      int o_dtype, int64_t T, int64_t k, int64_t N) {
  pdl_enter();
  const int64_t groups = (N + 7) / 8;
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= T * groups) return;
  const int64_t t = i / groups, n0 = (i - t * groups) * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int64_t j0 = 0; j0 < k; j0 += kCombineBatch) {
    if (VEC) {
      uint4 q[kCombineBatch];
      float wj[kCombineBatch];
#pragma unroll
      for (int u = 0; u < kCombineBatch; ++u) {
        const int64_t j = j0 + u;
        if (j < k) {
          const int64_t r = t * k + j;
          const int64_t row = rows ? rows[r] : r;
          q[u] = *reinterpret_cast<const uint4*>(static_cast<const char*>(src) + (row * N + n0) * 2);
        }
      }
      // weights after the row loads are issued (see combine_vec_kernel)
#pragma unroll
      for (int u = 0; u < kCombineBatch; ++u)
        wj[u] = (w && j0 + u < k) ? round_to(load_as_float(w, w_dtype, t * k + j0 + u), s_dtype) : 1.f;
#pragma unroll
      for (int u = 0; u < kCombineBatch; ++u) {
        if (j0 + u >= k) break;
        const uint32_t wd[4] = {q[u].x, q[u].y, q[u].z, q[u].w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          acc[2 * c] = fmaf(wj[u], bits_to_float((uint16_t)(wd[c] & 0xffffu), s_dtype), acc[2 * c]);
          acc[2 * c + 1] = fmaf(wj[u], bits_to_float((uint16_t)(wd[c] >> 16), s_dtype), acc[2 * c + 1]);
        }
      }
    } else {
      for (int64_t j = j0; j < k && j < j0 + kCombineBatch; ++j) {
        const int64_t r = t * k + j;
        const int64_t row = rows ? rows[r] : r;
        const float wj = w ? round_to(load_as_float(w, w_dtype, r), s_dtype) : 1.f;
        for (int c = 0; c < 8 && n0 + c < N; ++c) acc[c] = fmaf(wj, load_as_float(src, s_dtype, row * N + n0 + c), acc[c]);
      }
    }
  }
  if (VEC) {
    uint32_t wd[4];
#pragma unroll
    for (int c = 0; c < 4; ++c)
      wd[c] = pack2(acc[2 * c], acc[2 * c + 1], o_dtype);
    *reinterpret_cast<uint4*>(static_cast<char*>(out) + (t * N + n0) * 2) = make_uint4(wd[0], wd[1], wd[2], wd[3]);
  } else {
    for (int c = 0; c < 8 && n0 + c < N; ++c) store_from_float(out, o_dtype, t * N + n0 + c, acc[c]);
  }
}

// 16-bit rows, 16-byte accesses: one thread per CPT chunks of 8 columns of
// one token (chunks sub, sub + tpt, ... so consecutive lanes read consecutive
// 16 bytes), with the route rows of up to kVecRoutes routes times CPT chunks
// (8 x 16 bytes) in flight per thread, and at most 85 registers per thread so
// that 3 CTAs (24 warps) share an SM: a CTA-per-SM occupancy of 1 (CPT = 4,
// 141 registers) measured 2.1 TB/s, latency-bound. Same arithmetic and route
// order as combine_kernel, so the results are bit-identical.
constexpr int kVecRoutes = 4;

template <int CPT>
__global__ void __launch_bounds__(256, 3) combine_vec_kernel(const uint4* __restrict__ src, int s_dtype,
                                                          const void* __restrict__ w, int w_dtype,
                                                          const int32_t* __restrict__ rows, uint4* __restrict__ out,
                                                          int o_dtype, int64_t T, int64_t k, int64_t groups) {
  pdl_enter();
  const int64_t tpt = groups / CPT;  // threads per token
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= T * tpt) return;
  const int64_t t = i / tpt, sub = i - t * tpt;
  float acc[CPT][8];
#pragma unroll
  for (int c = 0; c < CPT; ++c)
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[c][e] = 0.f;
  for (int64_t j0 = 0; j0 < k; j0 += kVecRoutes) {
    uint4 q[kVecRoutes][CPT];
    float wj[kVecRoutes];
    // Row loads first, then the weights: the weight conversion branches on
    // the dtype, and a load inside that branch followed by its rounding made
    // every route wait for its weight before its row loads were issued
    // (weighted combine 54 us against 40 us for the plain k-sum). A
    // grid-stride variant that prefetched the next token's row indices
    // measured slower (46-52 us) than this one-item-per-thread form.
#pragma unroll
    for (int u = 0; u < kVecRoutes; ++u) {
      const int64_t j = j0 + u;
      if (j < k) {
        const int64_t r = t * k + j;
        const int64_t row = rows ? rows[r] : r;
#pragma unroll
        for (int c = 0; c < CPT; ++c) q[u][c] = src[row * groups + sub + c * tpt];
      }
    }
    if (w) {
      if (w_dtype == F32) {
#pragma unroll
        for (int u = 0; u < kVecRoutes; ++u)
          wj[u] = j0 + u < k ? static_cast<const float*>(w)[t * k + j0 + u] : 0.f;
      } else {
#pragma unroll
        for (int u = 0; u < kVecRoutes; ++u) wj[u] = j0 + u < k ? load_as_float(w, w_dtype, t * k + j0 + u) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < kVecRoutes; ++u) wj[u] = round_to(wj[u], s_dtype);
    } else {
#pragma unroll
      for (int u = 0; u < kVecRoutes; ++u) wj[u] = 1.f;
    }
#pragma unroll
    for (int u = 0; u < kVecRoutes; ++u) {
      if (j0 + u >= k) break;
#pragma unroll
      for (int c = 0; c < CPT; ++c) {
        const uint32_t wd[4] = {q[u][c].x, q[u][c].y, q[u][c].z, q[u][c].w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          acc[c][2 * h] = fmaf(wj[u], bits_to_float((uint16_t)(wd[h] & 0xffffu), s_dtype), acc[c][2 * h]);
          acc[c][2 * h + 1] = fmaf(wj[u], bits_to_float((uint16_t)(wd[h] >> 16), s_dtype), acc[c][2 * h + 1]);
        }
      }
    }
  }
#pragma unroll
  for (int c = 0; c < CPT; ++c) {
    uint32_t wd[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) wd[h] = pack2(acc[c][2 * h], acc[c][2 * h + 1], o_dtype);
    out[t * groups + sub + c * tpt] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
  }
}

// dz = dh * gelu'(z), fp32 math on the 16-bit values, rounded once (the
// elementwise backward of F.gelu that follows the down projection's grad-x).
__global__ void __launch_bounds__(256) gelu_backward_kernel(const void* __restrict__ grad, const void* __restrict__ z,
                                                            void* __restrict__ out, int dtype, int64_t n, bool vec) {
  pdl_enter();
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  if (vec) {
    const uint4* g4 = static_cast<const uint4*>(grad);
    const uint4* z4 = static_cast<const uint4*>(z);
    uint4* o4 = static_cast<uint4*>(out);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n / 8; i += stride) {
      const uint4 gv = g4[i], zv = z4[i];
      const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, zw[4] = {zv.x, zv.y, zv.z, zv.w};
      uint32_t ow[4];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float lo = bits_to_float((uint16_t)(gw[h] & 0xffffu), dtype) *
                         gelu_erf_grad(bits_to_float((uint16_t)(zw[h] & 0xffffu), dtype));
        const float hi = bits_to_float((uint16_t)(gw[h] >> 16), dtype) *
                         gelu_erf_grad(bits_to_float((uint16_t)(zw[h] >> 16), dtype));
        ow[h] = pack2(lo, hi, dtype);
      }
      o4[i] = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    }
    return;
  }
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    store_from_float(out, dtype, i, load_as_float(grad, dtype, i) * gelu_erf_grad(load_as_float(z, dtype, i)));
}

// Router of the sigma-MoE layer (the caller of CVMM, benchmark_ffn_moe.py:89-92):
// probs = softmax(float(logits)); (w, sel) = top-k(probs) in descending order;
// w /= max(sum(w), 1e-20) when renormalize. One warp per token, the token's
// logits held in registers (n_experts <= 1024: 32 per lane); the top-k are k
// rounds of a warp arg-max (ties to the lower expert id).
constexpr int kRouterMaxExperts = 1024;

__global__ void __launch_bounds__(256) router_topk_kernel(const void* __restrict__ logits, int dtype, int64_t T,
                                                          int64_t E, int64_t k, int renorm,
                                                          int64_t* __restrict__ sel, float* __restrict__ weights) {
  pdl_enter();
  constexpr int kPer = kRouterMaxExperts / 32;
  const int lane = threadIdx.x & 31;
  const int64_t t = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (t >= T) return;
  float v[kPer];
  float mx = -INFINITY;
#pragma unroll
  for (int q = 0; q < kPer; ++q) {
    const int64_t e = lane + 32 * q;
    v[q] = e < E ? load_as_float(logits, dtype, t * E + e) : -INFINITY;
    mx = fmaxf(mx, v[q]);
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int q = 0; q < kPer; ++q) {
    v[q] = (lane + 32 * q) < E ? expf(v[q] - mx) : 0.f;
    sum += v[q];
  }
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
  for (int q = 0; q < kPer; ++q) v[q] = (lane + 32 * q) < E ? v[q] / sum : -1.f;
  float mine = 0.f;  // lane j < k keeps the j-th selected probability
  int64_t my_e = 0;
  float tot = 0.f;
  for (int j = 0; j < (int)k; ++j) {
    float bv = -2.f;
    int be = 0x7fffffff;
#pragma unroll
    for (int q = 0; q < kPer; ++q)
      if (v[q] > bv) {
        bv = v[q];
        be = lane + 32 * q;
      }
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
#pragma unroll
    for (int q = 0; q < kPer; ++q)
      if (lane + 32 * q == be) v[q] = -1.f;  // remove the winner (only its lane holds it)
    if (lane == j) {
      mine = bv;
      my_e = be;
    }
    tot += bv;
  }
  if (lane < k) {
    sel[t * k + lane] = my_e;
    weights[t * k + lane] = renorm ? mine / fmaxf(tot, 1e-20f) : mine;
  }
}

// Self-test of the bounded-wait path every persistent kernel relies on: one
// thread waits on an mbarrier that nothing ever arrives on, through the same
// bounded wait as the GEMM roles, so the wait runs out after `limit_ns`, the
// status word records CVMM_DEV_TIMEOUT at kSelfTestTag and the kernel returns.
constexpr int kSelfTestTag = 99;

__global__ void wait_timeout_selftest_kernel(uint64_t limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    ptx::mbar_init(&bar, 1);
    abort_flag = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) ptx::mbar_wait_or_abort(&bar, 0, kSelfTestTag, &abort_flag, limit_ns);
}

// rows[route[v]] = pad_start[e] + v - seg_begin(e) for every sorted position v.
__global__ void padded_route_rows_kernel(const int64_t* __restrict__ route, const int32_t* __restrict__ sorted_sel,
                                         const int64_t* __restrict__ offsets, const int32_t* __restrict__ pad_start,
                                         int64_t n_routes, int32_t* __restrict__ rows) {
  pdl_enter();
  const int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (v >= n_routes) return;
  const int64_t e = sorted_sel[v];
  rows[route[v]] = (int32_t)(pad_start[e] + v - seg_begin(offsets, e));
}

// One CTA per token: grad_x[t] = sum_j w'[t,j] rg[t,j,:],  gsel[t,j] = <rg[t,j,:], x[t,:]>.
__global__ void weighted_token_bwd_kernel(const void* __restrict__ rg, int rg_dtype,
                                          const void* __restrict__ w, int w_dtype,
                                          const void* __restrict__ x, int x_dtype,
                                          void* __restrict__ gx, int gx_dtype,
                                          float* __restrict__ gsel, int64_t k, int64_t d) {
  pdl_enter();
  const int64_t t = blockIdx.x;
  extern __shared__ float red[];  // [blockDim.x / 32]
  for (int64_t j = 0; j < k; ++j) {
    if (!gsel) break;
    float part = 0.f;
    for (int64_t c = threadIdx.x; c < d; c += blockDim.x)
      part = fmaf(load_as_float(rg, rg_dtype, (t * k + j) * d + c), load_as_float(x, x_dtype, t * d + c), part);
    for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = part;
    __syncthreads();
    if (threadIdx.x == 0) {
      float s = 0.f;
      for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
      gsel[t * k + j] = s;
    }
    __syncthreads();
  }
  if (!gx) return;
  for (int64_t c = threadIdx.x; c < d; c += blockDim.x) {
    float acc = 0.f;
    for (int64_t j = 0; j < k; ++j) {
      const float wj = round_to(load_as_float(w, w_dtype, t * k + j), rg_dtype);
      acc = fmaf(wj, load_as_float(rg, rg_dtype, (t * k + j) * d + c), acc);
    }
    store_from_float(gx, gx_dtype, t * d + c, acc);
  }
}

__global__ void cast_kernel(const void* __restrict__ src, int s_dtype, void* __restrict__ dst,
                            int d_dtype, int64_t n) {
  pdl_enter();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    store_from_float(dst, d_dtype, i, load_as_float(src, s_dtype, i));
}

// fp32 -> bf16/fp16, two groups of 8 elements per thread (a block's groups
// are blockDim.x apart, so every warp access stays coalesced): four 16-byte
// loads in flight per thread before the two 16-byte stores.
__global__ void cast_f32_to_16_vec(const float4* __restrict__ src, uint4* __restrict__ dst,
                                   int d_dtype, int64_t n8) {
  pdl_enter();
  for (int64_t i = blockIdx.x * 2 * (int64_t)blockDim.x + threadIdx.x; i < n8;
       i += (int64_t)gridDim.x * 2 * blockDim.x) {
    const int64_t j = i + blockDim.x;
    const bool two = j < n8;
    const float4 a = src[2 * i], b = src[2 * i + 1];
    float4 c = a, d = b;
    if (two) {
      c = src[2 * j];
      d = src[2 * j + 1];
    }
    uint4 o;
    o.x = pack2(a.x, a.y, d_dtype);
    o.y = pack2(a.z, a.w, d_dtype);
    o.z = pack2(b.x, b.y, d_dtype);
    o.w = pack2(b.z, b.w, d_dtype);
    dst[i] = o;
    if (two) {
      o.x = pack2(c.x, c.y, d_dtype);
      o.y = pack2(c.z, c.w, d_dtype);
      o.z = pack2(d.x, d.y, d_dtype);
      o.w = pack2(d.z, d.w, d_dtype);
      dst[j] = o;
    }
  }
}

// The same cast with its first loads ahead of the previous kernel on the
// stream: every thread loads its first kCastAhead groups of 8 fp32 values
// into registers, then waits for the predecessor (pdl_wait) and only then
// converts and stores. Reads of src may overlap the predecessor because no
// kernel of this library writes src; writes wait, because dst may reuse
// memory the predecessor still uses (stream-ordered allocation). Groups a
// block touches are blockDim.x apart, so warp accesses stay coalesced.
constexpr int kCastAhead = 4;
__global__ void __launch_bounds__(256) cast_f32_to_16_ahead(const float4* __restrict__ src,
                                                            uint4* __restrict__ dst, int d_dtype, int64_t n8) {
  pdl_trigger();
  const int64_t step = (int64_t)gridDim.x * blockDim.x * kCastAhead;
  bool waited = false;
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x * kCastAhead + threadIdx.x; base < n8; base += step) {
    float4 v[kCastAhead][2];
#pragma unroll
    for (int g = 0; g < kCastAhead; ++g) {
      const int64_t i = base + (int64_t)g * blockDim.x;
      if (i < n8) {
        v[g][0] = src[2 * i];
        v[g][1] = src[2 * i + 1];
      }
    }
    if (!waited) {
      pdl_wait();
      waited = true;
    }
#pragma unroll
    for (int g = 0; g < kCastAhead; ++g) {
      const int64_t i = base + (int64_t)g * blockDim.x;
      if (i < n8) {
        uint4 o;
        o.x = pack2(v[g][0].x, v[g][0].y, d_dtype);
        o.y = pack2(v[g][0].z, v[g][0].w, d_dtype);
        o.z = pack2(v[g][1].x, v[g][1].y, d_dtype);
        o.w = pack2(v[g][1].z, v[g][1].w, d_dtype);
        dst[i] = o;
      }
    }
  }
  if (!waited) pdl_wait();
}

static inline int grid_for(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  return (int)std::max<int64_t>(1, std::min<int64_t>(g, 148 * 16));
}

static inline bool al16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// ------------------------------------------------------------------ GEMM plumbing
// Workspace layout shared by the GEMM entry points:
//   [0, 256)           tile / unit count
//   tiles or units     int4 x max_row_tiles(n_routes, n_experts, 64)
//   expert_slots       int2 x n_experts                 (grad-W only)
//   partials           fp32 x max_slots x m_dim x n_dim (grad-W only)
struct GemmWs {
  int* count;
  void* tiles;
  int2* expert_slots;
  float* partials;
};

static size_t table_bytes(int64_t n_routes, int64_t n_experts) {
  return 256 + align_up((size_t)max_row_tiles(n_routes, n_experts, 64) * sizeof(int4), 256);
}

// Split-K chunk of the grad-W units (routes per unit): no split when the
// expert tiles alone fill the GPU several times; otherwise 1024 routes (16
// tensor-core stages), halved while the grid would not fill two CTAs per SM,
// and doubled while the partial slots would exceed 256 MiB.
static int64_t segw_chunk(int64_t n_routes, int64_t n_experts, int64_t m_dim, int64_t n_dim, bool tensor) {
  const int64_t mt = (m_dim + (tensor ? 127 : 63)) / (tensor ? 128 : 64);
  const int64_t nt = (n_dim + (tensor ? 255 : 63)) / (tensor ? 256 : 64);
  if (n_experts * mt * nt >= 8 * 148) return std::max<int64_t>(64, (n_routes + 63) / 64 * 64);
  // Experts longer than `chunk` routes are split into partial slots that
  // seg_reduce adds. Units run longest first over the SMs, so a unit only has
  // to be short next to one SM's share of the work (n_routes * mt * nt / 148
  // route-tiles): chunks of at least half that share keep the SMs balanced
  // while splitting only the heavy experts (at ff_up_1024, 2048 instead of
  // 1024 routes, which split about half of the 64 experts).
  int64_t chunk = 1024;
  while (chunk < 8192 && chunk * 2 <= n_routes * mt * nt / 148) chunk *= 2;
  // Tuning override (routes per split-K chunk, a multiple of 64) for measurements.
  if (const char* ev = getenv("CVMM_B200_GRADW_CHUNK")) {
    const long long v = atoll(ev);
    if (v >= 64 && v % 64 == 0) return v;
  }
  // ... but at least one unit tile per SM (every expert is at least one unit).
  while (chunk > 128 && std::max<int64_t>(n_experts, n_routes / chunk) * mt * nt < 148) chunk /= 2;
  while (2 * ((n_routes + chunk - 1) / chunk) * m_dim * n_dim * 4 > ((int64_t)256 << 20)) chunk *= 2;
  return chunk;
}

static int64_t segw_max_slots(int64_t n_routes, int64_t chunk) { return 2 * ((n_routes + chunk - 1) / chunk); }

static size_t segw_ws_bytes(int64_t n_routes, int64_t n_experts, int64_t m_dim, int64_t n_dim, bool tensor) {
  const int64_t chunk = segw_chunk(n_routes, n_experts, m_dim, n_dim, tensor);
  return table_bytes(n_routes, n_experts) + align_up((size_t)n_experts * sizeof(int2), 256) +
         align_up((size_t)segw_max_slots(n_routes, chunk) * m_dim * n_dim * sizeof(float), 256) +
         3 * align_up((size_t)(n_routes + kRouteRowsPad) * 4, 256);
}

static int carve_ws(void* ws, size_t bytes, size_t need, int64_t n_routes, int64_t n_experts, GemmWs* out,
                    const char* who) {
  if (!ws || bytes < need) {
    snprintf(t_err, sizeof(t_err), "%s: workspace too small (need %zu bytes)", who, need);
    return CVMM_ERR_WORKSPACE;
  }
  char* b = static_cast<char*>(ws);
  out->count = reinterpret_cast<int*>(b);
  out->tiles = b + 256;
  b += table_bytes(n_routes, n_experts);
  out->expert_slots = reinterpret_cast<int2*>(b);
  b += align_up((size_t)n_experts * sizeof(int2), 256);
  out->partials = reinterpret_cast<float*>(b);
  return CVMM_OK;
}

static int run_row_gemm(RowGemm& p, void* ws, size_t ws_bytes, cudaStream_t stream, const char* who) {
  GemmWs g;
  int rc = carve_ws(ws, ws_bytes, table_bytes(p.n_routes, p.n_experts), p.n_routes, p.n_experts, &g, who);
  if (rc) return rc;
  const bool tensor = p.op_dtype != F32;
  const int bm = tensor ? 128 : 64;
  if (tensor && p.n_experts <= kRowPlanExperts) {
    // The tensor-core kernel derives its tile table from the offsets itself.
    p.tiles = nullptr;
    p.n_tiles = nullptr;
  } else {
    int4* tiles = static_cast<int4*>(g.tiles);
    rc = build_tiles(p.offsets, p.n_experts, bm, tiles, g.count, stream);
    if (rc) return rc;
    p.tiles = tiles;
    p.n_tiles = g.count;
  }
  const int64_t max_tiles = max_row_tiles(p.n_routes, p.n_experts, bm);
  return tensor ? launch_row_gemm_umma(p, max_tiles, stream) : launch_row_gemm_simt(p, max_tiles, stream);
}

}  // namespace cvmm

using namespace cvmm;

// ================================================================== C ABI
extern "C" {

int cvmm_abi_version(void) { return 10; }

int cvmm_set_pdl(int enable) {
  const int prev = pdl_enabled() ? 1 : 0;
  g_pdl.store(enable ? 1 : 0);
  return prev;
}

int cvmm_set_sm_limit(int n_sms) {
  if (n_sms < 0) return fail(CVMM_ERR_INVALID_ARG, "cvmm_set_sm_limit: n_sms must be >= 0");
  return g_sm_limit.exchange(n_sms);
}

const char* cvmm_last_error(void) { return t_err; }

int cvmm_device_status(int reset, int* where, long long* aux, cvmm_stream_t stream) {
  DeviceStatus st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemcpyFromSymbolAsync(&st, g_status, sizeof(st), 0, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return fail_cuda("cvmm_device_status");
  if (where) *where = st.where;
  if (aux) *aux = st.aux;
  if (reset) {
    DeviceStatus z = {0, 0, 0};
    if (cudaMemcpyToSymbolAsync(g_status, &z, sizeof(z), 0, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
      return fail_cuda("cvmm_device_status(reset)");
  }
  return st.code;
}

size_t cvmm_sel_prepare_workspace_size(int64_t n_routes) {
  return sel_prepare_workspace_size(n_routes < 0 ? 0 : n_routes);
}

int cvmm_sel_prepare(const void* sel, int sel_dtype, int64_t n_routes, int64_t top_k,
                     int route_input, int32_t* raw_sel, int32_t* sorted_sel, int64_t* sel_index,
                     int64_t* out_index, void* workspace, size_t workspace_bytes,
                     cvmm_stream_t stream) {
  // Tuning override (fewest routes per sort CTA) for measurements. It can
  // only raise the default, so the workspace sized for the default suffices.
  int64_t min_chunk = kSelMinChunk;
  if (const char* ev = getenv("CVMM_B200_SEL_MIN_CHUNK")) min_chunk = std::max<int64_t>(kSelMinChunk, atoll(ev));
  return sel_prepare(sel, sel_dtype, n_routes, top_k, route_input, raw_sel, sorted_sel, sel_index,
                     out_index, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream), min_chunk);
}

int cvmm_expert_offsets(const int32_t* sorted_sel, int64_t n_routes, int64_t n_experts,
                        int64_t* offsets, cvmm_stream_t stream) {
  return expert_offsets(sorted_sel, n_routes, n_experts, offsets, reinterpret_cast<cudaStream_t>(stream));
}

size_t cvmm_gemm_workspace_size(int64_t n_routes, int64_t n_experts, int64_t k_dim, int64_t n_dim,
                                int x_dtype, int keys_dtype, int op_dtype, int64_t x_rows) {
  (void)x_dtype; (void)keys_dtype; (void)x_rows;
  n_routes = n_routes < 0 ? 0 : n_routes;
  n_experts = n_experts < 1 ? 1 : n_experts;
  size_t b = table_bytes(n_routes, n_experts);
  if (k_dim > 0 && n_dim > 0)
    b = std::max(b, segw_ws_bytes(n_routes, n_experts, k_dim, n_dim, op_dtype != CVMM_F32));
  return b;
}

int cvmm_forward(const void* x, int x_dtype, int64_t x_rows, int64_t x_ld, const int64_t* sel_index,
                 const int64_t* out_index, const int64_t* offsets, int64_t n_routes,
                 const void* keys, int keys_dtype, int64_t n_experts, int64_t k_dim, int64_t n_dim,
                 int64_t ks_e, int64_t ks_k, int64_t ks_n, void* out, int out_dtype, int64_t out_ld,
                 int op_dtype, const int32_t* x_pad_start, const int32_t* out_pad_start, void* x_copy,
                 void* workspace, size_t workspace_bytes, cvmm_stream_t stream) {
  if (!is_float_dtype(x_dtype) || !is_float_dtype(keys_dtype) || !is_float_dtype(out_dtype) ||
      !is_float_dtype(op_dtype))
    return fail(CVMM_ERR_UNSUPPORTED_DTYPE, "cvmm_forward: unsupported dtype");
  if (x_pad_start && (op_dtype == F32 || x_dtype != op_dtype))
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_forward: the padded sorted layout needs x_dtype == op_dtype (bf16/fp16)");
  if (out_pad_start && op_dtype == F32)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_forward: a padded sorted output needs a bf16/fp16 op_dtype");
  if (x_copy && (op_dtype == F32 || x_pad_start))
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_forward: x_copy needs a bf16/fp16 op_dtype and a row-indexed x");
  if (n_routes < 0 || n_experts <= 0 || k_dim < 0 || n_dim <= 0 || x_rows < 0 || x_ld < k_dim ||
      out_ld < n_dim)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_forward: bad sizes");
  if (n_routes == 0) return CVMM_OK;
  if (n_routes > (int64_t)INT32_MAX || x_rows > (int64_t)INT32_MAX)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_forward: more than 2^31 routes or rows");
  if (!x || !sel_index || !offsets || !keys || !out)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_forward: null pointer");
  RowGemm p = {};
  p.a = x; p.a_dtype = x_dtype; p.a_ld = x_ld; p.a_rows = x_pad_start ? n_routes + n_experts * kPadRows : x_rows;
  p.a_index = sel_index; p.a_div = 1; p.a_pad_start = x_pad_start;
  p.b = keys; p.b_dtype = keys_dtype; p.bs_e = ks_e; p.bs_k = ks_k; p.bs_n = ks_n;
  p.c = out; p.c_dtype = out_dtype; p.c_ld = out_ld; p.c_index = out_index ? out_index : sel_index;
  p.c_pad_start = out_pad_start;
  p.a_copy = x_copy;
  p.offsets = offsets; p.n_routes = n_routes; p.n_experts = n_experts; p.K = k_dim; p.N = n_dim;
  p.mode = 0; p.op_dtype = op_dtype;
  return run_row_gemm(p, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream), "cvmm_forward");
}

int cvmm_forward_gelu(const void* x, int x_dtype, int64_t x_rows, int64_t x_ld, const int64_t* sel_index,
                      const int64_t* out_index, const int64_t* offsets, int64_t n_routes, const void* keys,
                      int keys_dtype, int64_t n_experts, int64_t k_dim, int64_t n_dim, int64_t ks_e, int64_t ks_k,
                      int64_t ks_n, void* out, void* pre_act, int out_dtype, int64_t out_ld, int op_dtype,
                      void* x_copy, void* workspace, size_t workspace_bytes, cvmm_stream_t stream) {
  if (op_dtype == F32 || (out_dtype != BF16 && out_dtype != F16) || out_dtype != op_dtype)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_forward_gelu: needs a bf16/fp16 op_dtype and out_dtype == op_dtype");
  if (!pre_act) return fail(CVMM_ERR_INVALID_ARG, "cvmm_forward_gelu: null pre_act");
  if (!is_float_dtype(x_dtype) || !is_float_dtype(keys_dtype))
    return fail(CVMM_ERR_UNSUPPORTED_DTYPE, "cvmm_forward_gelu: unsupported dtype");
  if (n_routes < 0 || n_experts <= 0 || k_dim < 0 || n_dim <= 0 || x_rows < 0 || x_ld < k_dim || out_ld < n_dim)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_forward_gelu: bad sizes");
  if (n_routes == 0) return CVMM_OK;
  if (n_routes > (int64_t)INT32_MAX || x_rows > (int64_t)INT32_MAX)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_forward_gelu: more than 2^31 routes or rows");
  if (!x || !sel_index || !offsets || !keys || !out)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_forward_gelu: null pointer");
  RowGemm p = {};
  p.a = x; p.a_dtype = x_dtype; p.a_ld = x_ld; p.a_rows = x_rows;
  p.a_index = sel_index; p.a_div = 1;
  p.b = keys; p.b_dtype = keys_dtype; p.bs_e = ks_e; p.bs_k = ks_k; p.bs_n = ks_n;
  p.c = out; p.c_dtype = out_dtype; p.c_ld = out_ld; p.c_index = out_index ? out_index : sel_index;
  p.a_copy = x_copy;
  p.offsets = offsets; p.n_routes = n_routes; p.n_experts = n_experts; p.K = k_dim; p.N = n_dim;
  p.mode = 0; p.op_dtype = op_dtype; p.act = 1; p.c2 = pre_act;
  return run_row_gemm(p, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream), "cvmm_forward_gelu");
}

int cvmm_gelu_backward(const void* grad, const void* pre_act, void* grad_pre_act, int dtype, int64_t n,
                       cvmm_stream_t stream) {
  if (dtype != BF16 && dtype != F16) return fail(CVMM_ERR_UNSUPPORTED_DTYPE, "cvmm_gelu_backward: bf16/fp16 only");
  if (n < 0) return fail(CVMM_ERR_INVALID_ARG, "cvmm_gelu_backward: bad size");
  if (n == 0) return CVMM_OK;
  if (!grad || !pre_act || !grad_pre_act) return fail(CVMM_ERR_INVALID_ARG, "cvmm_gelu_backward: null pointer");
  const bool vec = n % 8 == 0 && al16(grad) && al16(pre_act) && al16(grad_pre_act);
  const int64_t items = vec ? n / 8 : n;
  const unsigned grid = (unsigned)std::min<int64_t>((items + 255) / 256, 148 * 16);
  launch(gelu_backward_kernel, grid, 256, 0, reinterpret_cast<cudaStream_t>(stream), grad, pre_act, grad_pre_act,
                                                                                dtype, n, vec);
  return check_launch("cvmm_gelu_backward");
}

int cvmm_router_topk(const void* logits, int logits_dtype, int64_t n_tokens, int64_t n_experts, int64_t top_k,
                     int renormalize, int64_t* sel, float* weights, cvmm_stream_t stream) {
  if (logits_dtype != F32 && logits_dtype != BF16 && logits_dtype != F16)
    return fail(CVMM_ERR_UNSUPPORTED_DTYPE, "cvmm_router_topk: unsupported logits dtype");
  if (n_tokens < 0 || n_experts <= 0 || n_experts > kRouterMaxExperts || top_k <= 0 || top_k > n_experts ||
      top_k > 32)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_router_topk: needs 1 <= top_k <= min(32, n_experts), n_experts <= 1024");
  if (n_tokens == 0) return CVMM_OK;
  if (!logits || !sel || !weights) return fail(CVMM_ERR_INVALID_ARG, "cvmm_router_topk: null pointer");
  const unsigned grid = (unsigned)((n_tokens + 7) / 8);
  launch(router_topk_kernel, grid, 256, 0, reinterpret_cast<cudaStream_t>(stream),
      logits, logits_dtype, n_tokens, n_experts, top_k, renormalize, sel, weights);
  return check_launch("cvmm_router_topk");
}

int cvmm_weighted_combine(const void* y, int y_dtype, const void* w, int w_dtype, void* out,
                          int out_dtype, int64_t n_tokens, int64_t top_k, int64_t n_dim,
                          const int32_t* y_rows, cvmm_stream_t stream) {
  if (!is_float_dtype(y_dtype) || (w && !is_float_dtype(w_dtype)) || !is_float_dtype(out_dtype))
    return fail(CVMM_ERR_UNSUPPORTED_DTYPE, "cvmm_weighted_combine: unsupported dtype");
  if (n_tokens < 0 || top_k <= 0 || n_dim <= 0)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_weighted_combine: bad sizes");
  if (n_tokens == 0) return CVMM_OK;
  if (!y || !out) return fail(CVMM_ERR_INVALID_ARG, "cvmm_weighted_combine: null pointer");
  const bool vec = n_dim % 8 == 0 && y_dtype != F32 && out_dtype != F32 && al16(y) && al16(out);
  const int64_t groups = (n_dim + 7) / 8;
  const int64_t work = n_tokens * groups;
  const unsigned grid = (unsigned)((work + 255) / 256);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (vec && groups % 2 == 0) {
    const unsigned g2 = (unsigned)((n_tokens * (groups / 2) + 255) / 256);
    launch(combine_vec_kernel<2>, g2, 256, 0, s, static_cast<const uint4*>(y), y_dtype, w, w_dtype, y_rows,
                                             static_cast<uint4*>(out), out_dtype, n_tokens, top_k, groups);
  } else if (vec)
    launch(combine_kernel<true>, grid, 256, 0, s, y, y_dtype, w, w_dtype, y_rows, out, out_dtype, n_tokens, top_k, n_dim);
  else
    launch(combine_kernel<false>, grid, 256, 0, s, y, y_dtype, w, w_dtype, y_rows, out, out_dtype, n_tokens, top_k, n_dim);
  return check_launch("cvmm_weighted_combine");
}

int cvmm_sum_routes(const void* src, int src_dtype, void* out, int out_dtype, int64_t n_tokens,
                    int64_t top_k, int64_t d, const int32_t* src_rows, cvmm_stream_t stream) {
  return cvmm_weighted_combine(src, src_dtype, nullptr, CVMM_F32, out, out_dtype, n_tokens, top_k, d, src_rows,
                               stream);
}

int cvmm_selftest_wait_timeout(int64_t limit_ns, cvmm_stream_t stream) {
  if (limit_ns < 1000 || limit_ns > 100000000)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_selftest_wait_timeout: limit must be in [1 us, 100 ms]");
  wait_timeout_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>((uint64_t)limit_ns);
  return check_launch("cvmm_selftest_wait_timeout");
}

int cvmm_padded_route_rows(const int64_t* route, const int32_t* sorted_sel, const int64_t* offsets,
                           const int32_t* pad_start, int64_t n_routes, int64_t n_experts, int32_t* rows,
                           cvmm_stream_t stream) {
  if (n_routes < 0 || n_experts <= 0 || n_routes + n_experts * kPadRows > (int64_t)INT32_MAX)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_padded_route_rows: bad sizes");
  if (n_routes == 0) return CVMM_OK;
  if (!route || !sorted_sel || !offsets || !pad_start || !rows)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_padded_route_rows: null pointer");
  launch(padded_route_rows_kernel, (unsigned)((n_routes + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream),
      route, sorted_sel, offsets, pad_start, n_routes, rows);
  return check_launch("cvmm_padded_route_rows");
}

int cvmm_backward_x(const void* g, int g_dtype, int64_t g_ld, const int64_t* g_index, int64_t g_div,
                    const int64_t* out_index, const int64_t* offsets, int64_t n_routes,
                    const void* keys, int keys_dtype, int64_t n_experts, int64_t k_dim, int64_t n_dim,
                    int64_t ks_e, int64_t ks_k, int64_t ks_n, void* out, int out_dtype, int64_t out_ld,
                    int mode, const void* w, int w_dtype, const void* x, int x_dtype, int64_t x_ld,
                    int64_t x_div, float* gsel, int op_dtype, const int32_t* g_pad_start,
                    const int32_t* out_pad_start, void* workspace, size_t workspace_bytes, cvmm_stream_t stream) {
  if (!is_float_dtype(g_dtype) || !is_float_dtype(keys_dtype) || !is_float_dtype(out_dtype) ||
      !is_float_dtype(op_dtype))
    return fail(CVMM_ERR_UNSUPPORTED_DTYPE, "cvmm_backward_x: unsupported dtype");
  if (mode != 0 && mode != 1) return fail(CVMM_ERR_INVALID_ARG, "cvmm_backward_x: mode must be 0 or 1");
  if (n_routes < 0 || n_experts <= 0 || k_dim <= 0 || n_dim < 0 || g_div <= 0 || g_ld < n_dim ||
      out_ld < k_dim)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_backward_x: bad sizes");
  if (n_routes == 0) return CVMM_OK;
  if (n_routes > (int64_t)INT32_MAX) return fail(CVMM_ERR_INVALID_ARG, "cvmm_backward_x: too many routes");
  if (!g || (!g_index && !g_pad_start) || (!out_index && !out_pad_start) || !offsets || !keys || !out)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_backward_x: null pointer");
  if (out_pad_start && (mode != 0 || op_dtype == F32))
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_backward_x: a padded sorted output needs mode 0 and a bf16/fp16 op_dtype");
  if (g_pad_start && op_dtype == F32)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_backward_x: the padded sorted gradient layout needs bf16/fp16 op_dtype");
  if (mode == 1 && (!w || !x || !gsel || !is_float_dtype(w_dtype) || !is_float_dtype(x_dtype) || x_ld < k_dim ||
                    x_div <= 0))
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_backward_x: mode 1 needs w, x and gsel");
  RowGemm p = {};
  // B_e[kk][nn] = keys[e][nn][kk]: contract over n_dim, produce k_dim columns.
  p.a = g; p.a_dtype = g_dtype; p.a_ld = g_ld; p.a_rows = g_pad_start ? n_routes + n_experts * kPadRows : n_routes;
  p.a_index = g_index; p.a_div = g_pad_start ? 1 : g_div;
  p.b = keys; p.b_dtype = keys_dtype; p.bs_e = ks_e; p.bs_k = ks_n; p.bs_n = ks_k;
  p.c = out; p.c_dtype = out_dtype; p.c_ld = out_ld; p.c_index = out_index;
  p.offsets = offsets; p.n_routes = n_routes; p.n_experts = n_experts; p.K = n_dim; p.N = k_dim;
  p.mode = mode; p.w = w; p.w_dtype = w_dtype; p.x = x; p.x_dtype = x_dtype; p.x_ld = x_ld;
  p.x_div = x_div > 0 ? x_div : 1;
  p.gsel = gsel; p.op_dtype = op_dtype; p.a_pad_start = g_pad_start; p.c_pad_start = out_pad_start;
  return run_row_gemm(p, workspace, workspace_bytes, reinterpret_cast<cudaStream_t>(stream), "cvmm_backward_x");
}

int cvmm_backward_w(const void* x, int x_dtype, int64_t x_ld, const int64_t* x_index, int64_t x_div,
                    const void* g, int g_dtype, int64_t g_ld, const int64_t* g_index, int64_t g_div,
                    const void* w, int w_dtype, const int64_t* w_index, const int64_t* offsets,
                    int64_t n_routes, int64_t n_experts, int64_t m_dim, int64_t n_dim, float* grad_w,
                    int op_dtype, const int32_t* x_pad_start, const int32_t* g_pad_start, void* workspace,
                    size_t workspace_bytes, cvmm_stream_t stream) {
  if (!is_float_dtype(x_dtype) || !is_float_dtype(g_dtype) || !is_float_dtype(op_dtype) ||
      (w && !is_float_dtype(w_dtype)))
    return fail(CVMM_ERR_UNSUPPORTED_DTYPE, "cvmm_backward_w: unsupported dtype");
  if (n_routes < 0 || n_experts <= 0 || m_dim <= 0 || n_dim <= 0 || x_div <= 0 || g_div <= 0 ||
      x_ld < m_dim || g_ld < n_dim || n_routes > (int64_t)INT32_MAX)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_backward_w: bad sizes");
  if (!grad_w || !offsets || (n_routes > 0 && (!x || !g || (!x_index && !x_pad_start) || (!g_index && !g_pad_start))) ||
      (w && !w_index))
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_backward_w: null pointer");
  if ((g_pad_start && (op_dtype == F32 || g_dtype != op_dtype)) || (x_pad_start && (op_dtype == F32 || x_dtype != op_dtype)))
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_backward_w: padded sorted operands need operand dtype == op_dtype (bf16/fp16)");
  if (n_experts > 65535) return fail(CVMM_ERR_INVALID_ARG, "cvmm_backward_w: too many experts");
  const bool tensor = op_dtype != F32;
  GemmWs ws;
  int rc = carve_ws(workspace, workspace_bytes, segw_ws_bytes(n_routes, n_experts, m_dim, n_dim, tensor),
                    n_routes, n_experts, &ws, "cvmm_backward_w");
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  SegGemm p = {};
  p.x = x; p.x_dtype = x_dtype; p.x_ld = x_ld; p.x_index = x_index; p.x_div = x_div;
  p.g = g; p.g_dtype = g_dtype; p.g_ld = g_ld; p.g_index = g_index; p.g_div = g_div;
  p.w = w; p.w_dtype = w_dtype; p.w_index = w_index;
  p.offsets = offsets; p.n_routes = n_routes; p.n_experts = n_experts; p.M = m_dim; p.N = n_dim;
  p.out = grad_w; p.op_dtype = op_dtype; p.x_pad_start = x_pad_start; p.g_pad_start = g_pad_start;
  p.chunk = segw_chunk(n_routes, n_experts, m_dim, n_dim, tensor);
  p.units = static_cast<int4*>(ws.tiles);
  p.n_units = ws.count;
  p.expert_slots = ws.expert_slots;
  p.partials = ws.partials;
  // The tensor-core kernel builds a short unit list itself (one launch less);
  // seg_reduce then reads the expert slots its CTA 0 wrote.
  const bool own_units = tensor && n_routes > 0 && n_experts <= kOwnUnitExperts &&
                         max_row_tiles(n_routes, n_experts, (int)p.chunk) <= kOwnUnits;
  if (own_units) {
    p.units = nullptr;
  } else {
    rc = build_units(offsets, n_experts, p.chunk, static_cast<int4*>(ws.tiles), ws.count, ws.expert_slots, s);
    if (rc) return rc;
  }
  // Both operands padded: the GEMM derives every row from its unit and needs
  // no resolved route rows.
  if (tensor && n_routes > 0 && (!(x_pad_start && g_pad_start) || w)) {
    char* rr = reinterpret_cast<char*>(ws.partials) +
               align_up((size_t)segw_max_slots(n_routes, p.chunk) * m_dim * n_dim * sizeof(float), 256);
    const size_t arr = align_up((size_t)(n_routes + kRouteRowsPad) * 4, 256);
    int* xrow = reinterpret_cast<int*>(rr);
    int* grow = reinterpret_cast<int*>(rr + arr);
    float* wsc = reinterpret_cast<float*>(rr + 2 * arr);
    rc = resolve_route_rows(p, xrow, grow, wsc, s);
    if (rc) return rc;
    p.xrow = xrow;
    p.grow = grow;
    p.wsc = wsc;
  }
  if (n_routes > 0) {
    const int64_t max_units = max_row_tiles(n_routes, n_experts, (int)p.chunk);
    rc = tensor ? launch_seg_gemm_umma(p, max_units, s) : launch_seg_gemm_simt(p, max_units, s);
    if (rc) return rc;
  }
  // Sums split experts' partial slots in chunk order and zero-fills experts
  // without routes (the reference writes 0 for them, cvmm.py:476-478).
  return seg_reduce(ws.expert_slots, ws.partials, grad_w, n_experts, m_dim * n_dim, s);
}

int cvmm_backward_w_launches(int64_t n_routes, int64_t n_experts, int64_t m_dim, int64_t n_dim, int op_dtype,
                             int both_padded, int weighted) {
  const bool tensor = op_dtype != F32;
  if (n_routes <= 0) return 2;  // unit list + reduction (zero fill)
  const int64_t chunk = segw_chunk(n_routes, n_experts, m_dim, n_dim, tensor);
  const bool own_units = tensor && n_experts <= kOwnUnitExperts && max_row_tiles(n_routes, n_experts, (int)chunk) <= kOwnUnits;
  const bool resolve = tensor && (!both_padded || weighted);
  return (own_units ? 0 : 1) + (resolve ? 1 : 0) + 1 + 1;
}

int cvmm_pad_starts(const int64_t* offsets, int64_t n_experts, int32_t* pad_start, cvmm_stream_t stream) {
  if (n_experts <= 0 || !offsets || !pad_start) return fail(CVMM_ERR_INVALID_ARG, "cvmm_pad_starts: bad arguments");
  return pad_starts(offsets, n_experts, kPadRows, reinterpret_cast<int*>(pad_start),
                    reinterpret_cast<cudaStream_t>(stream));
}

static int sort_rows_padded_abi(const void* src, int src_dtype, int64_t src_ld, const int64_t* index, int64_t div,
                          const void* scale, int scale_dtype, const int32_t* sorted_sel, const int64_t* offsets,
                          int64_t n_routes, int64_t n_experts, int64_t cols, void* dst, int dst_dtype,
                          int32_t* pad_start, bool pad_ready, int32_t* route_rows,
                                cvmm_stream_t stream) {
  if (!is_float_dtype(src_dtype) || !is_float_dtype(dst_dtype) || (scale && !is_float_dtype(scale_dtype)))
    return fail(CVMM_ERR_UNSUPPORTED_DTYPE, "cvmm_sort_rows_padded: unsupported dtype");
  if (n_routes < 0 || n_experts <= 0 || cols <= 0 || div <= 0 || src_ld < cols ||
      n_routes + n_experts * kPadRows > (int64_t)INT32_MAX)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_sort_rows_padded: bad sizes");
  if (!dst || !pad_start || !offsets || (n_routes > 0 && (!src || !index || !sorted_sel)))
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_sort_rows_padded: null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int rc = pad_ready ? 0 : pad_starts(offsets, n_experts, kPadRows, reinterpret_cast<int*>(pad_start), s);
  if (rc || n_routes == 0) return rc;
  return sort_rows_padded(src, src_dtype, src_ld, index, div, scale, scale_dtype, sorted_sel, offsets,
                          reinterpret_cast<int*>(pad_start), n_routes, n_experts, cols, dst, dst_dtype, s,
                          route_rows);
}

int cvmm_sort_rows_padded(const void* src, int src_dtype, int64_t src_ld, const int64_t* index, int64_t div,
                          const void* scale, int scale_dtype, const int32_t* sorted_sel, const int64_t* offsets,
                          int64_t n_routes, int64_t n_experts, int64_t cols, void* dst, int dst_dtype,
                          int32_t* pad_start, cvmm_stream_t stream) {
  return sort_rows_padded_abi(src, src_dtype, src_ld, index, div, scale, scale_dtype, sorted_sel, offsets, n_routes,
                              n_experts, cols, dst, dst_dtype, pad_start, false, nullptr, stream);
}

int cvmm_sort_rows_padded_ex(const void* src, int src_dtype, int64_t src_ld, const int64_t* index, int64_t div,
                             const void* scale, int scale_dtype, const int32_t* sorted_sel, const int64_t* offsets,
                             int64_t n_routes, int64_t n_experts, int64_t cols, void* dst, int dst_dtype,
                             int32_t* pad_start, int pad_start_ready, int32_t* route_rows, cvmm_stream_t stream) {
  return sort_rows_padded_abi(src, src_dtype, src_ld, index, div, scale, scale_dtype, sorted_sel, offsets, n_routes,
                              n_experts, cols, dst, dst_dtype, pad_start, pad_start_ready != 0, route_rows, stream);
}

int cvmm_weighted_token_backward(const void* route_grad, int rg_dtype, const void* w, int w_dtype,
                                 const void* x, int x_dtype, void* grad_x, int gx_dtype,
                                 float* grad_sel, int64_t n_tokens, int64_t top_k, int64_t d,
                                 cvmm_stream_t stream) {
  if (!is_float_dtype(rg_dtype) || !is_float_dtype(w_dtype) || !is_float_dtype(x_dtype) ||
      (grad_x && !is_float_dtype(gx_dtype)))
    return fail(CVMM_ERR_UNSUPPORTED_DTYPE, "cvmm_weighted_token_backward: unsupported dtype");
  if (n_tokens < 0 || top_k <= 0 || d <= 0)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_weighted_token_backward: bad sizes");
  if (n_tokens == 0) return CVMM_OK;
  if (!route_grad || !w || (grad_sel && !x))
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_weighted_token_backward: null pointer");
  const int threads = 256;
  launch(weighted_token_bwd_kernel, (unsigned)n_tokens, threads, (threads / 32) * sizeof(float), reinterpret_cast<cudaStream_t>(stream),
      route_grad, rg_dtype, w, w_dtype, x, x_dtype, grad_x, gx_dtype, grad_sel, top_k, d);
  return check_launch("cvmm_weighted_token_backward");
}

int cvmm_cast(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t n, cvmm_stream_t stream) {
  if (!is_float_dtype(src_dtype) || !is_float_dtype(dst_dtype))
    return fail(CVMM_ERR_UNSUPPORTED_DTYPE, "cvmm_cast: unsupported dtype");
  if (n < 0) return fail(CVMM_ERR_INVALID_ARG, "cvmm_cast: bad size");
  if (n == 0) return CVMM_OK;
  if (!src || !dst) return fail(CVMM_ERR_INVALID_ARG, "cvmm_cast: null pointer");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (src_dtype == F32 && dst_dtype != F32 && n % 8 == 0 && al16(src) && al16(dst)) {
    launch(cast_f32_to_16_vec, grid_for((n / 8 + 1) / 2, 256), 256, 0, s, static_cast<const float4*>(src),
                                                            static_cast<uint4*>(dst), dst_dtype, n / 8);
  } else {
    launch(cast_kernel, grid_for(n, 256), 256, 0, s, src, src_dtype, dst, dst_dtype, n);
  }
  return check_launch("cvmm_cast");
}

int cvmm_cast_ahead(const void* src, int src_dtype, void* dst, int dst_dtype, int64_t n, cvmm_stream_t stream) {
  if (src_dtype == F32 && (dst_dtype == BF16 || dst_dtype == F16) && n > 0 && n % 8 == 0 && src && dst &&
      al16(src) && al16(dst)) {
    const int64_t per_block = 256 * kCastAhead;
    const int grid = (int)std::min<int64_t>((n / 8 + per_block - 1) / per_block, 148 * 8);
    launch(cast_f32_to_16_ahead, grid, 256, 0, reinterpret_cast<cudaStream_t>(stream),
           static_cast<const float4*>(src), static_cast<uint4*>(dst), dst_dtype, n / 8);
    return check_launch("cvmm_cast_ahead");
  }
  return cvmm_cast(src, src_dtype, dst, dst_dtype, n, stream);
}

}  // extern "C"
