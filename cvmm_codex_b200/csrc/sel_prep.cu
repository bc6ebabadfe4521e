// Selector preparation: stable device radix sort of routes by expert id.
//
// Reference semantics (cvmm.py:1786-1803): fsel = sel.flatten().to(int32);
// (ssel, idx) = fsel.sort(); token input: sel_index = idx // k, out_index = idx;
// route input: sel_index = idx. Our sort is stable (ties keep route order), the
// order torch.sort(stable=True) gives.
//
// Design (B200): the keys are tiny integers (expert ids), so instead of a
// general sort we run an LSD radix sort with 11-bit digits over the key range
// actually present (max - min). For every realistic expert count (< 2048
// experts) that is ONE pass of histogram -> scan -> scatter. The whole sort is
// one persistent launch (sort_kernel): at most one CTA per SM, each owning a
// contiguous slice of routes, with grid-wide barriers (bounded waits) between
// the phases, so the step costs one launch instead of a chain of small
// kernels whose launch gaps dominated the sort.
#include "common.cuh"
#include "launch.h"

namespace cvmm {

namespace sel {

constexpr int kDigitBits = 11;
constexpr int kBins = 1 << kDigitBits;  // 2048
constexpr int kMaxPasses = 3;           // 33 bits >= 32-bit key range
constexpr int kWarps = kSelWarps;       // warps per CTA; each owns a contiguous slice of the CTA's routes
constexpr int kThreads = kWarps * 32;
constexpr int kGridTag = 20;            // status-word site of a grid barrier that ran out

// Zeroed by the host before every call.
struct Header {
  unsigned int max_u;    // max over biased keys (key ^ 0x80000000)
  unsigned int max_nu;   // max over ~biased keys  => min = ~max_nu
  unsigned int arrived;  // grid-barrier arrivals (monotonic within the call)
  int abort;             // a barrier wait ran out: every CTA stops
};

__device__ __forceinline__ unsigned int bias(int32_t k) { return (unsigned int)k ^ 0x80000000u; }

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid-wide barrier of the persistent sort kernel. Every CTA of the grid is
// resident (the grid is at most one CTA per SM and the kernel needs no more
// than one SM's resources), so all arrivals eventually come; the wait is
// still bounded: if it runs out the CTA records CVMM_DEV_TIMEOUT, raises the
// shared abort flag and every CTA returns at its next barrier.
__device__ __forceinline__ bool grid_barrier(Header* h, unsigned int target, int* sh_ok) {
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    __threadfence();
    atomicAdd(&h->arrived, 1u);
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
      if (ld_acquire(&h->arrived) >= target) break;
      if ((it & 31u) == 31u) {
        if (*reinterpret_cast<volatile int*>(&h->abort)) { ok = 0; break; }
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
          report(CVMM_DEV_TIMEOUT, kGridTag, (long long)target);
          atomicExch(&h->abort, 1);
          ok = 0;
          break;
        }
      }
      __nanosleep(32);
    }
    __threadfence();
    *sh_ok = ok;
  }
  __syncthreads();
  return *sh_ok != 0;
}

__device__ __forceinline__ int warp_incl_scan(int v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += y;
  }
  return v;
}

// Exclusive scan of one int per thread over the CTA.
__device__ __forceinline__ int cta_excl_scan(int v, int* warp_tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int incl = warp_incl_scan(v);
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int t = lane < kWarps ? warp_tot[lane] : 0;
    const int s = warp_incl_scan(t);
    if (lane < kWarps) warp_tot[lane] = s - t;
  }
  __syncthreads();
  const int r = incl - v + warp_tot[warp];
  __syncthreads();
  return r;
}

// Stable LSD radix sort of the routes by expert id in ONE persistent launch.
// CTA c owns routes [c * cta_len, (c + 1) * cta_len); its warp w owns a
// contiguous slice of those, so (CTA, warp, lane) order is route order. Per
// 11-bit digit pass (one pass whenever the ids present span fewer than 2048
// values, i.e. for every realistic expert count):
//   1. per-warp digit histograms in shared memory (equal digits of a warp
//      step counted once by __match_any_sync), CTA totals to counts[bin][cta];
//   2. grid barrier; CTA c scans bins c, c + G, ... over the CTAs (exclusive,
//      in place) and records each bin's total;
//   3. grid barrier; every CTA scans the bin totals, adds its own prefix and
//      the counts of its earlier warps, and scatters: position = warp base of
//      the digit + rank among equal digits of the lanes before it.
// Before the first pass the CTAs convert the ids to int32 (raw_sel) and find
// the key range, after which a barrier makes it known to all. The digits are
// relative to the minimum id, so ids 0..E-1 of any E <= 2048 need one pass.
__global__ void __launch_bounds__(kThreads, 1)
sort_kernel(const void* __restrict__ sel, int sel_dtype, int64_t n, int64_t cta_len, int32_t* __restrict__ raw,
            Header* __restrict__ h, int* __restrict__ counts, int* __restrict__ bin_total, int32_t* __restrict__ kbuf0,
            int32_t* __restrict__ vbuf0, int32_t* __restrict__ kbuf1, int32_t* __restrict__ vbuf1,
            int32_t* __restrict__ sorted_sel, int64_t* __restrict__ sel_index, int64_t* __restrict__ out_index,
            int64_t top_k, int route_input) {
  pdl_enter();
  extern __shared__ int hist[];  // [kWarps][kBins] per-warp digit counts, then per-warp write positions
  __shared__ int bin_base[kBins];
  __shared__ int warp_tot[kWarps];
  __shared__ unsigned int red[2][kWarps];
  __shared__ int sh_ok;
  const int G = (int)gridDim.x, c = (int)blockIdx.x;
  const int tid = (int)threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t beg = (int64_t)c * cta_len, end = min(beg + cta_len, n);
  const int64_t wlen = cta_len / kWarps;  // a multiple of 32
  const int64_t wbeg = min(beg + warp * wlen, end), wend = min(wbeg + wlen, end);
  unsigned int barriers = 0;

  // ---- int32 conversion and key range
  unsigned int mx = 0u, mnx = 0u;
  for (int64_t i = beg + tid; i < end; i += kThreads) {
    const int32_t v = sel_dtype == CVMM_I64 ? (int32_t)reinterpret_cast<const int64_t*>(sel)[i]
                                            : reinterpret_cast<const int32_t*>(sel)[i];
    raw[i] = v;
    const unsigned int u = bias(v);
    mx = max(mx, u);
    mnx = max(mnx, ~u);
  }
  for (int o = 16; o > 0; o >>= 1) {
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    mnx = max(mnx, __shfl_xor_sync(0xffffffffu, mnx, o));
  }
  if (lane == 0) {
    red[0][warp] = mx;
    red[1][warp] = mnx;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < kWarps; ++w) {
      mx = max(mx, red[0][w]);
      mnx = max(mnx, red[1][w]);
    }
    if (end > beg) {
      atomicMax(&h->max_u, mx);
      atomicMax(&h->max_nu, mnx);
    }
  }
  if (!grid_barrier(h, ++barriers * G, &sh_ok)) return;
  const unsigned int mn = ~ld_acquire(&h->max_nu);
  const unsigned int range = ld_acquire(&h->max_u) - mn;
  int passes = 1;
  while (passes < kMaxPasses && (range >> (kDigitBits * passes)) != 0u) ++passes;

  int* my = hist + warp * kBins;
  const unsigned int lt_mask = (1u << lane) - 1u;
  const int32_t* kin = raw;
  const int32_t* vin = nullptr;
  for (int p = 0; p < passes; ++p) {
    const int shift = p * kDigitBits;
    const int nb = (range >> shift) >= (unsigned int)(kBins - 1) ? kBins : (int)(range >> shift) + 1;
    const bool last = p == passes - 1;
    int32_t* kout = (p & 1) ? kbuf1 : kbuf0;
    int32_t* vout = (p & 1) ? vbuf1 : vbuf0;
    // 1. per-warp histograms
    for (int b = lane; b < nb; b += 32) my[b] = 0;
    __syncwarp();
    for (int64_t i0 = wbeg; i0 < wend; i0 += 32) {
      const int64_t i = i0 + lane;
      const unsigned int d = i < wend ? ((bias(__ldcg(kin + i)) - mn) >> shift) & (kBins - 1) : 0xffffffffu;
      const unsigned int peers = __match_any_sync(0xffffffffu, d);
      if (i < wend && (peers & lt_mask) == 0u) my[d] += __popc(peers);
      __syncwarp();
    }
    __syncthreads();
    for (int b = tid; b < nb; b += kThreads) {
      int t = 0;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) t += hist[w * kBins + b];
      counts[(int64_t)b * G + c] = t;
    }
    if (!grid_barrier(h, ++barriers * G, &sh_ok)) return;
    // 2. per-bin exclusive scan over the CTAs (one warp per bin)
    for (int b = c + warp * G; b < nb; b += G * kWarps) {
      int run = 0;
      for (int j0 = 0; j0 < G; j0 += 32) {
        const int j = j0 + lane;
        const int v = j < G ? __ldcg(&counts[(int64_t)b * G + j]) : 0;
        const int incl = warp_incl_scan(v);
        if (j < G) counts[(int64_t)b * G + j] = run + incl - v;
        run += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) bin_total[b] = run;
    }
    if (!grid_barrier(h, ++barriers * G, &sh_ok)) return;
    // 3. positions: bin bases, this CTA's prefix, then its warps in order
    constexpr int kPer = kBins / kThreads;
    int loc[kPer];
    int sum = 0;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int b = tid * kPer + q;
      loc[q] = b < nb ? __ldcg(&bin_total[b]) : 0;
      sum += loc[q];
    }
    int run = cta_excl_scan(sum, warp_tot);
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int b = tid * kPer + q;
      if (b < nb) bin_base[b] = run;
      run += loc[q];
    }
    __syncthreads();
    for (int b = tid; b < nb; b += kThreads) {
      int pos = bin_base[b] + __ldcg(&counts[(int64_t)b * G + c]);
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const int t = hist[w * kBins + b];
        hist[w * kBins + b] = pos;
        pos += t;
      }
    }
    __syncthreads();
    for (int64_t i0 = wbeg; i0 < wend; i0 += 32) {
      const int64_t i = i0 + lane;
      const bool valid = i < wend;
      // Keys and values of later passes were written by other CTAs: read
      // them (and every other cross-CTA value) from L2, never a stale L1 line.
      const int32_t key = valid ? __ldcg(kin + i) : 0;
      const int32_t val = valid ? (vin ? __ldcg(vin + i) : (int32_t)i) : 0;
      const unsigned int d = valid ? ((bias(key) - mn) >> shift) & (kBins - 1) : 0xffffffffu;
      const unsigned int peers = __match_any_sync(0xffffffffu, d);
      int pos = 0;
      if (valid) pos = my[d] + __popc(peers & lt_mask);
      __syncwarp();
      if (valid && (peers & lt_mask) == 0u) my[d] += __popc(peers);
      __syncwarp();
      if (!valid) continue;
      if (last) {
        sorted_sel[pos] = key;
        if (route_input) {
          sel_index[pos] = (int64_t)val;
        } else {
          sel_index[pos] = (int64_t)val / top_k;
          out_index[pos] = (int64_t)val;
        }
      } else {
        kout[pos] = key;
        vout[pos] = val;
      }
    }
    if (last) break;
    if (!grid_barrier(h, ++barriers * G, &sh_ok)) return;
    kin = kout;
    vin = vout;
  }
}

// offsets[e] = #sorted keys <= e, the reference's inclusive end offsets
// (cvmm.py:315-335). One thread per sorted position i writes the experts in
// [sorted[i], sorted[i+1]) (clipped to [0, n_experts)) with i + 1; thread -1
// (i.e. position 0's extra work) writes the experts below sorted[0] with 0, and
// the last position the experts from sorted[n-1] on with n. Every expert is
// written exactly once, with no search.
__global__ void offsets_kernel(const int32_t* __restrict__ sorted, int64_t n, int64_t n_experts,
                               int64_t* __restrict__ offsets) {
  pdl_enter();
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (n == 0) {
    if (i < n_experts) offsets[i] = 0;
    return;
  }
  if (i >= n) return;
  const int64_t a = sorted[i];
  // An expert id outside [0, n_experts) would index past the weights: record
  // it (site 1 = sorted position) in the status word; the GEMMs never read
  // such routes (they only visit the routes inside [0, offsets[E-1])).
  if (a < 0 || a >= n_experts) report(CVMM_DEV_BAD_INDEX, 1, (long long)a);
  if (i == 0)
    for (int64_t e = 0; e < min(a, n_experts); ++e) offsets[e] = 0;
  const int64_t b = i + 1 < n ? (int64_t)sorted[i + 1] : n_experts;
  for (int64_t e = max(a, (int64_t)0); e < min(b, n_experts); ++e) offsets[e] = i + 1;
}

}  // namespace sel

namespace sel {
constexpr size_t kSmemBytes = (size_t)kWarps * kBins * sizeof(int);

static int sm_count() {
  static int cached[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int v = 0;
    cached[dev] = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0 ? v : 148;
  }
  return cached[dev];
}
}  // namespace sel

size_t sel_prepare_workspace_size(int64_t n, int64_t min_chunk) { return sel_ws_bytes(n, min_chunk); }

int sel_prepare(const void* sel_ptr, int sel_dtype, int64_t n, int64_t top_k, int route_input,
                int32_t* raw_sel, int32_t* sorted_sel, int64_t* sel_index, int64_t* out_index,
                void* workspace, size_t ws_bytes, cudaStream_t stream, int64_t min_chunk) {
  if (n < 0 || top_k <= 0) return fail(CVMM_ERR_INVALID_ARG, "cvmm_sel_prepare: bad n_routes/top_k");
  if (sel_dtype != CVMM_I64 && sel_dtype != CVMM_I32)
    return fail(CVMM_ERR_UNSUPPORTED_DTYPE, "cvmm_sel_prepare: sel must be int64 or int32");
  if (n == 0) return CVMM_OK;
  if (!sel_ptr || !raw_sel || !sorted_sel || !sel_index || (!route_input && !out_index))
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_sel_prepare: null pointer");
  if (n > (int64_t)INT32_MAX) return fail(CVMM_ERR_INVALID_ARG, "cvmm_sel_prepare: too many routes");
  if (!workspace || ws_bytes < sel_prepare_workspace_size(n, min_chunk))
    return fail(CVMM_ERR_WORKSPACE, "cvmm_sel_prepare: workspace too small");

  // One CTA per SM at most (the grid barriers need every CTA resident), each
  // a multiple of kSelWarps * 32 routes and at least min_chunk routes.
  const int64_t g_max = std::min<int64_t>(sel::sm_count(), kSelMaxGrid);
  const int64_t cta_len = std::max(sel_cta_len_min(min_chunk), sel_round(
                                       (n + g_max - 1) / g_max));
  const int grid = (int)((n + cta_len - 1) / cta_len);
  char* ws = static_cast<char*>(workspace);
  sel::Header* h = reinterpret_cast<sel::Header*>(ws);
  ws += 256;
  int* counts = reinterpret_cast<int*>(ws);
  ws += align_up((size_t)sel::kBins * sel_grid_bound(n, min_chunk) * sizeof(int), 256);
  int* bin_total = reinterpret_cast<int*>(ws);
  ws += align_up((size_t)sel::kBins * sizeof(int), 256);
  int32_t* buf[4];
  for (int i = 0; i < 4; ++i) {
    buf[i] = reinterpret_cast<int32_t*>(ws);
    ws += align_up((size_t)n * sizeof(int32_t), 256);
  }
  if (cudaFuncSetAttribute(sel::sort_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sel::kSmemBytes) !=
      cudaSuccess)
    return fail_cuda("cvmm_sel_prepare: cudaFuncSetAttribute");
  if (cudaMemsetAsync(h, 0, sizeof(sel::Header), stream) != cudaSuccess)
    return fail_cuda("cvmm_sel_prepare: memset");
  launch(sel::sort_kernel, grid, sel::kThreads, sel::kSmemBytes, stream,
      sel_ptr, sel_dtype, n, cta_len, raw_sel, h, counts, bin_total, buf[0], buf[1], buf[2], buf[3], sorted_sel,
      sel_index, out_index, top_k, route_input);
  return check_launch("cvmm_sel_prepare");
}

int expert_offsets(const int32_t* sorted, int64_t n, int64_t n_experts, int64_t* offsets,
                   cudaStream_t stream) {
  if (n < 0 || n_experts <= 0 || !offsets || (n > 0 && !sorted))
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_expert_offsets: bad arguments");
  const int64_t work = n > 0 ? n : n_experts;
  launch(sel::offsets_kernel, (unsigned)((work + 255) / 256), 256, 0, stream, sorted, n, n_experts, offsets);
  return check_launch("cvmm_expert_offsets");
}

}  // namespace cvmm
