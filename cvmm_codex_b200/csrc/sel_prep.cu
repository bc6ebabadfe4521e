// Selector preparation: stable device radix sort of routes by expert id.
//
// Reference semantics (cvmm.py:1786-1803): fsel = sel.flatten().to(int32);
// (ssel, idx) = fsel.sort(); token input: sel_index = idx // k, out_index = idx;
// route input: sel_index = idx. Our sort is stable (ties keep route order), the
// order torch.sort(stable=True) gives.
//
// Design (B200): the keys are tiny integers (expert ids), so instead of a
// general sort we run an LSD radix sort with 11-bit digits over the biased key
// range actually present (max - min). For every realistic expert count
// (< 2048 experts) that is ONE pass of histogram -> scan -> scatter. Each warp
// owns a chunk of consecutive routes (128 or more, at most 2048 chunks, so
// that even 64k routes spread over ~128 CTAs). Digit counts are kept per CTA
// (4 warp chunks), which keeps the single-CTA scan short; the scatter orders
// the warps of its CTA by their own histograms and ranks equal digits inside
// a warp with __match_any_sync, so the sort is stable. Extra passes (keys spread over > 2048
// values) are launched unconditionally but exit on the device when the key
// range does not need them, so the host never synchronises.
#include "common.cuh"
#include "launch.h"

namespace cvmm {

namespace sel {

constexpr int kDigitBits = 11;
constexpr int kBins = 1 << kDigitBits;  // 2048
constexpr int64_t kMaxChunks = 2048;    // bounds the single-CTA scan to kBins * kMaxChunks counts
constexpr int kWarpsPerCta = 4;
constexpr int kMaxPasses = 3;           // 33 bits >= 32-bit key range

struct Header {
  unsigned int max_u;   // max over biased keys (key ^ 0x80000000)
  unsigned int max_nu;  // max over ~biased keys  => min = ~max_nu
};

__device__ __forceinline__ unsigned int bias(int32_t k) { return (unsigned int)k ^ 0x80000000u; }

__device__ __forceinline__ unsigned int key_range(const Header* h) {
  unsigned int mn = ~h->max_nu;
  return h->max_u - mn;
}

// Pass p is needed iff the key range has bits at or above its shift.
__device__ __forceinline__ bool pass_needed(const Header* h, int shift) {
  return shift == 0 || (key_range(h) >> shift) != 0u;
}

__device__ __forceinline__ int n_bins(const Header* h, int shift) {
  unsigned int r = key_range(h) >> shift;
  return r >= (unsigned int)(kBins - 1) ? kBins : (int)r + 1;
}

__global__ void convert_minmax_kernel(const void* __restrict__ sel, int sel_dtype, int64_t n,
                                      int32_t* __restrict__ raw, Header* __restrict__ h) {
  unsigned int mx = 0u, mnx = 0u;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    int32_t v = sel_dtype == CVMM_I64 ? (int32_t)reinterpret_cast<const int64_t*>(sel)[i]
                                      : reinterpret_cast<const int32_t*>(sel)[i];
    raw[i] = v;
    unsigned int u = bias(v);
    mx = max(mx, u);
    mnx = max(mnx, ~u);
  }
  for (int o = 16; o > 0; o >>= 1) {
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    mnx = max(mnx, __shfl_xor_sync(0xffffffffu, mnx, o));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMax(&h->max_u, mx);
    atomicMax(&h->max_nu, mnx);
  }
}

__device__ __forceinline__ unsigned int digit_of(int32_t key, unsigned int mn, int shift) {
  return ((bias(key) - mn) >> shift) & (kBins - 1);
}

// Digit histogram of this CTA's warp chunks, one row per warp, in `hist`.
__device__ __forceinline__ void cta_histogram(const int32_t* __restrict__ keys, int64_t n, int64_t n_chunks,
                                              int64_t chunk_len, unsigned int mn, int shift, int nb,
                                              int (*hist)[kBins]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t chunk = (int64_t)blockIdx.x * kWarpsPerCta + warp;
  for (int b = lane; b < nb; b += 32) hist[warp][b] = 0;
  __syncwarp();
  if (chunk < n_chunks) {
    const int64_t beg = chunk * chunk_len;
    const int64_t end = min(beg + chunk_len, n);
    for (int64_t i = beg + lane; i < end; i += 32) atomicAdd(&hist[warp][digit_of(keys[i], mn, shift)], 1);
  }
  __syncthreads();
}

// counts layout: counts[bin * n_cta + cta] (one column per CTA of kWarpsPerCta
// warp chunks), so that one exclusive scan in memory order yields every
// (bin, CTA) base position; the warps of a CTA are ordered inside the scatter.
__global__ void __launch_bounds__(kWarpsPerCta * 32)
hist_kernel(const int32_t* __restrict__ keys, int64_t n, int64_t n_chunks, int64_t chunk_len,
            const Header* __restrict__ h, int shift, int* __restrict__ counts) {
  if (!pass_needed(h, shift)) return;
  __shared__ int hist[kWarpsPerCta][kBins];
  const int nb = n_bins(h, shift);
  cta_histogram(keys, n, n_chunks, chunk_len, ~h->max_nu, shift, nb, hist);
  for (int b = threadIdx.x; b < nb; b += blockDim.x) {
    int c = 0;
#pragma unroll
    for (int w = 0; w < kWarpsPerCta; ++w) c += hist[w][b];
    counts[(int64_t)b * gridDim.x + blockIdx.x] = c;
  }
}

// Single-CTA exclusive scan over nb * n_chunks counts, in place. Thread t
// owns a contiguous, 16-byte aligned slice; it reads the slice in batches of
// kScanBatch counts with int4 loads all in flight (the slice sum), the CTA
// scans the 1024 slice sums, and the slice is rewritten the same way.
constexpr int kScanBatch = 32;

__device__ __forceinline__ void scan_load(const int* __restrict__ c, int64_t i, int64_t end, int (&v)[kScanBatch]) {
#pragma unroll
  for (int q = 0; q < kScanBatch / 4; ++q) {
    const int64_t k = i + 4 * q;
    if (k + 3 < end) {
      const int4 x = *reinterpret_cast<const int4*>(c + k);
      v[4 * q] = x.x; v[4 * q + 1] = x.y; v[4 * q + 2] = x.z; v[4 * q + 3] = x.w;
    } else {
#pragma unroll
      for (int r = 0; r < 4; ++r) v[4 * q + r] = k + r < end ? c[k + r] : 0;
    }
  }
}

__global__ void __launch_bounds__(1024)
scan_kernel(int* __restrict__ counts, int64_t n_chunks, const Header* __restrict__ h, int shift) {
  if (!pass_needed(h, shift)) return;
  const int64_t total = (int64_t)n_bins(h, shift) * n_chunks;
  const int t = threadIdx.x;
  const int64_t per = ((total + blockDim.x - 1) / blockDim.x + 3) & ~(int64_t)3;
  const int64_t beg = min((int64_t)t * per, total), end = min(beg + per, total);
  int v[kScanBatch];
  int local = 0;
  for (int64_t b = beg; b < end; b += kScanBatch) {
    scan_load(counts, b, end, v);
#pragma unroll
    for (int j = 0; j < kScanBatch; ++j) local += v[j];
  }
  __shared__ int warp_sums[32];
  int x = local;
  const int lane = t & 31, warp = t >> 5;
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int s = lane < (int)(blockDim.x >> 5) ? warp_sums[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    warp_sums[lane] = s;  // inclusive over warps
  }
  __syncthreads();
  int run = x - local + (warp > 0 ? warp_sums[warp - 1] : 0);  // exclusive prefix
  for (int64_t b = beg; b < end; b += kScanBatch) {
    if (per > kScanBatch) scan_load(counts, b, end, v);  // else v still holds the slice
#pragma unroll
    for (int j = 0; j < kScanBatch; ++j) {
      const int c = v[j];
      v[j] = run;
      run += c;
    }
#pragma unroll
    for (int q = 0; q < kScanBatch / 4; ++q) {
      const int64_t k = b + 4 * q;
      if (k + 3 < end) {
        *reinterpret_cast<int4*>(counts + k) = make_int4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      } else {
#pragma unroll
        for (int r = 0; r < 4; ++r)
          if (k + r < end) counts[k + r] = v[4 * q + r];
      }
    }
  }
}

// Stable scatter. Pass 0 reads keys = raw_sel with implicit values = route id.
__global__ void __launch_bounds__(kWarpsPerCta * 32)
scatter_kernel(const int32_t* __restrict__ keys_in, const int32_t* __restrict__ vals_in,
               int64_t n, int64_t n_chunks, int64_t chunk_len, const Header* __restrict__ h, int shift,
               const int* __restrict__ base, int32_t* __restrict__ keys_out,
               int32_t* __restrict__ vals_out, int32_t* __restrict__ sorted_sel,
               int64_t* __restrict__ sel_index, int64_t* __restrict__ out_index,
               int64_t top_k, int route_input) {
  if (!pass_needed(h, shift)) return;
  __shared__ int ctr[kWarpsPerCta][kBins];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t chunk = (int64_t)blockIdx.x * kWarpsPerCta + warp;
  const int nb = n_bins(h, shift);
  const unsigned int mn = ~h->max_nu;
  const bool last = shift + kDigitBits >= 32 || (key_range(h) >> (shift + kDigitBits)) == 0u;
  // Each warp's first position per bin: the CTA's base plus the counts of the
  // CTA's earlier warps (stable: warp chunks are in route order).
  cta_histogram(keys_in, n, n_chunks, chunk_len, mn, shift, nb, ctr);
  for (int b = threadIdx.x; b < nb; b += blockDim.x) {
    int run = base[(int64_t)b * gridDim.x + blockIdx.x];
#pragma unroll
    for (int w = 0; w < kWarpsPerCta; ++w) {
      const int c = ctr[w][b];
      ctr[w][b] = run;
      run += c;
    }
  }
  __syncthreads();
  if (chunk >= n_chunks) return;
  int* my = ctr[warp];
  const int64_t beg = chunk * chunk_len;
  const int64_t end = min(beg + chunk_len, n);
  const unsigned int lt_mask = (1u << lane) - 1u;
  for (int64_t i0 = beg; i0 < end; i0 += 32) {
    const int64_t i = i0 + lane;
    const bool valid = i < end;
    int32_t key = valid ? keys_in[i] : 0;
    int32_t val = valid ? (vals_in ? vals_in[i] : (int32_t)i) : 0;
    unsigned int d = valid ? digit_of(key, mn, shift) : 0xffffffffu;
    unsigned int peers = __match_any_sync(0xffffffffu, d);
    int pos = 0;
    if (valid) pos = my[d] + __popc(peers & lt_mask);
    __syncwarp();
    if (valid && (peers & lt_mask) == 0u) my[d] += __popc(peers);
    __syncwarp();
    if (valid) {
      if (last) {
        sorted_sel[pos] = key;
        if (route_input) {
          sel_index[pos] = (int64_t)val;
        } else {
          sel_index[pos] = (int64_t)val / top_k;
          out_index[pos] = (int64_t)val;
        }
      } else {
        keys_out[pos] = key;
        vals_out[pos] = val;
      }
    }
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
// Routes per warp chunk: at least min_chunk, a multiple of 32, at most kMaxChunks chunks.
static int64_t chunk_len(int64_t n, int64_t min_chunk) {
  int64_t c = std::max<int64_t>(min_chunk, (n + kMaxChunks - 1) / kMaxChunks);
  return (c + 31) / 32 * 32;
}
}  // namespace sel

size_t sel_prepare_workspace_size(int64_t n, int64_t min_chunk) {
  const int64_t n_chunks = (n + sel::chunk_len(n, min_chunk) - 1) / sel::chunk_len(n, min_chunk);
  size_t bytes = 256;                                             // header
  bytes += align_up((size_t)n_chunks * sel::kBins * sizeof(int), 256);  // counts
  bytes += 4 * align_up((size_t)n * sizeof(int32_t), 256);         // ping-pong keys/vals
  return bytes;
}

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

  const int64_t clen = sel::chunk_len(n, min_chunk);
  const int64_t n_chunks = (n + clen - 1) / clen;
  char* ws = static_cast<char*>(workspace);
  sel::Header* h = reinterpret_cast<sel::Header*>(ws);
  ws += 256;
  int* counts = reinterpret_cast<int*>(ws);
  ws += align_up((size_t)n_chunks * sel::kBins * sizeof(int), 256);
  int32_t* buf[4];
  for (int i = 0; i < 4; ++i) {
    buf[i] = reinterpret_cast<int32_t*>(ws);
    ws += align_up((size_t)n * sizeof(int32_t), 256);
  }

  if (cudaMemsetAsync(h, 0, sizeof(sel::Header), stream) != cudaSuccess)
    return fail_cuda("cvmm_sel_prepare: memset");
  int grid = (int)std::min<int64_t>((n + 255) / 256, 148 * 8);
  sel::convert_minmax_kernel<<<grid, 256, 0, stream>>>(sel_ptr, sel_dtype, n, raw_sel, h);
  const int cta = (int)((n_chunks + sel::kWarpsPerCta - 1) / sel::kWarpsPerCta);
  const int32_t* kin = raw_sel;
  const int32_t* vin = nullptr;
  for (int p = 0; p < sel::kMaxPasses; ++p) {
    const int shift = p * sel::kDigitBits;
    int32_t* kout = buf[(p & 1) * 2];
    int32_t* vout = buf[(p & 1) * 2 + 1];
    sel::hist_kernel<<<cta, sel::kWarpsPerCta * 32, 0, stream>>>(kin, n, n_chunks, clen, h, shift, counts);
    sel::scan_kernel<<<1, 1024, 0, stream>>>(counts, cta, h, shift);
    sel::scatter_kernel<<<cta, sel::kWarpsPerCta * 32, 0, stream>>>(
        kin, vin, n, n_chunks, clen, h, shift, counts, kout, vout, sorted_sel, sel_index, out_index,
        top_k, route_input);
    kin = kout;
    vin = vout;
  }
  return check_launch("cvmm_sel_prepare");
}

int expert_offsets(const int32_t* sorted, int64_t n, int64_t n_experts, int64_t* offsets,
                   cudaStream_t stream) {
  if (n < 0 || n_experts <= 0 || !offsets || (n > 0 && !sorted))
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_expert_offsets: bad arguments");
  const int64_t work = n > 0 ? n : n_experts;
  sel::offsets_kernel<<<(unsigned)((work + 255) / 256), 256, 0, stream>>>(sorted, n, n_experts, offsets);
  return check_launch("cvmm_expert_offsets");
}

}  // namespace cvmm
