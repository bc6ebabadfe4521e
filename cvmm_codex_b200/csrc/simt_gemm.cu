// Expert-segment tile scheduler and the exact-fp32 (FFMA) GEMM engine.
//
// The fp32 engine serves op_dtype == float32, the reference's autocast-off
// path, which runs tl.dot with allow_tf32=False (cvmm.py:862 and every other
// launcher): a true fp32 dot product. sm_100 has no fp32 tensor-core MMA, so
// this path runs on the FMA pipes.
#include "gemm.cuh"
#include "launch.h"

namespace cvmm {

// ---------------------------------------------------------------- tiles
// One CTA: every thread owns a contiguous run of experts, counts their M tiles,
// and a block scan turns the counts into the write positions.
__global__ void __launch_bounds__(1024)
build_tiles_kernel(const int64_t* __restrict__ offsets, int64_t n_experts, int bm,
                   int4* __restrict__ tiles, int* __restrict__ n_tiles) {
  pdl_enter();
  const int t = threadIdx.x;
  const int64_t per = (n_experts + blockDim.x - 1) / blockDim.x;
  const int64_t e0 = min((int64_t)t * per, n_experts), e1 = min(e0 + per, n_experts);
  int cnt = 0;
  for (int64_t e = e0; e < e1; ++e) {
    int64_t len = offsets[e] - seg_begin(offsets, e);
    cnt += (int)((len + bm - 1) / bm);
  }
  __shared__ int warp_tot[32];
  const int lane = t & 31, warp = t >> 5;
  int v = cnt;
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += y;
  }
  if (lane == 31) warp_tot[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int s = lane < (int)(blockDim.x >> 5) ? warp_tot[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    warp_tot[lane] = s;
  }
  __syncthreads();
  int pos = v - cnt + (warp > 0 ? warp_tot[warp - 1] : 0);
  for (int64_t e = e0; e < e1; ++e) {
    int64_t b = seg_begin(offsets, e), end = offsets[e];
    for (int64_t r = b; r < end; r += bm, ++pos) tiles[pos] = make_int4((int)e, (int)r, (int)min((int64_t)bm, end - r), pos);
  }
  if (t == blockDim.x - 1) *n_tiles = pos;
}

int build_tiles(const int64_t* offsets, int64_t n_experts, int bm, int4* tiles, int* n_tiles,
                cudaStream_t stream) {
  launch(build_tiles_kernel, 1, 1024, 0, stream, offsets, n_experts, bm, tiles, n_tiles);
  return check_launch("build_tiles");
}

// Block-wide exclusive prefix of one int per thread (blockDim.x <= 1024).
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_tot) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  int incl = v;
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  __syncthreads();
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int s = lane < (int)(blockDim.x >> 5) ? warp_tot[lane] : 0;
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, s, o);
      if (lane >= o) s += y;
    }
    warp_tot[lane] = s;
  }
  __syncthreads();
  return incl - v + (warp > 0 ? warp_tot[warp - 1] : 0);
}

// Work units of the split-K grad-W: every expert segment is cut into chunks
// of `chunk` routes. An expert with a single chunk writes grad_w directly
// (slot -1); the chunks of a split expert write consecutive partial slots
// that seg_reduce_kernel later sums in chunk order, so the result does not
// depend on scheduling.
constexpr int kUnitSortMaxExperts = 1024;

// Builds the unit list of all experts into `units` (global or shared memory;
// room for max_row_tiles(n_routes, n_experts, chunk) entries) with every
// thread of the block, writes expert_slots when non-null, and returns the
// number of units in every thread. tail_len: n_experts ints of scratch (used
// up to kUnitSortMaxExperts experts), scratch: 34 ints. Ends with a barrier,
// so shared-memory units are visible to the whole block on return.
__device__ __noinline__ int build_unit_list(const int64_t* __restrict__ offsets, int64_t n_experts, int64_t chunk,
                                            int4* units, int2* __restrict__ expert_slots, int* tail_len,
                                            int* scratch) {
  int* warp_tot = scratch;
  const int t = threadIdx.x;
  const int64_t per = (n_experts + blockDim.x - 1) / blockDim.x;
  const int64_t e0 = min((int64_t)t * per, n_experts), e1 = min(e0 + per, n_experts);
  // Full chunks of every expert come first (in expert order), then the
  // shorter tail chunks, longest first (for up to kUnitSortMaxExperts
  // experts; expert order otherwise): CTAs take units round-robin, so this
  // longest-first order spreads the long units evenly over the CTAs. Slots of
  // split experts are numbered per expert in chunk order whatever the
  // emission order, so seg_reduce's fixed summation order is unchanged.
  const bool sort_tails = n_experts <= kUnitSortMaxExperts;
  int full = 0, tails = 0, slots = 0;
  for (int64_t e = e0; e < e1; ++e) {
    const int64_t len = offsets[e] - seg_begin(offsets, e);
    const int nch = (int)((len + chunk - 1) / chunk);
    full += (int)(len / chunk);
    tails += (len % chunk) != 0;
    if (nch > 1) slots += nch;
    if (sort_tails) tail_len[e] = (int)(len % chunk);
  }
  int fpos = block_exclusive_scan(full, warp_tot);
  int tpos = block_exclusive_scan(tails, warp_tot);
  int sbase = block_exclusive_scan(slots, warp_tot);
  if (t == blockDim.x - 1) {
    scratch[32] = fpos + full;
    scratch[33] = tpos + tails;
  }
  __syncthreads();
  const int n_full = scratch[32], n_total = n_full + scratch[33];
  for (int64_t e = e0; e < e1; ++e) {
    const int64_t b = seg_begin(offsets, e), end = offsets[e];
    const int nch = (int)((end - b + chunk - 1) / chunk);
    if (expert_slots) expert_slots[e] = make_int2(nch > 1 ? sbase : -1, nch);
    int c = 0;
    for (int64_t r = b; r < end; r += chunk, ++c) {
      const int4 u = make_int4((int)e, (int)r, nch > 1 ? sbase + c : -1, (int)min(r + chunk, end));
      if (r + chunk <= end) {
        units[fpos++] = u;
      } else {
        int rank = tpos;
        if (sort_tails) {  // tails longer than this one, ties by expert id
          const int L = (int)(end - r);
          rank = 0;
          for (int64_t f = 0; f < n_experts; ++f) rank += tail_len[f] > L || (tail_len[f] == L && f < e);
        }
        units[n_full + rank] = u;
        ++tpos;
      }
    }
    if (nch > 1) sbase += nch;
  }
  __syncthreads();
  return n_total;
}

__global__ void __launch_bounds__(1024)
build_units_kernel(const int64_t* __restrict__ offsets, int64_t n_experts, int64_t chunk,
                   int4* __restrict__ units, int* __restrict__ n_units, int2* __restrict__ expert_slots) {
  pdl_enter();
  __shared__ int scratch[34];
  __shared__ int tail_len[kUnitSortMaxExperts];  // each expert's tail chunk length (0: none)
  const int n = build_unit_list(offsets, n_experts, chunk, units, expert_slots, tail_len, scratch);
  if (threadIdx.x == 0) *n_units = n;
}

int build_units(const int64_t* offsets, int64_t n_experts, int64_t chunk, int4* units, int* n_units,
                int2* expert_slots, cudaStream_t stream) {
  launch(build_units_kernel, 1, 1024, 0, stream, offsets, n_experts, chunk, units, n_units, expert_slots);
  return check_launch("build_units");
}

// x row, grad row and op-rounded weight of every sorted route (for the
// tensor-core grad-W, whose index warp bulk-copies them into shared memory).
__global__ void resolve_route_rows_kernel(SegGemm p, int* __restrict__ xrow, int* __restrict__ grow,
                                          float* __restrict__ wsc, int64_t padded) {
  pdl_enter();
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < padded; r += (int64_t)gridDim.x * blockDim.x) {
    const bool ok = r < p.n_routes;
    int64_t lo = 0;  // expert of sorted position r (padded layouts): first e with offsets[e] > r
    if (p.x_pad_start || p.g_pad_start) {
      int64_t hi = p.n_experts - 1;
      while (ok && lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if (p.offsets[mid] > r) hi = mid; else lo = mid + 1;
      }
    }
    const int padded_row = ok ? (int)(r - seg_begin(p.offsets, lo)) : 0;
    if (p.x_pad_start) xrow[r] = ok ? p.x_pad_start[lo] + padded_row : -1;
    else xrow[r] = ok ? (int)idx_div(p.x_index[r], p.x_div) : -1;
    if (p.g_pad_start) grow[r] = ok ? p.g_pad_start[lo] + padded_row : -1;
    else grow[r] = ok ? (int)idx_div(p.g_index[r], p.g_div) : -1;
    if (p.w) wsc[r] = ok ? round_to(load_as_float(p.w, p.w_dtype, p.w_index[r]), p.op_dtype) : 0.f;
  }
}

int resolve_route_rows(const SegGemm& p, int* xrow, int* grow, float* wsc, cudaStream_t stream) {
  const int64_t padded = p.n_routes + kRouteRowsPad;
  const int grid = (int)std::min<int64_t>((padded + 255) / 256, 148 * 8);
  launch(resolve_route_rows_kernel, grid, 256, 0, stream, p, xrow, grow, wsc, padded);
  return check_launch("resolve_route_rows");
}

// pad_start[e] = sum over e' < e of round_up(count(e'), pad): one CTA scan.
// Counts and pad starts are below 2^31 (checked by the callers): 32-bit math.
__global__ void __launch_bounds__(512)
pad_starts_kernel(const int64_t* __restrict__ offsets, int64_t n_experts, int64_t pad, int* __restrict__ pad_start) {
  pdl_enter();
  __shared__ int warp_tot[32];
  const int t = threadIdx.x, n = (int)n_experts, pd = (int)pad;
  const int per = (n + (int)blockDim.x - 1) / (int)blockDim.x;
  const int e0 = min(t * per, n), e1 = min(e0 + per, n);
  auto padded = [&](int e) {
    const int c = (int)(offsets[e] - (e > 0 ? offsets[e - 1] : 0));
    return (c + pd - 1) / pd * pd;
  };
  int tot = 0;
  for (int e = e0; e < e1; ++e) tot += padded(e);
  int run = block_exclusive_scan(tot, warp_tot);
  for (int e = e0; e < e1; ++e) {
    pad_start[e] = run;
    run += padded(e);
  }
}

int pad_starts(const int64_t* offsets, int64_t n_experts, int64_t pad, int* pad_start, cudaStream_t stream) {
  launch(pad_starts_kernel, 1, 512, 0, stream, offsets, n_experts, pad, pad_start);
  return check_launch("pad_starts");
}

// Eight consecutive elements as fp32 (16-byte aligned source).
__device__ __forceinline__ void load8(const char* from, int dtype, float (&v)[8]) {
  if (dtype == F32) {
    const float4 a = reinterpret_cast<const float4*>(from)[0], b = reinterpret_cast<const float4*>(from)[1];
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    return;
  }
  const uint4 q = *reinterpret_cast<const uint4*>(from);
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = bits_to_float((uint16_t)(w[i] & 0xffffu), dtype);
    v[2 * i + 1] = bits_to_float((uint16_t)(w[i] >> 16), dtype);
  }
}

__device__ __forceinline__ void store8(char* to, int dtype, const float (&v)[8]) {
  if (dtype == F32) {
    reinterpret_cast<float4*>(to)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(to)[1] = make_float4(v[4], v[5], v[6], v[7]);
    return;
  }
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w[i] = pack2(v[2 * i], v[2 * i + 1], dtype);
  *reinterpret_cast<uint4*>(to) = make_uint4(w[0], w[1], w[2], w[3]);
}

// Expert-padded sorted copy. Virtual rows [0, n_routes) are the sorted routes:
// dst[pad_start[e] + p - seg_begin(e)] = op(src[index[p] / div]) (times
// op(scale[index[p]]), rounded again); rows [n_routes, n_routes + n_experts *
// kPadRows) enumerate every expert's candidate padding rows, and those inside
// the expert's padded segment are zeroed.
// Each CTA owns ROWS consecutive virtual rows: thread r < ROWS resolves row
// r's source, destination and scale (one round of dependent index loads for
// all rows, in parallel), then the CTA's 256 threads stream the rows' chunks
// with kSortBatch loads in flight per thread before converting and storing.
// Short rows (<= 512 bytes) take 128 rows per CTA, so that the index round
// is paid once per 32 KiB or more instead of once per 8 KiB.
// MODE 0: 16-byte copy (same dtype, no scale), 1: 8-element vectors with
// conversion (and scale), 2: scalar elements, 3: 16-byte chunks of one 16-bit
// dtype with the scale applied in registers (the weighted grad copy).
constexpr int kSortBatch = 8;

struct SortRowMeta {
  long long src;  // source element offset of the row, -1: zero row
  long long dst;  // destination element offset, -1: no row
  float scale;
  int pad;
};

template <int MODE, int ROWS>
__global__ void __launch_bounds__(256) sort_rows_padded_kernel(
    const char* __restrict__ src, int src_dtype, int64_t src_ld, const int64_t* __restrict__ index, int64_t div,
    const void* __restrict__ scale, int scale_dtype, const int32_t* __restrict__ sorted_sel,
    const int64_t* __restrict__ offsets, const int* __restrict__ pad_start, int64_t n_routes, int64_t n_experts,
    int64_t cols, char* __restrict__ dst, int dst_dtype, int32_t* __restrict__ route_rows) {
  pdl_enter();
  __shared__ SortRowMeta meta[ROWS];
  const int tid = threadIdx.x, lane = tid & 31;
  const int64_t v0 = blockIdx.x * (int64_t)ROWS;
  const int64_t total = n_routes + n_experts * kPadRows;
  if (tid < ROWS) {
    const int64_t v = v0 + tid;
    SortRowMeta m = {-1, -1, 1.f, 0};
    if (v < n_routes) {
      const int64_t r = index[v];
      const int64_t e = sorted_sel[v];
      m.src = idx_div(r, div) * src_ld;
      const int64_t row = pad_start[e] + v - seg_begin(offsets, e);
      m.dst = row * cols;
      if (route_rows) route_rows[r] = (int32_t)row;
      if (scale) m.scale = round_to(load_as_float(scale, scale_dtype, r), dst_dtype);
    } else if (v < total) {
      const int64_t e = (v - n_routes) / kPadRows, i = (v - n_routes) % kPadRows;
      const int64_t cnt = offsets[e] - seg_begin(offsets, e);
      if (cnt + i < (cnt + kPadRows - 1) / kPadRows * kPadRows) m.dst = (pad_start[e] + cnt + i) * cols;
    }
    meta[tid] = m;
  }
  __syncthreads();
  const int ssz = dtype_bytes(src_dtype), dsz = dtype_bytes(dst_dtype);
  if (MODE == 2) {
    for (int rr = tid >> 5; rr < ROWS; rr += blockDim.x >> 5) {
      const SortRowMeta m = meta[rr];
      if (m.dst < 0) continue;
      for (int64_t c = lane; c < cols; c += 32) {
        float x = m.src < 0 ? 0.f : round_to(load_as_float(src, src_dtype, m.src + c), dst_dtype);
        if (scale && m.src >= 0) x = x * m.scale;
        store_from_float(dst, dst_dtype, m.dst + c, x);
      }
    }
    return;
  }
  // Work items: (row, 8-element chunk) pairs; MODE 0 / 3 move 16-byte chunks.
  const int64_t per_row = (MODE == 0 || MODE == 3) ? cols * dsz / 16 : cols / 8;
  const int64_t items = ROWS * per_row;
  const uint32_t pr = (uint32_t)per_row;  // items < 2^32: 32-bit row / chunk split
  constexpr int kBatch = (MODE == 0 || MODE == 3) ? kSortBatch : kSortBatch / 2;
  for (int64_t base = 0; base < items; base += (int64_t)blockDim.x * kBatch) {
    if (MODE == 3) {
      // Same 16-bit dtype in and out, scaled: 16-byte loads, the 8 values
      // times the op-rounded route weight in fp32, rounded once (as MODE 1).
      uint4 buf[kSortBatch];
#pragma unroll
      for (int u = 0; u < kSortBatch; ++u) {
        const int64_t it = base + tid + (int64_t)blockDim.x * u;
        buf[u] = make_uint4(0, 0, 0, 0);
        if (it < items) {
          const SortRowMeta& m = meta[(uint32_t)it / pr];
          if (m.dst >= 0 && m.src >= 0)
            buf[u] = reinterpret_cast<const uint4*>(src + m.src * ssz)[(uint32_t)it % pr];
        }
      }
#pragma unroll
      for (int u = 0; u < kSortBatch; ++u) {
        const int64_t it = base + tid + (int64_t)blockDim.x * u;
        if (it >= items) continue;
        const SortRowMeta& m = meta[(uint32_t)it / pr];
        if (m.dst < 0) continue;
        uint32_t w[4] = {buf[u].x, buf[u].y, buf[u].z, buf[u].w};
#pragma unroll
        for (int h = 0; h < 4; ++h)
          w[h] = pack2(bits_to_float((uint16_t)(w[h] & 0xffffu), dst_dtype) * m.scale,
                       bits_to_float((uint16_t)(w[h] >> 16), dst_dtype) * m.scale, dst_dtype);
        reinterpret_cast<uint4*>(dst + m.dst * dsz)[(uint32_t)it % pr] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    } else if (MODE == 0) {
      uint4 buf[kSortBatch];
#pragma unroll
      for (int u = 0; u < kSortBatch; ++u) {
        const int64_t it = base + tid + (int64_t)blockDim.x * u;
        buf[u] = make_uint4(0, 0, 0, 0);
        if (it < items) {
          const SortRowMeta& m = meta[(uint32_t)it / pr];
          if (m.dst >= 0 && m.src >= 0)
            buf[u] = reinterpret_cast<const uint4*>(src + m.src * ssz)[(uint32_t)it % pr];
        }
      }
#pragma unroll
      for (int u = 0; u < kSortBatch; ++u) {
        const int64_t it = base + tid + (int64_t)blockDim.x * u;
        if (it < items) {
          const SortRowMeta& m = meta[(uint32_t)it / pr];
          if (m.dst >= 0) reinterpret_cast<uint4*>(dst + m.dst * dsz)[(uint32_t)it % pr] = buf[u];
        }
      }
    } else {
      constexpr int B = kBatch;
      float x[B][8];
#pragma unroll
      for (int u = 0; u < B; ++u) {
        const int64_t it = base + tid + (int64_t)blockDim.x * u;
#pragma unroll
        for (int j = 0; j < 8; ++j) x[u][j] = 0.f;
        if (it < items) {
          const SortRowMeta& m = meta[(uint32_t)it / pr];
          if (m.dst >= 0 && m.src >= 0) load8(src + (m.src + ((uint32_t)it % pr) * 8) * ssz, src_dtype, x[u]);
        }
      }
#pragma unroll
      for (int u = 0; u < B; ++u) {
        const int64_t it = base + tid + (int64_t)blockDim.x * u;
        if (it >= items) continue;
        const SortRowMeta& m = meta[(uint32_t)it / pr];
        if (m.dst < 0) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          // Values already in dst_dtype need no re-rounding (identity).
          if (src_dtype != dst_dtype) x[u][j] = round_to(x[u][j], dst_dtype);
          if (scale) x[u][j] = x[u][j] * m.scale;
        }
        store8(dst + (m.dst + ((uint32_t)it % pr) * 8) * dsz, dst_dtype, x[u]);
      }
    }
  }
}

// Wide rows (>= 1 KiB, one 16-bit dtype, MODE 0 copy or MODE 3 scaled): one
// warp per row, rows strided over a grid of resident warps. Every lane
// resolves the row's source, destination and scale (the same addresses, one
// transaction), the next row's metadata is loaded before the current row is
// copied, and each lane keeps 4 x 16 bytes of the row in flight. The CTA-per-32
// -rows kernel spent most of its time on its per-CTA index round at these row
// lengths (the weight-scaled grad copy of ff_down moved 284 MB in 60 us).
template <int MODE>
__global__ void __launch_bounds__(256) sort_rows_wide_kernel(
    const char* __restrict__ src, int64_t src_ld, const int64_t* __restrict__ index, int64_t div,
    const void* __restrict__ scale, int scale_dtype, const int32_t* __restrict__ sorted_sel,
    const int64_t* __restrict__ offsets, const int* __restrict__ pad_start, int64_t n_routes, int64_t n_experts,
    int64_t cols, char* __restrict__ dst, int dtype, int32_t* __restrict__ route_rows) {
  pdl_enter();
  const int lane = threadIdx.x & 31;
  const int64_t nw = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t total = n_routes + n_experts * kPadRows;
  const int cpr = (int)(cols / 8);  // 16-byte chunks per row
  auto meta = [&](int64_t v) {
    SortRowMeta m = {-1, -1, 1.f, 0};
    if (v < n_routes) {
      const int64_t r = index[v];
      const int64_t e = sorted_sel[v];
      m.src = idx_div(r, div) * src_ld;
      const int64_t row = pad_start[e] + v - seg_begin(offsets, e);
      m.dst = row * cols;
      if (route_rows) route_rows[r] = (int32_t)row;
      if (MODE == 3) m.scale = round_to(load_as_float(scale, scale_dtype, r), dtype);
    } else if (v < total) {
      const int64_t e = (v - n_routes) / kPadRows, i = (v - n_routes) % kPadRows;
      const int64_t cnt = offsets[e] - seg_begin(offsets, e);
      if (cnt + i < (cnt + kPadRows - 1) / kPadRows * kPadRows) m.dst = (pad_start[e] + cnt + i) * cols;
    }
    return m;
  };
  int64_t v = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  SortRowMeta m = meta(v);
  for (; v < total; v += nw) {
    const SortRowMeta nxt = meta(v + nw);
    if (m.dst >= 0) {
      const uint4* s4 = reinterpret_cast<const uint4*>(src + m.src * 2);
      uint4* d4 = reinterpret_cast<uint4*>(dst + m.dst * 2);
      for (int c0 = 0; c0 < cpr; c0 += 128) {
        uint4 buf[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = c0 + lane + 32 * j;
          buf[j] = (c < cpr && m.src >= 0) ? s4[c] : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = c0 + lane + 32 * j;
          if (c >= cpr) continue;
          if (MODE == 3) {
            uint32_t w[4] = {buf[j].x, buf[j].y, buf[j].z, buf[j].w};
#pragma unroll
            for (int h = 0; h < 4; ++h)
              w[h] = pack2(bits_to_float((uint16_t)(w[h] & 0xffffu), dtype) * m.scale,
                           bits_to_float((uint16_t)(w[h] >> 16), dtype) * m.scale, dtype);
            buf[j] = make_uint4(w[0], w[1], w[2], w[3]);
          }
          d4[c] = buf[j];
        }
      }
    }
    m = nxt;
  }
}

int sort_rows_padded(const void* src, int src_dtype, int64_t src_ld, const int64_t* index, int64_t div,
                     const void* scale, int scale_dtype, const int32_t* sorted_sel, const int64_t* offsets,
                     const int* pad_start, int64_t n_routes, int64_t n_experts, int64_t cols, void* dst,
                     int dst_dtype, cudaStream_t stream, int32_t* route_rows) {
  const int ssz = dtype_bytes(src_dtype), dsz = dtype_bytes(dst_dtype);
  const bool aligned = ((cols * ssz) % 16 == 0) && ((src_ld * ssz) % 16 == 0) && ((cols * dsz) % 16 == 0) &&
                       (((uintptr_t)src & 15u) == 0) && (((uintptr_t)dst & 15u) == 0) && cols % 8 == 0;
  const int64_t rows = n_routes + n_experts * kPadRows;
  const bool same16 = src_dtype == dst_dtype && dst_dtype != F32;
  const int mode = !aligned ? 2 : (src_dtype == dst_dtype && scale == nullptr ? 0 : (same16 ? 3 : 1));
  const bool short_rows = mode != 2 && cols * std::max(ssz, dsz) <= 512;
  const int64_t rpc = short_rows ? 128 : 32;  // rows per CTA
  const unsigned grid = (unsigned)std::max<int64_t>((rows + rpc - 1) / rpc, 1);
  const char* s = static_cast<const char*>(src);
  char* d = static_cast<char*>(dst);
#define CVMM_SORT_LAUNCH(MODE, ROWS)                                                                              \
  launch(sort_rows_padded_kernel<MODE, ROWS>, grid, 256, 0, stream, s, src_dtype, src_ld, index, div, scale,        \
                                                                scale_dtype, sorted_sel, offsets, pad_start,      \
                                                                n_routes, n_experts, cols, d, dst_dtype, route_rows)
  const bool wide = (mode == 0 || mode == 3) && src_dtype != F32 && cols * dsz >= 1024;
  const unsigned wgrid = (unsigned)std::min<int64_t>((rows + 7) / 8, 148 * 8);
  if (wide && mode == 0)
    launch(sort_rows_wide_kernel<0>, wgrid, 256, 0, stream, s, src_ld, index, div, scale, scale_dtype, sorted_sel,
                                                        offsets, pad_start, n_routes, n_experts, cols, d, dst_dtype, route_rows);
  else if (wide)
    launch(sort_rows_wide_kernel<3>, wgrid, 256, 0, stream, s, src_ld, index, div, scale, scale_dtype, sorted_sel,
                                                        offsets, pad_start, n_routes, n_experts, cols, d, dst_dtype, route_rows);
  else if (mode == 0 && short_rows) CVMM_SORT_LAUNCH(0, 128);
  else if (mode == 0) CVMM_SORT_LAUNCH(0, 32);
  else if (mode == 3 && short_rows) CVMM_SORT_LAUNCH(3, 128);
  else if (mode == 3) CVMM_SORT_LAUNCH(3, 32);
  else if (mode == 1 && short_rows) CVMM_SORT_LAUNCH(1, 128);
  else if (mode == 1) CVMM_SORT_LAUNCH(1, 32);
  else CVMM_SORT_LAUNCH(2, 32);
#undef CVMM_SORT_LAUNCH
  return check_launch("sort_rows_padded");
}

// grad_w[e] = sum over the expert's partial slots in chunk order (split
// experts), or 0 for experts without routes; single-chunk experts were
// written by their unit and are skipped.
__global__ void seg_reduce_kernel(const int2* __restrict__ expert_slots, const float4* __restrict__ partials,
                                  float4* __restrict__ out, int64_t mn4) {
  pdl_enter();
  const int64_t e = blockIdx.y;
  const int2 es = expert_slots[e];
  if (es.y == 1) return;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < mn4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int c = 0; c < es.y; ++c) {
      const float4 v = partials[(int64_t)(es.x + c) * mn4 + i];
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    out[e * mn4 + i] = acc;
  }
}

__global__ void seg_reduce_scalar_kernel(const int2* __restrict__ expert_slots, const float* __restrict__ partials,
                                         float* __restrict__ out, int64_t mn) {
  pdl_enter();
  const int64_t e = blockIdx.y;
  const int2 es = expert_slots[e];
  if (es.y == 1) return;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < mn; i += (int64_t)gridDim.x * blockDim.x) {
    float acc = 0.f;
    for (int c = 0; c < es.y; ++c) acc += partials[(int64_t)(es.x + c) * mn + i];
    out[e * mn + i] = acc;
  }
}

int seg_reduce(const int2* expert_slots, const float* partials, float* out, int64_t n_experts, int64_t mn,
               cudaStream_t stream) {
  const bool vec = mn % 4 == 0 && ((uintptr_t)partials & 15u) == 0 && ((uintptr_t)out & 15u) == 0;
  const int64_t work = vec ? mn / 4 : mn;
  dim3 grid((unsigned)std::min<int64_t>((work + 255) / 256, 64), (unsigned)n_experts);
  if (vec)
    launch(seg_reduce_kernel, grid, 256, 0, stream, expert_slots, reinterpret_cast<const float4*>(partials),
                                                reinterpret_cast<float4*>(out), mn / 4);
  else
    launch(seg_reduce_scalar_kernel, grid, 256, 0, stream, expert_slots, partials, out, mn);
  return check_launch("seg_reduce");
}

// ---------------------------------------------------------------- fp32 row GEMM
namespace simt {

constexpr int TM = 64, TN = 64, TK = 16, THREADS = 256;

__global__ void __launch_bounds__(THREADS) row_gemm_kernel(RowGemm p) {
  pdl_enter();
  if ((int)blockIdx.x >= *p.n_tiles) return;
  const int4 tile = p.tiles[blockIdx.x];
  const int64_t e = tile.x, r0 = tile.y;
  const int rows = tile.z;
  const int64_t n0 = (int64_t)blockIdx.y * TN;

  __shared__ float As[TK][TM + 4];
  __shared__ float Bs[TK][TN + 4];
  const int t = threadIdx.x;
  const int ty = t >> 4, tx = t & 15;

  // A rows this thread loads: row = t/16 + 16*i, k = t%16.
  int64_t a_row[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    int rr = (t >> 4) + 16 * i;
    a_row[i] = rr < rows ? idx_div(p.a_index[r0 + rr], p.a_div) : -1;
  }
  const char* bbase = static_cast<const char*>(p.b);
  const size_t bsz = p.b_dtype == F32 ? 4 : 2;

  float acc[4][4] = {};
  for (int64_t k0 = 0; k0 < p.K; k0 += TK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int rr = (t >> 4) + 16 * i, kk = t & 15;
      float v = 0.f;
      if (a_row[i] >= 0 && k0 + kk < p.K)
        v = round_to(load_as_float(p.a, p.a_dtype, a_row[i] * p.a_ld + k0 + kk), p.op_dtype);
      As[kk][rr] = v;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int idx = t + THREADS * i;
      int kk = idx / TN, nn = idx % TN;
      float v = 0.f;
      if (k0 + kk < p.K && n0 + nn < p.N) {
        int64_t off = e * p.bs_e + (k0 + kk) * p.bs_k + (n0 + nn) * p.bs_n;
        v = round_to(load_as_float(bbase, p.b_dtype, off), p.op_dtype);
      }
      Bs[kk][nn] = v;
    }
    (void)bsz;
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int rr = ty * 4 + i;
    const bool row_ok = rr < rows;
    int64_t c_row = row_ok ? p.c_index[r0 + rr] : 0;
    float wv = 0.f, dot = 0.f;
    if (p.mode == 1 && row_ok) wv = round_to(load_as_float(p.w, p.w_dtype, c_row), p.op_dtype);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t n = n0 + tx * 4 + j;
      if (!row_ok || n >= p.N) continue;
      if (p.mode == 0) {
        store_from_float(p.c, p.c_dtype, c_row * p.c_ld + n, acc[i][j]);
      } else {
        const float a = round_to(acc[i][j], p.op_dtype);
        store_from_float(p.c, p.c_dtype, c_row * p.c_ld + n, round_to(a * wv, p.op_dtype));
        dot = fmaf(a, load_as_float(p.x, p.x_dtype, idx_div(c_row, p.x_div) * p.x_ld + n), dot);
      }
    }
    if (p.mode == 1) {
      // The 16 threads sharing `ty` form one half-warp: reduce the row's dot there.
      for (int o = 8; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      if (tx == 0 && row_ok) atomicAdd(p.gsel + c_row, dot);
    }
  }
}

// ---------------------------------------------------------------- fp32 segment GEMM
// Split-K like the tensor-core kernel: one CTA per (work unit, m tile, n tile),
// writing grad_w directly or the unit's partial slot.
__global__ void __launch_bounds__(THREADS) seg_gemm_kernel(SegGemm p) {
  pdl_enter();
  if ((int)blockIdx.x >= *p.n_units) return;
  const int4 unit = p.units[blockIdx.x];
  const int64_t e = unit.x;
  const int64_t m0 = (int64_t)blockIdx.y * TM, n0 = (int64_t)blockIdx.z * TN;
  const int64_t beg = unit.y, end = unit.w;
  float* dst_base = unit.z < 0 ? p.out + e * p.M * p.N : p.partials + (int64_t)unit.z * p.M * p.N;
  __shared__ float Xs[TK][TM + 4];
  __shared__ float Gs[TK][TN + 4];
  const int t = threadIdx.x;
  const int ty = t >> 4, tx = t & 15;
  float acc[4][4] = {};
  for (int64_t r0 = beg; r0 < end; r0 += TK) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = t + THREADS * i;
      const int kk = idx / TM, mm = idx % TM;
      const int64_t r = r0 + kk;
      float xv = 0.f, gv = 0.f;
      if (r < end) {
        if (m0 + mm < p.M) {
          const int64_t xr = idx_div(p.x_index[r], p.x_div);
          xv = round_to(load_as_float(p.x, p.x_dtype, xr * p.x_ld + m0 + mm), p.op_dtype);
        }
        if (n0 + mm < p.N) {
          const int64_t gr = idx_div(p.g_index[r], p.g_div);
          gv = round_to(load_as_float(p.g, p.g_dtype, gr * p.g_ld + n0 + mm), p.op_dtype);
          if (p.w) {
            const float wv = round_to(load_as_float(p.w, p.w_dtype, p.w_index[r]), p.op_dtype);
            gv = round_to(gv * wv, p.op_dtype);
          }
        }
      }
      Xs[kk][mm] = xv;
      Gs[kk][mm] = gv;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < TK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = Xs[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Gs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + ty * 4 + i;
    if (m >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t n = n0 + tx * 4 + j;
      if (n < p.N) dst_base[m * p.N + n] = acc[i][j];
    }
  }
}

}  // namespace simt

int launch_row_gemm_simt(const RowGemm& p, int64_t max_tiles, cudaStream_t stream) {
  dim3 grid((unsigned)max_tiles, (unsigned)((p.N + simt::TN - 1) / simt::TN));
  launch(simt::row_gemm_kernel, grid, simt::THREADS, 0, stream, p);
  return check_launch("row_gemm_simt");
}

int launch_seg_gemm_simt(const SegGemm& p, int64_t max_units, cudaStream_t stream) {
  dim3 grid((unsigned)max_units, (unsigned)((p.M + simt::TM - 1) / simt::TM),
            (unsigned)((p.N + simt::TN - 1) / simt::TN));
  launch(simt::seg_gemm_kernel, grid, simt::THREADS, 0, stream, p);
  return check_launch("seg_gemm_simt");
}

}  // namespace cvmm
