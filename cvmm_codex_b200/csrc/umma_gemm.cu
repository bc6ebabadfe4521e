// tcgen05 (5th-generation tensor core) grouped GEMMs for bf16/fp16 arithmetic.
//
// Both kernels are warp-specialised, one output tile per CTA:
//   warps 0-3 (128 threads): producers, then epilogue. They gather operand
//     rows with 16-byte cp.async straight into the 128-byte-swizzled
//     shared-memory layout tcgen05.mma reads (zero-filling ragged edges), and
//     after the accumulator is complete read it back from TMEM (one TMEM lane
//     = one output row per thread) and store it.
//   warp 4: allocates the TMEM accumulator; its lane 0 issues tcgen05.mma
//     (M=128, N=BN, K=16 per instruction) and tcgen05.commit.
// Stages are handed over with mbarriers: full[s] (128 producer arrivals, after
// each producer's copies landed and a generic->async proxy fence) and empty[s]
// (tcgen05.commit when the MMAs reading stage s finished).
//
// Row gathering is the heart of CVMM: the A rows of a forward tile are
// x[sel_index[p]] for 128 consecutive sorted routes p of one expert, so no
// gathered copy of x is ever materialised in HBM. Tiles never straddle two
// experts (the tile scheduler cuts every expert segment into its own tiles),
// unlike the reference kernel which re-runs the K loop per expert present in
// a tile (cvmm.py:167,236-238).
//
// Every wait is bounded (ptx::mbar_wait); on a timeout the CTA records the
// failure in the device status word, stops issuing work, waits for what it
// already issued and frees its TMEM before returning.
#include <stdlib.h>

#include "gemm.cuh"
#include "launch.h"
#include "ptx.cuh"

namespace cvmm {
namespace umma {

constexpr int BM = 128;             // MMA M (TMEM lanes)
constexpr int BK = 64;              // K per stage: one 128-byte swizzle atom of bf16
constexpr int kProducers = 128;
constexpr int kThreads = 160;
constexpr uint32_t kAtomRowsBytes = 64 * 128;  // one 64-row x 128-byte MN-major atom column

// Development-only phase timestamps (compiled in with -DCVMM_TRACE; absent
// from the shipped library).
#ifdef CVMM_TRACE
__device__ unsigned long long* g_trace;
#define CVMM_TRACE_AT(slot)                                                                     \
  do {                                                                                        \
    if (g_trace) {                                                                            \
      unsigned smid;                                                                          \
      asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));                                      \
      const size_t b = blockIdx.x + (size_t)gridDim.x * (blockIdx.y + (size_t)gridDim.y * blockIdx.z); \
      g_trace[b * 10 + (slot)] = globaltimer_ns();                                            \
      g_trace[b * 10 + 9] = smid;                                                             \
    }                                                                                         \
  } while (0)
#else
#define CVMM_TRACE_AT(slot) \
  do {                      \
  } while (0)
#endif

// Wait-site tags reported with CVMM_DEV_TIMEOUT.
enum : int { kTagEmpty = 1, kTagFull = 2, kTagAccum = 3 };

template <int BN, int S, bool WEIGHTED>
struct Smem {
  static constexpr uint32_t a_bytes = BM * BK * 2;
  static constexpr uint32_t b_bytes = BN * BK * 2;
  static constexpr uint32_t stage_bytes = a_bytes + b_bytes;
  static constexpr uint32_t bars = S * stage_bytes;               // full[S], empty[S], accum
  static constexpr uint32_t misc = bars + (2 * S + 1) * 8;        // tmem slot, abort flag
  static constexpr uint32_t scales = misc + 16;                   // WEIGHTED: float[S+1][64]
  static constexpr uint32_t used = scales + (WEIGHTED ? (S + 1) * 64 * 4 : 0);
  static constexpr uint32_t alloc = used + 1024;                  // slack to align the base
};

// Byte offset of 16-byte chunk `chunk` of row `row` in a 128-byte-swizzled
// tile whose rows are 128 bytes (64 bf16) and whose 64-column atoms are
// `atom_stride` bytes apart.
__device__ __forceinline__ uint32_t swz(int row, int chunk, uint32_t atom_stride) {
  return (uint32_t)(chunk >> 3) * atom_stride + (uint32_t)(row >> 3) * 1024u +
         (uint32_t)(row & 7) * 128u + ((uint32_t)((chunk & 7) ^ (row & 7)) << 4);
}

// Copies 8 consecutive elements (columns col..col+7 of one row) into the
// 16-byte shared chunk at `dst`, converting to the op dtype; columns at or
// past `ncols` and rows with row == nullptr are zero.
__device__ __forceinline__ void load_chunk(uint32_t dst, const char* row, int64_t col,
                                           int64_t ncols, int src_dtype, int64_t col_stride,
                                           int op_dtype, bool fast, const void* safe) {
  const int64_t rem = ncols - col;
  if (fast) {
    uint32_t bytes = (row == nullptr || rem <= 0) ? 0u : (rem >= 8 ? 16u : (uint32_t)rem * 2u);
    const void* src = bytes ? (const void*)(row + col * 2) : safe;
    ptx::cp_async_16(dst, src, bytes);
    return;
  }
  uint32_t wds[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float lo = 0.f, hi = 0.f;
    if (row != nullptr) {
      if (2 * i < rem) lo = load_as_float(row, src_dtype, (col + 2 * i) * col_stride);
      if (2 * i + 1 < rem) hi = load_as_float(row, src_dtype, (col + 2 * i + 1) * col_stride);
    }
    wds[i] = (uint32_t)float_to_bits(lo, op_dtype) | ((uint32_t)float_to_bits(hi, op_dtype) << 16);
  }
  ptx::st_shared_v4(dst, wds[0], wds[1], wds[2], wds[3]);
}

__device__ __forceinline__ uint8_t* align_smem(uint8_t* p) {
  uint32_t a = ptx::smem_u32(p);
  return p + (((a + 1023u) & ~1023u) - a);
}

// Epilogue helper: 32 fp32 accumulator columns of one row -> output dtype.
__device__ __forceinline__ void store_row32(void* c, int c_dtype, int64_t off, const float* v,
                                            int ncols, bool vec) {
  if (vec && ncols == 32 && c_dtype != F32) {
    uint4* dst = reinterpret_cast<uint4*>(static_cast<char*>(c) + off * 2);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        w[i] = (uint32_t)float_to_bits(v[q * 8 + 2 * i], c_dtype) |
               ((uint32_t)float_to_bits(v[q * 8 + 2 * i + 1], c_dtype) << 16);
      dst[q] = make_uint4(w[0], w[1], w[2], w[3]);
    }
    return;
  }
  if (vec && ncols == 32 && c_dtype == F32) {
    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(c) + off);
#pragma unroll
    for (int q = 0; q < 8; ++q) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    return;
  }
#pragma unroll
  for (int j = 0; j < 32; ++j)
    if (j < ncols) store_from_float(c, c_dtype, off + j, v[j]);
}

// Multiplies this thread's G chunks of stage `j` by their route weights (kept
// in `scales`) and rounds to the op dtype: the reference multiplies the bf16
// grad row by the bf16 weight and rounds the product to bf16 before the dot
// (cvmm.py:591-599).
template <int BN, int S>
__device__ __forceinline__ void scale_rows(uint8_t* smem, const float* scales, int j, int t, int op) {
  using L = Smem<BN, S, true>;
  constexpr int GCPR = BN / 8;
  const int sj = j % S, sl = j % (S + 1);
  const int gc = t % GCPR;
  const uint32_t bj = ptx::smem_u32(smem + sj * L::stage_bytes) + L::a_bytes;
#pragma unroll
  for (int i = 0; i < BN / 16; ++i) {
    const int kr = t / GCPR + (kProducers / GCPR) * i;
    const float sc = scales[sl * 64 + kr];
    const uint32_t addr = bj + swz(kr, gc, kAtomRowsBytes);
    uint32_t w4[4];
    ptx::ld_shared_v4(addr, w4[0], w4[1], w4[2], w4[3]);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float lo = bits_to_float((uint16_t)(w4[q] & 0xffffu), op) * sc;
      const float hi = bits_to_float((uint16_t)(w4[q] >> 16), op) * sc;
      w4[q] = (uint32_t)float_to_bits(lo, op) | ((uint32_t)float_to_bits(hi, op) << 16);
    }
    ptx::st_shared_v4(addr, w4[0], w4[1], w4[2], w4[3]);
  }
}

// ============================================================ row-gathered GEMM
// flags bit0: A fast path (cp.async), bit1: B fast path, bit2: C vector stores.
template <int BN, int S, bool B_KMAJOR>
__global__ void __launch_bounds__(kThreads, 1) row_gemm_kernel(RowGemm p, int flags) {
  if ((int)blockIdx.x >= *p.n_tiles) return;
  if (threadIdx.x == 0) CVMM_TRACE_AT(0);
  using L = Smem<BN, S, false>;
  constexpr int LAG = S - 1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::bars);
  uint64_t* empty = full + S;
  uint64_t* accum = empty + S;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + L::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::misc + 4);

  const int2 tile = p.tiles[blockIdx.x];
  const int64_t e = tile.x, r0 = tile.y;
  const int rows = (int)imin64(BM, p.offsets[e] - r0);
  const int64_t n0 = (int64_t)blockIdx.y * BN;
  const int nkb = (int)((p.K + BK - 1) / BK);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool a_fast = flags & 1, b_fast = flags & 2, c_vec = flags & 4;
#ifdef CVMM_TRACE
  const bool dbg_no_mma = flags & 256, dbg_no_a = flags & 512, dbg_no_b = flags & 1024;
#else
  constexpr bool dbg_no_mma = false, dbg_no_a = false, dbg_no_b = false;
#endif
  const int op = p.op_dtype;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&full[s], kProducers);
      ptx::mbar_init(&empty[s], 1);
    }
    ptx::mbar_init(accum, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 4) {
    ptx::tmem_alloc(const_cast<uint32_t*>(tmem_slot), BN);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) CVMM_TRACE_AT(1);

  if (warp < 4) {
    const int t = threadIdx.x;
    // ---- producer: A (K-major): 128 gathered rows x 8 chunks per stage.
    const int ac = t & 7;
    const char* a_rows[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rr = (t >> 3) + 16 * i;
      a_rows[i] = rr < rows ? static_cast<const char*>(p.a) +
                                  idx_div(p.a_index[r0 + rr], p.a_div) * p.a_ld * (int64_t)dtype_bytes(p.a_dtype)
                            : nullptr;
    }
    const char* bbase = static_cast<const char*>(p.b);
    const int64_t bsz = dtype_bytes(p.b_dtype);
    // B K-major rows (n) are fixed over the K loop.
    constexpr int BKR = B_KMAJOR ? BN / 16 : 1;
    const char* b_rows[BKR];
    if (B_KMAJOR) {
#pragma unroll
      for (int i = 0; i < BKR; ++i) {
        const int64_t n = n0 + (t >> 3) + 16 * i;
        b_rows[i] = n < p.N ? bbase + (e * p.bs_e + n * p.bs_n) * bsz : nullptr;
      }
    }
    constexpr int CPR = BN / 8;  // MN-major B: 16-byte chunks per k row
    bool aborted = false;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % S;
      if (kb >= S && !ptx::mbar_wait(&empty[s], ((kb / S) - 1) & 1, kTagEmpty)) {
        *abort_flag = 1;
        aborted = true;
        break;
      }
      uint8_t* a_st = smem + s * L::stage_bytes;
      const uint32_t a_u = ptx::smem_u32(a_st), b_u = a_u + L::a_bytes;
      const int64_t k0 = (int64_t)kb * BK;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int rr = (t >> 3) + 16 * i;
        if (!dbg_no_a)
          load_chunk(a_u + swz(rr, ac, 0), a_rows[i], k0 + ac * 8, p.K, p.a_dtype, 1, op, a_fast, p.a);
      }
      if (dbg_no_b) {
      } else if (B_KMAJOR) {
#pragma unroll
        for (int i = 0; i < BKR; ++i) {
          const int nr = (t >> 3) + 16 * i;
          load_chunk(b_u + swz(nr, ac, 0), b_rows[i], k0 + ac * 8, p.K, p.b_dtype, p.bs_k, op,
                     b_fast, p.b);
        }
      } else {
        const int bc = t % CPR;
#pragma unroll
        for (int i = 0; i < BN / 16; ++i) {
          const int kr = t / CPR + (kProducers / CPR) * i;
          const int64_t k = k0 + kr;
          const char* row = k < p.K ? bbase + (e * p.bs_e + k * p.bs_k + n0 * p.bs_n) * bsz : nullptr;
          load_chunk(b_u + swz(kr, bc, kAtomRowsBytes), row, bc * 8, p.N - n0, p.b_dtype, p.bs_n,
                     op, b_fast, p.b);
        }
      }
      ptx::cp_async_commit();
      if (t == 0 && kb == 0) CVMM_TRACE_AT(2);
      if (kb >= LAG) {
        ptx::cp_async_wait<LAG>();
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(&full[(kb - LAG) % S]);
      }
    }
    if (t == 0) CVMM_TRACE_AT(3);
    ptx::cp_async_wait_all();
    ptx::fence_proxy_async_smem();
    if (!aborted)
      for (int j = max(0, nkb - LAG); j < nkb; ++j) ptx::mbar_arrive(&full[j % S]);

    // ---- epilogue: TMEM lane (32*warp + lane) holds output row rr.
    const int rr = warp * 32 + lane;
    const bool row_ok = rr < rows;
    const int64_t c_row = row_ok ? p.c_index[r0 + rr] : 0;
    const bool have_acc = nkb > 0 && ptx::mbar_wait(accum, 0, kTagAccum) && *abort_flag == 0;
    ptx::tc_fence_after();
    if (t == 0) CVMM_TRACE_AT(6);
    float wv = 0.f, dot = 0.f;
    if (p.mode == 1 && row_ok) wv = round_to(load_as_float(p.w, p.w_dtype, c_row), op);
    for (int ch = 0; ch < BN / 32; ++ch) {
      const int64_t nc = n0 + ch * 32;
      if (nc >= p.N) break;
      const int ncols = (int)imin64(32, p.N - nc);
      float v[32];
      if (have_acc) {
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(tmem + ((uint32_t)(warp * 32) << 16) + ch * 32, r);
        ptx::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
      }
      if (!row_ok || (nkb > 0 && !have_acc)) continue;
      if (p.mode == 1) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float a = round_to(v[j], op);
          if (j < ncols) dot = fmaf(a, load_as_float(p.x, p.x_dtype, c_row * p.x_ld + nc + j), dot);
          v[j] = round_to(a * wv, op);
        }
      }
      store_row32(p.c, p.c_dtype, c_row * p.c_ld + nc, v, ncols, c_vec);
    }
    if (p.mode == 1 && row_ok && (nkb == 0 || have_acc)) atomicAdd(p.gsel + c_row, dot);
  } else if (warp == 4 && lane == 0) {
    // ---- MMA issuer.
    const uint32_t idesc = ptx::instr_desc_f16(BM, BN, op == BF16, false, !B_KMAJOR);
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % S;
      if (*abort_flag || !ptx::mbar_wait(&full[s], (kb / S) & 1, kTagFull)) {
        *abort_flag = 1;
        break;
      }
      ptx::tc_fence_after();
      if (kb == 0) CVMM_TRACE_AT(4);
      const uint32_t a_u = ptx::smem_u32(smem + s * L::stage_bytes), b_u = a_u + L::a_bytes;
#pragma unroll
      for (int j = 0; j < BK / 16; ++j) {
        const uint64_t ad = ptx::smem_desc_sw128(a_u + j * 32, 16, 1024);
        const uint64_t bd = B_KMAJOR ? ptx::smem_desc_sw128(b_u + j * 32, 16, 1024)
                                     : ptx::smem_desc_sw128(b_u + j * 2048, kAtomRowsBytes, 1024);
        if (!dbg_no_mma) ptx::mma_f16(tmem, ad, bd, idesc, (kb | j) != 0 ? 1u : 0u);
      }
      ptx::mma_commit(&empty[s]);
    }
    ptx::mma_commit(accum);
    CVMM_TRACE_AT(5);
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) CVMM_TRACE_AT(7);
  if (warp == 4) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, BN);
  }
}

// ============================================================ segment GEMM (grad-W)
// Split-K over each expert segment: a work unit is (expert, chunk of at most
// p.chunk sorted routes) x (m tile) x (n tile), so a heavily loaded expert is
// spread over many CTAs instead of one CTA walking its whole segment. Partial
// sums go to per-chunk slots and are reduced in a fixed order (deterministic).
// flags bit0: X fast path, bit1: G fast path, bit2: out vector stores.
template <int BN, int S, bool WEIGHTED>
__global__ void __launch_bounds__(kThreads, 1) seg_gemm_kernel(SegGemm p, int flags) {
  if ((int)blockIdx.x >= *p.n_units) return;
  using L = Smem<BN, S, WEIGHTED>;
  constexpr int LAG = S - 1;
  constexpr int GCPR = BN / 8;            // G tile: 16-byte chunks per route row
  constexpr int GROWS = BN / 16;          // G rows per producer thread per stage
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::bars);
  uint64_t* empty = full + S;
  uint64_t* accum = empty + S;
  volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + L::misc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::misc + 4);
  float* scales = reinterpret_cast<float*>(smem + L::scales);

  const int4 unit = p.units[blockIdx.x];
  const int64_t e = unit.x;
  const int64_t beg = unit.y;
  const int64_t end = imin64(beg + p.chunk, p.offsets[e]);
  const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.z * BN;
  const int nkb = (int)((end - beg + BK - 1) / BK);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool x_fast = flags & 1, g_fast = flags & 2, o_vec = flags & 4;
  const int op = p.op_dtype;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&full[s], kProducers);
      ptx::mbar_init(&empty[s], 1);
    }
    ptx::mbar_init(accum, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
  }
  if (warp == 4) {
    ptx::tmem_alloc(const_cast<uint32_t*>(tmem_slot), BN);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    const int t = threadIdx.x;
    const char* xbase = static_cast<const char*>(p.x);
    const char* gbase = static_cast<const char*>(p.g);
    const int64_t xsz = dtype_bytes(p.x_dtype), gsz = dtype_bytes(p.g_dtype);
    const int xc = t & 15;       // X tile: 64 route rows x 16 chunks (128 m columns)
    const int gc = t % GCPR;     // G tile: 64 route rows x GCPR chunks
    // Row indices of the next stage are loaded one stage ahead so that their
    // latency overlaps the copies of the current stage.
    int64_t xi[8], gi[GROWS], wi[GROWS];
    auto fetch = [&](int kb) {
      const int64_t rb = beg + (int64_t)kb * BK;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int64_t r = rb + (t >> 4) + 8 * i;
        xi[i] = r < end ? p.x_index[r] : -1;
      }
#pragma unroll
      for (int i = 0; i < GROWS; ++i) {
        const int64_t r = rb + t / GCPR + (kProducers / GCPR) * i;
        gi[i] = r < end ? p.g_index[r] : -1;
        if (WEIGHTED) wi[i] = r < end ? p.w_index[r] : -1;
      }
    };
    if (nkb > 0) fetch(0);
    bool aborted = false;
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % S;
      bool bad = kb >= S && !ptx::mbar_wait(&empty[s], ((kb / S) - 1) & 1, kTagEmpty);
      // The weighted variant synchronises the producers below, so its abort
      // decision must be uniform across them.
      if (WEIGHTED) bad = ptx::named_bar_or(1, kProducers, bad);
      if (bad) {
        *abort_flag = 1;
        aborted = true;
        break;
      }
      const char* xrow[8];
      const char* grow[GROWS];
      float wsc[GROWS];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        xrow[i] = xi[i] >= 0 ? xbase + (idx_div(xi[i], p.x_div) * p.x_ld + m0) * xsz : nullptr;
#pragma unroll
      for (int i = 0; i < GROWS; ++i) {
        grow[i] = gi[i] >= 0 ? gbase + (idx_div(gi[i], p.g_div) * p.g_ld + n0) * gsz : nullptr;
        if (WEIGHTED) wsc[i] = wi[i] >= 0 ? round_to(load_as_float(p.w, p.w_dtype, wi[i]), op) : 0.f;
      }
      if (kb + 1 < nkb) fetch(kb + 1);
      const uint32_t a_u = ptx::smem_u32(smem + s * L::stage_bytes), b_u = a_u + L::a_bytes;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int kr = (t >> 4) + 8 * i;
        load_chunk(a_u + swz(kr, xc, kAtomRowsBytes), xrow[i], xc * 8, p.M - m0, p.x_dtype, 1, op,
                   x_fast, p.x);
      }
#pragma unroll
      for (int i = 0; i < GROWS; ++i) {
        const int kr = t / GCPR + (kProducers / GCPR) * i;
        load_chunk(b_u + swz(kr, gc, kAtomRowsBytes), grow[i], gc * 8, p.N - n0, p.g_dtype, 1, op,
                   g_fast, p.g);
        if (WEIGHTED && gc == 0) scales[(kb % (S + 1)) * 64 + kr] = wsc[i];
      }
      ptx::cp_async_commit();
      if (WEIGHTED) ptx::named_bar_sync(1, kProducers);
      if (kb >= LAG) {
        ptx::cp_async_wait<LAG>();
        if (WEIGHTED) scale_rows<BN, S>(smem, scales, kb - LAG, t, op);
        ptx::fence_proxy_async_smem();
        ptx::mbar_arrive(&full[(kb - LAG) % S]);
      }
    }
    ptx::cp_async_wait_all();
    if (WEIGHTED && !aborted)
      for (int j = max(0, nkb - LAG); j < nkb; ++j) scale_rows<BN, S>(smem, scales, j, t, op);
    ptx::fence_proxy_async_smem();
    if (!aborted)
      for (int j = max(0, nkb - LAG); j < nkb; ++j) ptx::mbar_arrive(&full[j % S]);

    // ---- epilogue: TMEM lane = m row of this expert's grad tile. A unit that
    // covers its whole expert writes grad_w; a chunk of a split expert writes
    // its partial slot (summed in order by seg_reduce).
    const int mr = warp * 32 + lane;
    const int64_t m = m0 + mr;
    const bool have_acc = nkb > 0 && ptx::mbar_wait(accum, 0, kTagAccum) && *abort_flag == 0;
    ptx::tc_fence_after();
    float* dst_base = unit.z < 0 ? p.out + e * p.M * p.N : p.partials + (int64_t)unit.z * p.M * p.N;
    if (have_acc) {
      for (int ch = 0; ch < BN / 32; ++ch) {
        const int64_t nc = n0 + ch * 32;
        if (nc >= p.N) break;
        const int ncols = (int)imin64(32, p.N - nc);
        uint32_t r[32];
        ptx::tmem_ld_32x32b_x32(tmem + ((uint32_t)(warp * 32) << 16) + ch * 32, r);
        ptx::tmem_wait_ld();
        if (m >= p.M) continue;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        store_row32(dst_base, F32, m * p.N + nc, v, ncols, o_vec);
      }
    }
  } else if (warp == 4 && lane == 0) {
    const uint32_t idesc = ptx::instr_desc_f16(BM, BN, op == BF16, true, true);
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % S;
      if (*abort_flag || !ptx::mbar_wait(&full[s], (kb / S) & 1, kTagFull)) {
        *abort_flag = 1;
        break;
      }
      ptx::tc_fence_after();
      const uint32_t a_u = ptx::smem_u32(smem + s * L::stage_bytes), b_u = a_u + L::a_bytes;
#pragma unroll
      for (int j = 0; j < BK / 16; ++j) {
        const uint64_t ad = ptx::smem_desc_sw128(a_u + j * 2048, kAtomRowsBytes, 1024);
        const uint64_t bd = ptx::smem_desc_sw128(b_u + j * 2048, kAtomRowsBytes, 1024);
        ptx::mma_f16(tmem, ad, bd, idesc, (kb | j) != 0 ? 1u : 0u);
      }
      ptx::mma_commit(&empty[s]);
    }
    ptx::mma_commit(accum);
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, BN);
  }
}

template <typename K>
static int set_smem(K kernel, uint32_t bytes) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) !=
      cudaSuccess)
    return fail_cuda("cudaFuncSetAttribute(max dynamic smem)");
  return CVMM_OK;
}

static inline bool aligned16(const void* ptr) { return ((uintptr_t)ptr & 15u) == 0; }

template <int BN, int S, bool BK_MAJOR>
static int row_launch(const RowGemm& p, int64_t max_tiles, int flags, cudaStream_t stream) {
  using L = Smem<BN, S, false>;
  auto kern = row_gemm_kernel<BN, S, BK_MAJOR>;
  int rc = set_smem(kern, L::alloc);
  if (rc) return rc;
  dim3 grid((unsigned)max_tiles, (unsigned)((p.N + BN - 1) / BN));
  kern<<<grid, kThreads, L::alloc, stream>>>(p, flags);
  return check_launch("row_gemm_umma");
}

template <int BN, int S, bool W>
static int seg_launch(const SegGemm& p, int64_t max_units, int flags, cudaStream_t stream) {
  using L = Smem<BN, S, W>;
  auto kern = seg_gemm_kernel<BN, S, W>;
  int rc = set_smem(kern, L::alloc);
  if (rc) return rc;
  dim3 grid((unsigned)max_units, (unsigned)((p.M + BM - 1) / BM), (unsigned)((p.N + BN - 1) / BN));
  kern<<<grid, kThreads, L::alloc, stream>>>(p, flags);
  return check_launch("seg_gemm_umma");
}

}  // namespace umma

#ifdef CVMM_TRACE
extern "C" int cvmm_debug_set_trace(void* buf) {
  unsigned long long* p = static_cast<unsigned long long*>(buf);
  return cudaMemcpyToSymbol(umma::g_trace, &p, sizeof(p)) == cudaSuccess ? 0 : -3;
}
#endif

int launch_row_gemm_umma(const RowGemm& p, int64_t max_tiles, cudaStream_t stream) {
  using namespace umma;
  const bool b_kmajor = p.bs_k == 1 && p.bs_n != 1;
  int flags = 0;
  if (p.a_dtype == p.op_dtype && p.a_ld % 8 == 0 && aligned16(p.a)) flags |= 1;
  if (p.b_dtype == p.op_dtype && aligned16(p.b) && p.bs_e % 8 == 0 &&
      (b_kmajor ? (p.bs_k == 1 && p.bs_n % 8 == 0) : (p.bs_n == 1 && p.bs_k % 8 == 0)))
    flags |= 2;
  if (p.c_ld % 8 == 0 && aligned16(p.c)) flags |= 4;
#ifdef CVMM_TRACE
  if (const char* e = getenv("CVMM_DBG_FLAGS")) flags |= atoi(e);
#endif
  if (p.N <= 64) {
    return b_kmajor ? row_launch<64, 6, true>(p, max_tiles, flags, stream)
                    : row_launch<64, 6, false>(p, max_tiles, flags, stream);
  } else if (p.N <= 128) {
    return b_kmajor ? row_launch<128, 4, true>(p, max_tiles, flags, stream)
                    : row_launch<128, 4, false>(p, max_tiles, flags, stream);
  }
  return b_kmajor ? row_launch<256, 4, true>(p, max_tiles, flags, stream)
                  : row_launch<256, 4, false>(p, max_tiles, flags, stream);
}

int launch_seg_gemm_umma(const SegGemm& p, int64_t max_units, cudaStream_t stream) {
  using namespace umma;
  int flags = 0;
  if (p.x_dtype == p.op_dtype && p.x_ld % 8 == 0 && aligned16(p.x)) flags |= 1;
  if (p.g_dtype == p.op_dtype && p.g_ld % 8 == 0 && aligned16(p.g)) flags |= 2;
  if (p.N % 4 == 0 && aligned16(p.out) && aligned16(p.partials)) flags |= 4;
  const bool w = p.w != nullptr;
  if (p.N <= 64) return w ? seg_launch<64, 6, true>(p, max_units, flags, stream) : seg_launch<64, 6, false>(p, max_units, flags, stream);
  if (p.N <= 128) return w ? seg_launch<128, 4, true>(p, max_units, flags, stream) : seg_launch<128, 4, false>(p, max_units, flags, stream);
  return w ? seg_launch<256, 4, true>(p, max_units, flags, stream) : seg_launch<256, 4, false>(p, max_units, flags, stream);
}

}  // namespace cvmm
