// tcgen05 (5th-generation tensor core) grouped GEMMs for bf16/fp16 arithmetic.
//
// Both kernels are persistent and warp-specialised (352 threads, one CTA per
// SM, tiles assigned round-robin):
//   warps 0-3  producers: gather the operand rows of every stage with 16-byte
//              cp.async straight into the 128-byte-swizzled shared-memory
//              layout tcgen05.mma reads (zero-filling ragged edges), then hand
//              the stage over with cp.async.mbarrier.arrive.noinc, which
//              arrives on the stage's `full` barrier when the copies land, so
//              the producers never wait for their own loads;
//   warps 4-7  epilogue: read finished accumulators from TMEM (one TMEM lane =
//              one output row per thread), convert and store them;
//   warp 8     allocates TMEM (two accumulator slots) and its lane 0 issues
//              tcgen05.mma (M=128, N=BN, K=16) and tcgen05.commit;
//   warp 9     lane 0 loads the expert-weight tiles with TMA (row GEMM) or
//              stages route rows for the grad-W index ring;
//   warp 10    lane 0 stores the gathered A tiles back as the expert-padded
//              sorted copy when the row GEMM is asked for one (forward).
// Barriers: full[s] / empty[s] per smem stage (S stages), acc_full[a] /
// acc_empty[a] per TMEM accumulator slot (2 slots), so the epilogue of tile i
// overlaps the main loop of tile i+1.
//
// Row gathering is the heart of CVMM: the A rows of a forward tile are
// x[sel_index[p]] for 128 consecutive sorted routes p of one expert, read
// straight from x. When the caller asks for it (kFlagACopy), warp 10 also
// stores those gathered tiles as the expert-padded sorted copy of x that the
// grad-W kernel reads as dense TMA boxes. Tiles never straddle two
// experts (the tile scheduler cuts every expert segment into its own tiles),
// unlike the reference kernel which re-runs the K loop per expert present in
// a tile (cvmm.py:167,236-238).
//
// Every wait is bounded; on a timeout the CTA records the failure in the
// device status word, stops issuing work, lets what it issued finish and
// frees its TMEM before returning.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdlib.h>

#include <mutex>

#include "gemm.cuh"
#include "launch.h"
#include "ptx.cuh"

namespace cvmm {
namespace umma {

constexpr int BM = 128;             // MMA M (TMEM lanes)
constexpr int BK = 64;              // K per stage: one 128-byte swizzle atom of bf16
constexpr int kProducers = 128;     // warps 0-3
constexpr int kEpilogue = 128;      // warps 4-7
constexpr int kMmaWarp = 8;
constexpr int kFlagACopy = 1 << 17;  // row GEMM: write the gathered A tiles to RowGemm::a_copy
constexpr int kLoaderWarp = 9;
constexpr int kStoreWarp = 10;  // row GEMM with an A copy: stores the gathered A tiles
constexpr int kThreads = 352;
constexpr uint32_t kAtomRowsBytes = 64 * 128;  // one 64-row x 128-byte MN-major atom column

// Development-only knobs (compiled in with -DCVMM_TRACE; absent from the
// shipped library): bit 8 skips the MMAs, bit 9 / bit 10 skip the A / B loads,
// bit 14 skips the epilogue stores, bit 15 keeps one epilogue warp group.
#ifdef CVMM_TRACE
#define CVMM_DBG(flags, bit) (((flags) & (bit)) != 0)
#else
#define CVMM_DBG(flags, bit) false
#endif

#ifdef CVMM_TRACE
// Per-stage timestamps of CTA 0: [role][stage] (roles: 0 producer t0 issued,
// 1 MMA saw full, 2 index warp published, 3 epilogue tile done).
__device__ unsigned long long* g_trace;
#define CVMM_STAMP(role, idx)                                                     \
  do {                                                                            \
    if (g_trace && blockIdx.x == 0 && (idx) < 4096) g_trace[(role) * 4096 + (idx)] = clock64(); \
  } while (0)
#else
#define CVMM_STAMP(role, idx) \
  do {                        \
  } while (0)
#endif

// Wait-site tags reported with CVMM_DEV_TIMEOUT.
enum : int { kTagEmpty = 1, kTagFull = 2, kTagAccFull = 3, kTagAccEmpty = 4, kTagDrain = 5 };

// Shared-memory plan of one CTA (offsets from a 1024-byte aligned base):
//   S operand stages (A tile 16 KiB + B tile BN x 128 B);
//   barriers: full[S] empty[S] acc_full[2] acc_empty[2] drain idx_full[S] idx_empty[S] ready[S];
//   epilogue staging (36 KiB, 1024-byte aligned): per epilogue warp either a
//   32 x 32 block (rows of 144 B; the 16-byte pad spreads the rows over the
//   shared-memory banks) or 32-row x 128-byte boxes in the 128-byte swizzle
//   that TMA stores read (two per warp with one epilogue warp group, one with two);
//   index ring (grad-W): S slots of the stage's x rows, grad rows and route
//   weights, bulk-copied from a 16-byte aligned start 0-3 entries before the
//   stage's first route (`off`).
constexpr uint32_t kStageRowBytes = 144;
constexpr uint32_t kStoreBox = 32 * 128;                  // one 32-row x 64-column 16-bit TMA store box
// Per epilogue warp: two store boxes (one warp group) or one (two groups), or
// 32 rows of kStageRowBytes.
constexpr uint32_t kStagingBytes = 8 * 32 * kStageRowBytes;
static_assert(kStagingBytes >= 8 * kStoreBox, "staging too small");
// BN = 256 tiles drained by two epilogue warp groups: two store boxes per warp (64 KiB).
constexpr uint32_t staging_bytes(int bn) { return bn >= 256 ? 16 * kStoreBox : kStagingBytes; }
static_assert(16 * kStoreBox >= kStagingBytes, "wide staging must also hold the row-transpose blocks");
constexpr int kRingEntries = 72;
constexpr int kPlanExperts = (int)kRowPlanExperts;  // experts up to which the row GEMM builds its tile table itself
struct IdxSlot {
  int x[kRingEntries];
  int g[kRingEntries];
  float w[kRingEntries];
  int off;
  int pad[3];
};

template <int BN, int S>
struct Smem {
  static constexpr uint32_t a_bytes = BM * BK * 2;
  static constexpr uint32_t b_bytes = BN * BK * 2;
  static constexpr uint32_t stage_bytes = a_bytes + b_bytes;
  static constexpr uint32_t bars = S * stage_bytes;
  static constexpr uint32_t misc = bars + (5 * S + 5) * 8;  // tmem slot, abort flag
  static constexpr uint32_t staging = (misc + 16 + 1023) / 1024 * 1024;  // swizzled TMA store boxes
  static constexpr uint32_t ring = staging + staging_bytes(BN);
  // Row GEMM tile plan built in the kernel: first tile and segment start of
  // every expert (kPlanExperts + 1 entries each) and the scan's warp totals.
  static constexpr uint32_t plan = ring + S * (uint32_t)sizeof(IdxSlot);
  static constexpr uint32_t used = plan + (2 * (kPlanExperts + 1) + 32) * 4;
  static constexpr uint32_t alloc = used + 1024;  // slack to align the base
  static_assert(alloc <= 232448, "shared memory plan exceeds 227 KiB");
  static_assert(staging % 1024 == 0 && kStageRowBytes % 16 == 0 && ring % 16 == 0, "misaligned smem region");
};

struct Bars {
  uint64_t* full;
  uint64_t* empty;
  uint64_t* accf;
  uint64_t* acce;
  uint64_t* drain;
  uint64_t* idxf;
  uint64_t* idxe;
  uint64_t* ready;
  volatile uint32_t* tmem_slot;
  volatile int* abort;
};

template <class L, int S>
__device__ __forceinline__ Bars carve_bars(uint8_t* smem) {
  Bars b;
  b.full = reinterpret_cast<uint64_t*>(smem + L::bars);
  b.empty = b.full + S;
  b.accf = b.empty + S;
  b.acce = b.accf + 2;
  b.drain = b.acce + 2;
  b.idxf = b.drain + 1;
  b.idxe = b.idxf + S;
  b.ready = b.idxe + S;
  b.tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + L::misc);
  b.abort = reinterpret_cast<volatile int*>(smem + L::misc + 4);
  return b;
}

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
    wds[i] = pack2(lo, hi, op_dtype);
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
        w[i] = pack2(v[q * 8 + 2 * i], v[q * 8 + 2 * i + 1], c_dtype);
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

// Two 32-column TMEM loads behind one wait (halves the load-latency stalls).
__device__ __forceinline__ void load_acc64(uint32_t taddr, float (&v)[64]) {
  uint32_t r0[32], r1[32];
  ptx::tmem_ld_32x32b_x32(taddr, r0);
  ptx::tmem_ld_32x32b_x32(taddr + 32, r1);
  ptx::tmem_wait_ld();
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    v[j] = __uint_as_float(r0[j]);
    v[32 + j] = __uint_as_float(r1[j]);
  }
}

__device__ __forceinline__ void load_acc32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  ptx::tmem_ld_32x32b_x32(taddr, r);
  ptx::tmem_wait_ld();
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

// Warp-cooperative store of a 32-row x 32-column block. Lane l holds row l's
// 32 accumulator values `v` and `row_off`, the element offset of the row's
// first column in `c` (-1: row not stored); `ncols` (<= 32) is warp-uniform.
// The block is transposed through the warp's staging area (32 rows of 144 B)
// so every st.global.v4 instruction writes whole row segments: 4 rows x 128 B
// for fp32 outputs, 8 rows x 64 B for 16-bit ones, instead of 32 scattered
// 16-byte pieces. Falls back to per-row stores for ragged or unaligned blocks.
__device__ __forceinline__ void warp_store_block(void* c, int c_dtype, int64_t row_off, const float* v, int ncols,
                                                 uint32_t stage, bool vec) {
  const int lane = threadIdx.x & 31;
  if (!vec || ncols != 32) {
    if (row_off >= 0) store_row32(c, c_dtype, row_off, v, ncols, false);
    return;
  }
  const uint32_t my = stage + lane * kStageRowBytes;
  if (c_dtype == F32) {
#pragma unroll
    for (int q = 0; q < 8; ++q)
      ptx::st_shared_v4(my + 16 * q, __float_as_uint(v[4 * q]), __float_as_uint(v[4 * q + 1]),
                        __float_as_uint(v[4 * q + 2]), __float_as_uint(v[4 * q + 3]));
    __syncwarp();
    const int q = lane & 7;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = (lane >> 3) + 4 * i;
      const int64_t off = __shfl_sync(0xffffffffu, row_off, r);
      uint32_t w0, w1, w2, w3;
      ptx::ld_shared_v4(stage + r * kStageRowBytes + 16 * q, w0, w1, w2, w3);
      if (off >= 0)
        *reinterpret_cast<uint4*>(static_cast<float*>(c) + off + 4 * q) = make_uint4(w0, w1, w2, w3);
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        w[i] = pack2(v[8 * q + 2 * i], v[8 * q + 2 * i + 1], c_dtype);
      ptx::st_shared_v4(my + 16 * q, w[0], w[1], w[2], w[3]);
    }
    __syncwarp();
    const int q = lane & 3;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = (lane >> 2) + 8 * i;
      const int64_t off = __shfl_sync(0xffffffffu, row_off, r);
      uint32_t w0, w1, w2, w3;
      ptx::ld_shared_v4(stage + r * kStageRowBytes + 16 * q, w0, w1, w2, w3);
      if (off >= 0)
        *reinterpret_cast<uint4*>(static_cast<char*>(c) + (off + 8 * q) * 2) = make_uint4(w0, w1, w2, w3);
    }
  }
  __syncwarp();
}

// Barrier set-up and TMEM allocation (2 accumulator slots of BN columns).
template <int BN, int S>
__device__ __forceinline__ uint32_t setup(const Bars& b, int full_count, int idxe_count = kProducers,
                                          int ready_count = 1, int epi_count = kEpilogue, int empty_count = 1) {
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&b.full[s], full_count);
      ptx::mbar_init(&b.empty[s], empty_count);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&b.accf[a], 1);
      ptx::mbar_init(&b.acce[a], epi_count);
    }
    ptx::mbar_init(b.drain, 1);
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&b.idxf[s], 1);
      ptx::mbar_init(&b.idxe[s], idxe_count);
      ptx::mbar_init(&b.ready[s], ready_count);
    }
    *b.abort = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    ptx::tmem_alloc(const_cast<uint32_t*>(b.tmem_slot), 2 * BN);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  return *b.tmem_slot;
}

// MMA issuer shared by both kernels: tile_nkb(t) gives the K stages of tile t.
template <int BN, int S, class NkbFn>
__device__ __forceinline__ void mma_loop(const Bars& b, uint64_t* consume, uint8_t* smem, uint32_t tmem,
                                         uint32_t idesc, bool a_mn, bool b_mn, int total, NkbFn tile_nkb,
                                         bool skip_mma) {
  using L = Smem<BN, S>;
  uint32_t it = 0;
  int local = 0;
  for (int tt = blockIdx.x; tt < total; tt += gridDim.x, ++local) {
    const int a = local & 1;
    if (local >= 2 && !ptx::mbar_wait_or_abort(&b.acce[a], ((local >> 1) - 1) & 1, kTagAccEmpty, b.abort))
      break;
    ptx::tc_fence_after();
    const uint32_t d = tmem + a * BN;
    const int nkb = tile_nkb(tt);
    bool ok = true;
    for (int kb = 0; kb < nkb; ++kb, ++it) {
      const int s = it % S;
      if (!ptx::mbar_wait_or_abort(&consume[s], (it / S) & 1, kTagFull, b.abort)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      CVMM_STAMP(1, it);
      ptx::fence_proxy_async_smem();
      const uint32_t a_u = ptx::smem_u32(smem + s * L::stage_bytes);
      const uint32_t b_u = a_u + L::a_bytes;
#pragma unroll
      for (int j = 0; j < BK / 16; ++j) {
        const uint64_t ad = a_mn ? ptx::smem_desc_sw128(a_u + j * 2048, kAtomRowsBytes, 1024)
                                 : ptx::smem_desc_sw128(a_u + j * 32, 16, 1024);
        const uint64_t bd = b_mn ? ptx::smem_desc_sw128(b_u + j * 2048, kAtomRowsBytes, 1024)
                                 : ptx::smem_desc_sw128(b_u + j * 32, 16, 1024);
        if (!skip_mma) ptx::mma_f16(d, ad, bd, idesc, (kb | j) != 0 ? 1u : 0u);
      }
      ptx::mma_commit(&b.empty[s]);
    }
    if (!ok) break;
    ptx::mma_commit(&b.accf[a]);
  }
  // Everything issued must finish before TMEM is released.
  ptx::mma_commit(b.drain);
  ptx::mbar_wait(b.drain, 0, kTagDrain);
}

// ============================================================ row-gathered GEMM
// flags bit0: A fast path (cp.async), bit1: B fast path (cp.async when not
// TMA), bit2: C vector stores, bit5: dense A (expert-padded layout), bit7:
// dense C (TMA stores), bit16: 16-byte x loads in the mode-1 epilogue.
// EPI2 (dense A, BN = 128): warp 9 issues the A box with the B tiles, and
// warps 0-3 become a second epilogue group: warps 4-7 drain accumulator
// columns 0-63, warps 0-3 columns 64-127 (warp w reaches TMEM lanes
// 32*(w%4)..+31), which halves the per-tile epilogue time that otherwise
// bounds the short-K shapes.
// ACT: the GELU epilogue (RowGemm::act), compiled only into the variants that
// use it, so the other variants keep their register allocation.
template <int BN, int S, bool B_KMAJOR, bool B_TMA, bool A_TMA, bool EPI2 = false, bool ACT = false>
__global__ void __launch_bounds__(kThreads, 1)
row_gemm_kernel(const RowGemm p, const __grid_constant__ CUtensorMap tmap_b,
                const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_c, int flags,
                int n_n) {
  static_assert(!A_TMA || B_TMA, "TMA row gathers are used together with TMA weight tiles");
  static_assert(!EPI2 || (A_TMA && (BN == 128 || BN == 256)), "two epilogue groups need dense TMA A tiles and BN >= 128");
  // Store boxes per epilogue warp: two (alternating) unless the two groups share a 128-column tile.
  constexpr int kBoxes = (EPI2 && BN == 128) ? 1 : 2;
  using L = Smem<BN, S>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem(smem_raw);
  const Bars bar = carve_bars<L, S>(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Tile table: 128-route M tiles of every expert segment, in expert order.
  // Without a table from the host (p.tiles == nullptr, at most kPlanExperts
  // experts) every CTA derives it from the offsets: tstart[e] = first tile of
  // expert e, sbeg[e] = its first sorted route (sbeg[E] = n_routes).
  int* tstart = reinterpret_cast<int*>(smem + L::plan);
  int* sbeg = tstart + kPlanExperts + 1;
  pdl_wait();  // before the first global access (the offsets below)
  const bool own_tiles = p.tiles == nullptr;
  const int n_exp = (int)p.n_experts;
  if (own_tiles) {
    const int per = (n_exp + (int)blockDim.x - 1) / (int)blockDim.x;
    const int e0 = min((int)threadIdx.x * per, n_exp), e1 = min(e0 + per, n_exp);
    int cnt = 0;
    for (int e = e0; e < e1; ++e) cnt += (int)((p.offsets[e] - seg_begin(p.offsets, e) + BM - 1) / BM);
    int run = block_exclusive_scan(cnt, sbeg + kPlanExperts + 1);
    for (int e = e0; e < e1; ++e) {
      const int64_t b = seg_begin(p.offsets, e);
      tstart[e] = run;
      sbeg[e] = (int)b;
      run += (int)((p.offsets[e] - b + BM - 1) / BM);
    }
    if (threadIdx.x == blockDim.x - 1) {
      tstart[n_exp] = run;
      sbeg[n_exp] = (int)p.offsets[n_exp - 1];
    }
    __syncthreads();
  }
  const int total = (own_tiles ? tstart[n_exp] : *p.n_tiles) * n_n;
  const uint32_t tmem = setup<BN, S>(bar, EPI2 ? 1 : (A_TMA ? 2 : kProducers + (B_TMA ? 1 : 0)), kProducers, 1,
                                     EPI2 ? 2 * kEpilogue : kEpilogue, (flags & kFlagACopy) ? 2 : 1);
  const int nkb = (int)((p.K + BK - 1) / BK);
  const int op = p.op_dtype;
  const bool a_fast = flags & 1, b_fast = flags & 2, c_vec = flags & 4;

  auto entry = [&](int tt) -> int4 {
    if (tt >= total) return make_int4(0, 0, 0, 0);
    const int m = tt / n_n;
    if (!own_tiles) return p.tiles[m];
    int lo = 0, hi = n_exp - 1;  // last expert with tstart[e] <= m (its tiles hold m)
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tstart[mid] <= m) lo = mid; else hi = mid - 1;
    }
    const int r0 = sbeg[lo] + BM * (m - tstart[lo]);
    return make_int4(lo, r0, min(BM, sbeg[lo + 1] - r0), m);
  };
  // A row (before a_div) of tile row rr: gathered index, or the row of the
  // expert-padded sorted layout.
  static_assert(BM == kPadRows, "padded rows follow from 128-row tile indices");
  auto a_row_of = [&](const int4& en, int rr) -> int {
    if (p.a_pad_start) return (int)kPadRows * en.w + rr;
    return (int)p.a_index[en.y + rr];
  };
  const bool a_dense = flags & 32;

  if (!EPI2 && A_TMA && warp < 4) {
    // ------------------------------------------------------------ A rows by TMA gather4
    // Warp 0: lane l gathers rows 4l..4l+3 of every tile, 4 rows x 128 bytes
    // per instruction, straight into the K-major swizzled A stage.
    if (warp == 0) {
      auto rows_of = [&](const int4& en, int (&r)[4]) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int rr = 4 * lane + q;
          r[q] = rr < en.z ? (int)idx_div(a_row_of(en, rr), p.a_div) : -1;
        }
      };
      int4 ent = entry(blockIdx.x);
      int rows[4], rows_next[4];
      rows_of(ent, rows);
      int4 ent_next = entry(blockIdx.x + gridDim.x);
      uint32_t it = 0;
      bool aborted = false;
      for (int tt = blockIdx.x; tt < total && !aborted; tt += gridDim.x) {
        rows_of(ent_next, rows_next);
        const int4 ent_after = entry(tt + 2 * gridDim.x);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % S;
          if (it >= S && !ptx::mbar_wait_or_abort(&bar.empty[s], ((it / S) - 1) & 1, kTagEmpty, bar.abort)) {
            aborted = true;
            break;
          }
          const uint32_t a_u = ptx::smem_u32(smem + s * L::stage_bytes);
          if (lane == 0) {
            if (CVMM_DBG(flags, 512)) ptx::mbar_arrive(&bar.full[s]);
            else ptx::mbar_arrive_expect_tx(&bar.full[s], L::a_bytes);
          }
          __syncwarp();
          if (CVMM_DBG(flags, 512)) {
          } else if (a_dense) {
            // Expert-padded sorted rows: the 128-row A tile is one dense box.
            if (lane == 0) ptx::tma_load_2d(a_u, &tmap_a, &bar.full[s], kb * BK, rows[0]);
          } else if (!CVMM_DBG(flags, 512)) {
            ptx::tma_gather4(a_u + lane * 512, &tmap_a, &bar.full[s], kb * BK, rows[0], rows[1], rows[2], rows[3]);
          }
        }
        ent = ent_next;
        ent_next = ent_after;
#pragma unroll
        for (int q = 0; q < 4; ++q) rows[q] = rows_next[q];
      }
    }
  } else if (!EPI2 && warp < 4) {
    // ------------------------------------------------------------ producers
    const int t = threadIdx.x;
    const int ac = t & 7;
    const int64_t asz = dtype_bytes(p.a_dtype);
    const char* bbase = static_cast<const char*>(p.b);
    const int64_t bsz = dtype_bytes(p.b_dtype);
    // Row indices of the next tile are loaded during the current one, and the
    // tile entry two tiles ahead, so tile changes do not stall on index loads.
    // Indices are below 2^31 (checked by the launcher): 32-bit registers.
    int4 ent = entry(blockIdx.x);
    int idx[8], idx_next[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rr = (t >> 3) + 16 * i;
      idx[i] = rr < ent.z ? a_row_of(ent, rr) : -1;
    }
    int4 ent_next = entry(blockIdx.x + gridDim.x);
    uint32_t it = 0;
    bool aborted = false;
    for (int tt = blockIdx.x; tt < total && !aborted; tt += gridDim.x) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int rr = (t >> 3) + 16 * i;
        idx_next[i] = rr < ent_next.z ? a_row_of(ent_next, rr) : -1;
      }
      const int4 ent_after = entry(tt + 2 * gridDim.x);
      const int64_t e = ent.x;
      const int64_t n0 = (int64_t)(tt % n_n) * BN;
      const char* a_rows[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        a_rows[i] = idx[i] >= 0 ? static_cast<const char*>(p.a) + idx_div(idx[i], p.a_div) * p.a_ld * asz : nullptr;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % S;
        if (it >= S && !ptx::mbar_wait_or_abort(&bar.empty[s], ((it / S) - 1) & 1, kTagEmpty, bar.abort)) {
          aborted = true;
          break;
        }
        const uint32_t a_u = ptx::smem_u32(smem + s * L::stage_bytes), b_u = a_u + L::a_bytes;
        const int64_t k0 = (int64_t)kb * BK;
        if (!CVMM_DBG(flags, 512)) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int rr = (t >> 3) + 16 * i;
            load_chunk(a_u + swz(rr, ac, 0), a_rows[i], k0 + ac * 8, p.K, p.a_dtype, 1, op, a_fast, p.a);
          }
        }
        if (!B_TMA && !CVMM_DBG(flags, 1024)) {
          if (B_KMAJOR) {
#pragma unroll
            for (int i = 0; i < BN / 16; ++i) {
              const int nr = (t >> 3) + 16 * i;
              const int64_t n = n0 + nr;
              const char* row = n < p.N ? bbase + (e * p.bs_e + n * p.bs_n) * bsz : nullptr;
              load_chunk(b_u + swz(nr, ac, 0), row, k0 + ac * 8, p.K, p.b_dtype, p.bs_k, op, b_fast, p.b);
            }
          } else {
            constexpr int CPR = BN / 8;
            const int bc = t % CPR;
#pragma unroll
            for (int i = 0; i < BN / 16; ++i) {
              const int kr = t / CPR + (kProducers / CPR) * i;
              const int64_t k = k0 + kr;
              const char* row = k < p.K ? bbase + (e * p.bs_e + k * p.bs_k + n0 * p.bs_n) * bsz : nullptr;
              load_chunk(b_u + swz(kr, bc, kAtomRowsBytes), row, bc * 8, p.N - n0, p.b_dtype, p.bs_n, op,
                         b_fast, p.b);
            }
          }
        }
        if (!a_fast || (!B_TMA && !b_fast)) ptx::fence_proxy_async_smem();
        ptx::cp_async_arrive_noinc(&bar.full[s]);
        if (t == 0) CVMM_STAMP(0, it);
      }
      ent = ent_next;
      ent_next = ent_after;
#pragma unroll
      for (int i = 0; i < 8; ++i) idx[i] = idx_next[i];
    }
    ptx::cp_async_wait_all();
  } else if (warp < 8) {
    // ------------------------------------------------------------ epilogue
    const int ew = warp & 3;                                // TMEM lane quadrant
    const int c_lo = EPI2 ? (warp < 4 ? BN / 2 : 0) : 0;    // this warp's accumulator columns
    const int c_hi = EPI2 ? c_lo + BN / 2 : BN;
    const bool stamper = warp == 4 && lane == 0;
    const int rr = ew * 32 + lane;
    const uint32_t stage = ptx::smem_u32(smem + L::staging) + (EPI2 ? warp : ew) * 32 * kStageRowBytes;
    // Dense C (expert-padded sorted output): each 32-row x 64-column block is
    // written to a swizzled box of the warp and stored by TMA.
    const bool c_dense = flags & 128;
    const uint32_t cbox = ptx::smem_u32(smem + L::staging) + (EPI2 ? warp : ew) * kBoxes * kStoreBox;
    int cbuf = 0;
    auto crow_of = [&](const int4& en) -> int64_t {
      return (c_dense || rr >= en.z) ? -1 : p.c_index[en.y + rr];
    };
    int4 ent = entry(blockIdx.x);
    int64_t crow = crow_of(ent);
    int4 ent_next = entry(blockIdx.x + gridDim.x);
    int local = 0;
    // Mode 1 reads the route's x row for the sel-weight dot product: 64
    // columns as eight 16-byte loads, issued ahead of the accumulator they
    // pair with (x_vec: 16-bit x with 16-byte aligned rows).
    const bool x_vec = p.mode == 1 && (flags & 65536);
    uint4 xr[8];
    auto load_x = [&](int64_t row, int64_t col0) {
      if (!x_vec || row < 0 || col0 + 64 > p.N) return;
      const uint4* src =
          reinterpret_cast<const uint4*>(static_cast<const char*>(p.x) + (idx_div(row, p.x_div) * p.x_ld + col0) * 2);
#pragma unroll
      for (int q = 0; q < 8; ++q) xr[q] = src[q];
    };
    for (int tt = blockIdx.x; tt < total; tt += gridDim.x, ++local) {
      const int64_t crow_next = crow_of(ent_next);
      const int4 ent_after = entry(tt + 2 * gridDim.x);
      const int a = local & 1;
      const int64_t n0 = (int64_t)(tt % n_n) * BN;
      load_x(crow, n0 + c_lo);
      if (!ptx::mbar_wait_or_abort(&bar.accf[a], (local >> 1) & 1, kTagAccFull, bar.abort)) break;
      ptx::tc_fence_after();
      if (stamper) CVMM_STAMP(2, local);
      const bool row_ok = crow >= 0;
      float wv = 0.f, dot = 0.f;
      if (p.mode == 1 && row_ok) wv = round_to(load_as_float(p.w, p.w_dtype, crow), op);
      const int prow0 = (int)kPadRows * ent.w + ew * 32;  // dense C: this warp's first padded row
      // The accumulator is handed back to the MMA warp as soon as this warp
      // has read its last columns out of TMEM, before converting and storing
      // them, so the next-but-one tile's MMAs start one chunk earlier.
      const int ch_end = min(c_hi / 64, (int)((p.N - n0 + 63) / 64));
      bool released = false;
      for (int ch = c_lo / 64; ch < c_hi / 64; ++ch) {
        if (n0 + ch * 64 >= p.N) break;
        if (ch > c_lo / 64) load_x(crow, n0 + ch * 64);
        const bool xv_ok = x_vec && n0 + ch * 64 + 64 <= p.N;
        float v2[64];
        load_acc64(tmem + ((uint32_t)(ew * 32) << 16) + a * BN + ch * 64, v2);
        if (ch == ch_end - 1) {
          ptx::tc_fence_before();
          ptx::mbar_arrive(&bar.acce[a]);
          released = true;
        }
        if (stamper && ch == 0) CVMM_STAMP(4, local);
        if (c_dense) {
          if (nkb == 0) {
#pragma unroll
            for (int j = 0; j < 64; ++j) v2[j] = 0.f;
          }
          // The store issued earlier from this box must have read it (two
          // boxes per warp: the one before last; one box: the last).
          if (lane == 0) {
            if (kBoxes == 1) ptx::bulk_wait_read<0>();
            else ptx::bulk_wait_read<1>();
          }
          __syncwarp();
          const uint32_t box = cbox + (kBoxes == 1 ? 0u : cbuf * kStoreBox);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            uint32_t w4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              w4[i] = pack2(v2[8 * q + 2 * i], v2[8 * q + 2 * i + 1], p.c_dtype);
            ptx::st_shared_v4(box + lane * 128 + ((uint32_t)(q ^ (lane & 7)) << 4), w4[0], w4[1], w4[2], w4[3]);
          }
          if (stamper && ch == 0) CVMM_STAMP(5, local);
          ptx::fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && !CVMM_DBG(flags, 16384)) {
            ptx::tma_store_2d(&tmap_c, box, (int)(n0 + ch * 64), prow0);
            ptx::bulk_commit();
          }
          if (stamper) CVMM_STAMP(6 + (ch & 1), local);
          cbuf ^= 1;
          continue;
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int64_t nc = n0 + ch * 64 + h * 32;
          if (nc >= p.N) break;
          const int ncols = (int)imin64(32, p.N - nc);
          float* v = v2 + 32 * h;
          if (nkb == 0) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.f;
          }
          if (p.mode == 1 && row_ok && xv_ok) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const uint4 q4 = xr[4 * h + (j >> 3)];
              const int c = (j >> 1) & 3;
              const uint32_t wd = c == 0 ? q4.x : (c == 1 ? q4.y : (c == 2 ? q4.z : q4.w));
              const float xval = bits_to_float((uint16_t)((j & 1) ? (wd >> 16) : (wd & 0xffffu)), p.x_dtype);
              const float av = round_to(v[j], op);
              dot = fmaf(av, xval, dot);
              v[j] = round_to(av * wv, op);
            }
          } else if (p.mode == 1 && row_ok) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float av = round_to(v[j], op);
              if (j < ncols) dot = fmaf(av, load_as_float(p.x, p.x_dtype, idx_div(crow, p.x_div) * p.x_ld + nc + j), dot);
              v[j] = round_to(av * wv, op);
            }
          }
          if (ACT) {
            // Pre-activation (rounded to the output dtype) to c2, GELU of it to c.
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = round_to(v[j], p.c_dtype);
            if (!CVMM_DBG(flags, 16384))
              warp_store_block(p.c2, p.c_dtype, row_ok ? crow * p.c_ld + nc : -1, v, ncols, stage, c_vec);
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = gelu_erf(v[j]);
          }
          if (!CVMM_DBG(flags, 16384))
            warp_store_block(p.c, p.c_dtype, row_ok ? crow * p.c_ld + nc : -1, v, ncols, stage, c_vec);
        }
      }
      if (p.mode == 1 && row_ok) atomicAdd(p.gsel + crow, dot);
      if (!released) {
        ptx::tc_fence_before();
        ptx::mbar_arrive(&bar.acce[a]);
      }
      if (stamper) CVMM_STAMP(3, local);
      ent = ent_next;
      ent_next = ent_after;
      crow = crow_next;
    }
    if (c_dense && lane == 0) ptx::bulk_wait_all();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = ptx::instr_desc_f16(BM, BN, op == BF16, false, !B_KMAJOR);
      mma_loop<BN, S>(bar, bar.full, smem, tmem, idesc, false, !B_KMAJOR, total, [&](int) { return nkb; },
                      CVMM_DBG(flags, 256));
    }
    __syncwarp();
  } else if (warp == kStoreWarp) {
    // ------------------------------------------------------------ A tile store-back
    // Each full stage's A tile (op dtype, already in the 128-byte swizzle TMA
    // uses) goes to its rows of the expert-padded sorted copy; the stage is
    // released (second arrival on `empty`, after the MMAs' commit) once the
    // store has read it, two stages later, so stores stay in flight while
    // this thread moves on. A separate warp keeps these waits off the MMA issue.
    if ((flags & kFlagACopy) && lane == 0) {
      uint32_t it = 0;
      int q0 = -1, q1 = -1;
      bool aborted = false;
      for (int tt = blockIdx.x; tt < total && !aborted; tt += gridDim.x) {
        const int prow = (int)kPadRows * entry(tt).w;
        const bool store = tt % n_n == 0;  // the A tile is the same for every column tile
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % S;
          if (!ptx::mbar_wait_or_abort(&bar.full[s], (it / S) & 1, kTagFull, bar.abort)) {
            aborted = true;
            break;
          }
          ptx::fence_proxy_async_smem();
          if (store && !CVMM_DBG(flags, 1 << 18))
            ptx::tma_store_2d(&tmap_a, ptx::smem_u32(smem + s * L::stage_bytes), kb * BK, prow);
          ptx::bulk_commit();
          if (q1 >= 0) {
            ptx::bulk_wait_read<2>();
            ptx::mbar_arrive(&bar.empty[q0]);
            q0 = q1;
            q1 = s;
          } else if (q0 >= 0) {
            q1 = s;
          } else {
            q0 = s;
          }
        }
      }
      ptx::bulk_wait_read<0>();
      if (q0 >= 0) ptx::mbar_arrive(&bar.empty[q0]);
      if (q1 >= 0) ptx::mbar_arrive(&bar.empty[q1]);
      ptx::bulk_wait_all();
    }
  } else if (warp == kLoaderWarp && B_TMA && lane == 0) {
    // ------------------------------------------------------------ B tiles by TMA
    ptx::tma_prefetch_desc(&tmap_b);
    if (EPI2) ptx::tma_prefetch_desc(&tmap_a);
    uint32_t it = 0;
    int4 ent = entry(blockIdx.x);
    for (int tt = blockIdx.x; tt < total; tt += gridDim.x) {
      const int4 ent_next = entry(tt + gridDim.x);
      const int e = ent.x;
      const int n0 = (tt % n_n) * BN;
      const int a_row0 = EPI2 ? a_row_of(ent, 0) : 0;  // dense A: the tile's first padded row
      bool aborted = false;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % S;
        if (it >= S && !ptx::mbar_wait_or_abort(&bar.empty[s], ((it / S) - 1) & 1, kTagEmpty, bar.abort)) {
          aborted = true;
          break;
        }
        const uint32_t b_u = ptx::smem_u32(smem + s * L::stage_bytes) + L::a_bytes;
        if (CVMM_DBG(flags, 1024)) {
          ptx::mbar_arrive(&bar.full[s]);
          continue;
        }
        ptx::mbar_arrive_expect_tx(&bar.full[s], (EPI2 ? L::a_bytes : 0u) + L::b_bytes);
        if (EPI2) ptx::tma_load_2d(b_u - L::a_bytes, &tmap_a, &bar.full[s], kb * BK, a_row0);
        if (B_KMAJOR) {
          ptx::tma_load_3d(b_u, &tmap_b, &bar.full[s], kb * BK, n0, e);
        } else {
#pragma unroll
          for (int q = 0; q < BN / 64; ++q)
            ptx::tma_load_3d(b_u + q * kAtomRowsBytes, &tmap_b, &bar.full[s], n0 + 64 * q, kb * BK, e);
        }
      }
      if (aborted) break;
      ent = ent_next;
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 2 * BN);
  }
}

// Multiplies this thread's G chunks of stage `j` by their route weights (from
// the index ring) and rounds to the op dtype: the reference multiplies the
// bf16 grad row by the bf16 weight and rounds the product to bf16 before the
// dot (cvmm.py:591-599).
template <int BN, int S>
__device__ __forceinline__ void scale_rows(uint8_t* smem, const IdxSlot* ring, uint32_t j, int t, int op) {
  using L = Smem<BN, S>;
  constexpr int GCPR = BN / 8;
  const int sj = j % S;
  const int gc = t % GCPR;
  const uint32_t bj = ptx::smem_u32(smem + sj * L::stage_bytes) + L::a_bytes;
#pragma unroll
  for (int i = 0; i < BN / 16; ++i) {
    const int kr = t / GCPR + (kProducers / GCPR) * i;
    const float sc = ring[sj].w[ring[sj].off + kr];
    const uint32_t addr = bj + swz(kr, gc, kAtomRowsBytes);
    uint32_t w4[4];
    ptx::ld_shared_v4(addr, w4[0], w4[1], w4[2], w4[3]);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float lo = bits_to_float((uint16_t)(w4[q] & 0xffffu), op) * sc;
      const float hi = bits_to_float((uint16_t)(w4[q] >> 16), op) * sc;
      w4[q] = pack2(lo, hi, op);
    }
    ptx::st_shared_v4(addr, w4[0], w4[1], w4[2], w4[3]);
  }
}

// ============================================================ segment GEMM (grad-W)
// Work = (unit, m tile, n tile) where a unit is a chunk of at most p.chunk
// sorted routes of one expert (split-K): a heavily loaded expert is spread
// over many tiles. A unit covering its whole expert writes grad_w; chunks of
// a split expert write partial slots that seg_reduce adds in a fixed order.
// Both operands are gathered rows: A = x^T (MN-major, rows = routes), B = the
// (weight-scaled) grad rows (MN-major). Warp 9 runs up to S stages ahead of
// the producers, resolving each stage's 64 route rows (x row, grad row, route
// weight) into the shared-memory index ring, so the producers never wait on
// index loads.
// flags bit0: X fast path, bit1: G fast path, bit2: out vector stores.
template <int BN, int S, bool WEIGHTED, bool G_TMA>
__global__ void __launch_bounds__(kThreads, 1)
seg_gemm_kernel(const SegGemm p, const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_g,
                int flags, int n_m, int n_n) {
  using L = Smem<BN, S>;
  constexpr int GCPR = BN / 8;    // G tile: 16-byte chunks per route row
  constexpr int GROWS = BN / 16;  // G rows per producer thread per stage
  // The weighted variant scales G in shared memory after it lands, so its
  // producers hand a stage over LAG stages after issuing it.
  constexpr int LAG = S / 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem(smem_raw);
  const Bars bar = carve_bars<L, S>(smem);
  IdxSlot* ring = reinterpret_cast<IdxSlot*>(smem + L::ring);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per_unit = n_m * n_n;
  constexpr int kTransform = kProducers - 32;  // warps 1-3 scale weighted grad rows
  const uint32_t tmem = G_TMA ? setup<BN, S>(bar, 1, WEIGHTED ? kProducers : 32, kTransform)
                              : setup<BN, S>(bar, kProducers);
  pdl_wait();
  // Unit list: from build_units, or built here in the (otherwise unused) tile
  // plan region when the host passes none (few experts and units).
  int4* own_units = reinterpret_cast<int4*>(smem + L::plan);
  static_assert(kOwnUnits * 16 + (kOwnUnitExperts + 34) * 4 <= (2 * (kPlanExperts + 1) + 32) * 4,
                "own unit list exceeds the plan region");
  const int n_units =
      p.units ? *p.n_units
              : build_unit_list(p.offsets, p.n_experts, p.chunk, own_units, blockIdx.x == 0 ? p.expert_slots : nullptr,
                                reinterpret_cast<int*>(own_units + kOwnUnits),
                                reinterpret_cast<int*>(own_units + kOwnUnits) + kOwnUnitExperts);
  const int4* units = p.units ? p.units : own_units;
  const int total = n_units * per_unit;
  const int op = p.op_dtype;
  const bool x_fast = flags & 1, g_fast = flags & 2, o_vec = flags & 4;

  auto entry = [&](int tt) -> int4 {
    return tt < total ? units[tt / per_unit] : make_int4(0, 0, -1, 0);
  };
  auto nkb_of = [&](const int4& u) -> int { return (int)((u.w - u.y + BK - 1) / BK); };

  if (G_TMA && warp == 0) {
    // ------------------------------------------------------------ gathers by TMA
    // Per stage: 64 route rows of x (the m slice) and of the grad (the n slice),
    // 4 rows per gather4, into the MN-major swizzled stages (route = k row).
    uint32_t it = 0;
    bool aborted = false;
    // The index ring carries the route weights of a weighted grad-W even when
    // both operands are dense boxes.
    const bool g_dense = flags & 32, x_dense = flags & 64, ring_on = WEIGHTED || !(g_dense && x_dense);
    for (int tt = blockIdx.x; tt < total && !aborted; tt += gridDim.x) {
      const int4 u = entry(tt);
      const int rem = tt % per_unit;
      const int m0 = (rem / n_n) * BM, n0 = (rem % n_n) * BN;
      const int nkb = nkb_of(u);
      const int64_t sbeg = (g_dense || x_dense) ? seg_begin(p.offsets, u.x) : 0;
      const int g_pstart = g_dense ? p.g_pad_start[u.x] : 0;
      const int x_pstart = x_dense ? p.x_pad_start[u.x] : 0;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % S;
        if ((it >= S && !ptx::mbar_wait_or_abort(&bar.empty[s], ((it / S) - 1) & 1, kTagEmpty, bar.abort)) ||
            (ring_on && !ptx::mbar_wait_or_abort(&bar.idxf[s], (it / S) & 1, kTagFull, bar.abort))) {
          aborted = true;
          break;
        }
        const IdxSlot& slot = ring[s];
        const int off = ring_on ? slot.off : 0;
        const int64_t rb = u.y + (int64_t)kb * BK;
        const uint32_t a_u = ptx::smem_u32(smem + s * L::stage_bytes), b_u = a_u + L::a_bytes;
        const bool skip_x = CVMM_DBG(flags, 512), skip_g = CVMM_DBG(flags, 1024);
        if (lane == 0) {
          const uint32_t tx = (skip_x ? 0u : L::a_bytes) + (skip_g ? 0u : L::b_bytes);
          if (tx) ptx::mbar_arrive_expect_tx(&bar.full[s], tx);
          else ptx::mbar_arrive(&bar.full[s]);
        }
        if (g_dense && !skip_g) {
          // Expert-padded sorted grad rows: the stage's 64 route rows are one
          // dense box per 64 columns. Units are whole multiples of 64 routes
          // except an expert's last one, whose tail rows are padding zeros.
          const int prow = g_pstart + (int)(rb - sbeg);
          if (lane < BN / 64) ptx::tma_load_2d(b_u + lane * kAtomRowsBytes, &tmap_g, &bar.full[s], n0 + 64 * lane, prow);
        }
        if (x_dense && !skip_x) {
          // Expert-padded sorted x rows: one dense 64-row box per 64 m columns.
          const int prow = x_pstart + (int)(rb - sbeg);
          if (lane < BM / 64) ptx::tma_load_2d(a_u + lane * kAtomRowsBytes, &tmap_x, &bar.full[s], m0 + 64 * lane, prow);
        }
        __syncwarp();
        if (!skip_x && !x_dense) {
          const int atom = lane >> 4, grp = lane & 15;
          int r[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int kr = 4 * grp + q;
            r[q] = rb + kr < u.w ? slot.x[off + kr] : -1;
          }
          ptx::tma_gather4(a_u + atom * kAtomRowsBytes + grp * 512, &tmap_x, &bar.full[s], m0 + 64 * atom, r[0],
                           r[1], r[2], r[3]);
        }
#pragma unroll
        for (int gi = lane; gi < (g_dense || skip_g ? 0 : BN / 4); gi += 32) {
          const int atom = gi >> 4, grp = gi & 15;
          int r[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int kr = 4 * grp + q;
            r[q] = rb + kr < u.w ? slot.g[off + kr] : -1;
          }
          ptx::tma_gather4(b_u + atom * kAtomRowsBytes + grp * 512, &tmap_g, &bar.full[s], n0 + 64 * atom, r[0],
                           r[1], r[2], r[3]);
        }
        if (ring_on) ptx::mbar_arrive(&bar.idxe[s]);
        if (lane == 0) CVMM_STAMP(0, it);
      }
    }
  } else if (G_TMA && warp < 4) {
    // ------------------------------------------------------------ transform (weighted)
    if (WEIGHTED) {
      const int tx = threadIdx.x - 32;
      constexpr int CPR = BN / 8;
      uint32_t it = 0;
      bool aborted = false;
      for (int tt = blockIdx.x; tt < total && !aborted; tt += gridDim.x) {
        const int nkb = nkb_of(entry(tt));
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % S;
          if (!ptx::mbar_wait_or_abort(&bar.full[s], (it / S) & 1, kTagFull, bar.abort)) {
            aborted = true;
            break;
          }
          const IdxSlot& slot = ring[s];
          const uint32_t b_u = ptx::smem_u32(smem + s * L::stage_bytes) + L::a_bytes;
          for (int c = tx; c < 64 * CPR; c += kTransform) {
            const int kr = c / CPR, col = c % CPR;
            const float sc = slot.w[slot.off + kr];
            const uint32_t addr = b_u + swz(kr, col, kAtomRowsBytes);
            uint32_t w4[4];
            ptx::ld_shared_v4(addr, w4[0], w4[1], w4[2], w4[3]);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float lo = bits_to_float((uint16_t)(w4[q] & 0xffffu), op) * sc;
              const float hi = bits_to_float((uint16_t)(w4[q] >> 16), op) * sc;
              w4[q] = pack2(lo, hi, op);
            }
            ptx::st_shared_v4(addr, w4[0], w4[1], w4[2], w4[3]);
          }
          ptx::fence_proxy_async_smem();
          ptx::mbar_arrive(&bar.ready[s]);
          ptx::mbar_arrive(&bar.idxe[s]);
        }
      }
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------ producers
    const int t = threadIdx.x;
    const char* xbase = static_cast<const char*>(p.x);
    const char* gbase = static_cast<const char*>(p.g);
    const int64_t xsz = dtype_bytes(p.x_dtype), gsz = dtype_bytes(p.g_dtype);
    const int xc = t & 15;    // X tile: 64 route rows x 16 chunks (128 m columns)
    const int gc = t % GCPR;  // G tile: 64 route rows x GCPR chunks
    uint32_t it = 0;
    bool aborted = false;
    for (int tt = blockIdx.x; tt < total && !aborted; tt += gridDim.x) {
      const int4 u = entry(tt);
      const int rem = tt % per_unit;
      const int64_t m0 = (int64_t)(rem / n_n) * BM, n0 = (int64_t)(rem % n_n) * BN;
      const int nkb = nkb_of(u);
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % S;
        if ((it >= S && !ptx::mbar_wait_or_abort(&bar.empty[s], ((it / S) - 1) & 1, kTagEmpty, bar.abort)) ||
            !ptx::mbar_wait_or_abort(&bar.idxf[s], (it / S) & 1, kTagFull, bar.abort)) {
          aborted = true;
          break;
        }
        const IdxSlot& slot = ring[s];
        const int off = slot.off;
        const int64_t rb = u.y + (int64_t)kb * BK;
        const uint32_t a_u = ptx::smem_u32(smem + s * L::stage_bytes), b_u = a_u + L::a_bytes;
        if (!CVMM_DBG(flags, 512)) {
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int kr = (t >> 4) + 8 * i;
            const int xr = slot.x[off + kr];
            const char* row = rb + kr < u.w ? xbase + ((int64_t)xr * p.x_ld + m0) * xsz : nullptr;
            load_chunk(a_u + swz(kr, xc, kAtomRowsBytes), row, xc * 8, p.M - m0, p.x_dtype, 1, op, x_fast, p.x);
          }
        }
        if (!CVMM_DBG(flags, 1024)) {
#pragma unroll
          for (int i = 0; i < GROWS; ++i) {
            const int kr = t / GCPR + (kProducers / GCPR) * i;
            const int gr = slot.g[off + kr];
            const char* row = rb + kr < u.w ? gbase + ((int64_t)gr * p.g_ld + n0) * gsz : nullptr;
            load_chunk(b_u + swz(kr, gc, kAtomRowsBytes), row, gc * 8, p.N - n0, p.g_dtype, 1, op, g_fast, p.g);
          }
        }
        if (t == 0) CVMM_STAMP(0, it);
        if (!WEIGHTED) {
          if (!x_fast || !g_fast) ptx::fence_proxy_async_smem();
          ptx::cp_async_arrive_noinc(&bar.full[s]);
          ptx::mbar_arrive(&bar.idxe[s]);
        } else {
          // Hand over stage it-LAG: its copies landed; scale it in place.
          ptx::cp_async_commit();
          if (it >= (uint32_t)LAG) {
            const uint32_t j = it - LAG;
            ptx::cp_async_wait<LAG>();
            scale_rows<BN, S>(smem, ring, j, t, op);
            ptx::fence_proxy_async_smem();
            ptx::mbar_arrive(&bar.full[j % S]);
            ptx::mbar_arrive(&bar.idxe[j % S]);
          }
        }
      }
    }
    ptx::cp_async_wait_all();
    if (WEIGHTED && !aborted) {
      const uint32_t first = it > (uint32_t)LAG ? it - LAG : 0;
      for (uint32_t j = first; j < it; ++j) scale_rows<BN, S>(smem, ring, j, t, op);
      ptx::fence_proxy_async_smem();
      for (uint32_t j = first; j < it; ++j) {
        ptx::mbar_arrive(&bar.full[j % S]);
        ptx::mbar_arrive(&bar.idxe[j % S]);
      }
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 4;
    const int mr = ew * 32 + lane;
    const uint32_t stage = ptx::smem_u32(smem + L::staging) + ew * 32 * kStageRowBytes;
    int local = 0;
    for (int tt = blockIdx.x; tt < total; tt += gridDim.x, ++local) {
      const int4 u = entry(tt);
      const int rem = tt % per_unit;
      const int64_t m0 = (int64_t)(rem / n_n) * BM, n0 = (int64_t)(rem % n_n) * BN;
      const int a = local & 1;
      if (!ptx::mbar_wait_or_abort(&bar.accf[a], (local >> 1) & 1, kTagAccFull, bar.abort)) break;
      ptx::tc_fence_after();
      const int64_t e = u.x;
      if (mr == 0) CVMM_STAMP(2, local);
      const int64_t m = m0 + mr;
      float* dst = u.z < 0 ? p.out + e * p.M * p.N : p.partials + (int64_t)u.z * p.M * p.N;
      const bool empty_unit = nkb_of(u) == 0;
      for (int ch = 0; ch < BN / 64; ++ch) {
        if (n0 + ch * 64 >= p.N) break;
        float v2[64];
        load_acc64(tmem + ((uint32_t)(ew * 32) << 16) + a * BN + ch * 64, v2);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int64_t nc = n0 + ch * 64 + h * 32;
          if (nc >= p.N) break;
          const int ncols = (int)imin64(32, p.N - nc);
          float* v = v2 + 32 * h;
          if (empty_unit) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0.f;
          }
          if (!CVMM_DBG(flags, 16384)) warp_store_block(dst, F32, m < p.M ? m * p.N + nc : -1, v, ncols, stage, o_vec);
        }
      }
      ptx::tc_fence_before();
      ptx::mbar_arrive(&bar.acce[a]);
      if (mr == 0) CVMM_STAMP(3, local);
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      const uint32_t idesc = ptx::instr_desc_f16(BM, BN, op == BF16, true, true);
      mma_loop<BN, S>(bar, WEIGHTED && G_TMA ? bar.ready : bar.full, smem, tmem, idesc, true, true, total, [&](int tt) { return nkb_of(entry(tt)); },
                      CVMM_DBG(flags, 256));
    }
    __syncwarp();
  } else if (warp == kLoaderWarp) {
    // ------------------------------------------------------------ index warp
    // (idle when both operands are dense: their rows follow from the unit)
    uint32_t it = 0;
    bool aborted = !WEIGHTED && (flags & 96) == 96;
    for (int tt = blockIdx.x; tt < total && !aborted; tt += gridDim.x) {
      const int4 u = entry(tt);
      const int nkb = nkb_of(u);
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % S;
        if (it >= S && !ptx::mbar_wait_or_abort(&bar.idxe[s], ((it / S) - 1) & 1, kTagEmpty, bar.abort)) {
          aborted = true;
          break;
        }
        if (lane == 0) {
          const int64_t rb = u.y + (int64_t)kb * BK;
          const int64_t al = rb & ~(int64_t)3;
          ring[s].off = (int)(rb - al);
          constexpr uint32_t kBytes = kRingEntries * 4;
          ptx::mbar_arrive_expect_tx(&bar.idxf[s], (WEIGHTED ? 3 : 2) * kBytes);
          ptx::bulk_load(ptx::smem_u32(ring[s].x), p.xrow + al, kBytes, &bar.idxf[s]);
          ptx::bulk_load(ptx::smem_u32(ring[s].g), p.grow + al, kBytes, &bar.idxf[s]);
          if (WEIGHTED) ptx::bulk_load(ptx::smem_u32(ring[s].w), p.wsc + al, kBytes, &bar.idxf[s]);
        }
        __syncwarp();
        if (lane == 0) CVMM_STAMP(2, it);
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, 2 * BN);
  }
}

// ------------------------------------------------------------ host side
template <typename K>
static int set_smem(K kernel, uint32_t bytes) {
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
    return fail_cuda("cudaFuncSetAttribute(max dynamic smem)");
  return CVMM_OK;
}

static inline bool aligned16(const void* ptr) { return ((uintptr_t)ptr & 15u) == 0; }

// SMs a persistent GEMM grid may use: the device's, capped by cvmm_set_sm_limit.
static int sm_count() {
  int dev = 0, v = 0;
  if (!(cudaGetDevice(&dev) == cudaSuccess && cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess &&
        v > 0))
    v = 148;
  const int lim = g_sm_limit.load(std::memory_order_relaxed);
  return lim > 0 ? std::min(v, lim) : v;
}

static int dbg_flags() {
#ifdef CVMM_TRACE
  if (const char* ev = getenv("CVMM_DBG_FLAGS")) return atoi(ev);
#endif
  return 0;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 3-D TMA map of the expert weights keys[e][r][c] (c contiguous) with a
// 64 x box_rows box and 128-byte swizzle. Returns false when the layout does
// not meet TMA's alignment rules (the caller then loads B with cp.async).
static bool make_b_map(CUtensorMap* map, const void* base, int dtype, int64_t cols, int64_t rows, int64_t experts,
                       int64_t row_stride, int64_t expert_stride, int box_rows) {
  auto fn = encode_fn();
  if (!fn || !aligned16(base) || (row_stride * 2) % 16 != 0 || (expert_stride * 2) % 16 != 0) return false;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)experts};
  cuuint64_t strides[2] = {(cuuint64_t)row_stride * 2, (cuuint64_t)expert_stride * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype == BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// 2-D TMA map over a row-major [rows, cols] operand for tile::gather4: a box
// of 64 columns (128 bytes) by one row, 128-byte swizzle.
static bool make_rows_map(CUtensorMap* map, const void* base, int dtype, int64_t cols, int64_t rows, int64_t ld,
                          int box_rows = 1) {
  auto fn = encode_fn();
  if (!fn || !aligned16(base) || (ld * 2) % 16 != 0 || rows <= 0 || cols <= 0 || rows > INT32_MAX) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dtype == BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <int BN, int S, bool BK_MAJOR>
static int row_launch(const RowGemm& p, int64_t max_tiles, int flags, cudaStream_t stream) {
  using L = Smem<BN, S>;
  const int n_n = (int)((p.N + BN - 1) / BN);
  CUtensorMap map;
  memset(&map, 0, sizeof(map));
  bool tma = false;
  if (flags & 2) {
    tma = BK_MAJOR ? make_b_map(&map, p.b, p.op_dtype, p.K, p.N, p.n_experts, p.bs_n, p.bs_e, BN)
                   : make_b_map(&map, p.b, p.op_dtype, p.N, p.K, p.n_experts, p.bs_k, p.bs_e, 64);
  }
  if (dbg_flags() & 2048) tma = false;
  CUtensorMap amap;
  memset(&amap, 0, sizeof(amap));
  // Dense A tiles (expert-padded sorted layout) always go through TMA; row
  // gathers stay on cp.async, which measured faster than gather4 here.
  const bool a_dense = tma && (flags & 1) && p.a_pad_start != nullptr &&
                       make_rows_map(&amap, p.a, p.op_dtype, p.K, p.a_rows, p.a_ld, BM);
  const bool a_tma = a_dense || (tma && (flags & 1) && (dbg_flags() & 8192) &&
                                 make_rows_map(&amap, p.a, p.op_dtype, p.K, p.a_rows, p.a_ld));
  if (a_dense) flags |= 32;
  // A copy (the forward writing the expert-padded sorted x): gathered A only;
  // the map over the copy takes tmap_a's place, unused on that path.
  if (p.a_copy) {
    if (a_tma ||
        !make_rows_map(&amap, p.a_copy, p.op_dtype, p.K, p.n_routes + kPadRows * p.n_experts, p.K, BM))
      return fail(CVMM_ERR_INVALID_ARG, "A copy needs a gathered A operand, 16-bit arithmetic and 16-byte aligned rows");
    flags |= kFlagACopy;
  }
  // Dense C: expert-padded sorted 16-bit output written by 32-row TMA boxes.
  CUtensorMap cmap;
  memset(&cmap, 0, sizeof(cmap));
  if (p.c_pad_start) {
    if (p.mode != 0 || (p.c_dtype != BF16 && p.c_dtype != F16) ||
        !make_rows_map(&cmap, p.c, p.c_dtype, p.N, p.n_routes + kPadRows * p.n_experts, p.c_ld, 32))
      return fail(CVMM_ERR_INVALID_ARG,
                  "padded sorted output needs mode 0, a bf16/fp16 out_dtype and 16-byte aligned rows");
    flags |= 128;
  }
  if (p.act == 1 && (a_tma || p.c_pad_start || p.mode != 0))
    return fail(CVMM_ERR_INVALID_ARG, "the GELU epilogue needs a row-gathered A, row-indexed outputs and mode 0");
  const int64_t work = max_tiles * n_n;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(work, sm_count()));
  if (a_dense && BN >= 128 && !(dbg_flags() & 32768)) {
    auto kern = row_gemm_kernel<BN, S, BK_MAJOR, true, true, (BN >= 128)>;
    int rc = set_smem(kern, L::alloc);
    if (rc) return rc;
    launch(kern, grid, kThreads, L::alloc, stream, p, map, amap, cmap, flags, n_n);
  } else if (a_tma) {
    auto kern = row_gemm_kernel<BN, S, BK_MAJOR, true, true>;
    int rc = set_smem(kern, L::alloc);
    if (rc) return rc;
    launch(kern, grid, kThreads, L::alloc, stream, p, map, amap, cmap, flags, n_n);
  } else if (tma && p.act == 1) {
    auto kern = row_gemm_kernel<BN, S, BK_MAJOR, true, false, false, true>;
    int rc = set_smem(kern, L::alloc);
    if (rc) return rc;
    launch(kern, grid, kThreads, L::alloc, stream, p, map, amap, cmap, flags, n_n);
  } else if (tma) {
    auto kern = row_gemm_kernel<BN, S, BK_MAJOR, true, false>;
    int rc = set_smem(kern, L::alloc);
    if (rc) return rc;
    launch(kern, grid, kThreads, L::alloc, stream, p, map, amap, cmap, flags, n_n);
  } else if (p.act == 1) {
    auto kern = row_gemm_kernel<BN, S, BK_MAJOR, false, false, false, true>;
    int rc = set_smem(kern, L::alloc);
    if (rc) return rc;
    launch(kern, grid, kThreads, L::alloc, stream, p, map, amap, cmap, flags, n_n);
  } else {
    auto kern = row_gemm_kernel<BN, S, BK_MAJOR, false, false>;
    int rc = set_smem(kern, L::alloc);
    if (rc) return rc;
    launch(kern, grid, kThreads, L::alloc, stream, p, map, amap, cmap, flags, n_n);
  }
  return check_launch("row_gemm_umma");
}

template <int BN, int S, bool W>
static int seg_launch(const SegGemm& p, int64_t max_units, int flags, cudaStream_t stream) {
  using L = Smem<BN, S>;
  const int n_m = (int)((p.M + BM - 1) / BM), n_n = (int)((p.N + BN - 1) / BN);
  const int64_t work = max_units * n_m * n_n;
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(work, sm_count()));
  CUtensorMap xmap, gmap;
  memset(&xmap, 0, sizeof(xmap));
  memset(&gmap, 0, sizeof(gmap));
  // Gathered rows index at most n_routes rows of x and of the grad; the
  // expert-padded sorted grad has n_routes + 128 * n_experts rows and is read
  // as dense 64-row boxes.
  const bool g_dense = p.g_pad_start != nullptr, x_dense = p.x_pad_start != nullptr;
  const int64_t padded_rows = p.n_routes + kPadRows * p.n_experts;
  // TMA needs both operands in the expert-padded layout (dense boxes): a
  // gathered grad operand goes through the cp.async producers, whose row
  // gathers measured about twice the throughput of tile::gather4 here
  // (4.1 vs 2.1 TB/s for 256-byte row pieces out of L2).
  const bool gt = (flags & 3) == 3 && g_dense && !(dbg_flags() & 4096) &&
                  make_rows_map(&xmap, p.x, p.op_dtype, p.M, x_dense ? padded_rows : p.n_routes, p.x_ld,
                                x_dense ? 64 : 1) &&
                  make_rows_map(&gmap, p.g, p.op_dtype, p.N, g_dense ? padded_rows : p.n_routes, p.g_ld,
                                g_dense ? 64 : 1);
  // Without TMA maps the cp.async producers read padded rows through the
  // resolved route rows like gathered ones.
  if (gt && g_dense) flags |= 32;
  if (gt && x_dense) flags |= 64;
  if (gt) {
    auto kern = seg_gemm_kernel<BN, S, W, true>;
    int rc = set_smem(kern, L::alloc);
    if (rc) return rc;
    launch(kern, grid, kThreads, L::alloc, stream, p, xmap, gmap, flags, n_m, n_n);
  } else {
    auto kern = seg_gemm_kernel<BN, S, W, false>;
    int rc = set_smem(kern, L::alloc);
    if (rc) return rc;
    launch(kern, grid, kThreads, L::alloc, stream, p, xmap, gmap, flags, n_m, n_n);
  }
  return check_launch("seg_gemm_umma");
}

}  // namespace umma

#ifdef CVMM_TRACE
extern "C" int cvmm_debug_set_trace(void* buf) {
  unsigned long long* q = static_cast<unsigned long long*>(buf);
  return cudaMemcpyToSymbol(umma::g_trace, &q, sizeof(q)) == cudaSuccess ? 0 : -3;
}
#endif

int launch_row_gemm_umma(const RowGemm& p, int64_t max_tiles, cudaStream_t stream) {
  using namespace umma;
  const bool b_kmajor = p.bs_k == 1 && p.bs_n != 1;
  int flags = dbg_flags() & ~2048;
  if (p.a_dtype == p.op_dtype && p.a_ld % 8 == 0 && aligned16(p.a)) flags |= 1;
  if (p.b_dtype == p.op_dtype && aligned16(p.b) && p.bs_e % 8 == 0 &&
      (b_kmajor ? (p.bs_k == 1 && p.bs_n % 8 == 0) : (p.bs_n == 1 && p.bs_k % 8 == 0)))
    flags |= 2;
  if (p.c_ld % 8 == 0 && aligned16(p.c)) flags |= 4;
  if (p.mode == 1 && (p.x_dtype == BF16 || p.x_dtype == F16) && p.x_ld % 8 == 0 && aligned16(p.x)) flags |= 65536;
  if (p.N <= 64) {
    return b_kmajor ? row_launch<64, 7, true>(p, max_tiles, flags, stream)
                    : row_launch<64, 7, false>(p, max_tiles, flags, stream);
  }
  // Dense A (expert-padded sorted rows) with a wide output: 128 x 256 tiles
  // read each A tile half as often as 128 x 128 ones (grad-x of ff_up, the
  // forward of ff_down: N = 1024), with both epilogue warp groups draining
  // 128 columns each.
  if (p.N >= 256 && p.a_pad_start && p.mode == 0 && (flags & 3) == 3) {
    return b_kmajor ? row_launch<256, 3, true>(p, max_tiles, flags, stream)
                    : row_launch<256, 3, false>(p, max_tiles, flags, stream);
  }
  return b_kmajor ? row_launch<128, 5, true>(p, max_tiles, flags, stream)
                  : row_launch<128, 5, false>(p, max_tiles, flags, stream);
}

int launch_seg_gemm_umma(const SegGemm& p, int64_t max_units, cudaStream_t stream) {
  using namespace umma;
  int flags = dbg_flags();
  if (p.x_dtype == p.op_dtype && p.x_ld % 8 == 0 && aligned16(p.x)) flags |= 1;
  if (p.g_dtype == p.op_dtype && p.g_ld % 8 == 0 && aligned16(p.g)) flags |= 2;
  if (p.N % 4 == 0 && aligned16(p.out) && aligned16(p.partials)) flags |= 4;
  const bool w = p.w != nullptr;
  if (p.N <= 64) return w ? seg_launch<64, 7, true>(p, max_units, flags, stream) : seg_launch<64, 7, false>(p, max_units, flags, stream);
  if (p.N <= 128) return w ? seg_launch<128, 5, true>(p, max_units, flags, stream) : seg_launch<128, 5, false>(p, max_units, flags, stream);
  return w ? seg_launch<256, 3, true>(p, max_units, flags, stream) : seg_launch<256, 3, false>(p, max_units, flags, stream);
}

}  // namespace cvmm
