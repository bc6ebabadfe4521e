// Host-side helpers shared by the entry points: error recording and sizes.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <utility>

#include "../../include/cvmm_sm100.h"

namespace cvmm {

// SMs the persistent tensor-core GEMMs may occupy (0: all). Set through
// cvmm_set_sm_limit while a collective must run next to them.
inline std::atomic<int> g_sm_limit{0};

// Programmatic dependent launches (on unless CVMM_B200_PDL=0): every kernel
// is launched with cudaLaunchAttributeProgrammaticStreamSerialization, so its
// CTAs are scheduled as the previous kernel on the stream drains and wait in
// pdl_wait() (device side) for that kernel's completion. In stream capture the
// attribute becomes a programmatic edge of the graph.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline void launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // Errors are picked up by check_launch (cudaGetLastError) like <<<>>> launches.
  (void)cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Records `msg` as the calling thread's last error and returns `code`.
int fail(int code, const char* msg);
// Records the pending CUDA error (if any) with `where` as context.
int fail_cuda(const char* where);
// Checks cudaGetLastError() after kernel launches.
int check_launch(const char* where);

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

inline bool is_float_dtype(int d) { return d == CVMM_F32 || d == CVMM_F16 || d == CVMM_BF16; }
inline size_t dtype_size(int d) {
  switch (d) {
    case CVMM_F32: return 4;
    case CVMM_F16: return 2;
    case CVMM_BF16: return 2;
    case CVMM_I32: return 4;
    case CVMM_I64: return 8;
  }
  return 0;
}

// Entry points implemented across the .cu files.
// Selector sort: one persistent CTA of kSelWarps warps per slice of routes, at
// most kSelMaxGrid CTAs (and never more than the SMs). min_chunk: fewest
// routes per CTA (rounded up to kSelWarps * 32; the allocation-free entry uses
// 1024 so its static scratch holds the counts of at most 64 CTAs).
constexpr int64_t kSelMinChunk = 512;
constexpr int kSelWarps = 16;
constexpr int64_t kSelMaxGrid = 256;
constexpr int64_t sel_round(int64_t v) { return (v + kSelWarps * 32 - 1) / (kSelWarps * 32) * (kSelWarps * 32); }
constexpr int64_t sel_cta_len_min(int64_t min_chunk) { return sel_round(min_chunk < 1 ? 1 : min_chunk); }
constexpr int64_t sel_grid_bound(int64_t n, int64_t min_chunk) {
  return (n + sel_cta_len_min(min_chunk) - 1) / sel_cta_len_min(min_chunk) < kSelMaxGrid
             ? (n + sel_cta_len_min(min_chunk) - 1) / sel_cta_len_min(min_chunk)
             : kSelMaxGrid;
}
constexpr size_t sel_align(size_t v) { return (v + 255) / 256 * 256; }
// Header, per-(bin, CTA) counts, bin totals, and the ping-pong key/value buffers of the extra passes.
constexpr size_t sel_ws_bytes(int64_t n, int64_t min_chunk) {
  return 256 + sel_align((size_t)2048 * sel_grid_bound(n, min_chunk) * 4) + sel_align(2048 * 4) +
         4 * sel_align((size_t)n * 4);
}
size_t sel_prepare_workspace_size(int64_t n, int64_t min_chunk = kSelMinChunk);
int sel_prepare(const void* sel, int sel_dtype, int64_t n, int64_t top_k, int route_input,
                int32_t* raw_sel, int32_t* sorted_sel, int64_t* sel_index, int64_t* out_index,
                void* workspace, size_t ws_bytes, cudaStream_t stream, int64_t min_chunk = kSelMinChunk);
int expert_offsets(const int32_t* sorted, int64_t n, int64_t n_experts, int64_t* offsets,
                   cudaStream_t stream);

}  // namespace cvmm
