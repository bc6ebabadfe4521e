// Host-side helpers shared by the entry points: error recording and sizes.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <algorithm>

#include "../../include/cvmm_sm100.h"

namespace cvmm {

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
// min_chunk: fewest routes per radix-sort warp chunk (128 by default; the
// allocation-free entry uses 1024 to keep its static scratch small).
constexpr int64_t kSelMinChunk = 128;
size_t sel_prepare_workspace_size(int64_t n, int64_t min_chunk = kSelMinChunk);
int sel_prepare(const void* sel, int sel_dtype, int64_t n, int64_t top_k, int route_input,
                int32_t* raw_sel, int32_t* sorted_sel, int64_t* sel_index, int64_t* out_index,
                void* workspace, size_t ws_bytes, cudaStream_t stream, int64_t min_chunk = kSelMinChunk);
int expert_offsets(const int32_t* sorted, int64_t n, int64_t n_experts, int64_t* offsets,
                   cudaStream_t stream);

}  // namespace cvmm
