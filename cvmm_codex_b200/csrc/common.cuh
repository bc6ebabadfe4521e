// Shared device helpers for the CVMM sm_100a kernels: dtype codes, element
// conversion, status reporting and the bounded-wait clock.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/cvmm_sm100.h"

namespace cvmm {

// Element dtype codes. The float codes are the reference's dtype_to_type_id
// values (cvmm.py:36-44): 0 = float32, 1 = float16, 2 = bfloat16.
enum DType : int { F32 = CVMM_F32, F16 = CVMM_F16, BF16 = CVMM_BF16 };

// Programmatic dependent launch. Every kernel of this library is launched
// with cudaLaunchAttributeProgrammaticStreamSerialization (unless disabled),
// so its CTAs may be scheduled while the previous kernel on the stream drains.
// pdl_wait() blocks the calling thread until every prerequisite grid has
// completed and its memory operations are visible; each kernel calls it before
// its first global-memory access (read or write). pdl_trigger() lets the next
// kernel's CTAs be scheduled once every CTA of this grid has issued it or
// exited. Both are no-ops in a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }
// Entry of the short element-wise / scan kernels: let the successor launch at
// once (its CTAs wait in pdl_wait until this grid completes), then wait for the
// predecessor. The persistent tensor-core GEMMs only wait: their trigger is
// implicit, at CTA exit. Measured on the ff_up / ff_down steps (CUDA graphs):
// early triggers in the short kernels alone took 3 % off the step; adding a
// trigger at the GEMMs' teardown made the step slower than no PDL at all.
__device__ __forceinline__ void pdl_enter() {
  pdl_trigger();
  pdl_wait();
}

__host__ __device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }

// Row index / divisor for non-negative 32-bit-range indices (every index
// array here indexes fewer than 2^31 rows): avoids 64-bit division.
__device__ __forceinline__ int64_t idx_div(int64_t v, int64_t d) {
  return d == 1 ? v : (int64_t)((uint32_t)v / (uint32_t)d);
}

__host__ __device__ __forceinline__ int dtype_bytes(int dtype) {
  return dtype == F32 ? 4 : (dtype == CVMM_I64 ? 8 : (dtype == CVMM_I32 ? 4 : 2));
}

__device__ __forceinline__ float load_as_float(const void* p, int dtype, int64_t i) {
  if (dtype == BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}

// Round an fp32 value to the operation dtype (round-to-nearest-even), returned
// as fp32. This is the "a.to(bf16)" step the reference applies to every GEMM
// operand before tl.dot (cvmm.py:198-204).
__device__ __forceinline__ float round_to(float v, int dtype) {
  if (dtype == BF16) return __bfloat162float(__float2bfloat16_rn(v));
  if (dtype == F16) return __half2float(__float2half_rn(v));
  return v;
}

__device__ __forceinline__ void store_from_float(void* p, int dtype, int64_t i, float v) {
  if (dtype == BF16) reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else if (dtype == F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else reinterpret_cast<float*>(p)[i] = v;
}

__device__ __forceinline__ uint16_t float_to_bits(float v, int dtype) {
  if (dtype == F16) return __half_as_ushort(__float2half_rn(v));
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// Two values rounded to a 16-bit dtype (round-to-nearest-even) and packed
// low | high << 16, with one paired conversion instead of two.
__device__ __forceinline__ uint32_t pack2(float lo, float hi, int dtype) {
  if (dtype == F16) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
  const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&b);
}

__device__ __forceinline__ float bits_to_float(uint16_t b, int dtype) {
  if (dtype == F16) return __half2float(__ushort_as_half(b));
  return __bfloat162float(__ushort_as_bfloat16(b));
}

// Device status word. Kernels never trap: a failed bounded wait or a bad
// index is recorded here and the kernel returns; the host reads it back with
// cvmm_device_status().
struct DeviceStatus {
  int code;       // first error code recorded (0 = none)
  int where;      // kernel-specific location tag
  long long aux;  // e.g. the offending index
};

// Defined here: the library is one translation unit (csrc/cvmm_sm100.cu).
__device__ DeviceStatus g_status;

__device__ __forceinline__ void report(int code, int where, long long aux) {
  if (atomicCAS(&g_status.code, 0, code) == 0) {
    g_status.where = where;
    g_status.aux = aux;
  }
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Upper bound of any single wait inside a kernel (2 s). A healthy wait lasts
// microseconds; exceeding it means a protocol bug, so the kernel records
// CVMM_DEV_TIMEOUT and unwinds instead of hanging the GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

}  // namespace cvmm
