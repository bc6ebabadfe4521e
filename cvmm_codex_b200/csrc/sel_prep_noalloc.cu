// Allocation-free variant of the selector preparation.
//
// Some callers of this library cannot allocate device memory on the call
// path: hosts that bind the C ABI from another language (Go, Java, Rust)
// while owning every device byte through their own fixed memory plan, and
// latency-critical serving loops that must not call cudaMalloc, because
// cudaMalloc can synchronise the device and fragment a planned pool. For them,
// cvmm_sel_prepare_noalloc takes only inputs and outputs and finds its
// scratch in the array below, reserved when the library is loaded.
#include <mutex>

#include "launch.h"

namespace cvmm {

// Sized for CVMM_NOALLOC_MAX_ROUTES routes: the radix-sort header, the
// per-(digit, CTA) counts and the ping-pong key/value buffers (about 1.6 MB).
// Every GPU that loads the library keeps this much memory until the process
// exits.
constexpr int64_t kNoAllocMaxRoutes = CVMM_NOALLOC_MAX_ROUTES;
constexpr int64_t kNoAllocChunk = 1024;  // fewest routes per sorting CTA
constexpr size_t kNoAllocScratchBytes = sel_ws_bytes(kNoAllocMaxRoutes, kNoAllocChunk);

static __device__ __align__(256) unsigned char g_sel_scratch[kNoAllocScratchBytes];

// In host code `g_sel_scratch` names a host-side stand-in, not device memory,
// so the device address is looked up once per device (with that device
// current) and cached here.
constexpr int kMaxDevices = 64;
static void* g_scratch_addr[kMaxDevices];
static std::mutex g_scratch_mutex;

static int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail_cuda("cvmm_sel_prepare_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(CVMM_ERR_DEVICE, "cvmm_sel_prepare_noalloc: device index out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_sel_scratch) != cudaSuccess || p == nullptr)
      return fail_cuda("cvmm_sel_prepare_noalloc: cudaGetSymbolAddress");
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return CVMM_OK;
}

}  // namespace cvmm

extern "C" int cvmm_sel_prepare_noalloc(const void* sel, int sel_dtype, int64_t n_routes, int64_t top_k,
                                        int route_input, int32_t* raw_sel, int32_t* sorted_sel,
                                        int64_t* sel_index, int64_t* out_index, cvmm_stream_t stream) {
  using namespace cvmm;
  if (n_routes > kNoAllocMaxRoutes)
    return fail(CVMM_ERR_INVALID_ARG,
                "cvmm_sel_prepare_noalloc: n_routes exceeds CVMM_NOALLOC_MAX_ROUTES (65536); "
                "use cvmm_sel_prepare with a caller-provided workspace");
  if (sel_prepare_workspace_size(n_routes < 0 ? 0 : n_routes, kNoAllocChunk) > kNoAllocScratchBytes)
    return fail(CVMM_ERR_INVALID_ARG, "cvmm_sel_prepare_noalloc: scratch too small for n_routes");
  void* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
  if (rc) return rc;
  // sel_prepare zeroes the part of the scratch that must start at zero (the
  // key-range header) on every call; the rest is fully written before use.
  return sel_prepare(sel, sel_dtype, n_routes, top_k, route_input, raw_sel, sorted_sel, sel_index, out_index,
                     scratch, kNoAllocScratchBytes, reinterpret_cast<cudaStream_t>(stream), kNoAllocChunk);
}
