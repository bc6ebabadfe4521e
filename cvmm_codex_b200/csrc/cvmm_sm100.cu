// Single translation unit of libcvmm_sm100.so. The kernels share the device
// status word (g_status), so they are compiled together rather than linked
// with relocatable device code.
#include "abi.cu"
#include "sel_prep.cu"
#include "sel_prep_noalloc.cu"
#include "simt_gemm.cu"
#include "umma_gemm.cu"
