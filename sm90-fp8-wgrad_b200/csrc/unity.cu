// Single translation unit for libsm100_fp8_wgrad.so: the device error word
// and the kernels that write it live in one module without relocatable
// device code.
#include "wgrad_gemm.cu"
#include "wgrad_sp.cu"
#include "quant.cu"
#include "meta.cu"
#include "capi.cu"
#include "noalloc.cu"
