// Single translation unit of libslimdit_b200.so: the kernel files share the device error
// word (slim::g_device_error) without relocatable device code.
#include "capi.cu"
#include "gemm_i8.cu"
#include "rotate_quant.cu"
#include "cert_quant.cu"
#include "linear_noalloc.cu"
#include "nvfp4_quant.cu"
#include "gemm_nvf4.cu"
#include "capi_nvfp4.cu"
#include "verify.cu"
#include "attn.cu"
