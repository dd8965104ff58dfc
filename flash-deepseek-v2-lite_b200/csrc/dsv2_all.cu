// Single translation unit for libdsv2.so: the kernels share one device-side error
// word (g_device_error), which a unity build links without relocatable device code.
#include "norm.cu"
#include "linear_gemv.cu"
#include "linear_tc.cu"
#include "linear_splitk.cu"
#include "moe_tc.cu"
#include "router.cu"
#include "mla.cu"
#include "mla_tc.cu"
#include "api.cu"
