// Single translation unit of libmeep2b: the device error word and every kernel share one module.
#include "capi.cu"
#include "route.cu"
#include "grouped_gemm.cu"
#include "reduce.cu"
#include "quant.cu"
#include "merge.cu"
#include "fp8_products.cu"
#include "swiglu.cu"
