// The whole library is one translation unit: the kernels, their launchers
// and the extern "C" entry points share the device error word directly.
#include "common.cuh"
#include "quant.cu"
#include "dequant.cu"
#include "hc.cu"
#include "gemm.cu"
#include "gemm_pair.cu"
#include "moe.cu"
#include "peer.cu"
#include "ep.cu"
#include "moe_fused.cu"
#include "capi.cu"
#include "noalloc.cu"
