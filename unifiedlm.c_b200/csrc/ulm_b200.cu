// Single translation unit of the library: the kernels share one device-side error flag, so they
// are compiled together (no relocatable device code needed).
#include "gemm.cu"
#include "stats.cu"
#include "memory.cu"
#include "decode.cu"
#include "address.cu"
#include "head.cu"
#include "norm.cu"
