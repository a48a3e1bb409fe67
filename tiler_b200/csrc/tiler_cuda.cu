// Single translation unit of libtiler_cuda.so: the per-device exp table
// (g_exp2_table) is one __device__ symbol shared by every family kernel, so
// the families are compiled together rather than with relocatable device code.
#include "reduce.cu"
#include "rows.cu"
#include "rms_scan.cu"
#include "rms_stream.cu"
#include "maps.cu"
#include "gemm.cu"
#include "abi.cu"
#include "no_alloc.cu"
#include "exchange.cu"
