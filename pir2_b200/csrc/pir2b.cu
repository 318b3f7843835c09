// Single translation unit of libpir2b.so: the kernels and the C ABI share
// one definition of the device status word without relocatable device code.
#include "quant.cuh"
#include "gemm_i8.cuh"
#include "gemm_pair.cuh"
#include "gemm_few.cuh"
#include "probe.cuh"
#include "gemm_fp4.cuh"
#include "dit_ffn.cuh"
#include "pointwise.cuh"
#include "attention.cuh"
#include "capi.cuh"
