// Argument blocks shared between the C ABI (capi.cu) and the kernels.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace pir2b {

struct QuantArgs {
  const __nv_bfloat16 *x;   // [rows, ldx]
  int64_t ldx;
  const __nv_bfloat16 *up;  // [rows, ldu] (gated mode) or null
  int64_t ldu;
  const uint16_t *lut;      // bf16 bits [65536] or null
  const float *smooth;      // [k] or null
  uint8_t *q;
  float *scales;
  int k;
  int kpad;
  int mode;
};

struct NormArgs {
  const __nv_bfloat16 *x;        // [rows, k]
  const __nv_bfloat16 *y_in;     // [rows, k] or null
  const __nv_bfloat16 *gate;     // [rows / tokens, ld_mod] or null (= 1)
  __nv_bfloat16 *res_out;        // [rows, k] or null
  const __nv_bfloat16 *gamma;    // [k] (RMS)
  const __nv_bfloat16 *scale;    // [rows / tokens, ld_mod] or null
  const __nv_bfloat16 *shift;
  const float *smooth;
  uint8_t *q;
  uint8_t *scales;               // fp32 [rows] or NVFP4 swizzled bytes
  int64_t ld_mod;
  int64_t tokens;
  int k;
  int kpad;
  float eps;
  // RMSNorm statistics in torch's row-mean order (integer outputs): the
  // threads per row torch's reduction uses for this [rows, k] shape, and
  // its fp32 factor rows / (rows * k).
  int rms_bw;
  float rms_factor;
};

struct GemmArgs {
  const float *sa;                  // [M] activation row scales
  const float *sw;                  // [Npad] weight channel scales
  const __nv_bfloat16 *bias;        // [Npad] or null
  const __nv_bfloat16 *out_lut;     // [65536] activation table or null
  const __nv_bfloat16 *residual;    // [M, ldr] added after rounding, or null
  int64_t ldr;                      // residual row stride (elements)
  __nv_bfloat16 *out;               // [M, ldo]
  int64_t ldo;                      // output row stride (elements)
  int m;                            // token rows
  int n_store;                      // channels written (<= Npad)
  int num_kb;                       // K blocks of 128 elements
  int bias_mode;                    // 0: none, 1: add +0, 2: add bias
  int bn;                           // token tile (multiple of 16, <= 256)
  int stages;                       // pipeline depth
  int splits;                       // cluster size along z (1,2,4,8)
  int tma_store;                    // 1: output tile leaves through TMA
  int wt;                           // 128-channel weight tiles per CTA (1, 2)
  int npairs;                       // (2-SM kernel) CTA pairs along the channels
  // SwiGLU epilogue (wt == 2, no split-K): weight tile 0 holds 128 gate
  // channels and tile 1 the matching up channels; the CTA writes
  // bf16(silu_lut[gate] * up) for those 128 output channels.
  const __nv_bfloat16 *silu_lut;    // [65536] or null
  // Fused activation pack (int8, one token tile): bf16 rows x[m, ldx]
  // replace the packed activations.  The CTA bulk-copies the rows (its K
  // slice when x_max gives the row maxima, else whole rows) into shared
  // memory, derives the row scales and writes the int8 codes of its K
  // slice in the swizzled operand layout.
  const __nv_bfloat16 *x;           // null: packed activations through TMA
  int64_t ldx;
  int k;                            // logical K of x (codes past k are 0)
  const float *x_max;               // [m, x_parts] partial |x| maxima, or null
  int x_parts;
  int fused_kb;                     // K blocks of codes the CTA holds
  int x_stride;                     // bytes per staged row
  int x_bytes;                      // staged rows region
  // Per-16-channel |y| maxima of the bf16 output, [m, max_parts], or null:
  // a later fused pack of this output reads them as its x_max.
  float *max_out;
  int max_parts;
};

cudaError_t run_quant_rows(const QuantArgs &a, int bits, int64_t rows,
                           bool vec, cudaStream_t st);
cudaError_t run_norm_quant(const NormArgs &a, int out_format, int64_t rows,
                           int norm, bool mod, bool res, cudaStream_t st);

template <int kBits, bool kWide = false>
__global__ void gemm_i8_kernel(const __grid_constant__ CUtensorMap tm_w,
                               const __grid_constant__ CUtensorMap tm_a,
                               const __grid_constant__ CUtensorMap tm_out,
                               const GemmArgs args);

} // namespace pir2b
