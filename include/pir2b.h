/*
 * pir2b — C ABI of the B200 (sm_100a) quantized-Linear library.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (cudaStream_t passed as void*), launches asynchronously on that stream,
 * allocates nothing, never synchronizes, and returns a status:
 *     0                 success
 *     PIR2B_EINVAL (1)  bad shape / size / mode / null pointer
 *     PIR2B_EALIGN (2)  pointer or stride alignment not met
 *     PIR2B_ECUDA (-1)  a CUDA runtime call failed (launch error)
 * pir2b_last_error() returns the message of the last failure on the calling
 * thread.  Because nothing allocates or syncs, calls can be captured into
 * CUDA graphs once the library has been loaded.
 *
 * Formats ("symmetric-row-v1", piR2 coexecution/kernels/ampere_ada/integer.py):
 *   Kpad = ceil(K / 128) * 128, Npad = ceil(N / 8) * 8, L = 2^(bits-1) - 1.
 *   Activations: per-row fp32 scale s = max|v| * (1/L) (1.0 for an all-zero
 *   row), q = clamp(rint(v / s), -L, L); int8 rows of Kpad bytes, or int4
 *   rows of Kpad/2 bytes, low nibble = even column.
 *   Weights: per-output-channel fp32 scale, same code layout, [Npad, Kpad].
 */
#ifndef PIR2B_H
#define PIR2B_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PIR2B_OK 0
#define PIR2B_EINVAL 1
#define PIR2B_EALIGN 2
#define PIR2B_ECUDA (-1)

/* Activation selection modes of the quantizer (integer.py:27-47). */
#define PIR2B_MODE_PLAIN 0 /* v = x                                  */
#define PIR2B_MODE_GATED 1 /* v = bf16(lut[x] * up)  (SiLU/GELU * up) */
#define PIR2B_MODE_LUT 2   /* v = lut[x]             (GELU)           */

/* Bias handling of the GEMM epilogue (integer_gemm.cu:73-76, 164-168). */
#define PIR2B_BIAS_NONE 0 /* gemm_biasless without bias: no add         */
#define PIR2B_BIAS_ZERO 1 /* gemm with a null bias: adds +0 (-0 -> +0)  */
#define PIR2B_BIAS_ADD 2  /* y + f32(bias[n])                           */

/* Norm kinds of the fused producer. */
#define PIR2B_NORM_NONE 0 /* input already normalized                      */
#define PIR2B_NORM_RMS 1  /* x * rsqrt(mean(x^2) + eps), then * gamma       */
#define PIR2B_NORM_LN 2   /* non-affine LayerNorm                          */

/* Output formats of the fused producer. */
#define PIR2B_OUT_INT8 8
#define PIR2B_OUT_INT4 4
#define PIR2B_OUT_NVFP4 16
/* First pass of the FP8 producers: bf16 values + the row's maximum finite
 * |value| (fp32), cast to E4M3 by pir2b_fp8_cast. */
#define PIR2B_OUT_FP8_VALUES 32

/* Library version (major * 100 + minor). */
int pir2b_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char *pir2b_last_error(void);

/* Reads, then clears, the device status word that bounded in-kernel waits
 * set when they give up (0: no wait expired).  Synchronizes `stream`.
 * No counterpart in the reference (which has no bounded device waits). */
int pir2b_device_status(int *status_out, void *stream);

/* Status word value left by pir2b_wait_probe. */
#define PIR2B_STATUS_TIMEOUT_PROBE 0x105

/* Self-test of the bounded device waits: launches one thread that waits on
 * an mbarrier nothing arrives at.  The wait gives up after its budget
 * (about 1 s), sets the device status word to PIR2B_STATUS_TIMEOUT_PROBE
 * and writes 0 to the device int `result`.  Asynchronous on `stream`.
 * No counterpart in the reference. */
int pir2b_wait_probe(int *result, void *stream);

/* Per-row symmetric quantization and packing of BF16 activations.
 * Replaces the Triton `_prepare` kernel and its native twin
 * `prepare_integer<Bits>`:
 *   coexecution/kernels/ampere_ada/integer.py:50-94, :107-173
 *   coexecution/kernels/ampere_ada/csrc/integer_dispatch.cu:11-65, :262-303
 *   coexecution/optimization/backends/integer/linear.py:51-90 (`prepare`)
 * x: bf16 [rows, k] with row stride ldx (elements); up: bf16 rows (stride
 * ldu) for MODE_GATED, else NULL; lut: bf16[65536] for MODE_GATED/MODE_LUT;
 * smooth: optional fp32 [k] SmoothQuant divisor applied as bf16(bf16(v)/s)
 * before quantization (thor/packing.py:69-73), NULL to skip.
 * q: int8 [rows, Kpad] (bits 8) or uint8 [rows, Kpad/2] (bits 4);
 * scales: fp32 [rows].  1 <= k <= 65536, rows >= 0. */
int pir2b_quant_rows(const void *x, int64_t ldx, const void *up, int64_t ldu,
                     const void *lut, const float *smooth, int mode, int bits,
                     int64_t rows, int64_t k, void *q, float *scales,
                     void *stream);

/* pir2b_quant_rows (plain values) for rows whose maximum |x| is already known
 * as partial maxima: x_max [rows, parts] fp32, e.g. the per-16-channel output
 * maxima of the GEMM that wrote x (pir2b_gemm_fused's max_out).  The row
 * scale comes from max_i x_max[row, i] and the codes are elementwise, so the
 * pack runs without a row reduction over x; codes and scales are bitwise
 * those of pir2b_quant_rows when x_max holds the rows' exact maxima.  The
 * same pack as the reference's `_prepare` (coexecution/kernels/ampere_ada/
 * integer.py:50-94) with its row statistic supplied by the producer.
 * q: int8 [rows, Kpad] (bits 8) or uint8 [rows, Kpad/2] (bits 4); scales:
 * fp32 [rows]. */
int pir2b_quant_rows_max(const void *x, int64_t ldx, const float *x_max, int64_t parts, int bits, int64_t rows,
                         int64_t k, void *q, float *scales, void *stream);

/* The values of pir2b_quant_rows (plain, LUT activation, SiLU * up; the
 * optional SmoothQuant division) to the floating formats of the piR2 Thor
 * producers:
 *   coexecution/optimization/backends/thor/packing.py:84-107 (_swiglu_pack,
 *     prepare_swiglu), :314-349 (_smooth_pack, prepare_smoothed), :352-392
 *     (_gelu_pack, prepare_gelu_packed), with _store_producer :57-82
 * out_format PIR2B_OUT_NVFP4: q = packed E2M1 [rows, k/2], scales = the
 *   swizzled UE4M3 block-16 factors (layout of pir2b_pack_nvfp4), k % 32 == 0;
 * out_format PIR2B_OUT_FP8_VALUES: q = bf16 values [rows, k], scales = fp32
 *   [rows, ceil(k / 1024)] partial maxima of the finite |value| (each row in
 *   slices of 1024 values), k % 16 == 0; pir2b_fp8_cast finishes the E4M3
 *   pack (packing.py:180-199).  q may be NULL here: the maxima alone, the
 *   first pass of a plain per-tensor quantization whose cast reads x in
 *   place.
 * 16 <= k <= 8192; q 16-byte aligned. */
int pir2b_floating_rows(const void *x, int64_t ldx, const void *up, int64_t ldu,
                        const void *lut, const float *smooth, int mode, int out_format,
                        int64_t rows, int64_t k, void *q, void *scales, void *stream);

/* Second pass of the FP8 producers and of the two-pass per-tensor
 * quantizer: the scale from the nmax partial maxima of the first pass (a
 * PIR2B_OUT_FP8_VALUES pass, or the per-row maxima of a norm producer) and
 * the E4M3 cast,
 *   coexecution/optimization/backends/thor/packing.py:180-199, :461-482
 *   (_finish_producer, _fp8_scale_and_cast), fast != 0:
 *     scale = max(max_i maxima[i] * (1/448), 1e-12);
 *     q = e4m3(clamp(v / scale, +-448)) with round-to-nearest division;
 *   fp8_cutlass_linear.cu:61-120 (quantize_bf16), fast == 0:
 *     scale = max(amax / 448, 1e-12); q = e4m3(clamp(v * (1 / scale), +-448)).
 * v: bf16 rows of stride ldv (elements, % 8 == 0), k % 8 == 0; q: [rows, k]
 * bytes; the scale is written to scale[0] and to scale_rep[0..n_rep) (null
 * when n_rep == 0). */
int pir2b_fp8_cast(const void *v, int64_t ldv, const float *maxima, int64_t nmax, int64_t rows, int64_t k,
                   int fast, void *q, float *scale, float *scale_rep, int64_t n_rep, void *stream);

/* Fused norm (+ AdaLN modulation) (+ gated residual) + quantize/pack.
 * Replaces the Triton producers of
 *   coexecution/kernels/ampere_ada/modulation.py:14-239 (modulation,
 *     non-affine LayerNorm + modulation, residual + LayerNorm + modulation)
 *   coexecution/kernels/ampere_ada/producers.py:19-90 (`prepare_rmsnorm`)
 *   coexecution/kernels/ampere_ada/csrc/layernorm_pack.cu:125-303
 *   coexecution/optimization/backends/thor/packing.py:84-448 (FP4 outputs)
 * Row r of x (bf16, contiguous [rows, k]):
 *   if y_in:  x' = bf16(x + bf16(y_in * gate[r / tokens]))  (written to
 *             res_out, modulation.py:212-216)
 *   norm:     NONE: n = x'; RMS: n = bf16(bf16(x' * rsqrt(var + eps)) *
 *             gamma); LN: n = bf16((x' - mean) * rsqrt(var + eps))
 *   if scale: v = bf16(bf16(n * bf16(1 + scale[r / tokens])) + shift[...])
 *             (modulation.py:103-107); scale/shift rows have stride ld_mod
 *   smooth:   optional SmoothQuant divisor as in pir2b_quant_rows
 *   out_format INT8 / INT4: symmetric-row-v1 q + scales;
 *   out_format NVFP4: q = packed E2M1 [rows, k/2], scales = swizzled UE4M3
 *             block-16 factors (layout of pir2b_pack_nvfp4);
 *   out_format FP8_VALUES: q = bf16 values [rows, k], scales = fp32 [rows]
 *             maximum finite |value| (then pir2b_fp8_cast).  The floating
 *             outputs take the Thor producers' RMS variance, sum(x^2) / k
 *             (packing.py:396-415).
 * 8 <= k <= 8192, k % 8 == 0 (k % 32 == 0 for NVFP4, % 16 for FP8_VALUES); pointers 16-byte
 * aligned.  (The reference RMS producer has the same k <= 8192 bound,
 * producers.py:295.) */
int pir2b_norm_quant_rows(const void *x, const void *y_in, const void *gate,
                          void *res_out, const void *gamma, const void *scale,
                          const void *shift, int64_t ld_mod, int64_t tokens,
                          const float *smooth, int norm_kind, float eps,
                          int out_format, int64_t rows, int64_t k, void *q,
                          void *scales, void *stream);

/* Quantized GEMM with fused dequant epilogue on tcgen05 (kind::i8).
 * Replaces pir2_integer::gemm / gemm_biasless
 *   coexecution/kernels/ampere_ada/csrc/integer_gemm.cu:22-195
 * and its Ada-only twins (split-K reduce_scale, integer_split_k.cu:27-52;
 * int4 small-M tiles, int4_small_m.cu:17-42; int4 GEMV, int4_gemv.cu:29-61).
 * qa: activations int8 [m, Kpad] / uint8 [m, Kpad/2]; sa fp32 [m];
 * qw: weights int8 [npad, Kpad] / uint8 [npad, Kpad/2]; sw fp32 [npad];
 * bias: bf16 [npad] (bias_mode ADD) or NULL; out_lut: optional bf16[65536]
 * table applied to the bf16 result (fuses GELU/SiLU producers);
 * residual: optional bf16 [m, ldr]; when given, out = bf16(f32(result) +
 * f32(residual)) -- the residual epilogue of integer_epilogue.cu:156-327
 * (pir2_integer_epilogue::gemm with a residual, epilogue.py:360-398);
 * out: bf16, row stride ldo, columns [0, n_store) written.
 * kpad % 128 == 0, npad % 8 == 0, n_store <= npad, m >= 1.
 * The weight tiles are requested before the kernel's programmatic-dependent
 * wait (they overlap the previous kernel): qw, like every GEMM weight in
 * this header, must not be written by the kernel launched just before on
 * the same stream (weights are packed at install time).
 * tactic: -1 selects the tile shape by heuristic; piR2's Ada tactic ids
 * 0..7 are accepted and ignored (tiles are chosen for B200). */
int pir2b_gemm(const void *qa, const float *sa, const void *qw,
               const float *sw, const void *bias, int bias_mode,
               const void *out_lut, const void *residual, int64_t ldr,
               int bits, int64_t m, int64_t npad, int64_t kpad, void *out,
               int64_t ldo, int64_t n_store, int tactic, void *stream);

/* NVFP4 (E2M1 values, UE4M3 scale per 16 elements) packing of bf16 rows.
 * Replaces pack_matrix_fp4_ue_rowmajor_kernel / pack_activation_gemm_bf16 /
 * pack_linear_weight_gemm_bf16:
 *   coexecution/kernels/blackwell/csrc/fp4_cutlass_linear.cu:789-842,
 *   :1530-1587, :1714-1749; Triton twin thor/packing.py:24-54.
 * x: bf16 [rows, k] contiguous, k % 32 == 0.  packed: uint8 [rows, k/2];
 * sf: uint8 [ceil(rows/128)*128, ceil(k/64)*4] in the 128x4 swizzled layout
 * (sfa_offset, fp4_cutlass_linear.cu:686-690).  Division is IEEE
 * round-to-nearest (the Triton variant). */
int pir2b_pack_nvfp4(const void *x, int64_t rows, int64_t k, void *packed,
                     void *sf, void *stream);

/* NVFP4 GEMM on tcgen05 kind::mxf4nvf4 (block16 UE4M3 scales), fp32
 * accumulate, out = bf16(alpha * acc [+ bias]).
 * Replaces linear_forward_packed_gemm_bf16_tactic
 *   coexecution/kernels/blackwell/csrc/fp4_cutlass_linear.cu:1751-1847.
 * qa [m, k/2] + sfa (swizzled, rows padded to 128); qw [n, k/2] + sfw;
 * bias bf16 [n] or NULL; out bf16 [m, ldo]; out = bf16(alpha * acc + bias).
 * k % 256 == 0 (one K block = 256 values + 16 factors per row; piR2 accepts
 * k % 32 == 0), operands 16-byte aligned. */
int pir2b_gemm_nvfp4(const void *qa, const void *sfa, const void *qw,
                     const void *sfw, const void *bias, float alpha,
                     int64_t m, int64_t n, int64_t k, void *out, int64_t ldo,
                     void *stream);

/* Fused per-head RMSNorm (Qwen3 q_norm / k_norm) + rotary embedding of the
 * q and k heads of a grouped q|k|v projection output, and the [B, H, T, D]
 * relayout of q, k and v for attention.  BF16 pointwise fusion next to the
 * quantized path; replaces the RoPE and RMSNorm kernels of
 *   coexecution/fused_ops.py:34-147 (rope), :150-232 (rmsnorm).
 * qkv: bf16 [rows = B*T, ld], q heads then k heads then v heads (head_dim
 * 128); cos/sin: bf16 [T, 128]; outputs bf16 [B, hq|hk, T, 128]. */
int pir2b_qk_norm_rope(const void *qkv, int64_t ld, const void *q_weight,
                       const void *k_weight, const void *cos, const void *sin,
                       int64_t rows, int64_t tokens, int hq, int hk,
                       int head_dim, float eps, void *q_out, void *k_out,
                       void *v_out, void *stream);

/* The W8A8 feed-forward half of a DiT block in one launch:
 *   out = residual + down(pack(gelu(up(x))))
 * with x the packed FFN input (int8 [m, d] codes + fp32 row scales, e.g. the
 * norm3 pack), up weights int8 [f, d] (+ sw_up [f], bias_up [f]), the GELU
 * table gelu_lut (torch-built, 65536 bf16), down weights int8 [d, f]
 * (+ sw_down [d], bias_down [d]).  Bitwise equal to the four launches piR2
 * runs for it (up GEMM, GELU pack of the down projection's input
 * (`forward_gelu`, coexecution/optimization/groot/integer.py:161-165), down
 * GEMM, residual add (integer_epilogue.cu:156-327)).  1 <= m <= 64,
 * d % 128 == 0, f % 1024 == 0, f/128 + 8*d/128 CTAs must fit the SMs at
 * once, and the whole grid must be resident at the same time (CTAs wait on
 * one another through counters, each wait bounded at about a second: do
 * not run other kernels concurrently on the device).  `workspace`
 * (256-byte aligned, pir2b_dit_ffn_workspace(m, f) bytes) holds the int8
 * codes of the intermediate activations, their row scales and three
 * counters; it must be zero before the first call and every call leaves
 * the counters zeroed; calls sharing a workspace must be stream-ordered. */
int64_t pir2b_dit_ffn_workspace(int64_t m, int64_t f);
int pir2b_dit_ffn(const void *qa, const float *sa, const void *up_w, const float *up_sw,
                  const void *up_bias, int up_bias_mode, const void *gelu_lut,
                  const void *down_w, const float *down_sw, const void *down_bias,
                  int down_bias_mode, const void *residual, int64_t ldr, int64_t m, int64_t d,
                  int64_t f, void *out, int64_t ldo, void *workspace, int64_t workspace_bytes,
                  void *stream);

/* pir2b_dit_ffn with its scratch in a static device array of this library
 * (about 530 KB on every device that loads it, held until the process
 * exits) instead of a caller workspace.  No counterpart in the reference.
 * It is for callers that cannot call cudaMalloc once they are running, such
 * as a robot control loop that must not allocate device memory after
 * start-up, or a host runtime that owns every device buffer and exposes no
 * allocator to its plugins: they pass inputs and outputs and nothing else.
 * It calls no cudaMalloc, cudaFree or allocating library routine.
 * 1 <= m <= 64 and f <= 8192 (the array's size; larger problems return
 * PIR2B_EINVAL), the other limits as pir2b_dit_ffn.  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress) with
 * that device current; make that first call before any stream capture.
 * Each call clears the array's counters on `stream` first; the rest of the
 * array keeps the last call's contents and is written before it is read.
 * All calls on one device share the array: calls that overlap on the GPU
 * (different streams, not ordered) race and corrupt each other's results,
 * so order them on one stream or synchronise between them; calls on
 * different devices are independent. */
int pir2b_dit_ffn_static(const void *qa, const float *sa, const void *up_w, const float *up_sw,
                         const void *up_bias, int up_bias_mode, const void *gelu_lut,
                         const void *down_w, const float *down_sw, const void *down_bias,
                         int down_bias_mode, const void *residual, int64_t ldr, int64_t m,
                         int64_t d, int64_t f, void *out, int64_t ldo, void *stream);

/* pir2b_gemm with two options for chains of small-M projections.
 *
 * Fused activation pack (x non-null, qa and sa null): bf16 rows x[m, ldx]
 * (m <= 64, k % 8 == 0, int8 weights) are quantized inside the GEMM by the
 * plain symmetric-row-v1 pack (coexecution/kernels/ampere_ada/integer.py:
 * 27-94, the pack pir2b_quant_rows runs), so the result is bitwise
 * pir2b_quant_rows followed by pir2b_gemm, with one launch instead of two.
 * Each CTA stages whole rows in shared memory to find the row maxima, or,
 * when x_max is given ([m, x_parts] partial maxima of |x|, x_parts % 4 ==
 * 0, e.g. the max_out of the GEMM that wrote x), only its own K slice.
 * Returns PIR2B_EINVAL when the rows do not fit (then pack separately).
 *
 * max_out (non-null): also writes max_out[r, g] = max |out[r, 16g..16g+15]|
 * for g < npad / 16 (the output's per-16-channel maxima, ready as the
 * x_max of a fused pack of `out`); needs npad % 16 == 0 and 16-byte aligned
 * output rows.  Exactly one of qa / x is non-null. */
int pir2b_gemm_fused(const void *qa, const float *sa, const void *x, int64_t ldx, int64_t k,
                     const float *x_max, int64_t x_parts, const void *qw, const float *sw,
                     const void *bias, int bias_mode, const void *out_lut, const void *residual,
                     int64_t ldr, int bits, int64_t m, int64_t npad, int64_t kpad, void *out,
                     int64_t ldo, int64_t n_store, float *max_out, void *stream);

/* Per-tensor E4M3 quantization of bf16 rows x[rows, ldx] (k % 8 == 0) into
 * q[rows, k] and one fp32 scale, the FP8 path's activation and weight pack:
 *   fast == 0: coexecution/kernels/blackwell/csrc/fp8_cutlass_linear.cu:
 *     61-120 (quantize_bf16 / pack_linear_weight): scale = max(amax/448,
 *     1e-12), q = e4m3_rn_satfinite(clamp(x * (1/scale), +-448));
 *   fast != 0: coexecution/optimization/backends/thor/packing.py:451-519
 *     (prepare_fp8): scale = max(amax * (1/448), 1e-12), q = e4m3(clamp(
 *     x / scale, +-448)) with round-to-nearest division;
 * amax is the maximum of the finite |x|.  The scale is also written to
 * scale_rep[0..n_rep) (null when n_rep == 0), the replicated vector the
 * FP8 GEMM reads as per-row or per-channel scales.  One launch.  weights
 * != 0 when q are GEMM weights: every GEMM entry of this library reads its
 * weights before its programmatic-dependent wait (they are normally packed
 * at install time), so a weight pack launched right before a GEMM must not
 * let it start early; with weights != 0 it does not. */
int pir2b_quant_fp8(const void *x, int64_t ldx, int64_t rows, int64_t k, int fast, int weights,
                    void *q, float *scale, float *scale_rep, int64_t n_rep, void *stream);

/* E4M3 GEMM on tcgen05 kind::f8f6f4 with fp32 accumulation:
 *   out[m, n] = bf16(f32(f32(acc * sa[m]) * sw[n]) [+ bias[n]]) [+ residual]
 * with the per-tensor scales given as replicated vectors (sa: m floats,
 * sw: npad floats, from pir2b_quant_fp8).  Replaces the CUTLASS FP8 GEMM
 * (fp8_cutlass_linear.cu:470-665, linear_forward_packed_tactic :1026-1145,
 * whose epilogue applies scale_a * scale_b and the per-column bias).
 * qa [m, kpad], qw [npad, kpad] E4M3 bytes, kpad % 128 == 0.  out_lut
 * (bf16[65536] or NULL) maps each bf16 result through an activation table
 * (GELU) before the residual; max_out (fp32 [m, npad / 16] or NULL; m <= 32)
 * receives per-16-column maxima of the finite |out|, the partial maxima
 * pir2b_fp8_cast packs `out` with (the GELU producer of the FP8 DiT FFN,
 * thor/packing.py:352-392, in the GEMM's epilogue). */
int pir2b_gemm_fp8(const void *qa, const float *sa, const void *qw, const float *sw,
                   const void *bias, int bias_mode, const void *residual, int64_t ldr, int64_t m,
                   int64_t npad, int64_t kpad, void *out, int64_t ldo, int64_t n_store,
                   const void *out_lut, float *max_out, void *stream);

/* W8A8 gate|up GEMM with the SwiGLU epilogue: out[m, c] =
 * bf16(f32(silu_lut[g]) * f32(u)) for c < half_n, where g and u are the
 * exact dequantized bf16 GEMM outputs of gate channel c and up channel c.
 * The weight rows (and sw, bias) are interleaved in blocks of 128: rows
 * 256j..256j+127 are gate channels 128j.., rows 256j+128..256j+255 the
 * matching up channels.  The result equals piR2's text MLP path, which
 * writes gate|up (coexecution/optimization/groot/integer.py:166-172) and
 * packs bf16(SiLU(gate) * up) in the down projection's gated pack
 * (coexecution/kernels/ampere_ada/integer.py:27-48); here the down
 * projection packs `out` plainly.  half_n % 128 == 0, kpad % 128 == 0.
 * max_out (fp32 [m, half_n / 16], or NULL) receives the per-16-column
 * maxima of |out|, the row statistic pir2b_quant_rows_max packs `out` with;
 * it needs a 16-byte aligned `out` with ldo % 8 == 0. */
int pir2b_gemm_swiglu(const void *qa, const float *sa, const void *qw, const float *sw,
                      const void *bias, int bias_mode, const void *silu_lut, int64_t m,
                      int64_t half_n, int64_t kpad, void *out, int64_t ldo, float *max_out,
                      void *stream);

/* Small-sequence attention (no mask) reading q, k, v from projection rows
 * (head h at columns h*head_dim..) and writing out[b*T + t, h*head_dim + d]
 * rows for the output projection's pack; fp32 scores and softmax, bf16 out.
 * Replaces the DiT's torch SDPA + transpose (coexecution/groot_pointwise.py:
 * 58-92) next to the quantized path.  head_dim in {32, 48, 64, 96, 128},
 * row strides of q/k/v multiples of 8 elements, q/k/v 16-byte aligned; S is
 * split over a cluster of up to 8 CTAs per head, each holding its keys in
 * shared memory (S up to about 5000 at head_dim 48). */
int pir2b_attention_rows(const void *q, int64_t ldq, const void *k,
                         int64_t ldk, const void *v, int64_t ldv, void *out,
                         int64_t ldo, int64_t batch, int64_t tq, int64_t skv,
                         int heads, int head_dim, float scale, void *stream);

/* Unpacks int4 codes (two per byte, low nibble first: the symmetric-row-v1
 * activation pack of coexecution/kernels/ampere_ada/integer.py:79-93 and
 * the weight packing of :234-238) into sign-extended int8 codes, one per
 * byte.
 * packed: [rows, k/2] bytes; out: [rows, k] int8; k a multiple of 32, both
 * 16-byte aligned.  The int8 GEMM of unpacked codes gives the int4 GEMM's
 * int32 sums exactly; W4A4 layers with many tokens run that way. */
int pir2b_unpack_int4(const void *packed, int64_t rows, int64_t k, void *out, void *stream);

/* Causal grouped-query attention of the VLM text layers (head_dim 128).
 * q: bf16 [batch, hq, T, 128], k and v: bf16 [batch, hk, T, 128] (the
 * outputs of pir2b_qk_norm_rope); out: bf16 rows out[b*T + t, h*128 + d]
 * with row stride ldo, the o_proj input.  Replaces the torch SDPA call
 * (is_causal, enable_gqa) and the [B, H, T, D] -> [B*T, H*D] transpose copy
 * around the quantized o_proj of the Qwen3-VL text attention; the
 * reference keeps transformers' "sdpa" attention there and checks for it
 * (coexecution/optimization/groot/vlm.py:312-313).  Query head h reads kv
 * head h / (hq / hk); key j is visible to query t when j <= t. */
int pir2b_attention_causal(const void *q, const void *k, const void *v, int64_t batch,
                           int64_t tokens, int hq, int hk, int head_dim, float scale, void *out,
                           int64_t ldo, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* PIR2B_H */
