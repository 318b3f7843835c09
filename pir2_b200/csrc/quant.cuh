// Activation producers: per-row symmetric int8/int4 quantization and packing
// (symmetric-row-v1), fused with the optional LUT activation (GELU, SiLU*up),
// SmoothQuant channel division, RMSNorm / non-affine LayerNorm, AdaLN
// modulation and the gated residual add, plus the NVFP4 (E2M1 + UE4M3
// block-16) output format.
//
// One CTA per row.  Each thread owns whole 8-element chunks (one 16-byte
// load of bf16), strided by the block size, keeps the row in registers
// across the reductions, and reduces with warp shuffles plus one
// shared-memory hop.  Every BF16 rounding boundary of the reference
// producers is kept (see the per-function citations).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdint>

#pragma once
#include "args.cuh"
#include "ptx.cuh"

namespace pir2b {





__device__ __forceinline__ float bf16r(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

__device__ __forceinline__ float lut_value(const uint16_t *lut,
                                           __nv_bfloat16 x) {
  return __bfloat162float(
      __ushort_as_bfloat16(__ldg(lut + __bfloat16_as_ushort(x))));
}

// Block-wide reductions over blockDim.x (a multiple of 32, <= 1024).
__device__ __forceinline__ float block_max(float v, float *red) {
  for (int d = 16; d; d >>= 1)
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0)
    red[w] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  v = l < nw ? red[l] : 0.f;
  for (int d = 16; d; d >>= 1)
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
  return v;
}

__device__ __forceinline__ float block_sum(float v, float *red) {
  for (int d = 16; d; d >>= 1)
    v += __shfl_xor_sync(0xffffffffu, v, d);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0)
    red[w] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  v = l < nw ? red[l] : 0.f;
  for (int d = 16; d; d >>= 1)
    v += __shfl_xor_sync(0xffffffffu, v, d);
  return v;
}

// Loads 8 consecutive bf16 starting at column c0 of a row (zero past k).
template <bool kVec>
__device__ __forceinline__ void load8(const __nv_bfloat16 *row, int c0, int k,
                                      __nv_bfloat16 (&v)[8]) {
  if (kVec) {
    if (c0 < k) {
      const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(row + c0));
      const __nv_bfloat16 *p = reinterpret_cast<const __nv_bfloat16 *>(&raw);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        v[i] = p[i];
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        v[i] = __ushort_as_bfloat16(0);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      v[i] = (c0 + i < k) ? row[c0 + i] : __ushort_as_bfloat16(0);
  }
}

// Quantize 8 values with the row scale and store them (int8: 8 bytes at
// q + c0; int4: 4 bytes at q + c0 / 2, low nibble = even column).
template <int kBits>
__device__ __forceinline__ void store_codes(const float (&v)[8], float s,
                                            uint8_t *qrow, int c0) {
  constexpr int L = (1 << (kBits - 1)) - 1;
  int c[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = __float2int_rn(__fdiv_rn(v[i], s));
    c[i] = max(-L, min(L, r));
  }
  if (kBits == 8) {
    uint32_t lo = (c[0] & 255) | ((c[1] & 255) << 8) | ((c[2] & 255) << 16) |
                  (uint32_t(c[3] & 255) << 24);
    uint32_t hi = (c[4] & 255) | ((c[5] & 255) << 8) | ((c[6] & 255) << 16) |
                  (uint32_t(c[7] & 255) << 24);
    *reinterpret_cast<uint2 *>(qrow + c0) = make_uint2(lo, hi);
  } else {
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      w |= uint32_t(c[i] & 15) << (4 * i);
    *reinterpret_cast<uint32_t *>(qrow + c0 / 2) = w;
  }
}

// Row scale from the absolute maximum: m * (1/L) as an fp32 multiply by the
// fp32 constant, 1.0 for an all-zero row (integer.py:69-71,
// integer_dispatch.cu:237).
template <int kBits>
__device__ __forceinline__ float row_scale(float m) {
  constexpr float inv = 1.0f / float((1 << (kBits - 1)) - 1);
  return m > 0.f ? __fmul_rn(m, inv) : 1.0f;
}

// ------------------------------------------------------------------ NVFP4
// Per 16-element block: m = max|v|; s = m / 6 (1 if m == 0); e = e4m3_rn(min(s,
// 448)); d = f32(e), or s when e decodes to 0; codes = e2m1_rn_satfinite(v *
// (1 / d)).  thor/packing.py:24-54 (IEEE division variant).
__device__ __forceinline__ uint32_t cvt_e2m1x2(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b8 p;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 p, %2, %1;\n\t"
      "cvt.u32.u8 %0, p;\n\t}"
      : "=r"(r)
      : "f"(lo), "f"(hi));
  return r;
}

__device__ __forceinline__ uint32_t cvt_e4m3(float v) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.f), "f"(v));
  return r & 0xFFu;
}

__device__ __forceinline__ float e4m3_to_f32(uint32_t e) {
  // e4m3fn: 1 sign, 4 exponent bits (bias 7), 3 mantissa bits; exact in fp32.
  const uint32_t sign = (e & 0x80u) << 24, ex = (e >> 3) & 0xFu, man = e & 7u;
  const float mag = ex == 0 ? __fmul_rn(float(man), 1.0f / 512.0f)
                            : __uint_as_float(((ex + 120u) << 23) | (man << 20));
  return __uint_as_float(__float_as_uint(mag) | sign);
}

__device__ __forceinline__ int64_t nvfp4_sf_offset(int64_t row, int64_t sf,
                                                   int64_t blocks_k) {
  // 128 rows x 4 factors per 512-byte atom (fp4_cutlass_linear.cu:686-690).
  return ((row >> 7) * blocks_k << 9) + ((row & 31) << 4) +
         (((row & 127) >> 5) << 2) + ((sf >> 2) << 9) + (sf & 3);
}

// One thread holds 8 values = half a 16-block; its neighbour lane holds the
// other half (chunks 2b and 2b+1 belong to lanes 2l and 2l+1).
__device__ __forceinline__ void store_nvfp4_chunk(const float (&v)[8],
                                                  int64_t row, int chunk,
                                                  int k, uint8_t *packed,
                                                  uint8_t *sf) {
  float m = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    m = fmaxf(m, fabsf(v[i]));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  const float s = m > 0.f ? __fdiv_rn(m, 6.0f) : 1.0f;
  const uint32_t e = cvt_e4m3(fminf(s, 448.0f));
  float d = e4m3_to_f32(e);
  if (!(d > 0.f))
    d = s;
  const float r = __fdiv_rn(1.0f, d);
  uint32_t w = 0;
#pragma unroll
  for (int i = 0; i < 8; i += 2)
    w |= cvt_e2m1x2(__fmul_rn(v[i], r), __fmul_rn(v[i + 1], r)) << (4 * i);
  const int c0 = chunk * 8;
  if (c0 < k) {
    *reinterpret_cast<uint32_t *>(packed + row * (k / 2) + c0 / 2) = w;
    if ((chunk & 1) == 0) {
      const int64_t blocks_k = (k / 16 + 3) / 4;
      sf[nvfp4_sf_offset(row, chunk / 2, blocks_k)] = uint8_t(e);
    }
  }
}

// Stores a thread's chunks of a row (values already bf16-exact) as bf16:
// chunk c = cbase + threadIdx.x + j * blockDim.x covers columns [8c, 8c + 8).
template <int kCpt>
__device__ __forceinline__ void store_bf16_row(const float (&v)[kCpt][8], __nv_bfloat16 *out, int k,
                                               int nchunks, int cbase = 0) {
#pragma unroll
  for (int j = 0; j < kCpt; ++j) {
    const int chunk = cbase + threadIdx.x + j * blockDim.x;
    if (chunk < nchunks && chunk * 8 < k) {
      uint4 raw;
      __nv_bfloat16 *p = reinterpret_cast<__nv_bfloat16 *>(&raw);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        p[i] = __float2bfloat16_rn(v[j][i]);
      *reinterpret_cast<uint4 *>(out + chunk * 8) = raw;
    }
  }
}

// ------------------------------------------------------------------ quant_rows
// integer.py:27-94 (_activation_values, _prepare).  The same values (plain,
// LUT activation, SiLU * up, SmoothQuant division) also go to the floating
// outputs of the piR2 Thor producers (thor/packing.py:57-107, :314-369):
// kBits 16 writes NVFP4 (store_nvfp4_chunk); kBits 32 the bf16 values and
// partial maxima of the finite |value| (the first pass of the FP8 producers,
// whose second pass is fp8_cast_kernel).  An FP8 value needs no row
// statistic, so a kBits 32 row is split over gridDim.y CTAs (blockIdx.y
// takes the chunks from blockIdx.y * blockDim.x * kCpt) and each CTA writes
// its own maximum, scales[row * gridDim.y + blockIdx.y].
template <int kBits, int kCpt, bool kVec>
__global__ void __launch_bounds__(256) quant_rows_kernel(const QuantArgs a) {
  __shared__ float red[32];
  // Programmatic dependent launch: inputs come from the previous kernel.
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x;
  const int nchunks = a.kpad >> 3;
  const int cbase = int(blockIdx.y) * int(blockDim.x) * kCpt;   // 0 unless kBits == 32
  const __nv_bfloat16 *xr = a.x + int64_t(row) * a.ldx;
  const __nv_bfloat16 *ur = a.up ? a.up + int64_t(row) * a.ldu : nullptr;
  float v[kCpt][8];
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < kCpt; ++j) {
    const int chunk = cbase + threadIdx.x + j * blockDim.x;
    const int c0 = chunk * 8;
    __nv_bfloat16 xv[8];
    load8<kVec>(xr, chunk < nchunks ? c0 : a.k, a.k, xv);
    __nv_bfloat16 uv[8];
    if (a.mode == 1)
      load8<kVec>(ur, chunk < nchunks ? c0 : a.k, a.k, uv);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float t;
      if (a.mode == 0) {
        t = __bfloat162float(xv[i]);
      } else {
        t = lut_value(a.lut, xv[i]);
        if (a.mode == 1)
          t = bf16r(__fmul_rn(t, __bfloat162float(uv[i])));
      }
      if (c0 + i >= a.k)
        t = 0.f;
      if (a.smooth != nullptr && c0 + i < a.k)
        t = bf16r(__fdiv_rn(bf16r(t), __ldg(a.smooth + c0 + i)));
      v[j][i] = t;
      // Non-finite values do not enter the FP8 producers' maximum
      // (packing.py:76-78); fmaxf already skips NaN.
      if (kBits != 32 || fabsf(t) != INFINITY)
        m = fmaxf(m, fabsf(t));
    }
  }
  if constexpr (kBits == 16) {
#pragma unroll
    for (int j = 0; j < kCpt; ++j) {
      const int chunk = threadIdx.x + j * blockDim.x;
      // Every lane takes part in the pairwise shuffle; stores are guarded.
      store_nvfp4_chunk(v[j], row, chunk < nchunks ? chunk : nchunks, a.k, a.q,
                        reinterpret_cast<uint8_t *>(a.scales));
    }
    return;
  }
  m = block_max(m, red);
  if constexpr (kBits == 32) {
    if (threadIdx.x == 0)
      a.scales[int64_t(row) * gridDim.y + blockIdx.y] = m;
    // q == null: the maxima alone (the plain FP8 activation quantizer,
    // whose cast reads x in place).
    if (a.q != nullptr)
      store_bf16_row(v, reinterpret_cast<__nv_bfloat16 *>(a.q) + int64_t(row) * a.k, a.k, nchunks, cbase);
    return;
  }
  const float s = row_scale<kBits>(m);
  if (threadIdx.x == 0)
    a.scales[row] = s;
  uint8_t *qrow = a.q + int64_t(row) * (kBits == 8 ? a.kpad : a.kpad / 2);
#pragma unroll
  for (int j = 0; j < kCpt; ++j) {
    const int chunk = threadIdx.x + j * blockDim.x;
    if (chunk < nchunks)
      store_codes<kBits>(v[j], s, qrow, chunk * 8);
  }
}

// Rows wider than 8192: pass 1 reduces the absolute maximum, pass 2
// recomputes each value (same arithmetic) and stores the codes.
template <int kBits, bool kVec>
__device__ __forceinline__ void chunk_values(const QuantArgs &a,
                                             const __nv_bfloat16 *xr,
                                             const __nv_bfloat16 *ur,
                                             int chunk, float (&v)[8]) {
  const int c0 = chunk * 8;
  __nv_bfloat16 xv[8], uv[8];
  load8<kVec>(xr, c0, a.k, xv);
  if (a.mode == 1)
    load8<kVec>(ur, c0, a.k, uv);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float t;
    if (a.mode == 0) {
      t = __bfloat162float(xv[i]);
    } else {
      t = lut_value(a.lut, xv[i]);
      if (a.mode == 1)
        t = bf16r(__fmul_rn(t, __bfloat162float(uv[i])));
    }
    if (c0 + i >= a.k)
      t = 0.f;
    if (a.smooth != nullptr && c0 + i < a.k)
      t = bf16r(__fdiv_rn(bf16r(t), __ldg(a.smooth + c0 + i)));
    v[i] = t;
  }
}

template <int kBits, bool kVec>
__global__ void __launch_bounds__(512) quant_rows_stream_kernel(const QuantArgs a) {
  __shared__ float red[32];
  // Programmatic dependent launch: inputs come from the previous kernel.
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.x;
  const int nchunks = a.kpad >> 3;
  const __nv_bfloat16 *xr = a.x + int64_t(row) * a.ldx;
  const __nv_bfloat16 *ur = a.up ? a.up + int64_t(row) * a.ldu : nullptr;
  float m = 0.f;
  for (int chunk = threadIdx.x; chunk < nchunks; chunk += blockDim.x) {
    float v[8];
    chunk_values<kBits, kVec>(a, xr, ur, chunk, v);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      m = fmaxf(m, fabsf(v[i]));
  }
  m = block_max(m, red);
  const float s = row_scale<kBits>(m);
  if (threadIdx.x == 0)
    a.scales[row] = s;
  uint8_t *qrow = a.q + int64_t(row) * (kBits == 8 ? a.kpad : a.kpad / 2);
  for (int chunk = threadIdx.x; chunk < nchunks; chunk += blockDim.x) {
    float v[8];
    chunk_values<kBits, kVec>(a, xr, ur, chunk, v);
    store_codes<kBits>(v, s, qrow, chunk * 8);
  }
}

// Rows split across a thread-block cluster (small M, long rows): CTA rank r
// of the cluster owns a contiguous slice of the row's 8-element chunks,
// reduces its block maximum, publishes it in shared memory, and every CTA
// reads all ranks' maxima through distributed shared memory.  Same
// arithmetic as quant_rows_kernel (the maximum is order independent).
template <int kBits, int kCpt, bool kVec>
__global__ void __launch_bounds__(256) quant_rows_cluster_kernel(const QuantArgs a) {
  __shared__ float red[32];
  __shared__ float slice_max;
  pdl_wait();
  pdl_launch_dependents();
  const int row = blockIdx.y;
  const uint32_t rank = cluster_ctarank();
  const uint32_t csize = gridDim.x;
  const int nchunks = a.kpad >> 3;
  const int per = (nchunks + int(csize) - 1) / int(csize);
  const int c_begin = int(rank) * per;
  const int c_end = min(nchunks, c_begin + per);
  const __nv_bfloat16 *xr = a.x + int64_t(row) * a.ldx;
  const __nv_bfloat16 *ur = a.up ? a.up + int64_t(row) * a.ldu : nullptr;
  float v[kCpt][8];
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < kCpt; ++j) {
    const int chunk = c_begin + int(threadIdx.x) + j * int(blockDim.x);
    if (chunk < c_end) {
      chunk_values<kBits, kVec>(a, xr, ur, chunk, v[j]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        v[j][i] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
      m = fmaxf(m, fabsf(v[j][i]));
  }
  m = block_max(m, red);
  if (threadIdx.x == 0)
    slice_max = m;
  cluster_sync();
  float row_max = 0.f;
  const uint32_t addr = smem_u32(&slice_max);
  for (uint32_t p = 0; p < csize; ++p)
    row_max = fmaxf(row_max, __int_as_float(ld_cluster_s32(map_peer(addr, p))));
  // No CTA may exit while a peer still reads its slice maximum.
  cluster_sync();
  const float s = row_scale<kBits>(row_max);
  if (rank == 0 && threadIdx.x == 0)
    a.scales[row] = s;
  uint8_t *qrow = a.q + int64_t(row) * (kBits == 8 ? a.kpad : a.kpad / 2);
#pragma unroll
  for (int j = 0; j < kCpt; ++j) {
    const int chunk = c_begin + int(threadIdx.x) + j * int(blockDim.x);
    if (chunk < c_end)
      store_codes<kBits>(v[j], s, qrow, chunk * 8);
  }
}

// ------------------------------------------------------------------ norm
// modulation.py:86-219 (AdaLN, LayerNorm + AdaLN, residual + LayerNorm +
// AdaLN), producers.py:19-53 (RMSNorm tail), thor/packing.py:109-150, :395-415
// (the same producers to NVFP4, kOut 16, and to FP8, kOut 32: bf16 values
// and the row's maximum finite |value|, cast by fp8_cast_kernel).
template <int kOut, int kCpt, int kNorm, bool kMod, bool kRes>
__global__ void __launch_bounds__(256) norm_quant_kernel(const NormArgs a) {
  __shared__ float red[32];
  // Programmatic dependent launch: inputs come from the previous kernel.
  pdl_wait();
  pdl_launch_dependents();
  const int64_t row = blockIdx.x;
  const int nchunks = a.kpad >> 3;
  const int64_t cond = row / a.tokens;
  float v[kCpt][8];
#pragma unroll
  for (int j = 0; j < kCpt; ++j) {
    const int chunk = threadIdx.x + j * blockDim.x;
    const int c0 = chunk < nchunks ? chunk * 8 : a.k;
    __nv_bfloat16 xv[8];
    load8<true>(a.x + row * a.k, c0, a.k, xv);
    if (kRes) {
      __nv_bfloat16 yv[8], gv[8];
      load8<true>(a.y_in + row * a.k, c0, a.k, yv);
      if (a.gate != nullptr)
        load8<true>(a.gate + cond * a.ld_mod, c0, a.k, gv);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        // A null gate is an ungated residual: bf16(y * 1) == y.
        const float prod =
            a.gate != nullptr
                ? bf16r(__fmul_rn(__bfloat162float(yv[i]), __bfloat162float(gv[i])))
                : __bfloat162float(yv[i]);
        xv[i] = __float2bfloat16_rn(__fadd_rn(__bfloat162float(xv[i]), prod));
      }
      if (c0 < a.k) {
        uint4 raw;
        __nv_bfloat16 *p = reinterpret_cast<__nv_bfloat16 *>(&raw);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          p[i] = xv[i];
        *reinterpret_cast<uint4 *>(a.res_out + row * a.k + c0) = raw;
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i)
      v[j][i] = (c0 + i < a.k) ? __bfloat162float(xv[i]) : 0.f;
  }
  const float kf = float(a.k);
  if constexpr (kNorm == 1) {
    // RMSNorm: var = mean(x^2); n = bf16(x * rsqrt(var + eps)); v = bf16(n*g)
    float var;
    if constexpr (kOut != 16 && kOut != 32) {
      // The integer producer's variance is the reference's B200 path
      // (producers.py:19-53 via rms_statistics.py:171-190): fp32 squares,
      // then torch's fp32 row mean, whose order this reproduces (ATen
      // Reduce.cuh, vectorised input of 4 floats): virtual thread t of
      // rms_bw sums the vectors t, t + bw, t + 2 bw, ... in four
      // accumulators (one per vector element), combines them as
      // ((a0 + a1) + a2) + a3, and the bw partials meet in a pairwise tree
      // with halving offsets (shared memory down to 32, then the warp);
      // the mean is that sum times rows / (rows * k).
      // The squares of the row ([k / 4] float4, dynamic shared memory
      // sized by the launch) and the partial sums of the virtual threads.
      extern __shared__ float4 sq4[];
      __shared__ float part[512];
#pragma unroll
      for (int j = 0; j < kCpt; ++j) {
        const int chunk = threadIdx.x + j * blockDim.x;
        if (chunk < nchunks && chunk * 8 < a.k) {
          const float *e = v[j];
          sq4[2 * chunk] = make_float4(__fmul_rn(e[0], e[0]), __fmul_rn(e[1], e[1]),
                                       __fmul_rn(e[2], e[2]), __fmul_rn(e[3], e[3]));
          sq4[2 * chunk + 1] = make_float4(__fmul_rn(e[4], e[4]), __fmul_rn(e[5], e[5]),
                                           __fmul_rn(e[6], e[6]), __fmul_rn(e[7], e[7]));
        }
      }
      __syncthreads();
      if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        const int bw = a.rms_bw;
        const int nvec = a.k >> 2;
        for (int t = lane; t < bw; t += 32) {
          float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
          for (int idx = t; idx < nvec; idx += bw) {
            const float4 q4 = sq4[idx];
            a0 = __fadd_rn(a0, q4.x);
            a1 = __fadd_rn(a1, q4.y);
            a2 = __fadd_rn(a2, q4.z);
            a3 = __fadd_rn(a3, q4.w);
          }
          part[t] = __fadd_rn(__fadd_rn(__fadd_rn(a0, a1), a2), a3);
        }
        __syncwarp();
        for (int off = bw >> 1; off >= 32; off >>= 1) {
          for (int t = lane; t < off; t += 32)
            part[t] = __fadd_rn(part[t], part[t + off]);
          __syncwarp();
        }
        float s = lane < bw ? part[lane] : 0.f;
        for (int off = min(bw, 32) >> 1; off > 0; off >>= 1)
          s = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, off));
        if (lane == 0)
          red[0] = __fmul_rn(s, a.rms_factor);
      }
      __syncthreads();
      var = red[0];
      __syncthreads();   // red is reused by the row maximum below
    } else {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < kCpt; ++j)
#pragma unroll
        for (int i = 0; i < 8; ++i)
          ss = __fadd_rn(ss, __fmul_rn(v[j][i], v[j][i]));
      ss = block_sum(ss, red);
      var = __fdiv_rn(ss, kf);
    }
    const float inv = rsqrtf(__fadd_rn(var, a.eps));
#pragma unroll
    for (int j = 0; j < kCpt; ++j) {
      const int chunk = threadIdx.x + j * blockDim.x;
      const int c0 = chunk < nchunks ? chunk * 8 : a.k;
      __nv_bfloat16 gv[8];
      load8<true>(a.gamma, c0, a.k, gv);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float n = bf16r(__fmul_rn(v[j][i], inv));
        v[j][i] = (c0 + i < a.k) ? bf16r(__fmul_rn(n, __bfloat162float(gv[i])))
                                 : 0.f;
      }
    }
  } else if constexpr (kNorm == 2) {
    // Non-affine LayerNorm: mean, centred variance, n = bf16(c * rsqrt(var+eps))
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < kCpt; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i)
        sum = __fadd_rn(sum, v[j][i]);
    sum = block_sum(sum, red);
    const float mean = __fdiv_rn(sum, kf);
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kCpt; ++j) {
      const int chunk = threadIdx.x + j * blockDim.x;
      const int c0 = chunk < nchunks ? chunk * 8 : a.k;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float c = (c0 + i < a.k) ? __fsub_rn(v[j][i], mean) : 0.f;
        v[j][i] = c;
        ss = __fadd_rn(ss, __fmul_rn(c, c));
      }
    }
    ss = block_sum(ss, red);
    const float inv = rsqrtf(__fadd_rn(__fdiv_rn(ss, kf), a.eps));
#pragma unroll
    for (int j = 0; j < kCpt; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i)
        v[j][i] = bf16r(__fmul_rn(v[j][i], inv));
  }
  if (kMod) {
#pragma unroll
    for (int j = 0; j < kCpt; ++j) {
      const int chunk = threadIdx.x + j * blockDim.x;
      const int c0 = chunk < nchunks ? chunk * 8 : a.k;
      __nv_bfloat16 sv[8], hv[8];
      load8<true>(a.scale + cond * a.ld_mod, c0, a.k, sv);
      load8<true>(a.shift + cond * a.ld_mod, c0, a.k, hv);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float factor = bf16r(__fadd_rn(1.0f, __bfloat162float(sv[i])));
        const float p = bf16r(__fmul_rn(v[j][i], factor));
        const float t = bf16r(__fadd_rn(p, __bfloat162float(hv[i])));
        v[j][i] = (c0 + i < a.k) ? t : 0.f;
      }
    }
  }
  if (a.smooth != nullptr) {
#pragma unroll
    for (int j = 0; j < kCpt; ++j) {
      const int chunk = threadIdx.x + j * blockDim.x;
      const int c0 = chunk * 8;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (chunk < nchunks && c0 + i < a.k)
          v[j][i] = bf16r(__fdiv_rn(v[j][i], __ldg(a.smooth + c0 + i)));
    }
  }
  if constexpr (kOut == 16) {
#pragma unroll
    for (int j = 0; j < kCpt; ++j) {
      const int chunk = threadIdx.x + j * blockDim.x;
      // Every lane takes part in the pairwise shuffle; stores are guarded.
      store_nvfp4_chunk(v[j], row, chunk < nchunks ? chunk : nchunks, a.k,
                        a.q, a.scales);
    }
  } else if constexpr (kOut == 32) {
    // Maximum of the finite |value| (packing.py:76-78).
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < kCpt; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (fabsf(v[j][i]) != INFINITY)
          m = fmaxf(m, fabsf(v[j][i]));
    m = block_max(m, red);
    if (threadIdx.x == 0)
      reinterpret_cast<float *>(a.scales)[row] = m;
    store_bf16_row(v, reinterpret_cast<__nv_bfloat16 *>(a.q) + row * a.k, a.k, nchunks);
  } else {
  float m = 0.f;
#pragma unroll
  for (int j = 0; j < kCpt; ++j)
#pragma unroll
    for (int i = 0; i < 8; ++i)
      m = fmaxf(m, fabsf(v[j][i]));
  m = block_max(m, red);
  const float s = row_scale<kOut>(m);
  if (threadIdx.x == 0)
    reinterpret_cast<float *>(a.scales)[row] = s;
  uint8_t *qrow = a.q + row * (kOut == 8 ? a.kpad : a.kpad / 2);
#pragma unroll
  for (int j = 0; j < kCpt; ++j) {
    const int chunk = threadIdx.x + j * blockDim.x;
    if (chunk < nchunks)
      store_codes<kOut>(v[j], s, qrow, chunk * 8);
  }
  }
}

// ------------------------------------------------------------------ launchers
// Threads per row: enough 8-wide chunks per thread to cover Kpad with at most
// kCpt chunks each, a multiple of 32, at most 1024.
static inline int pick_threads(int nchunks, int cpt) {
  int t = (nchunks + cpt - 1) / cpt;
  t = (t + 31) / 32 * 32;
  return t < 32 ? 32 : t;
}

// Launches `kernel<<<rows, threads>>>(args)` with programmatic dependent
// launch enabled, so its prologue may overlap the previous kernel's tail.
template <typename Args>
static cudaError_t launch_rows(void (*kernel)(Args), const Args &a,
                               int64_t rows, int threads, cudaStream_t st,
                               size_t smem = 0) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(rows), 1, 1);
  cfg.blockDim = dim3(unsigned(threads), 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, a);
}

template <int kBits, int kCpt>
static cudaError_t launch_quant(const QuantArgs &a, int64_t rows, bool vec,
                                cudaStream_t st) {
  const int threads = pick_threads(a.kpad / 8, kCpt);
  if (vec)
    return launch_rows(quant_rows_kernel<kBits, kCpt, true>, a, rows, threads, st);
  return launch_rows(quant_rows_kernel<kBits, kCpt, false>, a, rows, threads, st);
}

template <int kBits>
static cudaError_t launch_quant_cluster(const QuantArgs &a, int64_t rows,
                                        int csize, bool vec, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(csize), unsigned(rows), 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = unsigned(csize);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (vec)
    return cudaLaunchKernelEx(&cfg, quant_rows_cluster_kernel<kBits, 2, true>, a);
  return cudaLaunchKernelEx(&cfg, quant_rows_cluster_kernel<kBits, 2, false>, a);
}

// ------------------------------------------------------------------ packs
// with given maxima.  The symmetric-row-v1 pack of rows whose maximum |x| is
// already known as partial maxima (e.g. the per-16-channel maxima the GEMM
// that wrote x produced in its epilogue, `max_out`): the row scale
// row_scale(max_i x_max[row, i]) equals quant_rows_kernel's (a maximum does
// not depend on its order), and the codes are then elementwise, so a row is
// split over ceil(Kpad / 1024) CTAs of 128 threads, one 8-value chunk per
// thread, with no row reduction over x.  Bitwise the same bytes and scales
// as quant_rows_kernel (plain mode).
struct QuantMaxArgs {
  const __nv_bfloat16 *x;   // [rows, ldx]
  int64_t ldx;
  const float *x_max;       // [rows, parts]
  int parts;
  uint8_t *q;
  float *scales;
  int k;
  int kpad;
};

template <int kBits, bool kVec>
__global__ void __launch_bounds__(128) quant_rows_max_kernel(const QuantMaxArgs a) {
  __shared__ float red[32];
  pdl_wait();
  pdl_launch_dependents();
  const int64_t row = blockIdx.x;
  float m = 0.f;
  for (int i = threadIdx.x; i < a.parts; i += 128)
    m = fmaxf(m, __ldg(a.x_max + row * a.parts + i));
  m = block_max(m, red);
  const float s = row_scale<kBits>(m);
  if (blockIdx.y == 0 && threadIdx.x == 0)
    a.scales[row] = s;
  const int nchunks = a.kpad >> 3;
  const int chunk = int(blockIdx.y) * 128 + int(threadIdx.x);
  if (chunk < nchunks) {
    const int c0 = chunk * 8;
    __nv_bfloat16 xv[8];
    load8<kVec>(a.x + row * a.ldx, c0, a.k, xv);
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
      v[i] = c0 + i < a.k ? __bfloat162float(xv[i]) : 0.f;
    store_codes<kBits>(v, s, a.q + row * (kBits == 8 ? a.kpad : a.kpad / 2), c0);
  }
}

cudaError_t run_quant_rows_max(const QuantMaxArgs &a, int bits, int64_t rows, bool vec, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(rows), unsigned((a.kpad / 8 + 127) / 128), 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (bits == 8)
    return vec ? cudaLaunchKernelEx(&cfg, quant_rows_max_kernel<8, true>, a)
               : cudaLaunchKernelEx(&cfg, quant_rows_max_kernel<8, false>, a);
  return vec ? cudaLaunchKernelEx(&cfg, quant_rows_max_kernel<4, true>, a)
             : cudaLaunchKernelEx(&cfg, quant_rows_max_kernel<4, false>, a);
}

cudaError_t run_quant_rows(const QuantArgs &a, int bits, int64_t rows,
                           bool vec, cudaStream_t st) {
  const int nchunks = a.kpad / 8;
  // Floating outputs (NVFP4, FP8 first pass): rows of at most 8192 values
  // (1024 chunks) held in registers.
  if (bits == 16) {
    if (nchunks > 1024)
      return cudaErrorInvalidValue;
    return nchunks <= 256 ? launch_quant<16, 1>(a, rows, vec, st) : launch_quant<16, 4>(a, rows, vec, st);
  }
  if (bits == 32) {
    // One chunk per thread, 128 threads per CTA, fp8_value_splits(k) CTAs
    // per row.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(rows), unsigned((nchunks + 127) / 128), 1);
    cfg.blockDim = dim3(128, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return vec ? cudaLaunchKernelEx(&cfg, quant_rows_kernel<32, 1, true>, a)
               : cudaLaunchKernelEx(&cfg, quant_rows_kernel<32, 1, false>, a);
  }
  // Few long rows: spread each row over a cluster of CTAs (<= 8, each with
  // 128 threads x 2 chunks) so the launch covers more of the 148 SMs.
  if (rows <= 64 && nchunks > 256) {
    int csize = (nchunks + 255) / 256;
    csize = csize <= 2 ? 2 : (csize <= 4 ? 4 : 8);
    if (nchunks <= csize * 256)
      return bits == 8 ? launch_quant_cluster<8>(a, rows, csize, vec, st)
                       : launch_quant_cluster<4>(a, rows, csize, vec, st);
  }
  // <= 256 threads with up to 4 chunks each covers Kpad <= 8192 with the row
  // held in registers; wider rows (up to 65536) take two passes over x.
  if (nchunks <= 256)
    return bits == 8 ? launch_quant<8, 1>(a, rows, vec, st)
                     : launch_quant<4, 1>(a, rows, vec, st);
  if (nchunks <= 1024)
    return bits == 8 ? launch_quant<8, 4>(a, rows, vec, st)
                     : launch_quant<4, 4>(a, rows, vec, st);
  if (vec)
    return bits == 8 ? launch_rows(quant_rows_stream_kernel<8, true>, a, rows, 512, st)
                     : launch_rows(quant_rows_stream_kernel<4, true>, a, rows, 512, st);
  return bits == 8 ? launch_rows(quant_rows_stream_kernel<8, false>, a, rows, 512, st)
                   : launch_rows(quant_rows_stream_kernel<4, false>, a, rows, 512, st);
}

template <int kOut, int kCpt, int kNorm, bool kMod, bool kRes>
static cudaError_t launch_norm4(const NormArgs &a, int64_t rows,
                                cudaStream_t st) {
  const int threads = pick_threads(a.kpad / 8, kCpt);
  // Integer RMSNorm keeps the row's squares in dynamic shared memory.
  const size_t smem = (kNorm == 1 && kOut != 16 && kOut != 32) ? size_t(a.k) * 4 : 0;
  return launch_rows(norm_quant_kernel<kOut, kCpt, kNorm, kMod, kRes>, a, rows,
                     threads, st, smem);
}

template <int kOut, int kCpt>
static cudaError_t launch_norm3(const NormArgs &a, int64_t rows, int norm,
                                bool mod, bool res, cudaStream_t st) {
#define PIR2B_NORM_CASE(N, M, R)                                             \
  if (norm == N && mod == M && res == R)                                     \
    return launch_norm4<kOut, kCpt, N, M, R>(a, rows, st);
  PIR2B_NORM_CASE(0, true, false)
  PIR2B_NORM_CASE(1, false, false)
  PIR2B_NORM_CASE(1, true, false)
  PIR2B_NORM_CASE(2, false, false)
  PIR2B_NORM_CASE(2, true, false)
  PIR2B_NORM_CASE(2, true, true)
  PIR2B_NORM_CASE(2, false, true)
  PIR2B_NORM_CASE(0, false, false)
  PIR2B_NORM_CASE(1, false, true)
#undef PIR2B_NORM_CASE
  return cudaErrorInvalidValue;
}

template <int kOut>
static cudaError_t launch_norm2(const NormArgs &a, int64_t rows, int norm,
                                bool mod, bool res, cudaStream_t st) {
  const int nchunks = a.kpad / 8;
  if (nchunks <= 256)
    return launch_norm3<kOut, 1>(a, rows, norm, mod, res, st);
  return launch_norm3<kOut, 4>(a, rows, norm, mod, res, st);
}

cudaError_t run_norm_quant(const NormArgs &a, int out_format, int64_t rows,
                           int norm, bool mod, bool res, cudaStream_t st) {
  if (out_format == 8)
    return launch_norm2<8>(a, rows, norm, mod, res, st);
  if (out_format == 4)
    return launch_norm2<4>(a, rows, norm, mod, res, st);
  if (out_format == 32)
    return launch_norm2<32>(a, rows, norm, mod, res, st);
  return launch_norm2<16>(a, rows, norm, mod, res, st);
}

// ------------------------------------------------------------------ FP8
// Per-tensor E4M3 quantization of bf16 rows, both reference variants:
//  * default (fp8_cutlass_linear.cu:61-120, quantize_bf16): amax of the
//    finite |x|; scale = max(amax / 448, 1e-12); q = e4m3_rn_satfinite(
//    clamp(x * (1 / scale), -448, 448));
//  * fast (thor/packing.py:451-519, prepare_fp8): scale = max(amax *
//    (1/448), 1e-12); q = e4m3(clamp(x / scale, -448, 448)), with IEEE
//    round-to-nearest division here.
// One launch: a cluster of C CTAs splits the rows, each reduces its |x|
// maximum, every rank combines the C partial maxima through distributed
// shared memory, then casts its rows.  The scale is written to `scale` and
// replicated into `scale_rep` (the per-row / per-channel scale vector the
// E4M3 GEMM epilogue reads).
struct Fp8QuantArgs {
  const __nv_bfloat16 *x;
  int64_t ldx;
  int64_t rows;
  int k;                 // k % 8 == 0
  uint8_t *q;            // [rows, k]
  float *scale;          // [1]
  float *scale_rep;      // [n_rep] or null
  int64_t n_rep;
  int fast;
  // 1: the codes are GEMM weights.  The GEMM reads its weights before its
  // programmatic-dependent wait, so the kernel then lets dependent launches
  // start only at its end (no early trigger).
  int weights;
};

constexpr float kFp8Max = 448.0f;
constexpr float kFp8MinScale = 1.0e-12f;

__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

constexpr int kFp8Threads = 1024;
constexpr int kFp8Cached = 4;   // 16-byte chunks per thread kept in registers between the passes

__global__ void __launch_bounds__(kFp8Threads) fp8_quant_kernel(const Fp8QuantArgs a) {
  __shared__ float red[32];
  __shared__ float s_part;
  __shared__ float s_scale[2];
  pdl_wait();
  if (!a.weights)
    pdl_launch_dependents();
  uint32_t nranks;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(nranks));
  const uint32_t rank = cluster_ctarank();
  const int64_t r0 = a.rows * rank / nranks, r1 = a.rows * (rank + 1) / nranks;
  const int nch = a.k / 8;
  const int items = int((r1 - r0) * nch);   // 16-byte chunks of this CTA (< 2^31)
  const bool flat = a.ldx == a.k;           // rows back to back: chunk i at r0*k + 8i
  auto chunk_ptr = [&](int i) -> int64_t {  // element offset of chunk i in x
    if (flat)
      return r0 * a.k + int64_t(i) * 8;
    const int row = i / nch;
    return (r0 + row) * a.ldx + int64_t(i - row * nch) * 8;
  };
  auto out_ptr = [&](int i) -> int64_t {
    if (flat)
      return r0 * a.k + int64_t(i) * 8;
    const int row = i / nch;
    return (r0 + row) * int64_t(a.k) + int64_t(i - row * nch) * 8;
  };
  uint4 cache[kFp8Cached];
  float m = 0.f;
  auto absmax8 = [&](const uint4 &raw) {
    const __nv_bfloat16 *v = reinterpret_cast<const __nv_bfloat16 *>(&raw);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float f = fabsf(__bfloat162float(v[e]));
      if (isfinite(f))
        m = fmaxf(m, f);
    }
  };
  // Pass 1: maximum of the finite |x|.  The first kFp8Cached chunks of each
  // thread are loaded together and kept in registers for pass 2.
#pragma unroll
  for (int j = 0; j < kFp8Cached; ++j) {
    const int i = int(threadIdx.x) + j * kFp8Threads;
    cache[j] = i < items ? __ldg(reinterpret_cast<const uint4 *>(a.x + chunk_ptr(i)))
                         : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int j = 0; j < kFp8Cached; ++j)
    absmax8(cache[j]);
#pragma unroll 4
  for (int i = int(threadIdx.x) + kFp8Cached * kFp8Threads; i < items; i += kFp8Threads)
    absmax8(__ldg(reinterpret_cast<const uint4 *>(a.x + chunk_ptr(i))));
  m = block_max(m, red);
  if (threadIdx.x == 0)
    s_part = m;
  cluster_sync();
  if (threadIdx.x == 0) {
    float amax = 0.f;
    for (uint32_t p = 0; p < nranks; ++p)
      amax = fmaxf(amax, __int_as_float(ld_cluster_s32(map_peer(smem_u32(&s_part), p))));
    const float scale = a.fast ? fmaxf(__fmul_rn(amax, 1.0f / kFp8Max), kFp8MinScale)
                               : fmaxf(__fdiv_rn(amax, kFp8Max), kFp8MinScale);
    s_scale[0] = scale;
    s_scale[1] = __fdiv_rn(1.0f, scale);
  }
  // Every rank has read every partial maximum (no CTA leaves while a peer
  // still reads it), and s_scale is visible to the whole CTA.
  cluster_sync();
  const float scale = s_scale[0], inv = s_scale[1];
  // Pass 2: cast (chunks beyond the register cache are read again).
  auto cast8 = [&](int i, const uint4 &raw) {
    const __nv_bfloat16 *v = reinterpret_cast<const __nv_bfloat16 *>(&raw);
    float f[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float x = __bfloat162float(v[e]);
      const float y = a.fast ? __fdiv_rn(x, scale) : __fmul_rn(x, inv);
      f[e] = fminf(kFp8Max, fmaxf(-kFp8Max, y));
    }
    uint2 out;
    out.x = cvt_e4m3x2(f[0], f[1]) | (cvt_e4m3x2(f[2], f[3]) << 16);
    out.y = cvt_e4m3x2(f[4], f[5]) | (cvt_e4m3x2(f[6], f[7]) << 16);
    *reinterpret_cast<uint2 *>(a.q + out_ptr(i)) = out;
  };
#pragma unroll
  for (int j = 0; j < kFp8Cached; ++j) {
    const int i = int(threadIdx.x) + j * kFp8Threads;
    if (i < items)
      cast8(i, cache[j]);
  }
#pragma unroll 4
  for (int i = int(threadIdx.x) + kFp8Cached * kFp8Threads; i < items; i += kFp8Threads)
    cast8(i, __ldg(reinterpret_cast<const uint4 *>(a.x + chunk_ptr(i))));
  if (rank == 0 && threadIdx.x == 0)
    *a.scale = scale;
  if (a.scale_rep != nullptr)
    for (int64_t i = int64_t(rank) * kFp8Threads + threadIdx.x; i < a.n_rep;
         i += int64_t(nranks) * kFp8Threads)
      a.scale_rep[i] = scale;
}

cudaError_t run_fp8_quant(const Fp8QuantArgs &a, int ranks, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(ranks), 1, 1);
  cfg.blockDim = dim3(kFp8Threads, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = unsigned(ranks);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, fp8_quant_kernel, a);
}

// Second pass of the FP8 producers (thor/packing.py:180-199 with
// _fp8_scale_and_cast, :461-482) and of the per-tensor activation quantizer:
// the first pass wrote partial maxima of the finite |value| (a few per row);
// every CTA reduces them (a few KB) to the scale and casts its
// grid-stride share of 8-value chunks of v (rows of stride ldv):
//  * fast (prepare_fp8 and the producers): scale = max(amax * (1/448),
//    1e-12), q = e4m3_rn(clamp(v / scale, -448, 448)), IEEE division;
//  * default (quantize_bf16, fp8_cutlass_linear.cu:61-120): scale =
//    max(amax / 448, 1e-12), q = e4m3_rn(clamp(v * (1 / scale), -448, 448)).
// CTA 0 writes the scale; the CTAs together write its replicated copy (the
// per-row scale vector the E4M3 GEMM reads).
struct Fp8CastArgs {
  const __nv_bfloat16 *v;   // [rows, ldv]
  int64_t ldv;
  const float *row_max;     // [nmax] partial maxima of the first pass
  int64_t nmax;
  int64_t rows;
  int k;                    // k % 8 == 0
  int fast;
  uint8_t *q;               // [rows, k]
  float *scale;             // [1]
  float *scale_rep;         // [n_rep] or null
  int64_t n_rep;
};

constexpr int kFp8CastThreads = 256;

__global__ void __launch_bounds__(kFp8CastThreads) fp8_cast_kernel(const Fp8CastArgs a) {
  __shared__ float red[32];
  pdl_wait();
  pdl_launch_dependents();
  float m = 0.f;
  for (int64_t r = threadIdx.x; r < a.nmax; r += kFp8CastThreads)
    m = fmaxf(m, __ldg(a.row_max + r));
  m = block_max(m, red);
  const float scale = a.fast ? fmaxf(__fmul_rn(m, 1.0f / kFp8Max), kFp8MinScale)
                             : fmaxf(__fdiv_rn(m, kFp8Max), kFp8MinScale);
  const float inv = __fdiv_rn(1.0f, scale);
  const int nch = a.k / 8;
  const int64_t chunks = a.rows * int64_t(nch);
  const int64_t stride = int64_t(gridDim.x) * kFp8CastThreads;
  for (int64_t i = int64_t(blockIdx.x) * kFp8CastThreads + threadIdx.x; i < chunks; i += stride) {
    const int64_t row = i / nch;
    const uint4 raw = __ldg(reinterpret_cast<const uint4 *>(a.v + row * a.ldv + (i - row * nch) * 8));
    const __nv_bfloat16 *e = reinterpret_cast<const __nv_bfloat16 *>(&raw);
    float f[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float x = __bfloat162float(e[j]);
      f[j] = fminf(kFp8Max, fmaxf(-kFp8Max, a.fast ? __fdiv_rn(x, scale) : __fmul_rn(x, inv)));
    }
    uint2 out;
    out.x = cvt_e4m3x2(f[0], f[1]) | (cvt_e4m3x2(f[2], f[3]) << 16);
    out.y = cvt_e4m3x2(f[4], f[5]) | (cvt_e4m3x2(f[6], f[7]) << 16);
    reinterpret_cast<uint2 *>(a.q)[i] = out;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0)
    *a.scale = scale;
  if (a.scale_rep != nullptr)
    for (int64_t i = int64_t(blockIdx.x) * kFp8CastThreads + threadIdx.x; i < a.n_rep; i += stride)
      a.scale_rep[i] = scale;
}

cudaError_t run_fp8_cast(const Fp8CastArgs &a, int sms, cudaStream_t st) {
  const int64_t chunks = a.rows * int64_t(a.k / 8);
  const int64_t want = (std::max<int64_t>(chunks, a.n_rep) + kFp8CastThreads - 1) / kFp8CastThreads;
  const int grid = int(std::max<int64_t>(1, std::min<int64_t>(want, int64_t(sms) * 4)));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid), 1, 1);
  cfg.blockDim = dim3(kFp8CastThreads, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fp8_cast_kernel, a);
}

} // namespace pir2b
