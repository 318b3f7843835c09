// BF16 pointwise fusions around the quantized projections of the VLM text
// attention (piR2 coexecution/fused_ops.py: RoPE :34-147 and RMSNorm
// :150-232 run as separate Triton kernels; here one kernel does both for q
// and k and lays q, k, v out for attention).
//
// One warp per (token, head).  For q and k heads: per-head RMSNorm
//   n = bf16(f32(x) * rsqrt(mean(x^2) + eps)); h = bf16(w * n)
// (Qwen3 q_norm / k_norm), then rotary embedding with bf16 rounding at every
// step of torch's `q * cos + rotate_half(q) * sin`:
//   out = bf16(bf16(h * cos) + bf16(rotate_half(h) * sin)).
// v heads are copied.  Outputs are [B, H, T, D] contiguous.
#pragma once
#include <algorithm>

#include "args.cuh"
#include "gemm_i8.cuh"
#include "ptx.cuh"

namespace pir2b {

struct QkRopeArgs {
  const __nv_bfloat16 *qkv;   // [B*T, ld] rows: q | k | v heads
  int64_t ld;
  const __nv_bfloat16 *q_w;   // [D]
  const __nv_bfloat16 *k_w;   // [D]
  const __nv_bfloat16 *cos;   // [T, D]
  const __nv_bfloat16 *sin;   // [T, D]
  __nv_bfloat16 *q_out;       // [B, HQ, T, D]
  __nv_bfloat16 *k_out;       // [B, HK, T, D]
  __nv_bfloat16 *v_out;       // [B, HK, T, D]
  int rows;                   // B * T
  int tokens;                 // T
  int hq, hk;
  float eps;
};

__device__ __forceinline__ float bf16_round(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

// D == 128: each lane owns 4 consecutive elements; the rotate_half partner
// of lane l is lane l ^ 16.
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(const QkRopeArgs a) {
  pdl_wait();
  pdl_launch_dependents();
  constexpr int D = 128;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int heads = a.hq + 2 * a.hk;
  const int row = warp / heads;           // b * T + t
  const int head = warp % heads;
  if (row >= a.rows)
    return;
  const int b = row / a.tokens, t = row % a.tokens;
  const __nv_bfloat16 *src = a.qkv + int64_t(row) * a.ld + head * D + lane * 4;
  const uint2 raw = *reinterpret_cast<const uint2 *>(src);
  const __nv_bfloat16 *xv = reinterpret_cast<const __nv_bfloat16 *>(&raw);
  __nv_bfloat16 *dst;
  const bool is_q = head < a.hq;
  const bool is_k = !is_q && head < a.hq + a.hk;
  if (is_q)
    dst = a.q_out + ((int64_t(b) * a.hq + head) * a.tokens + t) * D;
  else if (is_k)
    dst = a.k_out + ((int64_t(b) * a.hk + (head - a.hq)) * a.tokens + t) * D;
  else
    dst = a.v_out + ((int64_t(b) * a.hk + (head - a.hq - a.hk)) * a.tokens + t) * D;
  if (!is_q && !is_k) {
    *reinterpret_cast<uint2 *>(dst + lane * 4) = raw;
    return;
  }
  float x[4];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[i] = __bfloat162float(xv[i]);
    ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
  }
  for (int d = 16; d; d >>= 1)
    ss += __shfl_xor_sync(0xffffffffu, ss, d);
  const float inv = rsqrtf(__fadd_rn(__fdiv_rn(ss, float(D)), a.eps));
  const __nv_bfloat16 *w = is_q ? a.q_w : a.k_w;
  const uint2 wraw = *reinterpret_cast<const uint2 *>(w + lane * 4);
  const __nv_bfloat16 *wv = reinterpret_cast<const __nv_bfloat16 *>(&wraw);
  float h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    h[i] = bf16_round(__fmul_rn(__bfloat162float(wv[i]), bf16_round(__fmul_rn(x[i], inv))));
  float p[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    p[i] = __shfl_xor_sync(0xffffffffu, h[i], 16);
  const uint2 craw = *reinterpret_cast<const uint2 *>(a.cos + int64_t(t) * D + lane * 4);
  const uint2 sraw = *reinterpret_cast<const uint2 *>(a.sin + int64_t(t) * D + lane * 4);
  const __nv_bfloat16 *cv = reinterpret_cast<const __nv_bfloat16 *>(&craw);
  const __nv_bfloat16 *sv = reinterpret_cast<const __nv_bfloat16 *>(&sraw);
  uint2 out;
  __nv_bfloat16 *ov = reinterpret_cast<__nv_bfloat16 *>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // rotate_half: first half takes -x[i + D/2], second half x[i - D/2].
    const float rot = lane < 16 ? -p[i] : p[i];
    const float c = bf16_round(__fmul_rn(h[i], __bfloat162float(cv[i])));
    const float s = bf16_round(__fmul_rn(rot, __bfloat162float(sv[i])));
    ov[i] = __float2bfloat16_rn(__fadd_rn(c, s));
  }
  *reinterpret_cast<uint2 *>(dst + lane * 4) = out;
}

cudaError_t run_qk_norm_rope(const QkRopeArgs &a, int64_t rows,
                             cudaStream_t st) {
  const int64_t warps = rows * (a.hq + 2 * a.hk);
  const int64_t blocks = (warps * 32 + 255) / 256;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(blocks), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, qk_norm_rope_kernel, a);
}

// Packed int4 codes (two per byte, low nibble first) -> sign-extended int8
// codes, one per byte: the int8 container layout of the same values, so the
// int8 GEMM produces the int4 GEMM's int32 sums.  16 packed bytes per
// thread and step, grid-stride.
__global__ void __launch_bounds__(256) unpack_int4_kernel(const uint4 *__restrict__ src,
                                                          uint4 *__restrict__ dst, int64_t chunks) {
  pdl_wait();
  pdl_launch_dependents();
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < chunks;
       i += int64_t(gridDim.x) * blockDim.x) {
    const uint4 w = src[i];
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    uint32_t out[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t lo = sext_nibbles(words[j] & 0x0F0F0F0Fu);
      const uint32_t hi = sext_nibbles((words[j] >> 4) & 0x0F0F0F0Fu);
      out[2 * j] = __byte_perm(lo, hi, 0x5140);
      out[2 * j + 1] = __byte_perm(lo, hi, 0x7362);
    }
    dst[2 * i] = make_uint4(out[0], out[1], out[2], out[3]);
    dst[2 * i + 1] = make_uint4(out[4], out[5], out[6], out[7]);
  }
}

cudaError_t run_unpack_int4(const void *src, void *dst, int64_t chunks, int sms,
                            cudaStream_t st) {
  const int64_t want = (chunks + 255) / 256;
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(want, int64_t(sms) * 8));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(blocks), 1, 1);
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, unpack_int4_kernel, static_cast<const uint4 *>(src),
                            static_cast<uint4 *>(dst), chunks);
}

} // namespace pir2b
