// Few-token W8A8 / W4A4 / E4M3 GEMM (M <= 32 token rows): the DiT's 17-row
// projections, single-row encoders.
//
// Same arithmetic as gemm_i8_kernel: exact int32 sums, then
// bf16(f32(f32(i2f(acc) * sa) * sw) [+ bias]), optional output table,
// residual and per-16-channel maxima.  For so few rows the tcgen05 kernel's
// cost is not the MMA but its fixed latency: TMA round trips into a
// per-CTA ring, TMEM set-up and, to spread the weights over enough SMs, a
// split-K reduction across a cluster (two cluster barriers and distributed
// shared-memory pulls).  Here:
//  * a CTA owns 16 output channels over the whole K; its 8 (16 for long K)
//    warps split K and add their partial tiles in shared memory (no
//    cluster, no global workspace), so Npad / 16 CTAs stream the weights
//    (96 for N = 1536);
//  * each warp runs warp-level integer MMAs (mma.sync m16n8k32, s8 x s8 ->
//    s32; int4 codes are sign-extended to int8 in registers) on operands
//    loaded straight from global memory with 16-byte loads: per 128-element
//    K chunk a thread holds 32 consecutive K bytes of weight rows g and
//    g + 8 and of token rows g + 8 t.  The K order inside a chunk is
//    permuted identically for weights and tokens, so the int32 sums are
//    the exact dot products;
//  * the first K chunks of weights are loaded before griddepcontrol.wait:
//    weights never depend on the previous kernel.
// kBits == 9: E4M3 codes (the FP8 path) in the int8 byte layout, warp-level
// e4m3 MMAs (m16n8k32, same fragments) with fp32 accumulators; the warps'
// fp32 partial tiles are added in warp order, a fixed order, so results are
// deterministic.
#pragma once
#include "args.cuh"
#include "gemm_i8.cuh"
#include "ptx.cuh"

namespace pir2b {

constexpr int kFewChannels = 16;     // channels per CTA (the MMA's M)
constexpr int kFewMaxRows = 32;      // token rows (4 MMA column tiles of 8)

struct FewArgs {
  const void *qa;                  // [m, lda] int8 codes or packed int4 bytes
  int64_t lda;                     // bytes per token row
  const float *sa;                 // [m]
  const void *qw;                  // [npad, ldw] int8 or packed int4
  int64_t ldw;                     // bytes per weight row
  const float *sw;                 // [npad]
  const __nv_bfloat16 *bias;       // [npad] or null
  int bias_mode;
  const __nv_bfloat16 *out_lut;    // [65536] or null
  const __nv_bfloat16 *residual;   // [m, ldr] or null
  int64_t ldr;
  __nv_bfloat16 *out;              // [m, ldo]
  int64_t ldo;
  float *max_out;                  // [m, max_parts] or null
  int max_parts;
  int m, npad, n_store;
  int chunks;                      // K chunks of 128 elements
};

// D (16 x 8, f32) += A (16 x 32, e4m3, row) * B (32 x 8, e4m3, col): the
// same fragment layout as the s8 form.
__device__ __forceinline__ void mma_e4m3_16832(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D (16 x 8, s32) += A (16 x 32, s8, row) * B (32 x 8, s8, col).
__device__ __forceinline__ void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 32 K elements of one row for one thread (8 words: K bytes in order).
struct Row32 {
  uint32_t w[8];
};

// Loads K elements [k0, k0 + 32) of a row: 32 int8 (or E4M3) bytes, or 16
// packed int4 bytes sign-extended to 32 int8 (low nibble = even element).
// Rows outside the matrix read as zeros.
template <int kBits>
__device__ __forceinline__ Row32 load_row32(const uint8_t *row, bool valid, int k0) {
  Row32 r;
  if (kBits != 4) {
    uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
    if (valid) {
      lo = __ldg(reinterpret_cast<const uint4 *>(row + k0));
      hi = __ldg(reinterpret_cast<const uint4 *>(row + k0 + 16));
    }
    r.w[0] = lo.x, r.w[1] = lo.y, r.w[2] = lo.z, r.w[3] = lo.w;
    r.w[4] = hi.x, r.w[5] = hi.y, r.w[6] = hi.z, r.w[7] = hi.w;
  } else {
    uint4 p = make_uint4(0, 0, 0, 0);
    if (valid)
      p = __ldg(reinterpret_cast<const uint4 *>(row + k0 / 2));
    const uint32_t words[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = sext_nibbles(words[i] & 0x0F0F0F0Fu);
      const uint32_t hi = sext_nibbles((words[i] >> 4) & 0x0F0F0F0Fu);
      r.w[2 * i] = __byte_perm(lo, hi, 0x5140);
      r.w[2 * i + 1] = __byte_perm(lo, hi, 0x7362);
    }
  }
  return r;
}

// Chunk of one warp: weight rows g and g + 8 and kTiles token rows g + 8 t.
template <int kBits, int kTiles>
struct FewChunk {
  Row32 wg, wg8;
  Row32 tok[kTiles];
};

template <int kBits, int kTiles>
__device__ __forceinline__ void few_load_weights(FewChunk<kBits, kTiles> &c, const uint8_t *wrow_g,
                                                 const uint8_t *wrow_g8, bool vg, bool vg8, int k0) {
  c.wg = load_row32<kBits>(wrow_g, vg, k0);
  c.wg8 = load_row32<kBits>(wrow_g8, vg8, k0);
}

template <int kBits, int kTiles>
__device__ __forceinline__ void few_load_tokens(FewChunk<kBits, kTiles> &c, const FewArgs &a, int g, int k0) {
#pragma unroll
  for (int t = 0; t < kTiles; ++t) {
    const int j = g + 8 * t;
    c.tok[t] = load_row32<kBits>(static_cast<const uint8_t *>(a.qa) + int64_t(j < a.m ? j : 0) * a.lda,
                                 j < a.m, k0);
  }
}

// Accumulator type: exact int32 for integer codes, fp32 for E4M3.
template <int kBits>
using FewAcc = typename std::conditional<kBits == 9, float, int>::type;

template <int kBits, int kTiles>
__device__ __forceinline__ void few_mma_chunk(FewAcc<kBits> (&acc)[kTiles][4], const FewChunk<kBits, kTiles> &c) {
#pragma unroll
  for (int s = 0; s < 4; ++s) {
#pragma unroll
    for (int t = 0; t < kTiles; ++t) {
      if constexpr (kBits == 9)
        mma_e4m3_16832(acc[t], c.wg.w[2 * s], c.wg8.w[2 * s], c.wg.w[2 * s + 1], c.wg8.w[2 * s + 1],
                       c.tok[t].w[2 * s], c.tok[t].w[2 * s + 1]);
      else
        mma_s8_16832(acc[t], c.wg.w[2 * s], c.wg8.w[2 * s], c.wg.w[2 * s + 1], c.wg8.w[2 * s + 1],
                     c.tok[t].w[2 * s], c.tok[t].w[2 * s + 1]);
    }
  }
}

template <int kBits, int kTiles, int kWarps>
__global__ void __launch_bounds__(kWarps * 32) gemm_few_kernel(const FewArgs a) {
  constexpr int kCols = 8 * kTiles;   // token columns of the CTA's tile
  constexpr int kThreads = kWarps * 32;
  using Acc = FewAcc<kBits>;
  __shared__ Acc red[kWarps][kCols][kFewChannels];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int c0 = blockIdx.x * kFewChannels;
  // This warp's K chunks (128 elements each).
  const int ch_begin = (warp * a.chunks) / kWarps;
  const int ch_end = ((warp + 1) * a.chunks) / kWarps;
  const uint8_t *w = static_cast<const uint8_t *>(a.qw);
  const bool vg = c0 + g < a.npad, vg8 = c0 + g + 8 < a.npad;
  const uint8_t *wrow_g = w + int64_t(vg ? c0 + g : 0) * a.ldw;
  const uint8_t *wrow_g8 = w + int64_t(vg8 ? c0 + g + 8 : 0) * a.ldw;
  Acc acc[kTiles][4];
#pragma unroll
  for (int t = 0; t < kTiles; ++t)
    acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = Acc(0);

  // Two chunks in flight: the weights of the first two are requested before
  // the previous kernel has finished (they do not depend on it).
  FewChunk<kBits, kTiles> cur, nxt;
  if (ch_begin < ch_end)
    few_load_weights(cur, wrow_g, wrow_g8, vg, vg8, ch_begin * 128 + tig * 32);
  if (ch_begin + 1 < ch_end)
    few_load_weights(nxt, wrow_g, wrow_g8, vg, vg8, (ch_begin + 1) * 128 + tig * 32);
  pdl_launch_dependents();
  pdl_wait();
  if (ch_begin < ch_end)
    few_load_tokens(cur, a, g, ch_begin * 128 + tig * 32);
  if (ch_begin + 1 < ch_end)
    few_load_tokens(nxt, a, g, (ch_begin + 1) * 128 + tig * 32);
  for (int ch = ch_begin; ch < ch_end; ch += 2) {
    few_mma_chunk(acc, cur);
    if (ch + 2 < ch_end) {
      few_load_weights(cur, wrow_g, wrow_g8, vg, vg8, (ch + 2) * 128 + tig * 32);
      few_load_tokens(cur, a, g, (ch + 2) * 128 + tig * 32);
    }
    if (ch + 1 < ch_end) {
      few_mma_chunk(acc, nxt);
      if (ch + 3 < ch_end) {
        few_load_weights(nxt, wrow_g, wrow_g8, vg, vg8, (ch + 3) * 128 + tig * 32);
        few_load_tokens(nxt, a, g, (ch + 3) * 128 + tig * 32);
      }
    }
  }
  // Partial tiles -> shared memory as [warp][token][channel]: accumulator
  // registers 0/1 hold channel g, tokens 8t + 2 tig (+1); 2/3 channel g + 8.
#pragma unroll
  for (int t = 0; t < kTiles; ++t) {
    const int j = 8 * t + 2 * tig;
    red[warp][j][g] = acc[t][0];
    red[warp][j + 1][g] = acc[t][1];
    red[warp][j][g + 8] = acc[t][2];
    red[warp][j + 1][g + 8] = acc[t][3];
  }
  __syncthreads();
  // Sum of the warps' partials and the epilogue: thread -> (token j,
  // channel c0 + cl), 16 consecutive threads per token row.
  const uint16_t *lut = reinterpret_cast<const uint16_t *>(a.out_lut);
  for (int idx = threadIdx.x; idx < kCols * kFewChannels; idx += kThreads) {
    const int j = idx / kFewChannels, cl = idx % kFewChannels;
    const int c = c0 + cl;
    Acc sum = Acc(0);
#pragma unroll
    for (int wp = 0; wp < kWarps; ++wp)
      sum += red[wp][j][cl];
    const bool live = j < a.m && c < a.n_store;
    float mag = 0.f;
    if (live) {
      const float b = a.bias_mode == 2 ? __bfloat162float(a.bias[c]) : 0.f;
      const float accf = kBits == 9 ? float(sum) : __int2float_rn(int(sum));
      __nv_bfloat16 o = epilogue_value(accf, a.sa[j], a.sw[c], b, a.bias_mode, lut);
      if (a.residual != nullptr)
        o = __float2bfloat16_rn(__fadd_rn(__bfloat162float(o), __bfloat162float(a.residual[int64_t(j) * a.ldr + c])));
      a.out[int64_t(j) * a.ldo + c] = o;
      mag = fabsf(__bfloat162float(o));
      // E4M3 (the FP8 cast's partial maxima): only finite values count
      // (thor/packing.py:76-78); fmaxf below already skips NaN.
      if (kBits == 9 && mag == INFINITY)
        mag = 0.f;
    }
    if (a.max_out != nullptr) {
      // Per-16-channel maximum of |y| for token j: the 16 threads of the row
      // (a half warp) hold this CTA's 16 channels.
#pragma unroll
      for (int off = 8; off > 0; off >>= 1)
        mag = fmaxf(mag, __shfl_xor_sync(0xffffffffu, mag, off));
      if (cl == 0 && j < a.m && c0 / 16 < a.max_parts)
        a.max_out[int64_t(j) * a.max_parts + c0 / 16] = mag;
    }
  }
}

} // namespace pir2b
