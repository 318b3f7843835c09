// W8A8 / W4A4 GEMM on the 5th-generation tensor cores (tcgen05 kind::i8).
//
// Computes, for the symmetric-row-v1 format
//   acc[m, n] = sum_k qa[m, k] * qw[n, k]                (exact int32)
//   y[m, n]   = bf16_rn( (f32_rn(f32_rn(i2f_rn(acc) * sa[m]) * sw[n])) [+ b] )
// which is the epilogue order of piR2's pir2_integer::gemm
// (coexecution/kernels/ampere_ada/csrc/integer_gemm.cu:37-59, accumulator
// times the per-row scale, times the per-column scale, plus the BF16 bias,
// one round-to-nearest per step) and of the explicit torch formula the
// reference pins it with (tests/gpu/test_quantization_gpu.py:37-44).
//
// Layout of the work:
//  * the weight matrix is the UMMA "A" operand: one CTA owns 128 output
//    channels (UMMA_M = 128) and a tile of BN tokens (UMMA_N = BN, 16..256),
//    so the accumulator tile lives in TMEM as 128 lanes (channels) x BN
//    columns (tokens).  Small token counts therefore cost no padding of the
//    weight stream, which is what bounds robot-control GEMMs;
//  * both operands are K-major; TMA brings 128-byte K slices with the
//    128-byte swizzle straight into the canonical UMMA shared-memory layout;
//  * warp 0 issues TMA, warp 1 owns TMEM and issues MMAs from one thread,
//    warps 2..5 read TMEM and run the epilogue (and, for W4A4, unpack int4
//    to int8 in shared memory during the main loop);
//  * split-K runs as a thread-block cluster along grid z; each CTA reduces a
//    channel slice of the cluster's partial sums through distributed shared
//    memory, so no global workspace is needed and the int32 sum stays exact.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <type_traits>

#pragma once
#include "args.cuh"
#include "ptx.cuh"
#include "quant.cuh"

namespace pir2b {


constexpr int kThreads = 192;
constexpr int kTileN = 128;          // channels per CTA (UMMA_M)
constexpr int kBlockK = 128;         // K elements per stage
constexpr int kWeightTileBytes = kTileN * kBlockK;  // 16 KB int8

// The accumulator word as fp32: an exact int32 sum (integer kinds) or an
// fp32 sum (E4M3, kind::f8f6f4).
template <bool kF8>
__device__ __forceinline__ float acc_value(uint32_t bits) {
  return kF8 ? __uint_as_float(bits) : __int2float_rn(int(bits));
}

__device__ __forceinline__ __nv_bfloat16 epilogue_value(float acc, float sa,
                                                        float sw, float bias,
                                                        int bias_mode,
                                                        const uint16_t *lut) {
  float y = __fmul_rn(__fmul_rn(acc, sa), sw);
  if (bias_mode != 0)
    y = __fadd_rn(y, bias);
  __nv_bfloat16 o = __float2bfloat16_rn(y);
  if (lut != nullptr) {
    uint16_t bits = __bfloat16_as_ushort(o);
    o = __ushort_as_bfloat16(__ldg(lut + bits));
  }
  return o;
}

// Residual variant (coexecution/kernels/ampere_ada/epilogue.py, module
// docstring): the bf16 GEMM result plus the bf16 residual, added in fp32 and
// rounded to bf16 again.
__device__ __forceinline__ __nv_bfloat16 add_residual(__nv_bfloat16 o,
                                                      const GemmArgs &args,
                                                      int64_t m, int c) {
  if (args.residual == nullptr)
    return o;
  const float r = __bfloat162float(args.residual[m * args.ldr + c]);
  return __float2bfloat16_rn(__fadd_rn(__bfloat162float(o), r));
}

// Unpacks a stage of low-nibble-first int4 bytes into sign-extended int8,
// written in the 128-byte-swizzled K-major layout UMMA reads.  `src` holds
// `rows` rows of 64 packed bytes (128 int4 values); `dst` holds `rows` rows
// of 128 bytes.
__device__ __forceinline__ uint32_t sext_nibbles(uint32_t v) {
  // Each byte of v holds a value 0..15 (two's-complement int4); return the
  // sign-extended int8 in every byte. ((v ^ 8) + 0x78) ^ 0x80 == v - 16*(v>=8)
  // with no carry between bytes.
  return (((v ^ 0x08080808u) + 0x78787878u) ^ 0x80808080u);
}

__device__ __forceinline__ void unpack_int4_stage(const uint8_t *src,
                                                  uint8_t *dst, int rows,
                                                  int tid, int nthreads) {
  // 16 packed bytes -> 32 int8 = two 16-byte chunks of one row.
  const int pieces = rows * 4;
  for (int p = tid; p < pieces; p += nthreads) {
    const int row = p >> 2;
    const int part = p & 3;
    const uint4 w = *reinterpret_cast<const uint4 *>(src + row * 64 + part * 16);
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    uint32_t out[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t lo = sext_nibbles(words[i] & 0x0F0F0F0Fu);
      const uint32_t hi = sext_nibbles((words[i] >> 4) & 0x0F0F0F0Fu);
      out[2 * i] = __byte_perm(lo, hi, 0x5140);
      out[2 * i + 1] = __byte_perm(lo, hi, 0x7362);
    }
    uint8_t *rowp = dst + row * 128;
    const int c0 = (2 * part) ^ (row & 7);
    const int c1 = (2 * part + 1) ^ (row & 7);
    *reinterpret_cast<uint4 *>(rowp + c0 * 16) =
        make_uint4(out[0], out[1], out[2], out[3]);
    *reinterpret_cast<uint4 *>(rowp + c1 * 16) =
        make_uint4(out[4], out[5], out[6], out[7]);
  }
}

// Per-16-channel maxima of |y| over a staged bf16 output tile [rows][width]
// (width a multiple of 16), written to max_out[m0 + j, group0 + g].
__device__ __forceinline__ void store_group_max(const GemmArgs &args, const __nv_bfloat16 *stage,
                                                int width, int rows, int m0, int group0, int et,
                                                int nthreads = 128) {
  const int groups = width / 16;
  for (int it = et; it < rows * groups; it += nthreads) {
    const int j = it / groups, g = it - j * groups;
    const uint4 *p = reinterpret_cast<const uint4 *>(stage + j * width + g * 16);
    float mx = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 u = p[h];
      const __nv_bfloat162 *v = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __bfloat1622float2(v[i]);
        mx = fmaxf(mx, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
    if (group0 + g < args.max_parts)
      args.max_out[int64_t(m0 + j) * args.max_parts + group0 + g] = mx;
  }
}

// Fused activation pack, run by the four epilogue warps (et = 0..127) of a
// CTA whose token tile starts at m0.  The symmetric-row-v1 quantization of
// the plain pack (integer.py:27-94: s = max|x| * (1/127), 1 for an all-zero
// row; q = clamp(rint(x / s), -127, 127); zero codes past K and for padding
// rows), written straight into this CTA's operand tiles:
//  1. one thread bulk-copies the rows (the K slice only when x_max holds
//     the row maxima, else whole rows) into shared memory;
//  2. row maxima from x_max (float bits compared as integers: every value
//     is a non-negative maximum) or from the staged whole rows;
//  3. the scales go to s_sa for the epilogue, and the codes of K blocks
//     [kb_begin, kb_begin + nkb) to the 128-byte-swizzled K-major tiles.
__device__ __forceinline__ void fused_pack(const GemmArgs &args, uint8_t *xs, uint8_t *codes,
                                           float *s_sa, uint64_t *xbar, int bn, int m0,
                                           int kb_begin, int nkb, int et) {
  const int rows = min(bn, args.m - m0);
  const int col0 = kb_begin * kBlockK;
  const bool parts = args.x_max != nullptr;
  const int xcol0 = parts ? col0 : 0;
  const int xcols = parts ? min(nkb * kBlockK, args.k - col0) : args.k;
  const int lane = et & 31;
  if (et == 0) {
    mbar_arrive_expect_tx(xbar, uint32_t(rows * xcols * 2));
    for (int r = 0; r < rows; ++r)
      bulk_load(xs + r * args.x_stride, args.x + int64_t(m0 + r) * args.ldx + xcol0,
                uint32_t(xcols * 2), xbar);
  }
  int *s_max = reinterpret_cast<int *>(s_sa);
  for (int j = et; j < bn; j += 128)
    s_max[j] = 0;
  named_barrier(1, 128);
  if (parts) {
    // x_parts % 4 == 0: every float4 lies within one row.
    const float4 *src = reinterpret_cast<const float4 *>(args.x_max + int64_t(m0) * args.x_parts);
    const int total4 = rows * args.x_parts / 4;
#pragma unroll 4
    for (int f = et; f < total4; f += 128) {
      const float4 v = __ldg(src + f);
      const float mx = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
      atomicMax(s_max + (4 * f) / args.x_parts, __float_as_int(mx));
    }
  }
  mbar_wait(xbar, 0, kStatusTimeoutConvert);
  if (!parts) {
    for (int r = et >> 5; r < rows; r += 4) {
      const uint4 *row = reinterpret_cast<const uint4 *>(xs + r * args.x_stride);
      float mx = 0.f;
      for (int c = lane; c < xcols / 8; c += 32) {
        const uint4 u = row[c];
        const __nv_bfloat162 *v = reinterpret_cast<const __nv_bfloat162 *>(&u);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(v[i]);
          mx = fmaxf(mx, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
      }
#pragma unroll
      for (int d = 16; d; d >>= 1)
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, d));
      if (lane == 0)
        s_max[r] = __float_as_int(mx);
    }
  }
  named_barrier(1, 128);
  for (int j = et; j < bn; j += 128) {
    const float mx = __int_as_float(s_max[j]);
    s_sa[j] = j < rows ? row_scale<8>(mx) : 0.f;
  }
  named_barrier(1, 128);
  const int per_block = bn * 8;   // 16-byte code chunks per K block
  for (int it = et; it < nkb * per_block; it += 128) {
    const int b = it / per_block, rem = it - b * per_block;
    const int j = rem >> 3, c = rem & 7;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (j < rows) {
      const float s = s_sa[j];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int col = col0 + b * kBlockK + c * 16 + h * 8;
        if (col < args.k) {
          const uint4 u = *reinterpret_cast<const uint4 *>(xs + j * args.x_stride + (col - xcol0) * 2);
          const __nv_bfloat16 *v = reinterpret_cast<const __nv_bfloat16 *>(&u);
          uint32_t q[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = __float2int_rn(__fdiv_rn(__bfloat162float(v[i]), s));
            q[i] = uint32_t(max(-127, min(127, r)) & 255);
          }
          w[2 * h] = q[0] | (q[1] << 8) | (q[2] << 16) | (q[3] << 24);
          w[2 * h + 1] = q[4] | (q[5] << 8) | (q[6] << 16) | (q[7] << 24);
        }
      }
    }
    *reinterpret_cast<uint4 *>(codes + b * per_block * 16 + j * 128 + ((c ^ (j & 7)) << 4)) =
        make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// kBits == 8: operands arrive as int8 through TMA in the swizzled layout.
// kBits == 9: the same for E4M3 bytes, multiplied by kind::f8f6f4 into fp32
// accumulators (per-tensor scales arrive replicated as the per-row and
// per-channel scale vectors; split-K partials are fp32, summed in rank order).
// kBits == 4: operands arrive as packed int4 (64 bytes per row and K block,
// no swizzle) and the four epilogue warps unpack them per stage.
//
// Launch with programmatic dependent launch: the prologue (barriers, TMEM,
// descriptor prefetch) and the first weight tiles, which do not depend on
// the previous kernel, overlap its tail; activation tiles and scales are
// read only after griddepcontrol.wait.
// kWide: a token tile of more than 64 rows (the split-K reduction batches
// its peer loads); a separate instantiation so the small-tile code is
// unchanged.
template <int kBits, bool kWide>
__global__ void __launch_bounds__(kThreads, 2)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tm_w,
                   const __grid_constant__ CUtensorMap tm_a,
                   const __grid_constant__ CUtensorMap tm_out,
                   const GemmArgs args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzle atoms.
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  const int bn = args.bn;
  const int stages = args.stages;
  // wt = 2 (int8, no split-K): two 128-channel weight tiles share each token
  // tile, two TMEM accumulators, twice the MMA work per staged byte.
  constexpr bool kF8 = kBits == 9;
  constexpr bool kByte = kBits != 4;   // one byte per operand element, TMA-swizzled
  const int wt = kByte ? args.wt : 1;
  const int op_a_bytes = wt * kWeightTileBytes;   // unpacked int8 weight tile(s)
  const int op_b_bytes = bn * kBlockK;            // unpacked int8 token tile
  // Fused pack: the token codes of all of this CTA's K blocks sit in their
  // own region, so the ring stages hold weights only.
  const bool fused = kBits == 8 && args.x != nullptr;
  const int stage_bytes = op_a_bytes + (fused ? 0 : op_b_bytes);
  // W4A4 keeps the packed TMA destination next to the unpacked operands.
  const int packed_bytes = (kBits == 4) ? (kTileN + bn) * 64 : 0;
  const int packed_stride = (packed_bytes + 1023) & ~1023;
  uint8_t *packed_base = smem + stages * stage_bytes;
  uint8_t *codes = packed_base + stages * packed_stride;            // [fused_kb][bn][128]
  uint8_t *xs = codes + (fused ? args.fused_kb * op_b_bytes : 0);   // staged bf16 rows
  float *s_sa = reinterpret_cast<float *>(xs + (fused ? args.x_bytes : 0));
  uint64_t *bars = reinterpret_cast<uint64_t *>(s_sa + 256);
  uint64_t *full = bars;                  // TMA -> consumer
  uint64_t *empty = bars + stages;        // MMA done -> producer
  uint64_t *ready = bars + 2 * stages;    // (W4A4) unpacked -> MMA
  uint64_t *accum_full = bars + 3 * stages;
  uint64_t *xbar = bars + 3 * stages + 1;   // (fused) staged rows landed
  uint64_t *cbar = bars + 3 * stages + 2;   // (fused) codes written -> MMA
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 3 * stages + 3);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * kTileN * wt;
  const int m0 = blockIdx.y * bn;
  const int split = blockIdx.z;
  const int kb_begin = (split * args.num_kb) / args.splits;
  const int kb_end = ((split + 1) * args.num_kb) / args.splits;
  const int nkb = kb_end - kb_begin;
  const uint32_t acc_cols = bn <= 32 ? 32 : (bn <= 64 ? 64 : (bn <= 128 ? 128 : 256));
  const uint32_t tmem_cols = acc_cols * uint32_t(wt);   // second accumulator at acc_cols

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&ready[s], 128);
    }
    mbar_init(accum_full, 1);
    if (fused) {
      mbar_init(xbar, 1);
      mbar_init(cbar, 128);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tm_w);
    if (!fused)
      tma_prefetch_desc(&tm_a);
    if (args.tma_store)
      tma_prefetch_desc(&tm_out);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Let the next kernel of the stream launch now: its prologue and weight
  // prefetch overlap this kernel; it reads our output only after its own
  // griddepcontrol.wait, which waits for this grid to complete.
  pdl_launch_dependents();

  // Split-K epilogue constants of an epilogue thread (token tiles of at most
  // 64 rows): the scales and bias of its four channels of the rank's slice
  // and the residual values of the tokens it writes.  They are loaded while
  // the main loop runs, so no load is outstanding at the cluster barrier.
  constexpr int kPreTok = 8;   // 64 / (smallest token stride, 8)
  float ep_sw[4] = {0.f, 0.f, 0.f, 0.f}, ep_b[4] = {0.f, 0.f, 0.f, 0.f};
  __nv_bfloat162 ep_res[kPreTok][2];   // bf16 pairs: channels (0, 1), (2, 3)

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one_sync()) {
      // Weights are streamed once when a single token tile covers M; with
      // several token tiles other CTAs re-read them from L2.
      const uint64_t wpolicy =
          gridDim.y == 1 ? policy_evict_first() : policy_evict_last();
      const uint32_t tx = kByte ? uint32_t(stage_bytes)
                                       : uint32_t((kTileN + bn) * 64);   // fused: weights only
      const int kstep = kByte ? kBlockK : 64;
      // Weight tiles of the first ring pass do not depend on the previous
      // kernel: issue them before waiting on it.
      const int pre = min(nkb, stages);
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], tx);
        uint8_t *dst = kByte ? smem + i * stage_bytes
                             : packed_base + i * packed_stride;
        tma_load_2d_hint(dst, &tm_w, &full[i], (kb_begin + i) * kstep, n0,
                         wpolicy);
        if (wt == 2)
          tma_load_2d_hint(dst + kWeightTileBytes, &tm_w, &full[i], (kb_begin + i) * kstep,
                           n0 + kTileN, wpolicy);
      }
      if (!fused) {
        pdl_wait();
        for (int i = 0; i < pre; ++i) {
          uint8_t *dst = kByte ? smem + i * stage_bytes + op_a_bytes
                               : packed_base + i * packed_stride + kTileN * 64;
          tma_load_2d(dst, &tm_a, &full[i], (kb_begin + i) * kstep, m0);
        }
      }
      for (int i = pre; i < nkb; ++i) {
        const int s = i % stages;
        const uint32_t phase = (i / stages) & 1;
        if (!mbar_wait(&empty[s], phase ^ 1, kStatusTimeoutProducer))
          break;
        mbar_arrive_expect_tx(&full[s], tx);
        const int kx = (kb_begin + i) * kstep;
        if (kByte) {
          uint8_t *a = smem + s * stage_bytes;
          tma_load_2d_hint(a, &tm_w, &full[s], kx, n0, wpolicy);
          if (wt == 2)
            tma_load_2d_hint(a + kWeightTileBytes, &tm_w, &full[s], kx, n0 + kTileN, wpolicy);
          if (!fused)
            tma_load_2d(a + op_a_bytes, &tm_a, &full[s], kx, m0);
        } else {
          uint8_t *p = packed_base + s * packed_stride;
          tma_load_2d_hint(p, &tm_w, &full[s], kx, n0, wpolicy);
          tma_load_2d(p + kTileN * 64, &tm_a, &full[s], kx, m0);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    if (elect_one_sync()) {
      const uint32_t idesc = kF8 ? idesc_f8(kTileN, bn) : idesc_i8(kTileN, bn);
      // Fused pack: every K block's codes are written before the first MMA.
      bool ok = !fused || mbar_wait(cbar, 0, kStatusTimeoutMma);
      for (int i = 0; i < nkb && ok; ++i) {
        const int s = i % stages;
        const uint32_t phase = (i / stages) & 1;
        ok = kByte ? mbar_wait(&full[s], phase, kStatusTimeoutMma)
                          : mbar_wait(&ready[s], phase, kStatusTimeoutMma);
        if (!ok)
          break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + s * stage_bytes);
        const uint32_t b_addr =
            fused ? smem_u32(codes + i * op_b_bytes) : a_addr + op_a_bytes;
#pragma unroll
        for (int k = 0; k < kBlockK / 32; ++k) {
          if (kF8)
            mma_f8(tmem_base, smem_desc_sw128(a_addr + k * 32),
                   smem_desc_sw128(b_addr + k * 32), idesc,
                   (i > 0 || k > 0) ? 1u : 0u);
          else
            mma_i8(tmem_base, smem_desc_sw128(a_addr + k * 32),
                   smem_desc_sw128(b_addr + k * 32), idesc,
                   (i > 0 || k > 0) ? 1u : 0u);
          if (wt == 2)
            if (kF8)
              mma_f8(tmem_base + acc_cols, smem_desc_sw128(a_addr + kWeightTileBytes + k * 32),
                     smem_desc_sw128(b_addr + k * 32), idesc, (i > 0 || k > 0) ? 1u : 0u);
            else
              mma_i8(tmem_base + acc_cols, smem_desc_sw128(a_addr + kWeightTileBytes + k * 32),
                     smem_desc_sw128(b_addr + k * 32), idesc, (i > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&empty[s]);
      }
      // Always signal the epilogue; the commit also orders every MMA issued
      // so far, so TMEM is quiescent once the epilogue has seen it.
      mma_commit(accum_full);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int et = threadIdx.x - 64;   // 0..127
    pdl_wait();
    if (fused) {
      fused_pack(args, xs, codes, s_sa, xbar, bn, m0, kb_begin, nkb, et);
      fence_proxy_async_smem();   // the codes are read by the tensor cores
      mbar_arrive(cbar);
    } else {
      // Token scales of this tile, once, while the main loop runs.
      for (int j = et; j < bn; j += 128)
        s_sa[j] = (m0 + j < args.m) ? __ldg(args.sa + m0 + j) : 0.f;
    }
    if (!kWide && args.splits > 1) {
      const int slice = kTileN / args.splits;
      const int tpt = slice / 4;
      const int cc = n0 + int(cluster_ctarank()) * slice + (et % tpt) * 4;
      const int first = et / tpt, tstride = 128 / tpt;
      const int valid_m = min(bn, args.m - m0);
      const __nv_bfloat16 zero = __float2bfloat16_rn(0.f);
      __nv_bfloat16 res[kPreTok][4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const bool in_range = cc + i < args.n_store;
        ep_sw[i] = in_range ? __ldg(args.sw + cc + i) : 0.f;
        ep_b[i] = (args.bias_mode == 2 && in_range) ? __bfloat162float(args.bias[cc + i]) : 0.f;
#pragma unroll
        for (int u = 0; u < kPreTok; ++u) {
          const int j = first + u * tstride;
          res[u][i] = (args.residual != nullptr && in_range && j < valid_m)
                          ? args.residual[int64_t(m0 + j) * args.ldr + cc + i]
                          : zero;
        }
      }
#pragma unroll
      for (int u = 0; u < kPreTok; ++u) {
        ep_res[u][0] = __halves2bfloat162(res[u][0], res[u][1]);
        ep_res[u][1] = __halves2bfloat162(res[u][2], res[u][3]);
      }
    }
    named_barrier(1, 128);
    if (kBits == 4) {
      for (int i = 0; i < nkb; ++i) {
        const int s = i % stages;
        const uint32_t phase = (i / stages) & 1;
        if (!mbar_wait(&full[s], phase, kStatusTimeoutConvert))
          break;
        const uint8_t *p = packed_base + s * packed_stride;
        uint8_t *a = smem + s * stage_bytes;
        unpack_int4_stage(p, a, kTileN, et, 128);
        unpack_int4_stage(p + kTileN * 64, a + op_a_bytes, bn, et, 128);
        fence_proxy_async_smem();
        mbar_arrive(&ready[s]);
      }
    }
    const bool have_acc = mbar_wait(accum_full, 0, kStatusTimeoutEpilogue);
    tc_fence_after();
    const int quarter = warp & 3;
    const int ch = quarter * 32 + lane;       // channel within the tile
    const int c = n0 + ch;
    const int valid_m = min(bn, args.m - m0);
    const uint32_t lane_addr = tmem_base + (uint32_t(quarter * 32) << 16);
    if (have_acc) {
      if (args.silu_lut != nullptr && wt == 2) {
        // SwiGLU: gate (accumulator 0) and up (accumulator 1) of the same
        // 128 output channels meet in this thread: h = bf16(silu(g) * u)
        // with silu(g) from the torch-built table, exactly the gated pack's
        // value (coexecution/kernels/ampere_ada/integer.py:27-48).
        const uint16_t *silu = reinterpret_cast<const uint16_t *>(args.silu_lut);
        const int bias_mode = args.bias_mode;
        const bool tma = args.tma_store != 0;
        const int co = blockIdx.x * kTileN + ch;          // output channel
        const bool in_range = co < args.n_store;
        const float sw_g = in_range ? __ldg(args.sw + c) : 0.f;
        const float sw_u = in_range ? __ldg(args.sw + c + kTileN) : 0.f;
        const float b_g = (bias_mode == 2 && in_range) ? __bfloat162float(args.bias[c]) : 0.f;
        const float b_u = (bias_mode == 2 && in_range) ? __bfloat162float(args.bias[c + kTileN]) : 0.f;
        __nv_bfloat16 *stage = reinterpret_cast<__nv_bfloat16 *>(smem);
        for (int j0 = 0; j0 < bn; j0 += 16) {
          uint32_t rg[16], ru[16];
          tmem_ld_16(lane_addr + j0, rg);
          tmem_ld_16(lane_addr + acc_cols + j0, ru);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const __nv_bfloat16 g = epilogue_value(acc_value<kF8>(rg[i]), s_sa[j0 + i], sw_g, b_g, bias_mode, nullptr);
            const __nv_bfloat16 u = epilogue_value(acc_value<kF8>(ru[i]), s_sa[j0 + i], sw_u, b_u, bias_mode, nullptr);
            const float sg = __bfloat162float(__ushort_as_bfloat16(__ldg(silu + __bfloat16_as_ushort(g))));
            const __nv_bfloat16 h = __float2bfloat16_rn(__fmul_rn(sg, __bfloat162float(u)));
            if (tma)
              stage[(j0 + i) * kTileN + ch] = h;
            else if (in_range && j0 + i < valid_m)
              args.out[int64_t(m0 + j0 + i) * args.ldo + co] = h;
          }
        }
        if (tma) {
          fence_proxy_async_smem();
          named_barrier(1, 128);
          if (et == 0) {
            tma_store_2d(&tm_out, stage, blockIdx.x * kTileN, m0);
            tma_store_commit_and_wait();
          }
          // Per-16-channel maxima of h for the next pack (read from the
          // staged tile, which the TMA store only reads as well).
          if (args.max_out != nullptr)
            store_group_max(args, stage, kTileN, valid_m, m0, blockIdx.x * kTileN / 16, et);
        }
      } else if (args.splits == 1) {
        const uint16_t *lut = reinterpret_cast<const uint16_t *>(args.out_lut);
        const int bias_mode = args.bias_mode;
        const bool tma = args.tma_store != 0;
        const bool with_res = args.residual != nullptr;
        for (int w = 0; w < wt; ++w) {
          const int cw = c + w * kTileN;            // channel of accumulator w
          const bool in_range = cw < args.n_store;
          const float sw = in_range ? __ldg(args.sw + cw) : 0.f;
          const float b = (bias_mode == 2 && in_range) ? __bfloat162float(args.bias[cw]) : 0.f;
          const uint32_t acc_addr = lane_addr + uint32_t(w) * acc_cols;
          // Staging tile [bn tokens][128 channels] bf16 per accumulator in
          // the idle stage buffers, written out by one TMA store each.
          __nv_bfloat16 *stage = reinterpret_cast<__nv_bfloat16 *>(smem) + size_t(w) * bn * kTileN;
          for (int j0 = 0; j0 < bn; j0 += 16) {
            // 16 token columns per step: bn is a multiple of 16.
            uint32_t r[16];
            tmem_ld_16(acc_addr + j0, r);
            float res[16];
            if (with_res) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                res[i] = (in_range && j0 + i < valid_m)
                             ? __bfloat162float(args.residual[int64_t(m0 + j0 + i) * args.ldr + cw])
                             : 0.f;
            }
            tmem_ld_wait();
            __nv_bfloat16 o[16];
#pragma unroll
            for (int i = 0; i < 16; ++i)
              o[i] = epilogue_value(acc_value<kF8>(r[i]), s_sa[j0 + i], sw, b, bias_mode, lut);
            if (with_res) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                o[i] = __float2bfloat16_rn(__fadd_rn(__bfloat162float(o[i]), res[i]));
            }
            if (tma) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                stage[(j0 + i) * kTileN + ch] = o[i];
            } else if (in_range) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (j0 + i < valid_m)
                  args.out[int64_t(m0 + j0 + i) * args.ldo + cw] = o[i];
            }
          }
          if (tma) {
            fence_proxy_async_smem();
            named_barrier(1, 128);
            // A tile that starts past the stored width has nothing to write.
            if (et == 0 && n0 + w * kTileN < args.n_store) {
              tma_store_2d(&tm_out, stage, n0 + w * kTileN, m0);
              tma_store_commit_and_wait();
            }
            if (args.max_out != nullptr)
              store_group_max(args, stage, kTileN, valid_m, m0, (n0 + w * kTileN) / 16, et);
          }
        }
      } else {
        // Partial sums to shared memory as [token][channel] int32, reusing
        // the (now idle) pipeline buffers.
        int *part = reinterpret_cast<int *>(smem);
        for (int j0 = 0; j0 < bn; j0 += 16) {
          uint32_t r[16];
          tmem_ld_16(lane_addr + j0, r);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 16; ++i)
            part[(j0 + i) * kTileN + ch] = int(r[i]);
        }
      }
    }
  }

  if (args.splits > 1) {
    // Every thread of every CTA in the cluster takes part in both phases of
    // the cluster barrier: phase 1 (a full sync) publishes the partial
    // tiles; phase 2 is split, each thread arriving once its reads of the
    // peers' tiles are done and waiting only before exit, so the epilogue
    // math and stores overlap it while no CTA leaves before its peers have
    // read its tile.
    cluster_sync();
    if (warp >= 2) {
      // Rank r reduces and writes channels [r*slice, (r+1)*slice) of the
      // tile.  Each thread owns four consecutive channels (scales and bias
      // loaded once) and walks the tokens; one 16-byte distributed-shared-
      // memory load per peer and token fetches the four partial sums.
      const int et = threadIdx.x - 64;
      const uint32_t rank = cluster_ctarank();
      const int splits = args.splits;
      const int slice = kTileN / splits;              // 64, 32 or 16 channels
      const int tpt = slice / 4;                      // threads per token
      const int cl = (et % tpt) * 4;
      const int cq = int(rank) * slice + cl;          // first channel in the tile
      const int cc = n0 + cq;
      const int tstride = 128 / tpt;
      const int valid_m = min(bn, args.m - m0);
      float sw[4], b[4];
      bool in_range[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        in_range[i] = cc + i < args.n_store;
        if (kWide) {
          sw[i] = in_range[i] ? __ldg(args.sw + cc + i) : 0.f;
          b[i] = (args.bias_mode == 2 && in_range[i]) ? __bfloat162float(args.bias[cc + i]) : 0.f;
        } else {
          sw[i] = ep_sw[i];
          b[i] = ep_b[i];
        }
      }
      const uint16_t *lut = reinterpret_cast<const uint16_t *>(args.out_lut);
      const uint32_t part_addr = smem_u32(smem) + uint32_t(cq * 4);
      uint32_t peer_base[8];
#pragma unroll
      for (int p = 0; p < 8; ++p)
        peer_base[p] = p < splits ? map_peer(part_addr, uint32_t(p)) : 0u;
      // Staging tile [bn][slice] bf16 after the partial sums.
      __nv_bfloat16 *stage = reinterpret_cast<__nv_bfloat16 *>(smem + size_t(bn) * kTileN * 4);
      // Small token tiles write their rows directly (8 bytes per thread and
      // token; nothing to wait for before exit) unless the per-16-channel
      // maxima are wanted, which are taken from the staged tile.
      const bool tma = args.tma_store != 0 && (kWide || args.max_out != nullptr);
      const bool vec8 = args.ldo % 4 == 0 && (reinterpret_cast<uintptr_t>(args.out) & 7) == 0;
      const bool with_res = args.residual != nullptr;
      const int jend = tma ? bn : valid_m;
      const int first = et / tpt;
      // Writes the four outputs of token j from its summed partials.
      auto finish = [&](int j, const int (&acc)[4], const float (&res)[4]) {
        __nv_bfloat16 o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          o[i] = epilogue_value(acc_value<kF8>(uint32_t(acc[i])), s_sa[j], sw[i], b[i], args.bias_mode, lut);
          if (with_res && in_range[i] && j < valid_m)
            o[i] = __float2bfloat16_rn(__fadd_rn(__bfloat162float(o[i]), res[i]));
        }
        if (tma) {
          __nv_bfloat162 *d = reinterpret_cast<__nv_bfloat162 *>(stage + j * slice + cl);
          d[0] = __halves2bfloat162(o[0], o[1]);
          d[1] = __halves2bfloat162(o[2], o[3]);
        } else if (vec8 && in_range[3]) {
          const __nv_bfloat162 lo = __halves2bfloat162(o[0], o[1]), hi = __halves2bfloat162(o[2], o[3]);
          *reinterpret_cast<uint2 *>(args.out + int64_t(m0 + j) * args.ldo + cc) =
              make_uint2(*reinterpret_cast<const uint32_t *>(&lo), *reinterpret_cast<const uint32_t *>(&hi));
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (in_range[i])
              args.out[int64_t(m0 + j) * args.ldo + cc + i] = o[i];
        }
      };
      // Sums the peers' partials of token j (and loads its residual values
      // alongside the distributed-shared-memory loads).
      auto gather = [&](int j, int (&acc)[4], float (&res)[4], bool load_res) {
        const uint32_t off = uint32_t(j * kTileN * 4);
        int4 v[8];
#pragma unroll
        for (int p = 0; p < 8; ++p)
          if (p < splits)
            v[p] = ld_cluster_v4(peer_base[p] + off);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          res[i] = 0.f;
          if (load_res && with_res && in_range[i] && j < valid_m)
            res[i] = __bfloat162float(args.residual[int64_t(m0 + j) * args.ldr + cc + i]);
        }
        acc[0] = acc[1] = acc[2] = acc[3] = 0;
        if (kF8) {
          // fp32 partial sums, added in rank order.
          float f[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int p = 0; p < 8; ++p)
            if (p < splits) {
              f[0] = __fadd_rn(f[0], __int_as_float(v[p].x));
              f[1] = __fadd_rn(f[1], __int_as_float(v[p].y));
              f[2] = __fadd_rn(f[2], __int_as_float(v[p].z));
              f[3] = __fadd_rn(f[3], __int_as_float(v[p].w));
            }
#pragma unroll
          for (int i = 0; i < 4; ++i)
            acc[i] = __float_as_int(f[i]);
        } else {
#pragma unroll
          for (int p = 0; p < 8; ++p)
            if (p < splits) {
              acc[0] += v[p].x;
              acc[1] += v[p].y;
              acc[2] += v[p].z;
              acc[3] += v[p].w;
            }
        }
      };
      // Large token tiles (kWide, many tokens per thread): 8 / S tokens
      // per round for S = 2 or 4 ranks, eight 16-byte peer loads in flight
      // (compile-time S keeps every index in registers).  544 x 2048 x 2048
      // with 2 ranks: 23.8 instead of 27.2 us back to back; small tiles
      // (one or two tokens per thread) keep the per-token loop.
      auto rounds = [&](auto split_count) {
        constexpr int S = decltype(split_count)::value;
        constexpr int per = 8 / S;
        for (int j = first; j < jend; j += per * tstride) {
          int4 v[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int jj = j + (q / S) * tstride;
            if (jj < jend)
              v[q] = ld_cluster_v4(peer_base[q % S] + uint32_t(jj * kTileN * 4));
          }
          // Every residual value of the round is requested before the
          // first one is used.
          float res_all[per][4];
#pragma unroll
          for (int u = 0; u < per; ++u) {
            const int jj = j + u * tstride;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              res_all[u][i] = 0.f;
              if (with_res && in_range[i] && jj < valid_m)
                res_all[u][i] = __bfloat162float(args.residual[int64_t(m0 + jj) * args.ldr + cc + i]);
            }
          }
#pragma unroll
          for (int u = 0; u < per; ++u) {
            const int jj = j + u * tstride;
            if (jj < jend) {
              const float (&res)[4] = res_all[u];
              int acc[4] = {0, 0, 0, 0};
              if (kF8) {
                float f[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int p = 0; p < S; ++p) {
                  f[0] = __fadd_rn(f[0], __int_as_float(v[u * S + p].x));
                  f[1] = __fadd_rn(f[1], __int_as_float(v[u * S + p].y));
                  f[2] = __fadd_rn(f[2], __int_as_float(v[u * S + p].z));
                  f[3] = __fadd_rn(f[3], __int_as_float(v[u * S + p].w));
                }
#pragma unroll
                for (int i = 0; i < 4; ++i)
                  acc[i] = __float_as_int(f[i]);
              } else {
#pragma unroll
                for (int p = 0; p < S; ++p) {
                  acc[0] += v[u * S + p].x;
                  acc[1] += v[u * S + p].y;
                  acc[2] += v[u * S + p].z;
                  acc[3] += v[u * S + p].w;
                }
              }
              finish(jj, acc, res);
            }
          }
        }
      };
      if (kWide && splits == 2) {
        rounds(std::integral_constant<int, 2>());
      } else if (kWide && splits == 4) {
        rounds(std::integral_constant<int, 4>());
      } else if (!kWide) {
        // At most kPreTok tokens per thread; residual values preloaded.
#pragma unroll
        for (int u = 0; u < kPreTok; ++u) {
          const int j = first + u * tstride;
          if (j < jend) {
            int acc[4];
            float res[4];
            gather(j, acc, res, false);
            const float2 r01 = __bfloat1622float2(ep_res[u][0]), r23 = __bfloat1622float2(ep_res[u][1]);
            res[0] = r01.x;
            res[1] = r01.y;
            res[2] = r23.x;
            res[3] = r23.y;
            finish(j, acc, res);
          }
        }
      } else {
        for (int j = first; j < jend; j += tstride) {
          int acc[4];
          float res[4];
          gather(j, acc, res, true);
          finish(j, acc, res);
        }
      }
      // Every read of a peer's tile by this thread is done.
      cluster_arrive();
      if (tma) {
        fence_proxy_async_smem();
        named_barrier(1, 128);
        if (et == 0) {
          tma_store_2d(&tm_out, stage, n0 + int(rank) * slice, m0);
          tma_store_commit_and_wait();
        }
        if (args.max_out != nullptr)
          store_group_max(args, stage, slice, valid_m, m0, (n0 + int(rank) * slice) / 16, et);
      }
    } else {
      cluster_arrive();
    }
    cluster_wait();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

} // namespace pir2b
