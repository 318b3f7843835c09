// Many-token W8A8 GEMM on 2-SM tiles (tcgen05.mma.cta_group::2).
//
// Same arithmetic as gemm_i8_kernel (exact int32 sums; epilogue
// bf16(f32(f32(i2f(acc) * sa) * sw) [+ bias]), then the optional output
// table, residual, per-16-channel maxima, or the SwiGLU value
// bf16(silu[gate] * up)), for token tiles of 64-256 rows, where a one-SM
// tile re-reads the token tile once per 128 channels:
//  * a cluster of two CTAs (a pair) owns 2 x 128 x kWt weight rows and BN
//    tokens.  CTA r loads its own 128 x kWt weight rows and tokens
//    [r BN/2, (r+1) BN/2) of the token tile into its own shared memory (no
//    multicast: each CTA reads only its own halves), with the .cta_group::2
//    TMA form whose completion counts on the even CTA's stage barrier;
//  * the even CTA issues tcgen05.mma.cta_group::2 (M = 256, N = BN) per
//    weight tile: the tensor cores of both SMs read their own halves of the
//    operands and write their own 128 TMEM lanes x BN columns; its commits
//    arrive on the stage and accumulator barriers of both CTAs;
//  * each CTA's eight epilogue warps read its 128 channels x BN tokens per
//    weight tile from TMEM and store each with one TMA store.
// Per K block a CTA stages kWt x 16 KB of weights and BN x 64 bytes of
// tokens for kWt x 128 x BN x 128 MACs: half the token bytes per MAC of the
// one-SM tile.  CTA r of pair p holds weight rows [128 kWt (2p + r),
// 128 kWt (2p + r + 1)); with SwiGLU (kWt = 2, gate|up interleaved in
// 128-row blocks [g0 u0 g1 u1 ...]) that is gate block 2p + r and its up
// block, so both accumulators of a thread hold the same output channel.
//
// Every mbarrier wait is bounded (about a second) and records a status word
// on expiry; the two cluster barriers (after set-up, before TMEM is freed)
// are reached by every thread on every path.
#pragma once
#include "args.cuh"
#include "gemm_i8.cuh"
#include "ptx.cuh"

namespace pir2b {

__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` (same offset) in both CTAs of the pair when the
// pair's previously issued tcgen05 operations have completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(uint16_t(3))
      : "memory");
}

// 2-D tile into this CTA's shared memory, counted on the mbarrier at the
// cluster address `bar` (the even CTA's stage barrier).
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const void *tmap, uint32_t bar, int32_t x, int32_t y,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(bar), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// Threads of a pair CTA: warp 0 TMA, warp 1 TMEM and (even CTA) MMA issue,
// warps 2..9 the epilogue.  Two epilogue warps per TMEM lane quarter (warp w
// may read lanes 32 (w % 4) .. +31) split the token columns in 16-column
// chunks, so each scheduler has a second warp to issue while one waits on
// TMEM or shared memory.
constexpr int kPairThreads = 320;
constexpr int kPairEpiThreads = 256;

// Epilogue of 16 tokens (j0 .. j0 + 15) of one channel: the exact order of
// epilogue_value, the two scale products two tokens per packed fp32
// multiply (each lane one IEEE round-to-nearest step).  The bias add stays
// scalar __fadd_rn: a packed __fadd2_rn after the packed multiply was
// contracted into a fused multiply-add (single rounding), which moved
// values that sit exactly on a bf16 rounding tie by one unit.
__device__ __forceinline__ void pair_values(const uint32_t (&r)[16], const float *s_sa, int j0, float sw,
                                            float b, int bias_mode, __nv_bfloat162 (&o)[8]) {
  const float4 *sa4 = reinterpret_cast<const float4 *>(s_sa + j0);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 sa = sa4[q];
    const float2 s01 = make_float2(sa.x, sa.y), s23 = make_float2(sa.z, sa.w);
    float2 y0 = make_float2(__int2float_rn(int(r[4 * q])), __int2float_rn(int(r[4 * q + 1])));
    float2 y1 = make_float2(__int2float_rn(int(r[4 * q + 2])), __int2float_rn(int(r[4 * q + 3])));
    y0 = __fmul2_rn(__fmul2_rn(y0, s01), make_float2(sw, sw));
    y1 = __fmul2_rn(__fmul2_rn(y1, s23), make_float2(sw, sw));
    if (bias_mode != 0) {
      y0 = make_float2(__fadd_rn(y0.x, b), __fadd_rn(y0.y, b));
      y1 = make_float2(__fadd_rn(y1.x, b), __fadd_rn(y1.y, b));
    }
    o[2 * q] = __float22bfloat162_rn(y0);
    o[2 * q + 1] = __float22bfloat162_rn(y1);
  }
}

template <int kWt>
__global__ void __launch_bounds__(kPairThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                     const __grid_constant__ CUtensorMap tm_out, const GemmArgs args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Both CTAs round the same dynamic base up identically, so a stage sits at
  // the same shared-memory offset in both, as the pair's MMAs require.
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int bn = args.bn;             // tokens of the pair's tile (multiple of 16)
  const int half = bn / 2;            // tokens this CTA loads
  const int stages = args.stages;
  const int a_bytes = kWt * kWeightTileBytes;
  const int stage_bytes = a_bytes + half * kBlockK;
  float *s_sa = reinterpret_cast<float *>(smem + size_t(stages) * stage_bytes);
  uint64_t *bars = reinterpret_cast<uint64_t *>(s_sa + 256);
  uint64_t *full = bars;                  // (even CTA) both halves of a stage landed
  uint64_t *empty = bars + stages;        // the pair's MMAs are done with a stage
  uint64_t *accum_full = bars + 2 * stages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * stages + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int block = int(blockIdx.x);      // 2 p + r: this CTA's weight block
  const int m0 = int(blockIdx.y) * bn;
  const int w_row0 = block * kWt * kTileN;
  const bool swiglu = kWt == 2 && args.silu_lut != nullptr;
  const int nkb = args.num_kb;
  const uint32_t acc_cols = bn <= 32 ? 32 : (bn <= 64 ? 64 : (bn <= 128 ? 128 : 256));
  const uint32_t tmem_cols = acc_cols * uint32_t(kWt);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum_full, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_out);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, tmem_cols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  // Both CTAs' barriers are initialised and their TMEM allocated before any
  // copy completes on, or any commit arrives at, the other CTA.
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (elect_one_sync()) {
      const uint64_t wpolicy = gridDim.y == 1 ? policy_evict_first() : policy_evict_last();
      const uint64_t apolicy = policy_evict_last();
      const uint32_t tx = uint32_t(2 * stage_bytes);   // both halves, counted on the even CTA
      auto weights = [&](int i, int s) {
        const uint32_t bar = map_peer(smem_u32(&full[s]), 0u);
        uint8_t *dst = smem + s * stage_bytes;
#pragma unroll
        for (int w = 0; w < kWt; ++w)
          tma_load_2d_pair(dst + w * kWeightTileBytes, &tm_w, bar, i * kBlockK, w_row0 + w * kTileN, wpolicy);
      };
      auto tokens = [&](int i, int s) {
        const uint32_t bar = map_peer(smem_u32(&full[s]), 0u);
        tma_load_2d_pair(smem + s * stage_bytes + a_bytes, &tm_a, bar, i * kBlockK, m0 + int(rank) * half,
                         apolicy);
      };
      // The first ring pass of weights does not depend on the previous kernel.
      const int pre = min(nkb, stages);
      for (int i = 0; i < pre; ++i) {
        if (leader)
          mbar_arrive_expect_tx(&full[i], tx);
        weights(i, i);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i)
        tokens(i, i);
      for (int i = pre; i < nkb; ++i) {
        const int s = i % stages;
        const uint32_t phase = (i / stages) & 1;
        if (!mbar_wait(&empty[s], phase ^ 1, kStatusTimeoutProducer))
          break;
        if (leader)
          mbar_arrive_expect_tx(&full[s], tx);
        weights(i, s);
        tokens(i, s);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue (even CTA)
    if (leader && elect_one_sync()) {
      const uint32_t idesc = idesc_i8(2 * kTileN, uint32_t(bn));
      for (int i = 0; i < nkb; ++i) {
        const int s = i % stages;
        const uint32_t phase = (i / stages) & 1;
        if (!mbar_wait(&full[s], phase, kStatusTimeoutMma))
          break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + s * stage_bytes);
        const uint32_t b_addr = a_addr + uint32_t(a_bytes);
#pragma unroll
        for (int k = 0; k < kBlockK / 32; ++k) {
          const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
#pragma unroll
          for (int w = 0; w < kWt; ++w)
            mma_i8_pair(tmem_base + uint32_t(w) * acc_cols, smem_desc_sw128(a_addr + w * kWeightTileBytes + k * 32),
                        smem_desc_sw128(b_addr + k * 32), idesc, acc);
        }
        mma_commit_pair(&empty[s]);
      }
      // Always signal both epilogues; the commit also orders every MMA.
      mma_commit_pair(accum_full);
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int et = threadIdx.x - 64;   // 0..255
    pdl_wait();
    for (int j = et; j < bn; j += kPairEpiThreads)
      s_sa[j] = (m0 + j < args.m) ? __ldg(args.sa + m0 + j) : 0.f;
    const int quarter = warp & 3;
    const int sub = (warp - 2) >> 2;   // this warp's chunks: c % 2 == sub
    const int ch = quarter * 32 + lane;
    const int bias_mode = args.bias_mode;
    // Scales and bias of this thread's weight row in each tile.
    float sw[kWt], b[kWt];
    bool in_range[kWt];
#pragma unroll
    for (int w = 0; w < kWt; ++w) {
      const int wr = w_row0 + w * kTileN + ch;
      // SwiGLU: both tiles feed output channel block * 128 + ch.
      in_range[w] = (swiglu ? block * kTileN + ch : wr) < args.n_store;
      sw[w] = in_range[w] ? __ldg(args.sw + wr) : 0.f;
      b[w] = (bias_mode == 2 && in_range[w]) ? __bfloat162float(args.bias[wr]) : 0.f;
    }
    named_barrier(1, kPairEpiThreads);
    const bool have_acc = mbar_wait(accum_full, 0, kStatusTimeoutEpilogue);
    tc_fence_after();
    const uint32_t lane_addr = tmem_base + (uint32_t(quarter * 32) << 16);
    const int valid_m = min(bn, args.m - m0);
    const int nchunks = bn / 16;
    const uint16_t *lut = reinterpret_cast<const uint16_t *>(args.out_lut);
    const uint16_t *silu = reinterpret_cast<const uint16_t *>(args.silu_lut);
    const bool with_res = args.residual != nullptr;
    uint16_t *stage16 = reinterpret_cast<uint16_t *>(smem);   // [bn][128] per tile, ring idle
    if (have_acc && swiglu) {
      const int c0 = block * kTileN;
      for (int c = sub; c < nchunks; c += 2) {
        const int j0 = c * 16;
        uint32_t rg[16], ru[16];
        tmem_ld_16(lane_addr + j0, rg);
        tmem_ld_16(lane_addr + acc_cols + j0, ru);
        tmem_ld_wait_regs(rg);
        tmem_ld_wait_regs(ru);
        __nv_bfloat162 g[8], u[8];
        pair_values(rg, s_sa, j0, sw[0], b[0], bias_mode, g);
        pair_values(ru, s_sa, j0, sw[kWt - 1], b[kWt - 1], bias_mode, u);
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const float2 uf = __bfloat1622float2(u[t]);
          const float2 sg = make_float2(
              __bfloat162float(__ushort_as_bfloat16(__ldg(silu + __bfloat16_as_ushort(g[t].x)))),
              __bfloat162float(__ushort_as_bfloat16(__ldg(silu + __bfloat16_as_ushort(g[t].y)))));
          const __nv_bfloat162 h = __float22bfloat162_rn(__fmul2_rn(sg, uf));
          stage16[(j0 + 2 * t) * kTileN + ch] = __bfloat16_as_ushort(h.x);
          stage16[(j0 + 2 * t + 1) * kTileN + ch] = __bfloat16_as_ushort(h.y);
        }
      }
      fence_proxy_async_smem();
      named_barrier(1, kPairEpiThreads);
      if (et == 0 && c0 < args.n_store) {
        tma_store_2d(&tm_out, stage16, c0, m0);
        tma_store_commit_and_wait();
      }
      if (args.max_out != nullptr)
        store_group_max(args, reinterpret_cast<const __nv_bfloat16 *>(stage16), kTileN, valid_m, m0, c0 / 16,
                        et, kPairEpiThreads);
    } else if (have_acc) {
#pragma unroll
      for (int w = 0; w < kWt; ++w) {
        const int c = w_row0 + w * kTileN + ch;
        uint16_t *stage = stage16 + size_t(w) * bn * kTileN;
        const uint32_t acc_addr = lane_addr + uint32_t(w) * acc_cols;
        // Writes the 16 tokens of chunk k from its accumulator registers.
        auto finish = [&](int k, const uint32_t (&r)[16]) {
          const int j0 = k * 16;
          float res[16];
          if (with_res) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              res[i] = (in_range[w] && j0 + i < valid_m)
                           ? __bfloat162float(args.residual[int64_t(m0 + j0 + i) * args.ldr + c])
                           : 0.f;
          }
          __nv_bfloat162 o[8];
          pair_values(r, s_sa, j0, sw[w], b[w], bias_mode, o);
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            uint16_t lo = __bfloat16_as_ushort(o[t].x), hi = __bfloat16_as_ushort(o[t].y);
            if (lut != nullptr) {
              lo = __ldg(lut + lo);
              hi = __ldg(lut + hi);
            }
            if (with_res) {
              const __nv_bfloat162 v = __floats2bfloat162_rn(
                  __fadd_rn(__bfloat162float(__ushort_as_bfloat16(lo)), res[2 * t]),
                  __fadd_rn(__bfloat162float(__ushort_as_bfloat16(hi)), res[2 * t + 1]));
              lo = __bfloat16_as_ushort(v.x);
              hi = __bfloat16_as_ushort(v.y);
            }
            stage[(j0 + 2 * t) * kTileN + ch] = lo;
            stage[(j0 + 2 * t + 1) * kTileN + ch] = hi;
          }
        };
        // Chunks sub, sub + 2, ...: the next chunk's TMEM load is in flight
        // while this one is finished.
        uint32_t r0[16], r1[16];
        int k = sub;
        if (k < nchunks)
          tmem_ld_16(acc_addr + k * 16, r0);
        tmem_ld_wait_regs(r0);
        while (k < nchunks) {
          const int k1 = k + 2;
          if (k1 < nchunks)
            tmem_ld_16(acc_addr + k1 * 16, r1);
          finish(k, r0);
          tmem_ld_wait_regs(r1);
          if (k1 >= nchunks)
            break;
          const int k2 = k1 + 2;
          if (k2 < nchunks)
            tmem_ld_16(acc_addr + k2 * 16, r0);
          finish(k1, r1);
          tmem_ld_wait_regs(r0);
          k = k2;
        }
        fence_proxy_async_smem();
        named_barrier(1, kPairEpiThreads);
        const int t0 = w_row0 + w * kTileN;
        if (et == 0 && t0 < args.n_store)
          tma_store_2d(&tm_out, stage, t0, m0);
        if (args.max_out != nullptr)
          store_group_max(args, reinterpret_cast<const __nv_bfloat16 *>(stage), kTileN, valid_m, m0, t0 / 16,
                          et, kPairEpiThreads);
      }
      if (et == 0)
        tma_store_commit_and_wait();
    }
  }

  // Both CTAs' epilogues have read their TMEM (and every MMA has completed)
  // before either frees the pair's allocation.
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, tmem_cols);
  }
}

} // namespace pir2b
