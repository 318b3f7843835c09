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

// E4M3 x E4M3 -> fp32 on 2-SM tiles (kind::f8f6f4, the operand layout of
// kind::i8).
__device__ __forceinline__ void mma_f8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
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

// Remote arrive (release, cluster scope) on an mbarrier given by its
// shared::cluster address (another CTA's barrier through mapa).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Waits until at most one (read_1) or none (read_0) of this thread's
// committed bulk-store groups is still reading shared memory.
__device__ __forceinline__ void bulk_wait_read_1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_read_0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Threads of a pair CTA: warp 0 TMA, warp 1 TMEM and (even CTA) MMA issue,
// warps 2..9 the epilogue.  Two epilogue warps per TMEM lane quarter (warp w
// may read lanes 32 (w % 4) .. +31) split the token columns in 16-column
// chunks, so each scheduler has a second warp to issue while one waits on
// TMEM or shared memory.
constexpr int kPairThreads = 320;
constexpr int kPairEpiThreads = 256;
// Output tiles leave in groups of 64 tokens x 128 channels (16 KB of bf16)
// through a two-buffer staging ring of their own, so the stage ring keeps
// loading the next tile meanwhile.  Token tiles are multiples of 64.
constexpr int kPairGroup = 64;
constexpr int kPairStagingBytes = 2 * kPairGroup * kTileN * 2;

// Epilogue of 16 tokens (j0 .. j0 + 15) of one channel: the exact order of
// epilogue_value, the two scale products two tokens per packed fp32
// multiply (each lane one IEEE round-to-nearest step).  The bias add stays
// scalar __fadd_rn: a packed __fadd2_rn after the packed multiply was
// contracted into a fused multiply-add (single rounding), which moved
// values that sit exactly on a bf16 rounding tie by one unit.  kF8: the
// accumulator words are fp32 sums (E4M3), else exact int32 sums.
template <bool kF8>
__device__ __forceinline__ void pair_values(const uint32_t (&r)[16], const float *s_sa, int j0, float sw,
                                            float b, int bias_mode, __nv_bfloat162 (&o)[8]) {
  const float4 *sa4 = reinterpret_cast<const float4 *>(s_sa + j0);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 sa = sa4[q];
    const float2 s01 = make_float2(sa.x, sa.y), s23 = make_float2(sa.z, sa.w);
    float2 y0 = make_float2(acc_value<kF8>(r[4 * q]), acc_value<kF8>(r[4 * q + 1]));
    float2 y1 = make_float2(acc_value<kF8>(r[4 * q + 2]), acc_value<kF8>(r[4 * q + 3]));
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

// Persistent over tiles: cluster c of the grid takes tiles c, c + clusters,
// ... of the (token tile, pair) grid, token-tile major.  The stage ring
// runs on across tiles; TMEM holds two accumulator sets when a tile needs
// at most 256 columns (kWt x BN), so the MMAs of the next tile run while
// the epilogue drains the previous one, else one set that the MMA warp
// reuses once both CTAs' epilogues have read it.  kF8: E4M3 operands
// (kind::f8f6f4) with fp32 accumulators, no SwiGLU epilogue.
template <int kWt, bool kF8 = false>
__global__ void __launch_bounds__(kPairThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                     const __grid_constant__ CUtensorMap tm_out, const GemmArgs args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // Both CTAs round the same dynamic base up identically, so a stage sits at
  // the same shared-memory offset in both, as the pair's MMAs require.
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int bn = args.bn;             // tokens of a tile (multiple of 64)
  const int half = bn / 2;            // tokens this CTA loads
  const int stages = args.stages;
  const int a_bytes = kWt * kWeightTileBytes;
  const int stage_bytes = a_bytes + half * kBlockK;
  uint16_t *staging = reinterpret_cast<uint16_t *>(smem + size_t(stages) * stage_bytes);
  float *s_sa = reinterpret_cast<float *>(smem + size_t(stages) * stage_bytes + kPairStagingBytes);
  uint64_t *bars = reinterpret_cast<uint64_t *>(s_sa + 256);
  uint64_t *full = bars;                  // (even CTA) both halves of a stage landed
  uint64_t *empty = bars + stages;        // the pair's MMAs are done with a stage
  uint64_t *acc_full = bars + 2 * stages;       // [2] accumulator set ready (both CTAs)
  uint64_t *acc_empty = bars + 2 * stages + 2;  // [2] (even CTA) both epilogues read it
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * stages + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = int(blockIdx.x) >> 1;
  const int clusters = int(gridDim.x) >> 1;
  const int npairs = args.npairs;
  const int ntiles = npairs * ((args.m + bn - 1) / bn);
  const bool swiglu = kWt == 2 && args.silu_lut != nullptr;
  const int nkb = args.num_kb;
  const uint32_t acc_cols = bn <= 64 ? 64 : (bn <= 128 ? 128 : 256);
  const uint32_t set_cols = acc_cols * uint32_t(kWt);
  const int nbuf = set_cols <= 256 ? 2 : 1;
  const uint32_t tmem_cols = set_cols * uint32_t(nbuf);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * (kPairEpiThreads / 32));
    }
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
  // copy completes on, or any commit or arrive reaches, the other CTA.
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (elect_one_sync()) {
      const uint64_t wpolicy = policy_evict_last();
      const uint64_t apolicy = policy_evict_last();
      const uint32_t tx = uint32_t(2 * stage_bytes);   // both halves, counted on the even CTA
      const uint32_t full0 = map_peer(smem_u32(&full[0]), 0u);
      auto weights = [&](int i, int s, int w_row0) {
        uint8_t *dst = smem + s * stage_bytes;
#pragma unroll
        for (int w = 0; w < kWt; ++w)
          tma_load_2d_pair(dst + w * kWeightTileBytes, &tm_w, full0 + uint32_t(s) * 8u, i * kBlockK,
                           w_row0 + w * kTileN, wpolicy);
      };
      // The first ring pass of the first tile's weights does not depend on
      // the previous kernel: it is issued before griddepcontrol.wait.
      const int pre = cluster < ntiles ? min(nkb, stages) : 0;
      for (int i = 0; i < pre; ++i) {
        if (leader)
          mbar_arrive_expect_tx(&full[i], tx);
        weights(i, i, (2 * (cluster % npairs) + int(rank)) * kWt * kTileN);
      }
      pdl_wait();
      uint32_t kbg = 0;   // K blocks issued so far (all tiles)
      bool ok = true;
      for (int t = cluster; t < ntiles && ok; t += clusters) {
        const int p = t % npairs, m0 = (t / npairs) * bn;
        const int w_row0 = (2 * p + int(rank)) * kWt * kTileN;
        for (int i = 0; i < nkb; ++i, ++kbg) {
          const int s = int(kbg % uint32_t(stages));
          if (kbg >= uint32_t(pre)) {
            if (kbg >= uint32_t(stages) &&
                !mbar_wait(&empty[s], ((kbg / stages) & 1) ^ 1, kStatusTimeoutProducer)) {
              ok = false;
              break;
            }
            if (leader)
              mbar_arrive_expect_tx(&full[s], tx);
            weights(i, s, w_row0);
          }
          tma_load_2d_pair(smem + s * stage_bytes + a_bytes, &tm_a, full0 + uint32_t(s) * 8u, i * kBlockK,
                           m0 + int(rank) * half, apolicy);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue (even CTA)
    if (leader && elect_one_sync()) {
      const uint32_t idesc = kF8 ? idesc_f8(2 * kTileN, uint32_t(bn)) : idesc_i8(2 * kTileN, uint32_t(bn));
      uint32_t kbg = 0;
      int it = 0;
      bool ok = true;
      for (int t = cluster; t < ntiles && ok; t += clusters, ++it) {
        const int b = it % nbuf, use = it / nbuf;
        if (use > 0 && !mbar_wait(&acc_empty[b], (use - 1) & 1, kStatusTimeoutMma))
          break;
        tc_fence_after();
        const uint32_t d = tmem_base + uint32_t(b) * set_cols;
        for (int i = 0; i < nkb; ++i, ++kbg) {
          const int s = int(kbg % uint32_t(stages));
          if (!mbar_wait(&full[s], (kbg / stages) & 1, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + s * stage_bytes);
          const uint32_t b_addr = a_addr + uint32_t(a_bytes);
#pragma unroll
          for (int k = 0; k < kBlockK / 32; ++k) {
            const uint32_t acc = (i > 0 || k > 0) ? 1u : 0u;
#pragma unroll
            for (int w = 0; w < kWt; ++w) {
              if constexpr (kF8)
                mma_f8_pair(d + uint32_t(w) * acc_cols, smem_desc_sw128(a_addr + w * kWeightTileBytes + k * 32),
                            smem_desc_sw128(b_addr + k * 32), idesc, acc);
              else
                mma_i8_pair(d + uint32_t(w) * acc_cols, smem_desc_sw128(a_addr + w * kWeightTileBytes + k * 32),
                            smem_desc_sw128(b_addr + k * 32), idesc, acc);
            }
          }
          mma_commit_pair(&empty[s]);
        }
        // Signals both epilogues (also after a failed wait, so they do not
        // wait out their own budget); orders every MMA of the tile.
        mma_commit_pair(&acc_full[b]);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int et = threadIdx.x - 64;   // 0..255
    const int quarter = warp & 3;
    const int sub = (warp - 2) >> 2;   // this warp's chunks: c % 2 == sub
    const int ch = quarter * 32 + lane;
    const int bias_mode = args.bias_mode;
    const uint32_t lane_off = uint32_t(quarter * 32) << 16;
    const uint16_t *lut = reinterpret_cast<const uint16_t *>(args.out_lut);
    const uint16_t *silu = reinterpret_cast<const uint16_t *>(args.silu_lut);
    const bool with_res = args.residual != nullptr;
    const uint32_t acc_empty0 = map_peer(smem_u32(&acc_empty[0]), 0u);
    const int groups = bn / kPairGroup;
    int gcount = 0;        // output groups staged so far (staging buffer gcount % 2)
    bool stored = false;   // (et == 0) the previous group was stored
    pdl_wait();
    int it = 0;
    for (int t = cluster; t < ntiles; t += clusters, ++it) {
      const int b = it % nbuf, use = it / nbuf;
      const int p = t % npairs, m0 = (t / npairs) * bn;
      const int block = 2 * p + int(rank);
      const int w_row0 = block * kWt * kTileN;
      const int valid_m = min(bn, args.m - m0);
      // The previous tile's last group barrier has passed: s_sa is free.
      for (int j = et; j < bn; j += kPairEpiThreads)
        s_sa[j] = (m0 + j < args.m) ? __ldg(args.sa + m0 + j) : 0.f;
      float sw[kWt], bias[kWt];
      bool in_range[kWt];
#pragma unroll
      for (int w = 0; w < kWt; ++w) {
        const int wr = w_row0 + w * kTileN + ch;
        // SwiGLU: both tiles feed output channel block * 128 + ch.
        in_range[w] = (swiglu ? block * kTileN + ch : wr) < args.n_store;
        sw[w] = in_range[w] ? __ldg(args.sw + wr) : 0.f;
        bias[w] = (bias_mode == 2 && in_range[w]) ? __bfloat162float(args.bias[wr]) : 0.f;
      }
      named_barrier(1, kPairEpiThreads);
      if (!mbar_wait(&acc_full[b], use & 1, kStatusTimeoutEpilogue))
        break;
      tc_fence_after();
      const uint32_t set = tmem_base + lane_off + uint32_t(b) * set_cols;
      const int outs = swiglu ? 1 : kWt;   // output tiles of 128 channels
#pragma unroll
      for (int w = 0; w < kWt; ++w) {
        if (w >= outs)
          break;
        const int c0 = swiglu ? block * kTileN : w_row0 + w * kTileN;   // first output channel
        const int c = c0 + ch;
#pragma unroll 1
        for (int g = 0; g < groups; ++g, ++gcount) {
          uint16_t *stage = staging + (gcount & 1) * (kPairGroup * kTileN);
          // The store that last read this buffer (two groups ago) is done:
          // at most the previous group's store may still be reading.
          if (et == 0) {
            if (stored)
              bulk_wait_read_1();
            else
              bulk_wait_read_0();
          }
          named_barrier(1, kPairEpiThreads);
          // This warp's two 16-token chunks of the group.
          const int k0 = g * 4 + sub, k1 = k0 + 2;
          uint32_t r0[16], r1[16];
          tmem_ld_16(set + uint32_t(w) * acc_cols + k0 * 16, r0);
          tmem_ld_16(set + uint32_t(w) * acc_cols + k1 * 16, r1);
          if (swiglu) {
            uint32_t u0[16], u1[16];
            tmem_ld_16(set + acc_cols + k0 * 16, u0);
            tmem_ld_16(set + acc_cols + k1 * 16, u1);
            tmem_ld_wait_regs(r0);
            tmem_ld_wait_regs(r1);
            tmem_ld_wait_regs(u0);
            tmem_ld_wait_regs(u1);
            auto gated = [&](int k, const uint32_t (&rg)[16], const uint32_t (&ru)[16]) {
              const int j0 = k * 16;
              __nv_bfloat162 gv[8], uv[8];
              pair_values<kF8>(rg, s_sa, j0, sw[0], bias[0], bias_mode, gv);
              pair_values<kF8>(ru, s_sa, j0, sw[kWt - 1], bias[kWt - 1], bias_mode, uv);
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                const float2 sg = make_float2(
                    __bfloat162float(__ushort_as_bfloat16(__ldg(silu + __bfloat16_as_ushort(gv[q].x)))),
                    __bfloat162float(__ushort_as_bfloat16(__ldg(silu + __bfloat16_as_ushort(gv[q].y)))));
                const __nv_bfloat162 h = __float22bfloat162_rn(__fmul2_rn(sg, __bfloat1622float2(uv[q])));
                const int jr = j0 - g * kPairGroup + 2 * q;
                stage[jr * kTileN + ch] = __bfloat16_as_ushort(h.x);
                stage[(jr + 1) * kTileN + ch] = __bfloat16_as_ushort(h.y);
              }
            };
            gated(k0, r0, u0);
            gated(k1, r1, u1);
          } else {
            tmem_ld_wait_regs(r0);
            tmem_ld_wait_regs(r1);
            auto plain = [&](int k, const uint32_t (&r)[16]) {
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
              pair_values<kF8>(r, s_sa, j0, sw[w], bias[w], bias_mode, o);
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                uint16_t lo = __bfloat16_as_ushort(o[q].x), hi = __bfloat16_as_ushort(o[q].y);
                if (lut != nullptr) {
                  lo = __ldg(lut + lo);
                  hi = __ldg(lut + hi);
                }
                if (with_res) {
                  const __nv_bfloat162 v = __floats2bfloat162_rn(
                      __fadd_rn(__bfloat162float(__ushort_as_bfloat16(lo)), res[2 * q]),
                      __fadd_rn(__bfloat162float(__ushort_as_bfloat16(hi)), res[2 * q + 1]));
                  lo = __bfloat16_as_ushort(v.x);
                  hi = __bfloat16_as_ushort(v.y);
                }
                const int jr = j0 - g * kPairGroup + 2 * q;
                stage[jr * kTileN + ch] = lo;
                stage[(jr + 1) * kTileN + ch] = hi;
              }
            };
            plain(k0, r0);
            plain(k1, r1);
          }
          if (w == outs - 1 && g == groups - 1) {
            // Every TMEM read of this warp for the tile is complete: release
            // the accumulator set to the even CTA's MMA warp.
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
              mbar_arrive_cluster(acc_empty0 + uint32_t(b) * 8u);
          }
          fence_proxy_async_smem();
          named_barrier(1, kPairEpiThreads);
          const int gm0 = m0 + g * kPairGroup;
          stored = et == 0 && c0 < args.n_store && gm0 < args.m;
          if (stored) {
            tma_store_2d(&tm_out, stage, c0, gm0);
            bulk_commit();
          }
          if (args.max_out != nullptr && gm0 < args.m)
            store_group_max(args, reinterpret_cast<const __nv_bfloat16 *>(stage), kTileN,
                            min(kPairGroup, args.m - gm0), gm0, c0 / 16, et, kPairEpiThreads);
        }
      }
    }
    if (et == 0)
      bulk_wait_read_0();
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
