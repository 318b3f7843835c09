// NVFP4 GEMM on tcgen05 (kind::mxf4nvf4, block16 UE4M3 scale factors).
//
// Computes y[m, n] = bf16(alpha * sum_k (a[m,k] * sfa) * (w[n,k] * sfw) [+ b])
// for E2M1 operands packed two per byte (low nibble = even column) with one
// UE4M3 factor per 16 elements, the format of piR2's Thor FP4 path
// (coexecution/kernels/blackwell/csrc/fp4_cutlass_linear.cu:686-842,
// :1751-1847; scale layout `sfa_offset`), accumulating in fp32 in TMEM.
//
// Same CTA structure as the integer GEMM: weights are the UMMA A operand
// (128 output channels per CTA), a token tile of BN <= 128 rows is B, warp 0
// issues TMA (packed operands, SWIZZLE_128B) and bulk copies of the scale
// atoms, warp 1 copies the scale atoms into TMEM (tcgen05.cp 32x128b.warpx4)
// and issues the block-scaled MMAs, warps 2-5 run the epilogue.  A 256-
// element K block is 128 bytes per row; its 16 factors per row are four
// 512-byte atoms (128 rows x 4 factors), contiguous in the global layout.
//
// Few tokens (one token tile) give few CTAs, so the K blocks are split over
// a cluster of `splits` CTAs along z: each writes its fp32 partial tile to
// its own (then idle) stage memory, and rank r sums channels
// [r*128/splits, (r+1)*128/splits) of all ranks through distributed shared
// memory in rank order before the alpha/bias epilogue.
#pragma once
#include "args.cuh"
#include "ptx.cuh"

namespace pir2b {

struct Fp4GemmArgs {
  const uint8_t *sfw;            // weight factors, atoms of 128 rows
  const uint8_t *sfa;            // activation factors, atoms of 128 rows
  const __nv_bfloat16 *bias;     // [n] or null
  __nv_bfloat16 *out;            // [m, ldo]
  int64_t ldo;
  int m, n;
  int num_kb;                    // K blocks of 256 elements
  int blocks_k;                  // ceil(K / 64): atoms per 128-row block
  int bn;                        // token tile (16..128, multiple of 16)
  int stages;
  float alpha;
  int tma_store;
  int splits;                    // K split over a cluster along z (1..8)
};

constexpr int kFp4Threads = 192;
constexpr int kFp4BlockBytes = 128;          // 256 fp4 elements per row
constexpr int kFp4WeightTile = 128 * kFp4BlockBytes;
constexpr int kSfStageBytes = 2048;          // four 512-byte atoms

// Descriptor of one scale atom in shared memory for tcgen05.cp: 32 rows of
// 16 contiguous bytes, no swizzle (8-row core matrices 128 bytes apart).
__device__ __forceinline__ uint64_t sf_atom_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1u) << 16;                 // LBO (single column)
  d |= static_cast<uint64_t>(128u >> 4) << 32;          // SBO: 8 rows x 16 B
  d |= static_cast<uint64_t>(1u) << 46;                 // descriptor version
  return d;                                             // SWIZZLE_NONE
}

__device__ __forceinline__ void tmem_cp_atom(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr),
               "l"(sdesc)
               : "memory");
}

__device__ __forceinline__ void mma_nvf4(uint32_t d_tmem, uint64_t adesc,
                                         uint64_t bdesc, uint32_t idesc,
                                         uint32_t tsfa, uint32_t tsfb,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, "
      "%2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tsfa),
      "r"(tsfb)
      : "memory");
}

// Block-scaled instruction descriptor: E2M1 A and B (format 1), UE4M3
// factors (scale format 0), fp32 accumulate implied, K-major, K = 64.
__host__ __device__ constexpr uint32_t idesc_nvf4(uint32_t m, uint32_t n) {
  return (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

__global__ void __launch_bounds__(kFp4Threads, 1)
    gemm_fp4_kernel(const __grid_constant__ CUtensorMap tm_w,
                    const __grid_constant__ CUtensorMap tm_a,
                    const __grid_constant__ CUtensorMap tm_out,
                    const Fp4GemmArgs args) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int bn = args.bn;
  const int stages = args.stages;
  const int op_b_bytes = bn * kFp4BlockBytes;
  const int stage_bytes = kFp4WeightTile + op_b_bytes + 2 * kSfStageBytes;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + stages * stage_bytes);
  uint64_t *full = bars;
  uint64_t *empty = bars + stages;
  uint64_t *accum_full = bars + 2 * stages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * stages + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * 128;
  const int m0 = blockIdx.y * 128;        // token tiles start on atom rows
  const int kb_begin = (int(blockIdx.z) * args.num_kb) / args.splits;
  const int kb_end = ((int(blockIdx.z) + 1) * args.num_kb) / args.splits;
  const int nkb = kb_end - kb_begin;
  constexpr uint32_t kTmemCols = 256;     // accumulator (<=128) + SFA + SFB
  const uint32_t sfa_col = 128, sfb_col = 144;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum_full, 1);
    fence_barrier_init();
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_a);
    if (args.tma_store)
      tma_prefetch_desc(&tm_out);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();

  const uint8_t *sfw_block = args.sfw + (size_t(n0 / 128) * args.blocks_k) * 512;
  const uint8_t *sfa_block = args.sfa + (size_t(m0 / 128) * args.blocks_k) * 512;

  if (warp == 0) {
    if (elect_one_sync()) {
      const uint32_t tx = uint32_t(stage_bytes);
      bool waited = false;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % stages;
        const uint32_t phase = (i / stages) & 1;
        if (!mbar_wait(&empty[s], phase ^ 1, kStatusTimeoutProducer))
          break;
        const int kb = kb_begin + i;
        uint8_t *st = smem + s * stage_bytes;
        mbar_arrive_expect_tx(&full[s], tx);
        tma_load_2d(st, &tm_w, &full[s], kb * kFp4BlockBytes, n0);
        bulk_load(st + kFp4WeightTile + op_b_bytes, sfw_block + size_t(kb) * kSfStageBytes,
                  kSfStageBytes, &full[s]);
        if (!waited) {
          pdl_wait();   // activations and their factors come from the previous kernel
          waited = true;
        }
        tma_load_2d(st + kFp4WeightTile, &tm_a, &full[s], kb * kFp4BlockBytes, m0);
        bulk_load(st + kFp4WeightTile + op_b_bytes + kSfStageBytes,
                  sfa_block + size_t(kb) * kSfStageBytes, kSfStageBytes, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (elect_one_sync()) {
      const uint32_t idesc = idesc_nvf4(128, bn);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % stages;
        const uint32_t phase = (i / stages) & 1;
        if (!mbar_wait(&full[s], phase, kStatusTimeoutMma))
          break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(smem + s * stage_bytes);
        const uint32_t b_addr = a_addr + kFp4WeightTile;
        const uint32_t sfw_addr = b_addr + op_b_bytes;
        const uint32_t sfa_addr = sfw_addr + kSfStageBytes;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          tmem_cp_atom(tmem_base + sfa_col + 4 * k, sf_atom_desc(sfw_addr + 512 * k));
          tmem_cp_atom(tmem_base + sfb_col + 4 * k, sf_atom_desc(sfa_addr + 512 * k));
        }
#pragma unroll
        for (int k = 0; k < 4; ++k)
          mma_nvf4(tmem_base, smem_desc_sw128(a_addr + k * 32),
                   smem_desc_sw128(b_addr + k * 32), idesc,
                   tmem_base + sfa_col + 4 * k, tmem_base + sfb_col + 4 * k,
                   (i > 0 || k > 0) ? 1u : 0u);
        mma_commit(&empty[s]);
      }
      mma_commit(accum_full);
    }
  } else {
    const int et = threadIdx.x - 64;
    pdl_wait();
    const bool have_acc = mbar_wait(accum_full, 0, kStatusTimeoutEpilogue);
    tc_fence_after();
    const int quarter = warp & 3;
    const int ch = quarter * 32 + lane;
    const int c = n0 + ch;
    const bool in_range = c < args.n;
    const float b = (args.bias != nullptr && in_range) ? __bfloat162float(args.bias[c]) : 0.f;
    const int valid_m = min(bn, args.m - m0);
    const uint32_t lane_addr = tmem_base + (uint32_t(quarter * 32) << 16);
    __nv_bfloat16 *stage = reinterpret_cast<__nv_bfloat16 *>(smem);
    if (have_acc && args.splits > 1) {
      // fp32 partial tile [bn][128] over the stage memory: every MMA (and
      // so every read of the stages) completed before accum_full.
      float *part = reinterpret_cast<float *>(smem);
      for (int j0 = 0; j0 < bn; j0 += 16) {
        uint32_t r[16];
        tmem_ld_16(lane_addr + j0, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i)
          part[(j0 + i) * 128 + ch] = __uint_as_float(r[i]);
      }
    } else if (have_acc) {
      for (int j0 = 0; j0 < bn; j0 += 16) {
        uint32_t r[16];
        tmem_ld_16(lane_addr + j0, r);
        tmem_ld_wait();
        __nv_bfloat16 o[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          o[i] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(args.alpha, __uint_as_float(r[i])), b));
        if (args.tma_store) {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            stage[(j0 + i) * 128 + ch] = o[i];
        } else if (in_range) {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (j0 + i < valid_m)
              args.out[int64_t(m0 + j0 + i) * args.ldo + c] = o[i];
        }
      }
      if (args.tma_store) {
        fence_proxy_async_smem();
        named_barrier(1, 128);
        if (et == 0) {
          tma_store_2d(&tm_out, stage, n0, m0);
          tma_store_commit_and_wait();
        }
      }
    }
  }
  if (args.splits > 1) {
    // Every thread of every CTA in the cluster takes part in both barriers.
    cluster_sync();
    if (warp >= 2) {
      // Rank r owns channels [r*slice, (r+1)*slice); a thread takes four
      // consecutive channels and walks the tokens, one 16-byte load per
      // peer and token, summed in rank order.
      const int et = threadIdx.x - 64;
      const uint32_t rank = cluster_ctarank();
      const int splits = args.splits;
      const int slice = 128 / splits;
      const int tpt = slice / 4;
      const int cl = (et % tpt) * 4;
      const int cq = int(rank) * slice + cl;
      const int cc = n0 + cq;
      const int valid_m = min(bn, args.m - m0);
      float b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        b[i] = (args.bias != nullptr && cc + i < args.n) ? __bfloat162float(args.bias[cc + i]) : 0.f;
      const uint32_t part_addr = smem_u32(smem) + uint32_t(cq * 4);
      for (int j = et / tpt; j < valid_m; j += 128 / tpt) {
        const uint32_t off = uint32_t(j * 128 * 4);
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int p = 0; p < splits; ++p) {
          const int4 v = ld_cluster_v4(map_peer(part_addr, uint32_t(p)) + off);
          acc[0] = __fadd_rn(acc[0], __int_as_float(v.x));
          acc[1] = __fadd_rn(acc[1], __int_as_float(v.y));
          acc[2] = __fadd_rn(acc[2], __int_as_float(v.z));
          acc[3] = __fadd_rn(acc[3], __int_as_float(v.w));
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (cc + i < args.n)
            args.out[int64_t(m0 + j) * args.ldo + cc + i] =
                __float2bfloat16_rn(__fadd_rn(__fmul_rn(args.alpha, acc[i]), b[i]));
      }
    }
    cluster_sync();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

} // namespace pir2b
