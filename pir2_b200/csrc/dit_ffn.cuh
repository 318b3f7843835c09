// The W8A8 feed-forward half of a DiT block in one launch:
//
//   h   = bf16(gelu(bf16(up(x_q))))                     (up GEMM + output LUT)
//   h_q = symmetric-row-v1 int8 pack of h               (plain pack)
//   out = bf16(bf16(down(h_q)) + residual)              (down GEMM + residual)
//
// which is what piR2 runs as four launches after the norm3 pack: the up
// projection, the GELU pack of the down projection's input (`forward_gelu`,
// coexecution/optimization/groot/integer.py:161-165), the down GEMM and the
// residual add (integer_epilogue.cu:156-327).  The values are bitwise those of
// that chain: the GELU is the same torch-built table applied to the same bf16
// GEMM output, the pack's row maximum is order-independent, and every GEMM
// uses the exact epilogue of gemm_i8.cuh.
//
// One grid of F/128 "up" CTAs followed by (D/128) x 8 "down" CTAs, all
// resident at once (the host checks the count against the SMs):
//  * an up CTA owns 128 FFN channels over the full model width: it streams
//    its weights (issued before griddepcontrol.wait) and the packed input,
//    accumulates in TMEM, keeps h for its channels in registers and
//    publishes, per token, the maximum |h| over them (counter A).  Once all
//    up CTAs have, it forms each token's row scale, writes the int8 codes
//    of its own channels and (CTA 0) the row scales, and bumps counter B:
//    every element of h is quantized exactly once;
//  * a down CTA owns 128 output channels and 1/8 of the FFN width (a
//    cluster of 8 splits the K dimension): its whole weight slice is loaded
//    while the up CTAs run; after counter B it loads its slice of the codes
//    by TMA, runs the MMAs and reduces the 8 partial tiles through
//    distributed shared memory, adding the residual in the epilogue.  The
//    last down CTA to finish resets the counters for the next launch.
// Every wait is bounded (about a second); an expired wait records a status
// code and the kernel still runs to completion.
#pragma once
#include "args.cuh"
#include "gemm_i8.cuh"
#include "ptx.cuh"

namespace pir2b {

struct FfnArgs {
  const float *sa;                   // [M] row scales of the packed input
  const float *sw_up;                // [F]
  const __nv_bfloat16 *bias_up;      // [F] or null
  const __nv_bfloat16 *gelu_lut;     // [65536]
  const float *sw_down;              // [D]
  const __nv_bfloat16 *bias_down;    // [D] or null
  const __nv_bfloat16 *residual;     // [M, ldr]
  int64_t ldr;
  __nv_bfloat16 *out;                // [M, ldo]
  int64_t ldo;
  int8_t *codes;                     // workspace [M, F] int8 codes of h
  float *scales;                     // workspace [M] row scales of h
  float *row_max;                    // workspace [M, F / 128]
  unsigned *counters;                // workspace [3], zero between launches
  int m, d, f;
  int bias_mode_up, bias_mode_down;
  int bn;                            // token tile (16..64)
  int up_ctas;                       // F / 128
  int up_kb;                         // model width / 128
  int up_stages;
  int down_kb;                       // FFN width / 128 / kFfnSplits
};

constexpr int kFfnSplits = 8;
constexpr int kStatusTimeoutFfnCounter = 0x105;

__device__ __forceinline__ bool wait_counter(const unsigned *ctr, unsigned target) {
  const long long t0 = clock64();
  for (;;) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    if (v >= target)
      return true;
    if (clock64() - t0 > kWaitCycles) {
      atomicCAS(&g_device_status, 0, kStatusTimeoutFfnCounter);
      return false;
    }
    __nanosleep(32);
  }
}

__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Shared-memory bytes of either role (the launch takes the larger): stage
// buffers, then 2.5 KB of token scales and maxima and up to 1 KB of
// barriers, and 1 KB for the 1024-byte alignment of the dynamic shared
// memory.
__host__ __device__ inline size_t ffn_up_smem(int bn, int stages) {
  return size_t(stages) * (kWeightTileBytes + size_t(bn) * kBlockK) + 2560 + 1024 + 1024;
}
__host__ __device__ inline size_t ffn_down_smem(int bn, int down_kb) {
  return size_t(down_kb) * (kWeightTileBytes + size_t(bn) * kBlockK) + 2560 + 1024 + 1024;
}

__global__ void __launch_bounds__(kThreads, 1)
    dit_ffn_kernel(const __grid_constant__ CUtensorMap tm_up_w,
                   const __grid_constant__ CUtensorMap tm_act,
                   const __grid_constant__ CUtensorMap tm_down_w,
                   const __grid_constant__ CUtensorMap tm_codes, const FfnArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int bn = a.bn;
  const bool up = int(blockIdx.x) < a.up_ctas;
  const int stages = up ? a.up_stages : a.down_kb;
  const int op_b_bytes = bn * kBlockK;
  const int stage_bytes = kWeightTileBytes + op_b_bytes;
  // Up: a ring of [weights | token codes] stages.  Down: all weight tiles,
  // then all token-code tiles.
  float *s_sa = reinterpret_cast<float *>(smem + size_t(stages) * stage_bytes);
  float *s_max = s_sa + 64;                                  // [<= 8][64] (up to 512 floats)
  float *s_hs = s_sa + 576;                                  // [64] row scales of h
  float *s_abs = reinterpret_cast<float *>(smem);            // [128][bn + 1], up epilogue
  uint64_t *bars = reinterpret_cast<uint64_t *>(s_sa + 640);
  uint64_t *full = bars;
  uint64_t *empty = bars + stages;
  uint64_t *accum_full = bars + 2 * stages;
  uint64_t *act_full = bars + 2 * stages + 1;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * stages + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_down_ctas = int(gridDim.x) - a.up_ctas;
  const int down_idx = int(blockIdx.x) - a.up_ctas;
  const int n0 = up ? int(blockIdx.x) * kTileN : (down_idx / kFfnSplits) * kTileN;
  const uint32_t rank = up ? 0u : cluster_ctarank();
  const int num_kb = up ? a.up_kb : a.down_kb;
  const int kb0 = up ? 0 : int(rank) * a.down_kb;
  const uint32_t tmem_cols = bn <= 32 ? 32 : 64;
  const int valid_m = min(bn, a.m);
  unsigned *counter_max = a.counters;        // up CTAs that published maxima
  unsigned *counter_codes = a.counters + 1;  // up CTAs that wrote their codes
  unsigned *counter_done = a.counters + 2;   // down CTAs finished

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum_full, 1);
    mbar_init(act_full, 1);
    fence_barrier_init();
    tma_prefetch_desc(up ? &tm_up_w : &tm_down_w);
    tma_prefetch_desc(up ? &tm_act : &tm_codes);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one_sync()) {
      const uint64_t wpolicy = policy_evict_first();
      if (up) {
        const uint32_t tx = uint32_t(stage_bytes);
        const int pre = min(num_kb, stages);
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(&full[i], tx);
          tma_load_2d_hint(smem + i * stage_bytes, &tm_up_w, &full[i], i * kBlockK, n0, wpolicy);
        }
        pdl_wait();   // the packed input comes from the previous kernel
        for (int i = 0; i < pre; ++i)
          tma_load_2d(smem + i * stage_bytes + kWeightTileBytes, &tm_act, &full[i], i * kBlockK, 0);
        for (int i = pre; i < num_kb; ++i) {
          const int s = i % stages;
          const uint32_t phase = (i / stages) & 1;
          if (!mbar_wait(&empty[s], phase ^ 1, kStatusTimeoutProducer))
            break;
          mbar_arrive_expect_tx(&full[s], tx);
          tma_load_2d_hint(smem + s * stage_bytes, &tm_up_w, &full[s], i * kBlockK, n0, wpolicy);
          tma_load_2d(smem + s * stage_bytes + kWeightTileBytes, &tm_act, &full[s], i * kBlockK, 0);
        }
      } else {
        // The whole weight slice; it depends on nothing of this step.
        for (int i = 0; i < num_kb; ++i) {
          mbar_arrive_expect_tx(&full[i], uint32_t(kWeightTileBytes));
          tma_load_2d_hint(smem + i * kWeightTileBytes, &tm_down_w, &full[i],
                           (kb0 + i) * kBlockK, n0, wpolicy);
        }
        // Then the codes of h, once every up CTA has written them (generic
        // stores, read here through the async proxy).  The counters are
        // shared with the previous launch on this workspace, which resets
        // them as it finishes: wait for that grid before reading them, or a
        // stale count would release the loads of the previous call's codes.
        pdl_wait();
        wait_counter(counter_codes, unsigned(a.up_ctas));
        fence_proxy_async_global();
        uint8_t *codes = smem + num_kb * kWeightTileBytes;
        mbar_arrive_expect_tx(act_full, uint32_t(num_kb * op_b_bytes));
        for (int i = 0; i < num_kb; ++i)
          tma_load_2d(codes + i * op_b_bytes, &tm_codes, act_full, (kb0 + i) * kBlockK, 0);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    if (elect_one_sync()) {
      const uint32_t idesc = idesc_i8(kTileN, bn);
      bool ok = up ? true : mbar_wait(act_full, 0, kStatusTimeoutMma);
      for (int i = 0; i < num_kb && ok; ++i) {
        const int s = up ? i % stages : i;
        const uint32_t phase = up ? (i / stages) & 1 : 0;
        ok = mbar_wait(&full[s], phase, kStatusTimeoutMma);
        if (!ok)
          break;
        tc_fence_after();
        const uint32_t a_addr = up ? smem_u32(smem + s * stage_bytes)
                                   : smem_u32(smem + i * kWeightTileBytes);
        const uint32_t b_addr = up ? a_addr + kWeightTileBytes
                                   : smem_u32(smem + num_kb * kWeightTileBytes + i * op_b_bytes);
#pragma unroll
        for (int k = 0; k < kBlockK / 32; ++k)
          mma_i8(tmem_base, smem_desc_sw128(a_addr + k * 32), smem_desc_sw128(b_addr + k * 32),
                 idesc, (i > 0 || k > 0) ? 1u : 0u);
        if (up)
          mma_commit(&empty[s]);
      }
      mma_commit(accum_full);
    }
  } else {
    // ------------------------------------------------------------ epilogue warps
    const int et = threadIdx.x - 64;    // 0..127
    const int quarter = warp & 3;
    const int ch = quarter * 32 + lane;
    const uint32_t lane_addr = tmem_base + (uint32_t(quarter * 32) << 16);
    pdl_wait();
    if (up) {
      for (int j = et; j < bn; j += 128)
        s_sa[j] = j < a.m ? __ldg(a.sa + j) : 0.f;
      named_barrier(1, 128);
      const bool have_acc = mbar_wait(accum_full, 0, kStatusTimeoutEpilogue);
      tc_fence_after();
      const int c = n0 + ch;
      const float sw = __ldg(a.sw_up + c);
      const float b = a.bias_mode_up == 2 ? __bfloat162float(a.bias_up[c]) : 0.f;
      const uint16_t *lut = reinterpret_cast<const uint16_t *>(a.gelu_lut);
      // h of this thread's channel for every token, in registers (bn <= 64).
      float hv[4][16];
#pragma unroll
      for (int cj = 0; cj < 4; ++cj) {
        if (cj * 16 < bn) {
          uint32_t r[16];
          tmem_ld_16(lane_addr + cj * 16, r);
          tmem_ld_wait();
          __nv_bfloat16 o[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            o[i] = have_acc ? epilogue_value(acc_value<false>(r[i]), s_sa[cj * 16 + i], sw, b, a.bias_mode_up, lut)
                            : __float2bfloat16_rn(0.f);
#pragma unroll
          for (int i = 0; i < 16; ++i)
            hv[cj][i] = __bfloat162float(o[i]);
          // |h| per (channel, token) into the idle stage buffers, laid out
          // [channel][bn + 1] (conflict-free column reads below).
#pragma unroll
          for (int i = 0; i < 16; ++i)
            s_abs[ch * (bn + 1) + cj * 16 + i] = fabsf(hv[cj][i]);
        }
      }
      named_barrier(1, 128);
      // Per-token maximum over the CTA's 128 channels: 128 / bn threads per
      // token, each over a contiguous run of channels.
      {
        const int per = 128 / bn;             // threads per token (2..8)
        const int j = et % bn, part_id = et / bn;
        const int c0 = part_id * (128 / per);
        if (part_id < per) {
          float mx = 0.f;
          for (int cc2 = 0; cc2 < 128 / per; ++cc2)
            mx = fmaxf(mx, s_abs[(c0 + cc2) * (bn + 1) + j]);
          s_max[part_id * 64 + j] = mx;
        }
      }
      named_barrier(1, 128);
      for (int j = et; j < valid_m; j += 128) {
        float mx = 0.f;
        for (int p2 = 0; p2 < 128 / bn; ++p2)
          mx = fmaxf(mx, s_max[p2 * 64 + j]);
        a.row_max[int64_t(j) * a.up_ctas + blockIdx.x] = mx;
      }
      named_barrier(1, 128);
      if (et == 0) {
        __threadfence();
        atomicAdd(counter_max, 1u);
        wait_counter(counter_max, unsigned(a.up_ctas));
      }
      named_barrier(1, 128);
      // Row scales from every up CTA's maxima (all loads issued first).
      {
        const int wq = et >> 5;               // rows wq, wq + 4, ...
        float v[16][2];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const int j = wq + 4 * t;
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int i = lane + 32 * u;      // up CTA (f / 128 <= 64)
            v[t][u] = (j < a.m && i < a.up_ctas) ? __ldcg(a.row_max + int64_t(j) * a.up_ctas + i) : 0.f;
          }
        }
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          float mx = fmaxf(v[t][0], v[t][1]);
#pragma unroll
          for (int o2 = 16; o2; o2 >>= 1)
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o2));
          const int j = wq + 4 * t;
          if (lane == 0 && j < bn)
            s_hs[j] = row_scale<8>(mx);
        }
      }
      named_barrier(1, 128);
      // Codes of this CTA's channels (the plain pack of quant_rows).
#pragma unroll
      for (int cj = 0; cj < 4; ++cj) {
        if (cj * 16 < bn) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int j = cj * 16 + i;
            if (j < a.m) {
              const int q = max(-127, min(127, __float2int_rn(__fdiv_rn(hv[cj][i], s_hs[j]))));
              a.codes[int64_t(j) * a.f + c] = int8_t(q);
            }
          }
        }
      }
      if (blockIdx.x == 0)
        for (int j = et; j < valid_m; j += 128)
          a.scales[j] = s_hs[j];
      named_barrier(1, 128);
      if (et == 0) {
        __threadfence();
        fence_proxy_async_global();
        atomicAdd(counter_codes, 1u);
      }
    } else {
      if (et == 0)
        wait_counter(counter_codes, unsigned(a.up_ctas));
      named_barrier(1, 128);
      for (int j = et; j < bn; j += 128)
        s_sa[j] = j < a.m ? __ldcg(a.scales + j) : 0.f;
      const bool have_acc = mbar_wait(accum_full, 0, kStatusTimeoutEpilogue);
      tc_fence_after();
      // Partial tile [token][channel] int32 over the (now idle) weight tiles.
      int *part = reinterpret_cast<int *>(smem);
      for (int j0 = 0; j0 < bn; j0 += 16) {
        uint32_t r[16];
        tmem_ld_16(lane_addr + j0, r);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 16; ++i)
          part[(j0 + i) * kTileN + ch] = have_acc ? int(r[i]) : 0;
      }
    }
  }

  if (!up) {
    // Split-K reduction over the cluster: rank r writes channels
    // [16 r, 16 r + 16) of the tile, four per thread, one 16-byte
    // distributed-shared-memory load per peer and token.
    cluster_sync();
    if (warp >= 2) {
      const int et = threadIdx.x - 64;
      constexpr int kSlice = kTileN / kFfnSplits;        // 16 channels
      constexpr int kTpt = kSlice / 4;                    // threads per token
      const int cl = (et % kTpt) * 4;
      const int cq = int(rank) * kSlice + cl;
      const int cc = n0 + cq;
      float sw[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sw[i] = __ldg(a.sw_down + cc + i);
        b[i] = a.bias_mode_down == 2 ? __bfloat162float(a.bias_down[cc + i]) : 0.f;
      }
      const uint32_t part_addr = smem_u32(smem) + uint32_t(cq * 4);
      uint32_t peer_base[kFfnSplits];
#pragma unroll
      for (int p = 0; p < kFfnSplits; ++p)
        peer_base[p] = map_peer(part_addr, uint32_t(p));
      for (int j = et / kTpt; j < valid_m; j += 128 / kTpt) {
        const uint32_t off = uint32_t(j * kTileN * 4);
        int4 v[kFfnSplits];
#pragma unroll
        for (int p = 0; p < kFfnSplits; ++p)
          v[p] = ld_cluster_v4(peer_base[p] + off);
        int acc[4] = {0, 0, 0, 0};
#pragma unroll
        for (int p = 0; p < kFfnSplits; ++p) {
          acc[0] += v[p].x;
          acc[1] += v[p].y;
          acc[2] += v[p].z;
          acc[3] += v[p].w;
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const __nv_bfloat16 o = epilogue_value(acc_value<false>(uint32_t(acc[i])), s_sa[j], sw[i], b[i], a.bias_mode_down, nullptr);
          const float r = __bfloat162float(a.residual[int64_t(j) * a.ldr + cc + i]);
          a.out[int64_t(j) * a.ldo + cc + i] = __float2bfloat16_rn(__fadd_rn(__bfloat162float(o), r));
        }
      }
    }
    cluster_sync();
    if (threadIdx.x == 0) {
      // The last down CTA resets the counters for the next launch: by then
      // every up CTA has bumped both counters and every down CTA has passed
      // its waits.
      __threadfence();
      if (atomicAdd(counter_done, 1u) == unsigned(n_down_ctas - 1)) {
        atomicExch(counter_max, 0u);
        atomicExch(counter_codes, 0u);
        atomicExch(counter_done, 0u);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, tmem_cols);
  }
}

} // namespace pir2b
