// Issue-rate probe of the int8 tensor cores: the denominator the benchmark
// reports large-M GEMMs against.
//
// One CTA per SM; one elected thread issues `iters` x 4 tcgen05.mma
// kind::i8 instructions (M = 128, N = 256, K = 32 each, 1 M MACs) back to
// back into one TMEM accumulator, with both operands resident in shared
// memory (zeros: the rate does not depend on the values), then commits and
// waits (bounded) for their completion.  Each CTA writes the SM clock
// cycles from the first issue to the completion; the host divides the MACs
// by those cycles (MAC / clk / SM) and by the CUDA-event time of the launch.
#pragma once
#include "gemm_i8.cuh"
#include "ptx.cuh"

namespace pir2b {

constexpr int kProbeA = 128 * 128;   // A tile: 128 rows x 128 K bytes
constexpr int kProbeB = 256 * 128;   // B tile: 256 rows x 128 K bytes

__global__ void __launch_bounds__(128, 1) mma_peak_probe_kernel(int iters, long long *cycles) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t *done = reinterpret_cast<uint64_t *>(smem + kProbeA + kProbeB);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
  const int warp = threadIdx.x >> 5;
  for (int i = threadIdx.x; i < (kProbeA + kProbeB) / 16; i += blockDim.x)
    reinterpret_cast<int4 *>(smem)[i] = make_int4(0, 0, 0, 0);
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp == 1 && elect_one_sync()) {
    const uint32_t idesc = idesc_i8(128, 256);
    const uint32_t a = smem_u32(smem), b = smem_u32(smem + kProbeA);
    const long long t0 = clock64();
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int k = 0; k < 4; ++k)
        mma_i8(tmem, smem_desc_sw128(a + k * 32), smem_desc_sw128(b + k * 32), idesc, (it > 0 || k > 0) ? 1u : 0u);
    }
    mma_commit(done);
    mbar_wait(done, 0, kStatusTimeoutMma);
    cycles[blockIdx.x] = clock64() - t0;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

} // namespace pir2b
