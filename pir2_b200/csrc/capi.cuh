// C ABI of the library (include/pir2b.h): argument validation, tile-shape
// selection, TMA tensor-map encoding and kernel launches.  Nothing here
// allocates device memory or synchronizes, so every entry point can be
// captured into a CUDA graph once the library is loaded.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <atomic>
#include <mutex>

#include "../../include/pir2b.h"
#pragma once
#include "args.cuh"
#include "ptx.cuh"

namespace pir2b {





// ------------------------------------------------------------------ errors
static thread_local char g_last_error[512] = "";

static int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

static int cuda_status(cudaError_t e, const char *what) {
  if (e == cudaSuccess)
    return PIR2B_OK;
  return fail(PIR2B_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

static bool aligned(const void *p, uintptr_t a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0;
}

// ------------------------------------------------------------------ device info
struct DeviceInfo {
  int sms = 0;
  int max_smem = 0;
  bool attrs_set = false;
  void *ffn_scratch = nullptr;   // device address of g_ffn_scratch (set on first use)
};

static std::mutex g_mutex;
// Plan override for tests and measurement (pir2b_set_pair_mode): 0 lets the
// planner choose, 1 takes 2-SM tiles wherever they fit, 2 never takes them.
static std::atomic<int> g_pair_mode{0};
// Split-K override of the small-M plans for measurement
// (pir2b_set_small_m_splits): 0 lets the planner choose, else 1/2/4/8.
static std::atomic<int> g_small_m_splits{0};
// Few-token kernel override (pir2b_set_few_mode): 0 lets the planner
// choose, 1 takes gemm_few_kernel for every M <= 32, 2 never.
static std::atomic<int> g_few_mode{0};
static DeviceInfo g_devices[64];

static int device_info(DeviceInfo **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return cuda_status(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64)
    return fail(PIR2B_EINVAL, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceInfo &d = g_devices[dev];
  if (d.sms == 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0)
      return fail(PIR2B_EINVAL,
                  "pir2b kernels are built for sm_100a (B200); device %d is "
                  "sm_%d%d",
                  dev, major, minor);
    cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&d.max_smem,
                           cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  }
  if (!d.attrs_set) {
    const void *gemms[] = {
        reinterpret_cast<const void *>(gemm_i8_kernel<8, false>),
        reinterpret_cast<const void *>(gemm_i8_kernel<8, true>),
        reinterpret_cast<const void *>(gemm_i8_kernel<4, false>),
        reinterpret_cast<const void *>(gemm_i8_kernel<4, true>),
        reinterpret_cast<const void *>(gemm_i8_kernel<9, false>),
        reinterpret_cast<const void *>(gemm_i8_kernel<9, true>),
        reinterpret_cast<const void *>(gemm_pair_kernel<1>),
        reinterpret_cast<const void *>(gemm_pair_kernel<2>),
        reinterpret_cast<const void *>(gemm_pair_kernel<1, true>),
        reinterpret_cast<const void *>(gemm_pair_kernel<2, true>)};
    e = cudaSuccess;
    for (const void *f : gemms)
      if (e == cudaSuccess)
        e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, d.max_smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(gemm_fp4_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               d.max_smem);
    if (e == cudaSuccess)
      e = attention_set_smem_all(d.max_smem);
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(dit_ffn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               d.max_smem);
    if (e != cudaSuccess)
      return cuda_status(e, "cudaFuncSetAttribute");
    d.attrs_set = true;
  }
  *out = &d;
  return PIR2B_OK;
}

// ------------------------------------------------------------------ TMA maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t,
                                  void *, const cuuint64_t *, const cuuint64_t *,
                                  const cuuint32_t *, const cuuint32_t *,
                                  CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault,
                                &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D uint8 map over a row-major [rows, cols] byte matrix, box [box_rows,
// box_cols] (box_cols bytes innermost).
static int make_map(CUtensorMap *map, const void *base, uint64_t cols,
                    uint64_t rows, uint64_t row_bytes, uint32_t box_cols,
                    uint32_t box_rows, bool swizzle128) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr)
    return fail(PIR2B_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                  const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B
                             : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PIR2B_ECUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
  return PIR2B_OK;
}

// 2-D bf16 map over the [rows, cols] output (row stride ld elements), box
// [box_rows, box_cols], used by the epilogue's TMA store.
static int make_out_map(CUtensorMap *map, const void *base, uint64_t cols,
                        uint64_t rows, uint64_t ld, uint32_t box_rows,
                        uint32_t box_cols) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr)
    return fail(PIR2B_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                  const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PIR2B_ECUDA, "cuTensorMapEncodeTiled (output) failed (%d)", int(r));
  return PIR2B_OK;
}

// ------------------------------------------------------------------ RMS order
// The launch shape torch's fp32 row mean (x.float() ** 2).mean(-1) takes for
// a contiguous [rows, k] input (ATen Reduce.cuh, setReduceConfig): input
// vectorised by 4 floats (k >= 128), block width bw and height bh from
// 512 threads, one warp-row per output unless the per-thread value count
// reaches min(16 bh, 256) (then torch splits a row across warps, which this
// kernel does not reproduce).  Also returns torch's mean factor, the fp32
// quotient rows / (rows * k).
static int64_t last_pow2(int64_t n) {
  n |= n >> 1;
  n |= n >> 2;
  n |= n >> 4;
  n |= n >> 8;
  n |= n >> 16;
  n |= n >> 32;
  return std::max<int64_t>(1, n - (n >> 1));
}

static bool torch_row_mean_config(int64_t rows, int64_t k, int *bw_out, float *factor) {
  if (k < 128 || k % 4 != 0 || rows < 1)
    return false;
  const int64_t max_threads = 512;
  const int64_t dim0 = k / 4, dim1 = rows;
  const int64_t dim0_pow2 = dim0 < max_threads ? last_pow2(dim0) : max_threads;
  const int64_t dim1_pow2 = dim1 < max_threads ? last_pow2(dim1) : max_threads;
  int64_t bw = std::min<int64_t>(dim0_pow2, 32);
  const int64_t bh = std::min<int64_t>(dim1_pow2, max_threads / bw);
  bw = std::min<int64_t>(dim0_pow2, max_threads / bh);
  const int64_t values_per_thread = (k + bw - 1) / bw;
  if (values_per_thread >= std::min<int64_t>(bh * 16, 256))
    return false;
  *bw_out = int(bw);
  *factor = float(rows) / float(rows * k);
  return true;
}

// ------------------------------------------------------------------ GEMM plan
struct GemmPlan {
  int bn, mtiles, splits, stages;
  size_t smem;
  int wt = 1;          // 128-channel weight tiles per CTA
  int pair = 0;        // 1: 2-SM tiles (gemm_pair_kernel), bn tokens per pair
};

static size_t gemm_smem(int bits, int bn, int stages, int wt = 1) {
  const size_t stage = 16384 * size_t(wt) + size_t(bn) * 128;
  const size_t packed = bits == 4 ? ((size_t(128 + bn) * 64 + 1023) & ~size_t(1023)) : 0;
  // + 1 KB of staged token scales, + barriers and the TMEM address slot.
  return 1024 + stages * (stage + packed) + 1024 + (4 * stages + 1) * 8 + 16;
}

// Single-token-tile (small-M) GEMMs stay under ~110 KB of shared memory so
// two CTAs fit on an SM: with programmatic dependent launch the next GEMM's
// prologue and weight prefetch then run while this one finishes.
constexpr int kCoResidentSmem = 110 * 1024;
// Larger-M GEMM CTAs stay under ~200 KB so a small kernel's CTA still fits
// beside them.
constexpr int kChainSmem = 200 * 1024;

static int stages_for(int bits, int bn, int max_smem, int cap = 8) {
  int s = cap;
  while (s > 2 && gemm_smem(bits, bn, s) > size_t(max_smem))
    --s;
  return s;
}

// Small M (one token tile of <= 64 tokens) is weight streaming, and the
// measured TMA round trip under load is ~2,500 SM cycles, so a CTA moves at
// most (stages x stage bytes) per round trip.  Weight tiles do not depend on
// the previous kernel and are issued before griddepcontrol.wait, so the best
// plan gives every CTA room for its whole K slice (all of its weights are in
// flight while the producer kernel still runs) and spreads the matrix over
// enough CTAs: the smallest split with >= 144 CTAs (about one per SM; the
// DiT step measured 3.09 ms with this target against 3.16 ms with 96 and
// 3.20 ms with 48) whose K slice fits the stage ring.  Matrices with >= 148
// channel tiles keep two CTAs per SM.
static bool plan_small_m(int bits, int64_t m, int ntiles, int num_kb, int max_smem,
                         GemmPlan *plan) {
  const int bn = int((m + 15) / 16 * 16);
  if (ntiles >= 148) {
    const int stages = stages_for(bits, bn, std::min(max_smem, kCoResidentSmem));
    *plan = GemmPlan{bn, 1, 1, stages, gemm_smem(bits, bn, stages)};
    return true;
  }
  const int smax = stages_for(bits, bn, max_smem, 12);
  int chosen = 0;
  for (int s = 1; s <= 8 && s <= num_kb; s *= 2) {
    const int kb_per = (num_kb + s - 1) / s;
    chosen = s;
    if (kb_per <= smax && ntiles * s >= 144)
      break;
  }
  const int forced = g_small_m_splits.load(std::memory_order_relaxed);
  if (forced > 0 && forced <= num_kb)
    chosen = forced;
  const int kb_per = (num_kb + chosen - 1) / chosen;
  int stages = std::max(2, std::min(smax, kb_per));
  // More CTAs than SMs: keep two per SM (one wave) rather than the whole K
  // slice of each in flight (N=12288 K=2048: 192 CTAs of 6 stages instead
  // of 1.3 waves of 8).
  if (ntiles * chosen > 148)
    while (stages > 2 && gemm_smem(bits, bn, stages) > size_t(std::min(max_smem, kCoResidentSmem)))
      --stages;
  const size_t smem = gemm_smem(bits, bn, stages);
  if (smem > size_t(max_smem))
    return false;
  // The split-K partial tile and staging slice live in the stage buffers.
  if (chosen > 1 && size_t(stages) * (16384 + size_t(bn) * 128) < size_t(bn) * (512 + 128))
    return false;
  *plan = GemmPlan{bn, 1, chosen, stages, smem};
  return true;
}

// Fused activation pack (bf16 rows in, int8 codes made by the GEMM CTA):
// the small-M plan with weight-only stages, plus a region for the codes of
// the CTA's K slice and one for the staged bf16 rows.
struct FusedInput {
  const void *x;
  int64_t ldx;
  int64_t k;
  const float *x_max;
  int64_t x_parts;
  int fused_kb;
  int x_stride;
  int x_bytes;
};

static size_t gemm_smem_fused(int bn, int stages, int fused_kb, int x_bytes) {
  return 1024 + size_t(stages) * 16384 + size_t(fused_kb) * bn * 128 + size_t(x_bytes) + 1024 +
         (4 * stages + 1) * 8 + 16;
}

static bool plan_fused(int64_t m, int ntiles, int num_kb, int max_smem, FusedInput *fin,
                       GemmPlan *plan) {
  GemmPlan p;
  if (m > 64 || !plan_small_m(8, m, ntiles, num_kb, max_smem, &p))
    return false;
  const int fused_kb = (num_kb + p.splits - 1) / p.splits;
  const bool parts = fin->x_max != nullptr;
  const int x_stride = parts ? fused_kb * 256 : int((fin->k * 2 + 15) / 16 * 16);
  const int x_bytes = int(m) * x_stride;
  // The split-K partial tile and the rank's staging slice reuse the stages.
  const int min_stages = p.splits > 1 ? int((size_t(p.bn) * 640 + 16383) / 16384) : 2;
  int stages = std::max(std::max(2, min_stages), std::min(p.stages, fused_kb));
  while (stages > std::max(2, min_stages) &&
         gemm_smem_fused(p.bn, stages, fused_kb, x_bytes) > size_t(max_smem))
    --stages;
  const size_t smem = gemm_smem_fused(p.bn, stages, fused_kb, x_bytes);
  if (smem > size_t(max_smem) || size_t(m) * x_stride >= (size_t(1) << 20))
    return false;
  fin->fused_kb = fused_kb;
  fin->x_stride = x_stride;
  fin->x_bytes = x_bytes;
  *plan = GemmPlan{p.bn, 1, p.splits, stages, smem};
  return true;
}

// Shared memory of a 2-SM pair CTA: the stage ring (wt weight tiles and
// half the token tile per stage), the 32 KB output staging ring, token
// scales, barriers, the TMEM slot.
static size_t pair_smem(int bn, int stages, int wt) {
  return 1024 + size_t(stages) * (16384 * size_t(wt) + size_t(bn) * 64) + size_t(kPairStagingBytes) + 1024 +
         (2 * stages + 4) * 8 + 16;
}

// Best 2-SM plan (int8, more than 64 tokens, no split-K) in SM cycles, on
// the cost terms of plan_gemm: a CTA stages half of the token tile per K
// block and the pair's two SMs take one 256 x BN MMA together, so a K block
// costs max(347, 2 BN) cycles per weight tile while the token bytes halve.
// The kernel is persistent (one CTA per SM, tiles strided over the
// clusters); its epilogue (measured ~0.22 SM cycles per output value of a
// CTA with eight epilogue warps) overlaps the next tile's main loop when
// TMEM holds two accumulator sets (kWt x BN <= 256 columns), else follows
// it.  Token tiles are multiples of 64 (the output staging groups).
// Returns the modelled cost (1e30 when no plan fits).
static double plan_pair(int64_t m, int64_t npad, int num_kb, int sms, int max_smem, bool swiglu,
                        GemmPlan *out) {
  double best_cost = 1e30;
  if (m <= 64)
    return best_cost;
  const int clusters_max = sms / 2;
  for (int wt = swiglu ? 2 : 1; wt <= 2; ++wt) {
    const int64_t npairs = (npad + 256 * wt - 1) / (256 * wt);
    for (int bn = 64; bn <= 256; bn += 64) {
      const int64_t mt = (m + bn - 1) / bn;
      if (mt > 1 && (mt - 1) * bn >= m)
        continue;
      int st = 8;
      while (st > 2 && pair_smem(bn, st, wt) > size_t(max_smem))
        --st;
      const size_t smem = pair_smem(bn, st, wt);
      if (smem > size_t(max_smem))
        continue;
      const int64_t tiles = npairs * mt;
      const int64_t clusters = std::min<int64_t>(tiles, clusters_max);
      const int64_t per_cluster = (tiles + clusters - 1) / clusters;
      const int active = int(2 * clusters);
      const double w_bw = std::min(128.0, (mt == 1 ? 3400.0 : 9000.0) / active);
      const double a_bw = std::min(128.0, 9000.0 / active);
      const double per_kb = std::max(std::max(wt * std::max(347.0, 2.0 * bn), 2700.0 / st),
                                     16384.0 * wt / w_bw + 64.0 * bn / a_bw);
      const double main = num_kb * per_kb;
      const double epi = 0.22 * 128.0 * double(swiglu ? 1 : wt) * bn * (swiglu ? 2.0 : 1.0);
      const bool two_sets = wt * bn <= 256;
      const double cost = two_sets ? 3000.0 + main + epi + double(per_cluster - 1) * std::max(main, epi)
                                   : 3000.0 + double(per_cluster) * (main + epi);
      if (cost < best_cost * 0.999) {
        best_cost = cost;
        GemmPlan p{bn, int(mt), 1, st, smem, wt};
        p.pair = 1;
        *out = p;
      }
    }
  }
  return best_cost;
}

// Picks the token tile, the number of token tiles, the split-K cluster size,
// the stage count and the weight tiles per CTA (small M: plan_small_m;
// larger M: the cost model below).
static GemmPlan plan_gemm(int bits, int64_t m, int64_t npad, int64_t kpad,
                          int sms, int max_smem, bool allow_pair = false) {
  const int ntiles = int((npad + 127) / 128);
  const int num_kb = int(kpad / 128);
  GemmPlan best{0, 0, 0, 0, 0};   // smem == 0 marks "no plan"
  if (m <= 64 && plan_small_m(bits, m, ntiles, num_kb, max_smem, &best))
    return best;
  // Larger M: a small cost model in SM cycles over the token tile, the
  // number of token tiles and the split-K cluster size:
  //  * a 128 x BN x 128 K block costs max(347, 2 BN) MMA cycles (measured
  //    kind::i8 issue rate: N <= 128 has a fixed ~87-cycle MMA, full rate is
  //    8192 MAC/clk/SM), and at least the TMA round trip (~2700 cycles) over
  //    the stages in flight: per-CTA traces show K blocks of ~540 cycles
  //    with 5 stages whatever the token tile.  With that term M=544 runs
  //    4 token tiles of 144 on 128 CTAs (6 stages) instead of 3 of 192 on
  //    96 (5 stages): VLM prefill 2.15 -> 2.03 ms in the control step;
  //  * its operands (16 KB of weights + 128 BN bytes) arrive at the CTA's
  //    share of HBM (~3400 B/clk for weights streamed once, single token
  //    tile) or of L2 (~9000 B/clk when several token tiles re-read the
  //    weights);
  //  * each CTA pays ~3000 cycles of launch, prologue and epilogue, +1500 for
  //    the cluster reduction of split-K;
  //  * CTAs under ~113 KB of shared memory run two per SM.
  // A model of the K-block latency alone (which wins on isolated launches)
  // gave a slower VLM prefill inside the full CUDA graph of the control
  // step, where each GEMM shares its SMs with the programmatically launched
  // kernels around it, than this combined one.
  double best_cost = 1e30;
  // Token tiles: the fewest of at most 256 rows and up to three more (M=256
  // as 2-4 tiles of 128-64 rows gives the channel tiles more CTAs than one
  // 256-row tile with split-K over large partial tiles).
  const int mt0 = int((m + 255) / 256);
  const int mt1 = mt0 + 3;
  for (int mt = mt0; mt <= mt1; ++mt) {
    int bn = int(((m + mt - 1) / mt + 15) / 16 * 16);
    if (bn > 256 || bn < 16)
      continue;
    if (int64_t(mt - 1) * bn >= m)
      continue;  // an empty token tile
    const int budget = (mt == 1 && bn <= 64) ? std::min(max_smem, kCoResidentSmem) : max_smem;
    const int stages = stages_for(bits, bn, budget);
    const size_t smem = gemm_smem(bits, bn, stages);
    if (smem > size_t(max_smem))
      continue;
    // Split-K reuses the stage buffers for the int32 partial tile and the
    // rank's bf16 staging slice.
    const bool split_fits =
        size_t(stages) * (16384 + size_t(bn) * 128) >= size_t(bn) * (512 + 128);
    const int per_sm = smem <= 113 * 1024 ? 2 : 1;
    const double scale = bits == 4 ? 0.5 : 1.0;
    const double w_bytes = 16384.0 * scale;     // weight tile per K block
    const double a_bytes = 128.0 * bn * scale;  // token tile per K block
    for (int s = 1; s <= 8; s *= 2) {
      if (s > num_kb || (s > 1 && !split_fits))
        break;
      const int ctas = ntiles * mt * s;
      const int slots = sms * per_sm;
      const int waves = (ctas + slots - 1) / slots;
      const int active = std::min(ctas, slots);
      // Weights come from HBM once (single token tile) or from L2; token
      // tiles are L2-resident.  Per-SM fill rate is capped at 128 B/clk.
      const double w_bw = std::min(128.0, (mt == 1 ? 3400.0 : 9000.0) / active);
      const double a_bw = std::min(128.0, 9000.0 / active);
      const double kb = double(num_kb) / s;
      const double per_kb = std::max(std::max(std::max(347.0, 2.0 * bn), 2700.0 / stages),
                                     w_bytes / w_bw + a_bytes / a_bw);
      const double per_cta = kb * per_kb + 3000.0 + (s > 1 ? 1500.0 : 0.0);
      const double cost = waves * per_cta;
      if (cost < best_cost * 0.999) {
        best_cost = cost;
        best = GemmPlan{bn, mt, s, stages, smem};
      }
    }
  }
  // 2-SM tiles for int8 with more than 64 tokens and a TMA-stored output
  // (back to back on B200 they beat the one-SM plans 1.04-1.9x from M=128
  // to M=34816), except where the one-SM plan splits a long K (>= 32 K
  // blocks) over a cluster and the pair grid would have at most 64 CTAs:
  // M=128/256 K=6144 N=2048 measured 15.5 vs 10.5 and 15.6 vs 12.3 us.
  const int pair_mode = g_pair_mode.load(std::memory_order_relaxed);
  if (allow_pair && bits == 8 && best.smem != 0 && pair_mode != 2) {
    GemmPlan pair;
    if (plan_pair(m, npad, num_kb, sms, max_smem, false, &pair) < 1e30) {
      const int64_t tiles = int64_t((npad + 256 * pair.wt - 1) / (256 * pair.wt)) * pair.mtiles;
      const int64_t ctas = 2 * std::min<int64_t>(tiles, sms / 2);
      if (pair_mode == 1 || !(best.splits > 1 && num_kb >= 32 && ctas <= 64))
        return pair;
    }
  }
  // A plan that needs more than one wave of CTAs runs in one wave with two
  // weight tiles per CTA (twice the MMA work per staged token byte): on
  // isolated launches M=544 N=12288 K=2048 takes 20.6 instead of 29.2 us,
  // M=1088 N=6144 K=1536 18.4 instead of 24.8 us.
  if (bits == 8 && best.smem != 0 && best.splits == 1) {
    const int per_sm = best.smem <= 113 * 1024 ? 2 : 1;
    const int64_t ctas = int64_t(ntiles) * best.mtiles;
    const int64_t ctas2 = int64_t((ntiles + 1) / 2) * best.mtiles;
    int st = 8;
    while (st > 3 && gemm_smem(bits, best.bn, st, 2) > size_t(std::min(max_smem, kChainSmem)))
      --st;
    const size_t smem2 = gemm_smem(bits, best.bn, st, 2);
    // Also when two tiles per CTA still take more than two waves (large
    // M): each staged token byte then feeds twice the MMA work, which
    // measured 17-19 % faster at M=34816 (K=2048 N=4096, K=6144 N=2048).
    if (ctas > int64_t(sms) * per_sm && (ctas2 <= sms || ctas2 > 2 * int64_t(sms)) &&
        smem2 <= size_t(max_smem))
      best = GemmPlan{best.bn, best.mtiles, 1, st, smem2, 2};
  }
  return best;
}

// Plan with two weight tiles per CTA and no split-K (the SwiGLU epilogue):
// the token tiling of the larger-M model above, restricted to wt = 2, with
// all of the opt-in shared memory for stages (M=544 gate|up: 4 stages of
// 56 KB instead of 3 under the 200 KB chain cap, VLM prefill 2.021 ->
// 2.009 ms in the control step).
static GemmPlan plan_gemm_wide(int64_t m, int64_t npad, int64_t kpad, int sms, int max_smem,
                               bool allow_pair = false) {
  const int ntw = int((npad + 255) / 256);
  const int num_kb = int(kpad / 128);
  GemmPlan best{0, 0, 0, 0, 0};
  double best_cost = 1e30;
  const int mt0 = int((m + 255) / 256);
  for (int mt = mt0; mt <= mt0 + 3; ++mt) {
    const int bn = int(((m + mt - 1) / mt + 15) / 16 * 16);
    if (bn > 256 || bn < 16 || int64_t(mt - 1) * bn >= m)
      continue;
    int st = 8;
    while (st > 3 && gemm_smem(8, bn, st, 2) > size_t(max_smem))
      --st;
    const size_t smem = gemm_smem(8, bn, st, 2);
    if (smem > size_t(max_smem))
      continue;
    const int ctas = ntw * mt;
    const int waves = (ctas + sms - 1) / sms;
    const double per_kb = std::max(2700.0 / st, 2.0 * std::max(347.0, 2.0 * bn));
    const double cost = waves * (4200.0 + num_kb * per_kb + 32.0 * bn) + (waves - 1) * 6000.0;
    if (cost < best_cost * 0.999) {
      best_cost = cost;
      best = GemmPlan{bn, mt, 1, st, smem, 2};
    }
  }
  if (allow_pair && best.smem != 0 && g_pair_mode.load(std::memory_order_relaxed) != 2) {
    GemmPlan pair;
    if (plan_pair(m, npad, num_kb, sms, max_smem, true, &pair) < 1e30)
      return pair;
  }
  return best;
}

// Whether a packed-input GEMM of m token rows (int8 / int4 codes, or E4M3
// as bits 9) runs the few-token kernel (gemm_few.cuh).
static bool use_few(int bits, int64_t m) {
  const int mode = g_few_mode.load(std::memory_order_relaxed);
  if ((bits != 8 && bits != 4 && bits != 9) || m > kFewMaxRows || mode == 2)
    return false;
  return true;
}

// Launch of the few-token kernel: one CTA per 16 output channels, token
// tiles of 8 rows (1-4), programmatic dependent launch.
static int launch_few(const void *qa, const float *sa, const void *qw, const float *sw, const void *bias,
                      int bias_mode, const void *out_lut, const void *residual, int64_t ldr, int bits, int64_t m,
                      int64_t npad, int64_t kpad, void *out, int64_t ldo, int64_t n_store, float *max_out,
                      void *stream) {
  FewArgs a;
  memset(&a, 0, sizeof(a));
  a.qa = qa;
  a.lda = bits == 4 ? kpad / 2 : kpad;
  a.sa = sa;
  a.qw = qw;
  a.ldw = a.lda;
  a.sw = sw;
  a.bias = bias_mode == PIR2B_BIAS_ADD ? static_cast<const __nv_bfloat16 *>(bias) : nullptr;
  a.bias_mode = bias_mode;
  a.out_lut = static_cast<const __nv_bfloat16 *>(out_lut);
  a.residual = static_cast<const __nv_bfloat16 *>(residual);
  a.ldr = ldr;
  a.out = static_cast<__nv_bfloat16 *>(out);
  a.ldo = ldo;
  a.max_out = max_out;
  a.max_parts = int(npad / 16);
  a.m = int(m);
  a.npad = int(npad);
  a.n_store = int(n_store);
  a.chunks = int(kpad / 128);
  if (m < 1 || m > kFewMaxRows)
    return fail(PIR2B_EINVAL, "internal: few-token GEMM with m=%lld", (long long)m);
  const int tiles = int((m + 7) / 8);
  // K split over 16 warps (twice the weight loads in flight per CTA) for
  // long K (>= 32 chunks of 128), and for K >= 1024 with 9-24 token rows
  // when the grid has at most one CTA per SM: 17 x 1536 -> 1536 2.5 vs
  // 3.1 us back to back, while wider grids (N = 4608: 4.6 vs 3.6 us) and
  // single rows are faster on 8 warps.
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  const int64_t ctas = (npad + kFewChannels - 1) / kFewChannels;
  const bool wide = tiles <= 3 && (a.chunks >= 32 || (tiles >= 2 && a.chunks >= 8 && ctas <= dev->sms));
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(unsigned((npad + kFewChannels - 1) / kFewChannels), 1u, 1u);
  cfg.blockDim = dim3(wide ? 512 : 256, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
#define PIR2B_FEW(B, T, W) cudaLaunchKernelEx(&cfg, gemm_few_kernel<B, T, W>, a)
  if (wide && bits == 9)
    e = tiles == 1 ? PIR2B_FEW(9, 1, 16) : tiles == 2 ? PIR2B_FEW(9, 2, 16) : PIR2B_FEW(9, 3, 16);
  else if (wide)
    e = bits == 8 ? (tiles == 1 ? PIR2B_FEW(8, 1, 16) : tiles == 2 ? PIR2B_FEW(8, 2, 16) : PIR2B_FEW(8, 3, 16))
                  : (tiles == 1 ? PIR2B_FEW(4, 1, 16) : tiles == 2 ? PIR2B_FEW(4, 2, 16) : PIR2B_FEW(4, 3, 16));
  else if (bits == 9)
    e = tiles == 1   ? PIR2B_FEW(9, 1, 8)
        : tiles == 2 ? PIR2B_FEW(9, 2, 8)
        : tiles == 3 ? PIR2B_FEW(9, 3, 8)
                     : PIR2B_FEW(9, 4, 8);
  else if (bits == 8)
    e = tiles == 1   ? PIR2B_FEW(8, 1, 8)
        : tiles == 2 ? PIR2B_FEW(8, 2, 8)
        : tiles == 3 ? PIR2B_FEW(8, 3, 8)
                     : PIR2B_FEW(8, 4, 8);
  else
    e = tiles == 1   ? PIR2B_FEW(4, 1, 8)
        : tiles == 2 ? PIR2B_FEW(4, 2, 8)
        : tiles == 3 ? PIR2B_FEW(4, 3, 8)
                     : PIR2B_FEW(4, 4, 8);
#undef PIR2B_FEW
  return cuda_status(e, "gemm (few tokens) launch");
}

// The epilogue stages output tiles in shared memory and writes them with TMA
// stores when the output rows are 16-byte aligned.
static bool tma_out(const void *out, int64_t ldo) { return ldo % 8 == 0 && aligned(out, 16); }

// Tensor maps, arguments and launch of one planned integer GEMM.  `n_store`
// is the number of output columns (half the weight rows for SwiGLU).
static int launch_gemm(const GemmPlan &plan, const void *qa, const float *sa, const void *qw,
                       const float *sw, const void *bias, int bias_mode, const void *out_lut,
                       const void *residual, int64_t ldr, const void *silu_lut, int bits,
                       int64_t m, int64_t npad, int64_t kpad, void *out, int64_t ldo,
                       int64_t n_store, void *stream, const FusedInput *fin = nullptr,
                       float *max_out = nullptr) {
  // bits: 8 (int8), 4 (packed int4) or 9 (E4M3 bytes).
  const bool byte_operands = bits != 4;
  const uint64_t row_bytes = byte_operands ? uint64_t(kpad) : uint64_t(kpad / 2);
  const uint32_t box_cols = byte_operands ? 128u : 64u;
  CUtensorMap tm_w, tm_a;
  memset(&tm_a, 0, sizeof(tm_a));
  if (int r = make_map(&tm_w, qw, row_bytes, uint64_t(npad), row_bytes,
                       box_cols, 128u, byte_operands))
    return r;
  if (fin == nullptr) {
    // A pair CTA loads half of the token tile.
    if (int r = make_map(&tm_a, qa, row_bytes, uint64_t(m), row_bytes, box_cols,
                         uint32_t(plan.pair ? plan.bn / 2 : plan.bn), byte_operands))
      return r;
  }
  GemmArgs args;
  memset(&args, 0, sizeof(args));
  if (fin != nullptr) {
    args.x = static_cast<const __nv_bfloat16 *>(fin->x);
    args.ldx = fin->ldx;
    args.k = int(fin->k);
    args.x_max = fin->x_max;
    args.x_parts = int(fin->x_parts);
    args.fused_kb = fin->fused_kb;
    args.x_stride = fin->x_stride;
    args.x_bytes = fin->x_bytes;
  }
  args.max_out = max_out;
  // Output columns per row: half the weight rows with SwiGLU.
  args.max_parts = int((silu_lut != nullptr ? n_store : npad) / 16);
  args.sa = sa;
  args.sw = sw;
  args.bias = bias_mode == PIR2B_BIAS_ADD
                  ? static_cast<const __nv_bfloat16 *>(bias)
                  : nullptr;
  args.out_lut = static_cast<const __nv_bfloat16 *>(out_lut);
  args.residual = static_cast<const __nv_bfloat16 *>(residual);
  args.ldr = ldr;
  args.out = static_cast<__nv_bfloat16 *>(out);
  args.ldo = ldo;
  args.m = int(m);
  args.n_store = int(n_store);
  args.num_kb = int(kpad / 128);
  args.bias_mode = bias_mode;
  args.bn = plan.bn;
  args.stages = plan.stages;
  args.splits = plan.splits;
  args.wt = plan.wt;
  args.silu_lut = static_cast<const __nv_bfloat16 *>(silu_lut);
  // A plan outside the kernel's shapes never reaches the device.
  if (args.bn < 16 || args.bn > 256 || args.bn % 16 != 0 || args.stages < 2 ||
      (args.splits != 1 && args.splits != 2 && args.splits != 4 && args.splits != 8) ||
      (args.wt != 1 && args.wt != 2) || args.num_kb < args.splits || plan.smem == 0)
    return fail(PIR2B_EINVAL, "internal: GEMM plan out of range (bn=%d stages=%d splits=%d wt=%d)",
                args.bn, args.stages, args.splits, args.wt);
  // The epilogue stages the tile (or, with split-K, each cluster rank's
  // channel slice) in shared memory and writes it with one TMA store when
  // the output rows are 16-byte aligned; otherwise it stores directly.
  args.tma_store = tma_out(out, ldo) ? 1 : 0;
  // The 2-SM kernel stores through TMA only and has no split-K or fused pack.
  if (plan.pair && (!args.tma_store || (bits != 8 && bits != 9) || fin != nullptr || plan.splits != 1 ||
                    plan.bn % kPairGroup != 0 || (silu_lut != nullptr && (plan.wt != 2 || bits != 8))))
    return fail(PIR2B_EINVAL, "internal: 2-SM GEMM plan on an unsupported call (bn=%d wt=%d)",
                plan.bn, plan.wt);
  CUtensorMap tm_out;
  memset(&tm_out, 0, sizeof(tm_out));
  if (args.tma_store) {
    // The 2-SM kernel stores 64-token groups.
    if (int r = make_out_map(&tm_out, out, uint64_t(n_store), uint64_t(m),
                             uint64_t(ldo), uint32_t(plan.pair ? kPairGroup : plan.bn),
                             uint32_t(128 / plan.splits)))
      return r;
  }

  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(unsigned((npad + 128 * plan.wt - 1) / (128 * plan.wt)),
                     unsigned(plan.mtiles), unsigned(plan.splits));
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = unsigned(plan.splits);
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (plan.pair) {
    // Persistent: one cluster of two CTAs per SM pair, tiles strided over them.
    const int64_t npairs = (npad + 256 * plan.wt - 1) / (256 * plan.wt);
    args.npairs = int(npairs);
    DeviceInfo *dev = nullptr;
    if (int r = device_info(&dev))
      return r;
    const int64_t clusters = std::min<int64_t>(npairs * plan.mtiles, std::max(1, dev->sms / 2));
    cfg.gridDim = dim3(unsigned(2 * clusters), 1u, 1u);
    cfg.blockDim = dim3(kPairThreads, 1, 1);
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.z = 1;
    cudaError_t e;
    if (bits == 9)
      e = plan.wt == 2 ? cudaLaunchKernelEx(&cfg, gemm_pair_kernel<2, true>, tm_w, tm_a, tm_out, args)
                       : cudaLaunchKernelEx(&cfg, gemm_pair_kernel<1, true>, tm_w, tm_a, tm_out, args);
    else
      e = plan.wt == 2 ? cudaLaunchKernelEx(&cfg, gemm_pair_kernel<2>, tm_w, tm_a, tm_out, args)
                       : cudaLaunchKernelEx(&cfg, gemm_pair_kernel<1>, tm_w, tm_a, tm_out, args);
    return cuda_status(e, "gemm (2-SM) launch");
  }
  // Token tiles above 64 rows take the wide instantiation.
  const bool wide = plan.bn > 64;
  cudaError_t e =
      !wide ? (bits == 8   ? cudaLaunchKernelEx(&cfg, gemm_i8_kernel<8, false>, tm_w, tm_a, tm_out, args)
               : bits == 9 ? cudaLaunchKernelEx(&cfg, gemm_i8_kernel<9, false>, tm_w, tm_a, tm_out, args)
                           : cudaLaunchKernelEx(&cfg, gemm_i8_kernel<4, false>, tm_w, tm_a, tm_out, args))
            : (bits == 8   ? cudaLaunchKernelEx(&cfg, gemm_i8_kernel<8, true>, tm_w, tm_a, tm_out, args)
               : bits == 9 ? cudaLaunchKernelEx(&cfg, gemm_i8_kernel<9, true>, tm_w, tm_a, tm_out, args)
                           : cudaLaunchKernelEx(&cfg, gemm_i8_kernel<4, true>, tm_w, tm_a, tm_out, args));
  return cuda_status(e, "gemm launch");
}

// Self-test of the bounded wait: one thread waits on an mbarrier that
// nothing arrives at.  After the wait budget (about 1 s of SM clock)
// `mbar_wait` gives up and records kStatusTimeoutProbe in the status word;
// the kernel then writes 0 to *result (1 would mean the wait completed).
__global__ void wait_probe_kernel(int *result) {
  __shared__ uint64_t bar;
  mbar_init(&bar, 1);
  fence_barrier_init();
  *result = mbar_wait(&bar, 0, kStatusTimeoutProbe) ? 1 : 0;
}

} // namespace pir2b

using namespace pir2b;

extern "C" {

int pir2b_version(void) { return 100; }

const char *pir2b_last_error(void) { return g_last_error; }

int pir2b_wait_probe(int *result, void *stream) {
  if (result == nullptr || !aligned(result, 4))
    return fail(PIR2B_EINVAL, "wait_probe needs a 4-byte aligned device int");
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  wait_probe_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(result);
  return cuda_status(cudaGetLastError(), "wait probe launch");
}

int pir2b_device_status(int *status_out, void *stream) {
  if (status_out == nullptr)
    return fail(PIR2B_EINVAL, "status_out is null");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int value = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&value, g_device_status,
                                            sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess)
    e = cudaStreamSynchronize(st);
  if (e != cudaSuccess)
    return cuda_status(e, "reading the device status word");
  if (value != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_device_status, &zero, sizeof(int), 0,
                                cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess)
      e = cudaStreamSynchronize(st);
    if (e != cudaSuccess)
      return cuda_status(e, "clearing the device status word");
  }
  *status_out = value;
  return PIR2B_OK;
}

int pir2b_quant_rows(const void *x, int64_t ldx, const void *up, int64_t ldu,
                     const void *lut, const float *smooth, int mode, int bits,
                     int64_t rows, int64_t k, void *q, float *scales,
                     void *stream) {
  if (bits != 4 && bits != 8)
    return fail(PIR2B_EINVAL, "bits must be 4 or 8, got %d", bits);
  if (mode < 0 || mode > 2)
    return fail(PIR2B_EINVAL, "mode must be 0, 1 or 2, got %d", mode);
  if (k < 1 || k > 65536)
    return fail(PIR2B_EINVAL, "row width k=%lld outside [1, 65536]",
                (long long)k);
  if (rows < 0 || rows > 0x7fffffffLL)
    return fail(PIR2B_EINVAL, "row count %lld out of range", (long long)rows);
  if (rows == 0)
    return PIR2B_OK;
  if (x == nullptr || q == nullptr || scales == nullptr)
    return fail(PIR2B_EINVAL, "x, q and scales must be non-null");
  if (ldx < k || (mode == 1 && ldu < k))
    return fail(PIR2B_EINVAL, "row stride smaller than the row width");
  if (mode != 0 && lut == nullptr)
    return fail(PIR2B_EINVAL, "mode %d needs a 65536-entry bf16 lookup table",
                mode);
  if (mode == 1 && up == nullptr)
    return fail(PIR2B_EINVAL, "mode 1 needs the multiplier rows (up)");
  if (!aligned(x, 2) || (up && !aligned(up, 2)) || !aligned(q, 16) ||
      !aligned(scales, 4) || (lut && !aligned(lut, 2)) ||
      (smooth && !aligned(smooth, 4)))
    return fail(PIR2B_EALIGN, "pointer alignment not met");
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  QuantArgs a;
  a.x = static_cast<const __nv_bfloat16 *>(x);
  a.ldx = ldx;
  a.up = mode == 1 ? static_cast<const __nv_bfloat16 *>(up) : nullptr;
  a.ldu = ldu;
  a.lut = static_cast<const uint16_t *>(lut);
  a.smooth = smooth;
  a.q = static_cast<uint8_t *>(q);
  a.scales = scales;
  a.k = int(k);
  a.kpad = int((k + 127) / 128 * 128);
  a.mode = mode;
  const bool vec = (k % 8 == 0) && (ldx % 8 == 0) && aligned(x, 16) &&
                   (mode != 1 || ((ldu % 8 == 0) && aligned(up, 16)));
  return cuda_status(
      run_quant_rows(a, bits, rows, vec, static_cast<cudaStream_t>(stream)),
      "quant_rows launch");
}

int pir2b_quant_rows_max(const void *x, int64_t ldx, const float *x_max, int64_t parts, int bits, int64_t rows,
                         int64_t k, void *q, float *scales, void *stream) {
  if (bits != 4 && bits != 8)
    return fail(PIR2B_EINVAL, "bits must be 4 or 8, got %d", bits);
  if (k < 1 || k > 65536)
    return fail(PIR2B_EINVAL, "row width k=%lld outside [1, 65536]", (long long)k);
  if (rows < 0 || rows > 0x7fffffffLL)
    return fail(PIR2B_EINVAL, "row count %lld out of range", (long long)rows);
  if (parts < 1 || parts > 65536)
    return fail(PIR2B_EINVAL, "parts (maxima per row) must be in [1, 65536]");
  if (rows == 0)
    return PIR2B_OK;
  if (x == nullptr || x_max == nullptr || q == nullptr || scales == nullptr)
    return fail(PIR2B_EINVAL, "x, x_max, q and scales must be non-null");
  if (ldx < k)
    return fail(PIR2B_EINVAL, "row stride smaller than the row width");
  if (!aligned(x, 2) || !aligned(q, 16) || !aligned(scales, 4) || !aligned(x_max, 4))
    return fail(PIR2B_EALIGN, "pointer alignment not met");
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  QuantMaxArgs a;
  a.x = static_cast<const __nv_bfloat16 *>(x);
  a.ldx = ldx;
  a.x_max = x_max;
  a.parts = int(parts);
  a.q = static_cast<uint8_t *>(q);
  a.scales = scales;
  a.k = int(k);
  a.kpad = int((k + 127) / 128 * 128);
  const bool vec = (k % 8 == 0) && (ldx % 8 == 0) && aligned(x, 16);
  return cuda_status(run_quant_rows_max(a, bits, rows, vec, static_cast<cudaStream_t>(stream)),
                     "quant_rows_max launch");
}

int pir2b_floating_rows(const void *x, int64_t ldx, const void *up, int64_t ldu,
                        const void *lut, const float *smooth, int mode, int out_format,
                        int64_t rows, int64_t k, void *q, void *scales, void *stream) {
  if (out_format != PIR2B_OUT_NVFP4 && out_format != PIR2B_OUT_FP8_VALUES)
    return fail(PIR2B_EINVAL, "out_format must be 16 (NVFP4) or 32 (FP8 values), got %d", out_format);
  if (mode < 0 || mode > 2)
    return fail(PIR2B_EINVAL, "mode must be 0, 1 or 2, got %d", mode);
  const int align_k = out_format == PIR2B_OUT_NVFP4 ? 32 : 16;
  if (k < 16 || k > 8192 || k % align_k != 0)
    return fail(PIR2B_EINVAL, "floating producer needs 16 <= k <= 8192 and k %% %d == 0 (k=%lld)", align_k,
                (long long)k);
  if (rows < 0 || rows > 0x7fffffffLL)
    return fail(PIR2B_EINVAL, "row count %lld out of range", (long long)rows);
  if (rows == 0)
    return PIR2B_OK;
  if (x == nullptr || scales == nullptr || (q == nullptr && out_format != PIR2B_OUT_FP8_VALUES))
    return fail(PIR2B_EINVAL, "x, q and scales must be non-null (q may be null for FP8 values)");
  if (ldx < k || (mode == 1 && ldu < k))
    return fail(PIR2B_EINVAL, "row stride smaller than the row width");
  if (mode != 0 && lut == nullptr)
    return fail(PIR2B_EINVAL, "mode %d needs a 65536-entry bf16 lookup table", mode);
  if (mode == 1 && up == nullptr)
    return fail(PIR2B_EINVAL, "mode 1 needs the multiplier rows (up)");
  if (!aligned(x, 2) || (up && !aligned(up, 2)) || (q && !aligned(q, 16)) || !aligned(scales, 4) ||
      (lut && !aligned(lut, 2)) || (smooth && !aligned(smooth, 4)))
    return fail(PIR2B_EALIGN, "pointer alignment not met");
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  QuantArgs a;
  a.x = static_cast<const __nv_bfloat16 *>(x);
  a.ldx = ldx;
  a.up = mode == 1 ? static_cast<const __nv_bfloat16 *>(up) : nullptr;
  a.ldu = ldu;
  a.lut = static_cast<const uint16_t *>(lut);
  a.smooth = smooth;
  a.q = static_cast<uint8_t *>(q);
  a.scales = static_cast<float *>(scales);
  a.k = int(k);
  a.kpad = int(k);
  a.mode = mode;
  const bool vec = (ldx % 8 == 0) && aligned(x, 16) && (mode != 1 || ((ldu % 8 == 0) && aligned(up, 16)));
  return cuda_status(run_quant_rows(a, out_format, rows, vec, static_cast<cudaStream_t>(stream)),
                     "floating_rows launch");
}

int pir2b_fp8_cast(const void *v, int64_t ldv, const float *maxima, int64_t nmax, int64_t rows, int64_t k,
                   int fast, void *q, float *scale, float *scale_rep, int64_t n_rep, void *stream) {
  if (rows < 1 || k < 8 || k % 8 != 0 || k > (1 << 20) || rows > (int64_t(1) << 33) / k || n_rep < 0 ||
      ldv < k || ldv % 8 != 0 || nmax < 1 || nmax > (int64_t(1) << 30))
    return fail(PIR2B_EINVAL,
                "fp8_cast needs rows >= 1, k %% 8 == 0, ldv >= k, ldv %% 8 == 0, nmax >= 1 and n_rep >= 0");
  const float *row_max = maxima;
  if (v == nullptr || row_max == nullptr || q == nullptr || scale == nullptr ||
      (n_rep > 0 && scale_rep == nullptr))
    return fail(PIR2B_EINVAL, "fp8_cast operands must be non-null");
  if (!aligned(v, 16) || !aligned(q, 8) || !aligned(row_max, 4) || !aligned(scale, 4) ||
      (scale_rep && !aligned(scale_rep, 4)))
    return fail(PIR2B_EALIGN, "fp8_cast: v 16-byte, q 8-byte, scales 4-byte aligned");
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  Fp8CastArgs a;
  a.v = static_cast<const __nv_bfloat16 *>(v);
  a.ldv = ldv;
  a.row_max = row_max;
  a.nmax = nmax;
  a.rows = rows;
  a.k = int(k);
  a.fast = fast ? 1 : 0;
  a.q = static_cast<uint8_t *>(q);
  a.scale = scale;
  a.scale_rep = n_rep > 0 ? scale_rep : nullptr;
  a.n_rep = n_rep;
  return cuda_status(run_fp8_cast(a, dev->sms, static_cast<cudaStream_t>(stream)), "fp8_cast launch");
}

int pir2b_norm_quant_rows(const void *x, const void *y_in, const void *gate,
                          void *res_out, const void *gamma, const void *scale,
                          const void *shift, int64_t ld_mod, int64_t tokens,
                          const float *smooth, int norm_kind, float eps,
                          int out_format, int64_t rows, int64_t k, void *q,
                          void *scales, void *stream) {
  if (out_format != PIR2B_OUT_INT8 && out_format != PIR2B_OUT_INT4 &&
      out_format != PIR2B_OUT_NVFP4 && out_format != PIR2B_OUT_FP8_VALUES)
    return fail(PIR2B_EINVAL, "out_format must be 8, 4, 16 or 32, got %d",
                out_format);
  if (norm_kind < 0 || norm_kind > 2)
    return fail(PIR2B_EINVAL, "norm_kind must be 0, 1 or 2");
  if (k < 8 || k > 8192 || k % 8 != 0)
    return fail(PIR2B_EINVAL,
                "fused producers need k %% 8 == 0 and 8 <= k <= 8192 (k=%lld)",
                (long long)k);
  if (out_format == PIR2B_OUT_NVFP4 && k % 32 != 0)
    return fail(PIR2B_EINVAL, "NVFP4 output needs k %% 32 == 0 (k=%lld)",
                (long long)k);
  if (out_format == PIR2B_OUT_FP8_VALUES && k % 16 != 0)
    return fail(PIR2B_EINVAL, "FP8 producer output needs k %% 16 == 0 (k=%lld)",
                (long long)k);
  if (rows < 0 || rows > 0x7fffffffLL)
    return fail(PIR2B_EINVAL, "row count out of range");
  if (rows == 0)
    return PIR2B_OK;
  const bool mod = scale != nullptr;
  const bool res = y_in != nullptr;
  if (x == nullptr || q == nullptr || scales == nullptr)
    return fail(PIR2B_EINVAL, "x, q and scales must be non-null");
  if (mod != (shift != nullptr))
    return fail(PIR2B_EINVAL, "modulation needs both scale and shift");
  if (res && res_out == nullptr)
    return fail(PIR2B_EINVAL, "a residual input needs res_out");
  if (norm_kind == PIR2B_NORM_RMS && gamma == nullptr)
    return fail(PIR2B_EINVAL, "RMSNorm needs gamma");
  if (norm_kind != PIR2B_NORM_NONE && !(eps > 0.f))
    return fail(PIR2B_EINVAL, "epsilon must be positive");
  if ((mod || gate) && (tokens < 1 || ld_mod < k || ld_mod % 8 != 0))
    return fail(PIR2B_EINVAL,
                "modulation rows need tokens >= 1 and ld_mod >= k, %% 8 == 0");
  if (tokens < 1)
    tokens = 1;
  const void *ptrs16[] = {x, y_in, gate, res_out, gamma, scale, shift, q};
  for (const void *p : ptrs16)
    if (p && !aligned(p, 16))
      return fail(PIR2B_EALIGN, "producer operands must be 16-byte aligned");
  if (!aligned(scales, 4) || (smooth && !aligned(smooth, 4)))
    return fail(PIR2B_EALIGN, "scale/smoothing pointer alignment not met");
  if (res && norm_kind == PIR2B_NORM_NONE)
    return fail(PIR2B_EINVAL, "a residual input needs a norm");
  int rms_bw = 0;
  float rms_factor = 0.f;
  const bool floating = out_format == PIR2B_OUT_NVFP4 || out_format == PIR2B_OUT_FP8_VALUES;
  if (norm_kind == PIR2B_NORM_RMS && !floating) {
    if (!torch_row_mean_config(rows, k, &rms_bw, &rms_factor))
      return fail(PIR2B_EINVAL,
                  "RMSNorm pack: rows=%lld k=%lld is outside the row-mean order this kernel "
                  "reproduces (k >= 128 and fewer than 16 values per thread-row step)",
                  (long long)rows, (long long)k);
  }
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  NormArgs a;
  a.rms_bw = rms_bw;
  a.rms_factor = rms_factor;
  a.x = static_cast<const __nv_bfloat16 *>(x);
  a.y_in = static_cast<const __nv_bfloat16 *>(y_in);
  a.gate = static_cast<const __nv_bfloat16 *>(gate);
  a.res_out = static_cast<__nv_bfloat16 *>(res_out);
  a.gamma = static_cast<const __nv_bfloat16 *>(gamma);
  a.scale = static_cast<const __nv_bfloat16 *>(scale);
  a.shift = static_cast<const __nv_bfloat16 *>(shift);
  a.smooth = smooth;
  a.q = static_cast<uint8_t *>(q);
  a.scales = static_cast<uint8_t *>(scales);
  a.ld_mod = ld_mod;
  a.tokens = tokens;
  a.k = int(k);
  a.kpad = floating ? int(k) : int((k + 127) / 128 * 128);
  a.eps = eps;
  return cuda_status(run_norm_quant(a, out_format, rows, norm_kind, mod, res,
                                    static_cast<cudaStream_t>(stream)),
                     "norm_quant_rows launch");
}

int pir2b_pack_nvfp4(const void *x, int64_t rows, int64_t k, void *packed,
                     void *sf, void *stream) {
  return pir2b_norm_quant_rows(x, nullptr, nullptr, nullptr, nullptr, nullptr,
                               nullptr, 0, 1, nullptr, PIR2B_NORM_NONE, 0.f,
                               PIR2B_OUT_NVFP4, rows, k, packed, sf, stream);
}

int pir2b_gemm(const void *qa, const float *sa, const void *qw,
               const float *sw, const void *bias, int bias_mode,
               const void *out_lut, const void *residual, int64_t ldr,
               int bits, int64_t m, int64_t npad, int64_t kpad, void *out,
               int64_t ldo, int64_t n_store, int tactic, void *stream) {
  (void)tactic;
  if (bits != 4 && bits != 8)
    return fail(PIR2B_EINVAL, "bits must be 4 or 8, got %d", bits);
  if (bias_mode < 0 || bias_mode > 2)
    return fail(PIR2B_EINVAL, "bias_mode must be 0, 1 or 2");
  if (m < 1 || m > 0x7fffffffLL || npad < 8 || npad % 8 != 0 || kpad < 128 ||
      kpad % 128 != 0 || npad > 0x7fffffffLL || kpad > (1LL << 20))
    return fail(PIR2B_EINVAL,
                "GEMM requires m >= 1, npad %% 8 == 0 and kpad %% 128 == 0 "
                "(m=%lld npad=%lld kpad=%lld)",
                (long long)m, (long long)npad, (long long)kpad);
  if (n_store < 1 || n_store > npad || ldo < n_store)
    return fail(PIR2B_EINVAL, "n_store must be in [1, npad] and ldo >= n_store");
  if (qa == nullptr || sa == nullptr || qw == nullptr || sw == nullptr ||
      out == nullptr)
    return fail(PIR2B_EINVAL, "GEMM operands must be non-null");
  if (bias_mode == PIR2B_BIAS_ADD && bias == nullptr)
    return fail(PIR2B_EINVAL, "bias_mode ADD needs a bias vector");
  if (!aligned(qa, 16) || !aligned(qw, 16))
    return fail(PIR2B_EALIGN, "packed operands must be 16-byte aligned");
  if (!aligned(out, 2) || !aligned(sa, 4) || !aligned(sw, 4) ||
      (bias && !aligned(bias, 2)) || (out_lut && !aligned(out_lut, 2)) ||
      (residual && !aligned(residual, 2)))
    return fail(PIR2B_EALIGN, "scale/bias/output alignment not met");
  if (residual != nullptr && ldr < n_store)
    return fail(PIR2B_EINVAL, "residual row stride ldr must be >= n_store");
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  if (use_few(bits, m))
    return launch_few(qa, sa, qw, sw, bias, bias_mode, out_lut, residual, ldr, bits, m, npad, kpad, out, ldo,
                      n_store, nullptr, stream);
  const GemmPlan plan = plan_gemm(bits, m, npad, kpad, dev->sms, dev->max_smem, tma_out(out, ldo));
  if (plan.smem == 0 || int64_t(plan.bn) * plan.mtiles < m || plan.stages < 2 ||
      plan.smem > size_t(dev->max_smem))
    return fail(PIR2B_EINVAL, "no GEMM tile plan fits m=%lld npad=%lld kpad=%lld",
                (long long)m, (long long)npad, (long long)kpad);
  return launch_gemm(plan, qa, sa, qw, sw, bias, bias_mode, out_lut, residual, ldr, nullptr,
                     bits, m, npad, kpad, out, ldo, n_store, stream);
}

int pir2b_qk_norm_rope(const void *qkv, int64_t ld, const void *q_weight,
                       const void *k_weight, const void *cos, const void *sin,
                       int64_t rows, int64_t tokens, int hq, int hk,
                       int head_dim, float eps, void *q_out, void *k_out,
                       void *v_out, void *stream) {
  if (head_dim != 128)
    return fail(PIR2B_EINVAL, "qk_norm_rope supports head_dim 128 (got %d)", head_dim);
  if (rows < 0 || tokens < 1 || rows % tokens != 0 || hq < 1 || hk < 1 ||
      rows > 0x7fffffffLL / (hq + 2 * hk))
    return fail(PIR2B_EINVAL, "qk_norm_rope: bad rows/tokens/heads");
  if (ld < int64_t(hq + 2 * hk) * head_dim || ld % 4 != 0)
    return fail(PIR2B_EINVAL, "qk_norm_rope: row stride too small or not a multiple of 4");
  if (!(eps > 0.f))
    return fail(PIR2B_EINVAL, "qk_norm_rope: epsilon must be positive");
  const void *ptrs[] = {qkv, q_weight, k_weight, cos, sin, q_out, k_out, v_out};
  for (const void *p : ptrs)
    if (p == nullptr || !aligned(p, 8))
      return fail(PIR2B_EALIGN, "qk_norm_rope operands must be non-null and 8-byte aligned");
  if (rows == 0)
    return PIR2B_OK;
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  QkRopeArgs a;
  a.qkv = static_cast<const __nv_bfloat16 *>(qkv);
  a.ld = ld;
  a.q_w = static_cast<const __nv_bfloat16 *>(q_weight);
  a.k_w = static_cast<const __nv_bfloat16 *>(k_weight);
  a.cos = static_cast<const __nv_bfloat16 *>(cos);
  a.sin = static_cast<const __nv_bfloat16 *>(sin);
  a.q_out = static_cast<__nv_bfloat16 *>(q_out);
  a.k_out = static_cast<__nv_bfloat16 *>(k_out);
  a.v_out = static_cast<__nv_bfloat16 *>(v_out);
  a.rows = int(rows);
  a.tokens = int(tokens);
  a.hq = hq;
  a.hk = hk;
  a.eps = eps;
  return cuda_status(run_qk_norm_rope(a, rows, static_cast<cudaStream_t>(stream)),
                     "qk_norm_rope launch");
}

int pir2b_attention_rows(const void *q, int64_t ldq, const void *k,
                         int64_t ldk, const void *v, int64_t ldv, void *out,
                         int64_t ldo, int64_t batch, int64_t tq, int64_t skv,
                         int heads, int head_dim, float scale, void *stream) {
  if (batch < 1 || tq < 1 || skv < 1 || heads < 1 ||
      !attention_head_dim_supported(head_dim) || skv > (int64_t(1) << 20) ||
      tq > (int64_t(1) << 30) || batch > 65535 || heads > 65535)
    return fail(PIR2B_EINVAL,
                "attention_rows: need batch, T, S >= 1 and head_dim in {32, 48, 64, 96, 128}");
  const int64_t width = int64_t(heads) * head_dim;
  if (ldq < width || ldk < width || ldv < width || ldo < width || ldq % 8 != 0 ||
      ldk % 8 != 0 || ldv % 8 != 0)
    return fail(PIR2B_EINVAL, "attention_rows: row strides too small or q/K/V strides not %% 8");
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr)
    return fail(PIR2B_EINVAL, "attention_rows operands must be non-null");
  if (!aligned(k, 16) || !aligned(v, 16) || !aligned(q, 16) || !aligned(out, 2))
    return fail(PIR2B_EALIGN, "attention_rows: q/K/V must be 16-byte aligned");
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  const int chunks = attention_chunks(int(skv));
  const int chunk = int((skv + chunks - 1) / chunks);
  if (attention_smem(chunk, head_dim, chunks) > size_t(dev->max_smem))
    return fail(PIR2B_EINVAL, "attention_rows: S too long for shared memory");
  AttnArgs a;
  a.q = static_cast<const __nv_bfloat16 *>(q);
  a.ldq = ldq;
  a.k = static_cast<const __nv_bfloat16 *>(k);
  a.ldk = ldk;
  a.v = static_cast<const __nv_bfloat16 *>(v);
  a.ldv = ldv;
  a.out = static_cast<__nv_bfloat16 *>(out);
  a.ldo = ldo;
  a.T = int(tq);
  a.S = int(skv);
  a.H = heads;
  a.D = head_dim;
  a.scale = scale;
  return cuda_status(run_attention_rows(a, int(batch), static_cast<cudaStream_t>(stream)),
                     "attention_rows launch");
}

int pir2b_unpack_int4(const void *packed, int64_t rows, int64_t k, void *out, void *stream) {
  if (rows < 1 || k < 32 || k % 32 != 0 || rows > (int64_t(1) << 31) || k > (int64_t(1) << 24))
    return fail(PIR2B_EINVAL, "unpack_int4 needs rows >= 1 and k a positive multiple of 32");
  if (packed == nullptr || out == nullptr)
    return fail(PIR2B_EINVAL, "unpack_int4 operands must be non-null");
  if (!aligned(packed, 16) || !aligned(out, 16))
    return fail(PIR2B_EALIGN, "unpack_int4 buffers must be 16-byte aligned");
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  return cuda_status(run_unpack_int4(packed, out, rows * k / 32, dev->sms,
                                     static_cast<cudaStream_t>(stream)),
                     "unpack_int4 launch");
}

int pir2b_attention_causal(const void *q, const void *k, const void *v, int64_t batch,
                           int64_t tokens, int hq, int hk, int head_dim, float scale, void *out,
                           int64_t ldo, void *stream) {
  if (batch < 1 || tokens < 1 || hq < 1 || hk < 1 || hq % hk != 0 || head_dim != kCausalD ||
      batch > 65535 || hq > 65535 || tokens > (int64_t(1) << 24))
    return fail(PIR2B_EINVAL,
                "attention_causal: need batch, T >= 1, hq a multiple of hk and head_dim 128");
  if (ldo < int64_t(hq) * head_dim)
    return fail(PIR2B_EINVAL, "attention_causal: ldo below hq * head_dim");
  if (q == nullptr || k == nullptr || v == nullptr || out == nullptr)
    return fail(PIR2B_EINVAL, "attention_causal operands must be non-null");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(out, 4) || ldo % 2 != 0)
    return fail(PIR2B_EALIGN, "attention_causal: q/k/v 16-byte, out 4-byte aligned, ldo even");
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  CausalArgs a;
  a.q = static_cast<const __nv_bfloat16 *>(q);
  a.k = static_cast<const __nv_bfloat16 *>(k);
  a.v = static_cast<const __nv_bfloat16 *>(v);
  a.out = static_cast<__nv_bfloat16 *>(out);
  a.ldo = ldo;
  a.T = int(tokens);
  a.hq = hq;
  a.hk = hk;
  a.scale = scale;
  return cuda_status(run_attention_causal(a, int(batch), static_cast<cudaStream_t>(stream)),
                     "attention_causal launch");
}

int pir2b_gemm_nvfp4(const void *qa, const void *sfa, const void *qw,
                     const void *sfw, const void *bias, float alpha,
                     int64_t m, int64_t n, int64_t k, void *out, int64_t ldo,
                     void *stream) {
  if (m < 1 || n < 1 || m > 0x7fffffffLL || n > 0x7fffffffLL)
    return fail(PIR2B_EINVAL, "NVFP4 GEMM needs m >= 1 and n >= 1");
  if (k < 256 || k % 256 != 0 || k > (1LL << 20))
    return fail(PIR2B_EINVAL,
                "NVFP4 GEMM needs k %% 256 == 0 (k=%lld): one K block is 256 "
                "E2M1 values with 16 UE4M3 factors per row",
                (long long)k);
  if (ldo < n)
    return fail(PIR2B_EINVAL, "ldo must be >= n");
  if (qa == nullptr || sfa == nullptr || qw == nullptr || sfw == nullptr ||
      out == nullptr)
    return fail(PIR2B_EINVAL, "NVFP4 GEMM operands must be non-null");
  const void *p16[] = {qa, sfa, qw, sfw};
  for (const void *p : p16)
    if (!aligned(p, 16))
      return fail(PIR2B_EALIGN, "NVFP4 operands and factors must be 16-byte aligned");
  if (!aligned(out, 2) || (bias && !aligned(bias, 2)))
    return fail(PIR2B_EALIGN, "output/bias alignment not met");
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  // Token tiles start on 128-row factor atoms: one tile of <= 128 tokens, or
  // tiles of 128.
  const int bn = m <= 128 ? int((m + 15) / 16 * 16) : 128;
  const int mtiles = int((m + 127) / 128);
  const size_t stage = size_t(kFp4WeightTile) + size_t(bn) * kFp4BlockBytes + 2 * kSfStageBytes;
  const int num_kb = int(k / 256);
  const int ntiles = int((n + 127) / 128);
  // One token tile: split K over a cluster (power of two up to 8, at least
  // one K block per rank) until about 96 CTAs stream the weights.
  int splits = 1;
  while (mtiles == 1 && splits < 8 && ntiles * splits < 96 && num_kb >= 2 * splits)
    splits *= 2;
  const int kb_per = (num_kb + splits - 1) / splits;
  int stages = splits > 1 ? std::max(2, std::min(8, kb_per)) : 8;
  auto smem_of = [&](int s) { return 1024 + s * stage + (2 * s + 1) * 8 + 16; };
  while (stages > 2 && smem_of(stages) > size_t(dev->max_smem))
    --stages;
  const uint64_t row_bytes = uint64_t(k / 2);
  CUtensorMap tm_w, tm_a, tm_out;
  memset(&tm_out, 0, sizeof(tm_out));
  if (int r = make_map(&tm_w, qw, row_bytes, uint64_t(n), row_bytes, 128u, 128u, true))
    return r;
  if (int r = make_map(&tm_a, qa, row_bytes, uint64_t(m), row_bytes, 128u, uint32_t(bn), true))
    return r;
  Fp4GemmArgs args;
  args.sfw = static_cast<const uint8_t *>(sfw);
  args.sfa = static_cast<const uint8_t *>(sfa);
  args.bias = static_cast<const __nv_bfloat16 *>(bias);
  args.out = static_cast<__nv_bfloat16 *>(out);
  args.ldo = ldo;
  args.m = int(m);
  args.n = int(n);
  args.num_kb = num_kb;
  args.blocks_k = int((k / 16 + 3) / 4);
  args.bn = bn;
  args.stages = stages;
  args.alpha = alpha;
  args.splits = splits;
  args.tma_store = (splits == 1 && ldo % 8 == 0 && aligned(out, 16)) ? 1 : 0;
  if (args.tma_store) {
    if (int r = make_out_map(&tm_out, out, uint64_t(n), uint64_t(m), uint64_t(ldo),
                             uint32_t(bn), 128u))
      return r;
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(unsigned(ntiles), unsigned(mtiles), unsigned(splits));
  cfg.blockDim = dim3(kFp4Threads, 1, 1);
  cfg.dynamicSmemBytes = smem_of(stages);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = unsigned(splits);
  cfg.attrs = attr;
  cfg.numAttrs = splits > 1 ? 2 : 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, gemm_fp4_kernel, tm_w, tm_a, tm_out, args),
                     "gemm_nvfp4 launch");
}

int pir2b_gemm_fused(const void *qa, const float *sa, const void *x, int64_t ldx, int64_t k,
                     const float *x_max, int64_t x_parts, const void *qw, const float *sw,
                     const void *bias, int bias_mode, const void *out_lut, const void *residual,
                     int64_t ldr, int bits, int64_t m, int64_t npad, int64_t kpad, void *out,
                     int64_t ldo, int64_t n_store, float *max_out, void *stream) {
  if (bits != 4 && bits != 8)
    return fail(PIR2B_EINVAL, "bits must be 4 or 8, got %d", bits);
  if (bias_mode < 0 || bias_mode > 2)
    return fail(PIR2B_EINVAL, "bias_mode must be 0, 1 or 2");
  if (m < 1 || m > 0x7fffffffLL || npad < 8 || npad % 8 != 0 || kpad < 128 ||
      kpad % 128 != 0 || npad > 0x7fffffffLL || kpad > (1LL << 20))
    return fail(PIR2B_EINVAL, "GEMM requires m >= 1, npad %% 8 == 0 and kpad %% 128 == 0");
  if (n_store < 1 || n_store > npad || ldo < n_store)
    return fail(PIR2B_EINVAL, "n_store must be in [1, npad] and ldo >= n_store");
  if ((qa == nullptr) == (x == nullptr))
    return fail(PIR2B_EINVAL, "gemm_fused takes packed activations (qa, sa) or bf16 rows x, not both");
  if (qw == nullptr || sw == nullptr || out == nullptr)
    return fail(PIR2B_EINVAL, "GEMM operands must be non-null");
  if (bias_mode == PIR2B_BIAS_ADD && bias == nullptr)
    return fail(PIR2B_EINVAL, "bias_mode ADD needs a bias vector");
  if (!aligned(qw, 16) || !aligned(out, 2) || !aligned(sw, 4) || (bias && !aligned(bias, 2)) ||
      (out_lut && !aligned(out_lut, 2)) || (residual && !aligned(residual, 2)))
    return fail(PIR2B_EALIGN, "weight/scale/bias/output alignment not met");
  if (residual != nullptr && ldr < n_store)
    return fail(PIR2B_EINVAL, "residual row stride ldr must be >= n_store");
  FusedInput fin;
  memset(&fin, 0, sizeof(fin));
  if (x != nullptr) {
    if (bits != 8 || m > 64)
      return fail(PIR2B_EINVAL, "the fused pack takes int8 weights and at most 64 token rows");
    if (k < 8 || k % 8 != 0 || (k + 127) / 128 * 128 != kpad || ldx < k || ldx % 8 != 0)
      return fail(PIR2B_EINVAL, "fused pack: need k %% 8 == 0, kpad = ceil(k/128)*128, ldx >= k, ldx %% 8 == 0");
    if (!aligned(x, 16))
      return fail(PIR2B_EALIGN, "fused pack: x must be 16-byte aligned");
    if (x_max != nullptr && (x_parts < 4 || x_parts % 4 != 0 || x_parts > (1 << 20) ||
                             !aligned(x_max, 16)))
      return fail(PIR2B_EINVAL, "fused pack: x_max needs x_parts %% 4 == 0 and 16-byte alignment");
    fin.x = x;
    fin.ldx = ldx;
    fin.k = k;
    fin.x_max = x_max;
    fin.x_parts = x_max != nullptr ? x_parts : 0;
  } else {
    if (sa == nullptr)
      return fail(PIR2B_EINVAL, "packed activations need their row scales");
    if (!aligned(qa, 16) || !aligned(sa, 4))
      return fail(PIR2B_EALIGN, "packed activations must be 16-byte aligned");
  }
  if (max_out != nullptr) {
    if (npad % 16 != 0 || !aligned(max_out, 4))
      return fail(PIR2B_EINVAL, "max_out needs npad %% 16 == 0 and a 4-byte aligned buffer");
    if (ldo % 8 != 0 || !aligned(out, 16))
      return fail(PIR2B_EINVAL, "max_out needs 16-byte aligned output rows (ldo %% 8 == 0)");
  }
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  GemmPlan plan;
  if (x != nullptr) {
    if (!plan_fused(m, int((npad + 127) / 128), int(kpad / 128), dev->max_smem, &fin, &plan))
      return fail(PIR2B_EINVAL, "fused pack: the rows do not fit one CTA's shared memory "
                                "(m=%lld k=%lld npad=%lld)", (long long)m, (long long)k,
                  (long long)npad);
  } else {
    if (use_few(bits, m))
      return launch_few(qa, sa, qw, sw, bias, bias_mode, out_lut, residual, ldr, bits, m, npad, kpad, out, ldo,
                        n_store, max_out, stream);
    plan = plan_gemm(bits, m, npad, kpad, dev->sms, dev->max_smem, tma_out(out, ldo));
    if (plan.smem == 0 || int64_t(plan.bn) * plan.mtiles < m || plan.stages < 2 ||
        plan.smem > size_t(dev->max_smem))
      return fail(PIR2B_EINVAL, "no GEMM tile plan fits m=%lld npad=%lld kpad=%lld",
                  (long long)m, (long long)npad, (long long)kpad);
  }
  return launch_gemm(plan, qa, sa, qw, sw, bias, bias_mode, out_lut, residual, ldr, nullptr, bits,
                     m, npad, kpad, out, ldo, n_store, stream, x != nullptr ? &fin : nullptr,
                     max_out);
}

int pir2b_quant_fp8(const void *x, int64_t ldx, int64_t rows, int64_t k, int fast, int weights,
                    void *q, float *scale, float *scale_rep, int64_t n_rep, void *stream) {
  if (rows < 1 || k < 8 || k % 8 != 0 || k > (1 << 20) || ldx < k || ldx % 8 != 0 ||
      rows > (int64_t(1) << 33) / k)
    return fail(PIR2B_EINVAL, "quant_fp8 needs rows >= 1, k %% 8 == 0 and ldx >= k, ldx %% 8 == 0");
  if (x == nullptr || q == nullptr || scale == nullptr || (n_rep > 0 && scale_rep == nullptr) ||
      n_rep < 0)
    return fail(PIR2B_EINVAL, "quant_fp8 operands must be non-null");
  if (!aligned(x, 16) || !aligned(q, 8) || !aligned(scale, 4) || (scale_rep && !aligned(scale_rep, 4)))
    return fail(PIR2B_EALIGN, "quant_fp8: x 16-byte, q 8-byte, scales 4-byte aligned");
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  Fp8QuantArgs a;
  a.x = static_cast<const __nv_bfloat16 *>(x);
  a.ldx = ldx;
  a.rows = rows;
  a.k = int(k);
  a.q = static_cast<uint8_t *>(q);
  a.scale = scale;
  a.scale_rep = n_rep > 0 ? scale_rep : nullptr;
  a.n_rep = n_rep;
  a.fast = fast ? 1 : 0;
  a.weights = weights ? 1 : 0;
  // About 32 K elements (4 chunks per thread) per CTA, at most a portable
  // cluster of 8 (and no more CTAs than rows).
  const int64_t want = (rows * k + 32767) / 32768;
  const int ranks = int(std::max<int64_t>(1, std::min<int64_t>(std::min<int64_t>(want, 8), rows)));
  return cuda_status(run_fp8_quant(a, ranks, static_cast<cudaStream_t>(stream)), "quant_fp8 launch");
}

int pir2b_gemm_fp8(const void *qa, const float *sa, const void *qw, const float *sw,
                   const void *bias, int bias_mode, const void *residual, int64_t ldr, int64_t m,
                   int64_t npad, int64_t kpad, void *out, int64_t ldo, int64_t n_store,
                   const void *out_lut, float *max_out, void *stream) {
  if (bias_mode < 0 || bias_mode > 2)
    return fail(PIR2B_EINVAL, "bias_mode must be 0, 1 or 2");
  if (m < 1 || m > 0x7fffffffLL || npad < 8 || npad % 8 != 0 || kpad < 128 ||
      kpad % 128 != 0 || npad > 0x7fffffffLL || kpad > (1LL << 20))
    return fail(PIR2B_EINVAL, "FP8 GEMM requires m >= 1, npad %% 8 == 0 and kpad %% 128 == 0");
  if (n_store < 1 || n_store > npad || ldo < n_store)
    return fail(PIR2B_EINVAL, "n_store must be in [1, npad] and ldo >= n_store");
  if (qa == nullptr || sa == nullptr || qw == nullptr || sw == nullptr || out == nullptr)
    return fail(PIR2B_EINVAL, "FP8 GEMM operands must be non-null");
  if (bias_mode == PIR2B_BIAS_ADD && bias == nullptr)
    return fail(PIR2B_EINVAL, "bias_mode ADD needs a bias vector");
  if (!aligned(qa, 16) || !aligned(qw, 16) || !aligned(out, 2) || !aligned(sa, 4) ||
      !aligned(sw, 4) || (bias && !aligned(bias, 2)) || (residual && !aligned(residual, 2)))
    return fail(PIR2B_EALIGN, "FP8 GEMM alignment not met");
  if (residual != nullptr && ldr < n_store)
    return fail(PIR2B_EINVAL, "residual row stride ldr must be >= n_store");
  if ((out_lut && !aligned(out_lut, 2)) || (max_out && !aligned(max_out, 4)))
    return fail(PIR2B_EALIGN, "FP8 GEMM alignment not met");
  if (max_out != nullptr && (!use_few(9, m) || npad % 16 != 0))
    return fail(PIR2B_EINVAL, "FP8 GEMM max_out needs m <= 32 token rows and npad %% 16 == 0");
  if (use_few(9, m))
    return launch_few(qa, sa, qw, sw, bias, bias_mode, out_lut, residual, ldr, 9, m, npad, kpad, out, ldo,
                      n_store, max_out, stream);
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  // E4M3 operands have the int8 byte layout: the same tile plans, 2-SM
  // tiles included (kind::f8f6f4 on cta_group::2).
  const GemmPlan plan = plan_gemm(8, m, npad, kpad, dev->sms, dev->max_smem, tma_out(out, ldo));
  if (plan.smem == 0 || int64_t(plan.bn) * plan.mtiles < m || plan.stages < 2 ||
      plan.smem > size_t(dev->max_smem))
    return fail(PIR2B_EINVAL, "no GEMM tile plan fits m=%lld npad=%lld kpad=%lld",
                (long long)m, (long long)npad, (long long)kpad);
  return launch_gemm(plan, qa, sa, qw, sw, bias, bias_mode, out_lut, residual, ldr, nullptr, 9, m,
                     npad, kpad, out, ldo, n_store, stream);
}

int pir2b_gemm_swiglu(const void *qa, const float *sa, const void *qw, const float *sw,
                      const void *bias, int bias_mode, const void *silu_lut, int64_t m,
                      int64_t half_n, int64_t kpad, void *out, int64_t ldo, float *max_out,
                      void *stream) {
  if (bias_mode < 0 || bias_mode > 2)
    return fail(PIR2B_EINVAL, "bias_mode must be 0, 1 or 2");
  if (m < 1 || m > 0x7fffffffLL || half_n < 128 || half_n % 128 != 0 ||
      half_n > (1LL << 28) || kpad < 128 || kpad % 128 != 0 || kpad > (1LL << 20))
    return fail(PIR2B_EINVAL,
                "SwiGLU GEMM requires m >= 1, half_n %% 128 == 0 and kpad %% 128 == 0");
  if (ldo < half_n)
    return fail(PIR2B_EINVAL, "ldo must be >= half_n");
  if (qa == nullptr || sa == nullptr || qw == nullptr || sw == nullptr || out == nullptr ||
      silu_lut == nullptr)
    return fail(PIR2B_EINVAL, "SwiGLU GEMM operands must be non-null");
  if (bias_mode == PIR2B_BIAS_ADD && bias == nullptr)
    return fail(PIR2B_EINVAL, "bias_mode ADD needs a bias vector");
  if (!aligned(qa, 16) || !aligned(qw, 16))
    return fail(PIR2B_EALIGN, "packed operands must be 16-byte aligned");
  if (!aligned(out, 2) || !aligned(sa, 4) || !aligned(sw, 4) || (bias && !aligned(bias, 2)) ||
      !aligned(silu_lut, 2) || (max_out && !aligned(max_out, 4)))
    return fail(PIR2B_EALIGN, "scale/bias/output alignment not met");
  // The maxima are taken from the staged output tile, written by TMA stores.
  if (max_out != nullptr && !tma_out(out, ldo))
    return fail(PIR2B_EINVAL, "max_out needs a 16-byte aligned output with ldo %% 8 == 0");
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  const GemmPlan plan = plan_gemm_wide(m, 2 * half_n, kpad, dev->sms, dev->max_smem, tma_out(out, ldo));
  if (plan.smem == 0 || int64_t(plan.bn) * plan.mtiles < m)
    return fail(PIR2B_EINVAL, "no SwiGLU tile plan fits m=%lld kpad=%lld", (long long)m,
                (long long)kpad);
  if (max_out != nullptr && plan.splits != 1)
    return fail(PIR2B_EINVAL, "internal: SwiGLU plan with split-K cannot write max_out");
  return launch_gemm(plan, qa, sa, qw, sw, bias, bias_mode, nullptr, nullptr, 0, silu_lut, 8, m,
                     2 * half_n, kpad, out, ldo, half_n, stream, nullptr, max_out);
}

// Workspace of pir2b_dit_ffn: [3 counters | pad to 256 B][row maxima f32
// [m, f/128]][row scales f32 [m]] padded to 256 B, then the int8 codes of h
// [m, f].
static int64_t ffn_workspace_layout(int64_t m, int64_t f, int64_t *max_off, int64_t *scale_off,
                                    int64_t *code_off) {
  *max_off = 256;
  *scale_off = *max_off + m * (f / 128) * 4;
  *code_off = ((*scale_off + m * 4 + 255) / 256) * 256;
  return *code_off + m * f;
}

int64_t pir2b_dit_ffn_workspace(int64_t m, int64_t f) {
  if (m < 1 || f < 128)
    return 0;
  int64_t a, b, c;
  return ffn_workspace_layout(m, f, &a, &b, &c);
}

int pir2b_dit_ffn(const void *qa, const float *sa, const void *up_w, const float *up_sw,
                  const void *up_bias, int up_bias_mode, const void *gelu_lut,
                  const void *down_w, const float *down_sw, const void *down_bias,
                  int down_bias_mode, const void *residual, int64_t ldr, int64_t m, int64_t d,
                  int64_t f, void *out, int64_t ldo, void *workspace, int64_t workspace_bytes,
                  void *stream) {
  if (m < 1 || m > 64 || d < 128 || d % 128 != 0 || d > 65536 || f < 1024 ||
      f % (128 * kFfnSplits) != 0 || f > 8192)
    return fail(PIR2B_EINVAL,
                "dit_ffn: need 1 <= m <= 64, d %% 128 == 0, f %% 1024 == 0 and f <= 8192");
  if (up_bias_mode < 0 || up_bias_mode > 2 || down_bias_mode < 0 || down_bias_mode > 2)
    return fail(PIR2B_EINVAL, "dit_ffn: bias modes must be 0, 1 or 2");
  if ((up_bias_mode == PIR2B_BIAS_ADD && up_bias == nullptr) ||
      (down_bias_mode == PIR2B_BIAS_ADD && down_bias == nullptr))
    return fail(PIR2B_EINVAL, "dit_ffn: bias mode ADD needs a bias vector");
  if (qa == nullptr || sa == nullptr || up_w == nullptr || up_sw == nullptr ||
      gelu_lut == nullptr || down_w == nullptr || down_sw == nullptr || residual == nullptr ||
      out == nullptr || workspace == nullptr)
    return fail(PIR2B_EINVAL, "dit_ffn operands must be non-null");
  if (ldr < d || ldo < d)
    return fail(PIR2B_EINVAL, "dit_ffn: row strides must be >= d");
  if (!aligned(qa, 16) || !aligned(up_w, 16) || !aligned(down_w, 16) ||
      !aligned(workspace, 256) || !aligned(out, 2) || !aligned(residual, 2))
    return fail(PIR2B_EALIGN, "dit_ffn: operand alignment not met");
  int64_t max_off, scale_off, code_off;
  if (workspace_bytes < ffn_workspace_layout(m, f, &max_off, &scale_off, &code_off))
    return fail(PIR2B_EINVAL, "dit_ffn: workspace too small");
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  const int bn = int((m + 15) / 16 * 16);
  const int up_ctas = int(f / 128);
  const int down_kb = int(f / 128 / kFfnSplits);
  const int ctas = up_ctas + int(d / 128) * kFfnSplits;
  if (ctas > dev->sms)
    return fail(PIR2B_EINVAL, "dit_ffn: %d CTAs do not fit the %d SMs at once", ctas, dev->sms);
  if (size_t(down_kb) * kWeightTileBytes < size_t(bn) * kTileN * 4)
    return fail(PIR2B_EINVAL, "dit_ffn: FFN width too small for the split-K partial tile");
  const int up_kb = int(d / 128);
  int up_stages = std::min(up_kb, 12);
  while (up_stages > 2 && ffn_up_smem(bn, up_stages) > size_t(dev->max_smem))
    --up_stages;
  const size_t smem = std::max(ffn_up_smem(bn, up_stages), ffn_down_smem(bn, down_kb));
  if (smem > size_t(dev->max_smem))
    return fail(PIR2B_EINVAL, "dit_ffn: shared memory plan does not fit");
  CUtensorMap tm_up, tm_act, tm_down;
  if (int r = make_map(&tm_up, up_w, uint64_t(d), uint64_t(f), uint64_t(d), 128u, 128u, true))
    return r;
  if (int r = make_map(&tm_act, qa, uint64_t(d), uint64_t(m), uint64_t(d), 128u, uint32_t(bn), true))
    return r;
  if (int r = make_map(&tm_down, down_w, uint64_t(f), uint64_t(d), uint64_t(f), 128u, 128u, true))
    return r;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  CUtensorMap tm_codes;
  if (int r = make_map(&tm_codes, ws + code_off, uint64_t(f), uint64_t(m), uint64_t(f), 128u,
                       uint32_t(bn), true))
    return r;
  FfnArgs a;
  a.sa = sa;
  a.sw_up = up_sw;
  a.bias_up = static_cast<const __nv_bfloat16 *>(up_bias);
  a.gelu_lut = static_cast<const __nv_bfloat16 *>(gelu_lut);
  a.sw_down = down_sw;
  a.bias_down = static_cast<const __nv_bfloat16 *>(down_bias);
  a.residual = static_cast<const __nv_bfloat16 *>(residual);
  a.ldr = ldr;
  a.out = static_cast<__nv_bfloat16 *>(out);
  a.ldo = ldo;
  a.codes = reinterpret_cast<int8_t *>(ws + code_off);
  a.scales = reinterpret_cast<float *>(ws + scale_off);
  a.row_max = reinterpret_cast<float *>(ws + max_off);
  a.counters = reinterpret_cast<unsigned *>(ws);
  a.m = int(m);
  a.d = int(d);
  a.f = int(f);
  a.bias_mode_up = up_bias_mode;
  a.bias_mode_down = down_bias_mode;
  a.bn = bn;
  a.up_ctas = up_ctas;
  a.up_kb = up_kb;
  a.up_stages = up_stages;
  a.down_kb = down_kb;
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(unsigned(ctas), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kFfnSplits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  // Up CTAs wait for every other up CTA (the row maxima), so all up clusters
  // must be resident together, and one down cluster beside them lets the
  // grid make progress while the rest queue.  Clusters of 8 are placed per
  // GPC, so the SM count alone does not show how many fit.
  int clusters = 0;
  cudaError_t oe = cudaOccupancyMaxActiveClusters(&clusters, dit_ffn_kernel, &cfg);
  if (oe != cudaSuccess)
    return cuda_status(oe, "dit_ffn cluster occupancy");
  const int up_clusters = up_ctas / kFfnSplits;
  if (clusters < up_clusters + 1)
    return fail(PIR2B_EINVAL,
                "dit_ffn: %d clusters of %d CTAs fit the device at once; this problem needs %d "
                "resident (all %d up clusters and one down cluster)",
                clusters, kFfnSplits, up_clusters + 1, up_clusters);
  return cuda_status(cudaLaunchKernelEx(&cfg, dit_ffn_kernel, tm_up, tm_act, tm_down, tm_codes, a),
                     "dit_ffn launch");
}

// pir2b_dit_ffn_static: the same launch with its scratch in a static
// device array instead of a caller workspace, for callers that allocate
// nothing.  Sized for the largest accepted problem (m = 64, f = 8192).
static_assert(sizeof(int64_t) == 8, "int64_t");
constexpr int64_t kFfnStaticM = 64, kFfnStaticF = 8192;
constexpr int64_t kFfnStaticBytes =
    ((256 + kFfnStaticM * (kFfnStaticF / 128) * 4 + kFfnStaticM * 4 + 255) / 256) * 256 +
    kFfnStaticM * kFfnStaticF;
__device__ __align__(256) uint8_t g_ffn_scratch[kFfnStaticBytes];

int pir2b_dit_ffn_static(const void *qa, const float *sa, const void *up_w, const float *up_sw,
                         const void *up_bias, int up_bias_mode, const void *gelu_lut,
                         const void *down_w, const float *down_sw, const void *down_bias,
                         int down_bias_mode, const void *residual, int64_t ldr, int64_t m,
                         int64_t d, int64_t f, void *out, int64_t ldo, void *stream) {
  if (m < 1 || m > kFfnStaticM || f < 1 || f > kFfnStaticF)
    return fail(PIR2B_EINVAL, "dit_ffn_static: need 1 <= m <= %lld and f <= %lld",
                (long long)kFfnStaticM, (long long)kFfnStaticF);
  int64_t max_off, scale_off, code_off;
  const int64_t need = ffn_workspace_layout(m, f, &max_off, &scale_off, &code_off);
  if (need > kFfnStaticBytes)
    return fail(PIR2B_EINVAL, "dit_ffn_static: problem exceeds the static scratch");
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  // Set-up, once per device on its first call (with that device current):
  // the array's address in this device's context.  In host code the symbol
  // itself is only a host-side stand-in, never a device address.
  void *scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (dev->ffn_scratch == nullptr) {
      void *p = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&p, g_ffn_scratch);
      if (e != cudaSuccess || p == nullptr)
        return cuda_status(e == cudaSuccess ? cudaErrorInvalidSymbol : e,
                           "dit_ffn_static scratch address");
      dev->ffn_scratch = p;
    }
    scratch = dev->ffn_scratch;
  }
  // The three counters must start at zero (a call that timed out may have
  // left them set); the rest of the scratch is written before it is read.
  cudaError_t e = cudaMemsetAsync(scratch, 0, 16, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return cuda_status(e, "dit_ffn_static counter reset");
  return pir2b_dit_ffn(qa, sa, up_w, up_sw, up_bias, up_bias_mode, gelu_lut, down_w, down_sw,
                       down_bias, down_bias_mode, residual, ldr, m, d, f, out, ldo, scratch,
                       kFfnStaticBytes, stream);
}

// Plan override for tests and the benchmark (not part of the public
// header's contract): 0 = the planner chooses, 1 = 2-SM tiles wherever they
// fit, 2 = never.  Returns the previous mode.
int pir2b_set_pair_mode(int mode) {
  if (mode < 0 || mode > 2)
    return fail(PIR2B_EINVAL, "pair mode must be 0, 1 or 2");
  return g_pair_mode.exchange(mode);
}

// Issue-rate probe of the int8 tensor cores (not part of the public
// header's contract; measurement): one CTA per SM issues iters x 4 MMAs of
// 128 x 256 x 32 back to back; cycles[sm] (device buffer of `ctas` int64)
// receives each CTA's SM clock cycles from first issue to completion.
int pir2b_int8_peak_probe(int iters, int ctas, long long *cycles, void *stream) {
  if (iters < 1 || ctas < 1 || cycles == nullptr || !aligned(cycles, 8))
    return fail(PIR2B_EINVAL, "peak probe needs iters >= 1, ctas >= 1 and an 8-byte aligned cycle buffer");
  DeviceInfo *dev = nullptr;
  if (int r = device_info(&dev))
    return r;
  const size_t smem = 1024 + kProbeA + kProbeB + 64;
  cudaError_t e = cudaFuncSetAttribute(mma_peak_probe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e == cudaSuccess) {
    mma_peak_probe_kernel<<<ctas, 128, smem, static_cast<cudaStream_t>(stream)>>>(iters, cycles);
    e = cudaGetLastError();
  }
  return cuda_status(e, "peak probe launch");
}

// Few-token kernel override for tests and measurement (not part of the
// public header's contract): 0 = the planner chooses, 1 = always for
// M <= 32, 2 = never.  Returns the previous mode.
int pir2b_set_few_mode(int mode) {
  if (mode < 0 || mode > 2)
    return fail(PIR2B_EINVAL, "few mode must be 0, 1 or 2");
  return g_few_mode.exchange(mode);
}

// Split-K override of the small-M (one token tile of <= 64 rows) plans for
// measurement (not part of the public header's contract): 0 = the planner
// chooses, 1/2/4/8 = that many K slices.  Returns the previous value.
int pir2b_set_small_m_splits(int splits) {
  if (splits != 0 && splits != 1 && splits != 2 && splits != 4 && splits != 8)
    return fail(PIR2B_EINVAL, "small-M splits must be 0, 1, 2, 4 or 8");
  return g_small_m_splits.exchange(splits);
}

// Plan introspection for tests and the benchmark (not part of the public
// header's contract; exported for diagnostics).
int pir2b_gemm_plan(int bits, int64_t m, int64_t npad, int64_t kpad,
                    int sms, int *bn, int *mtiles, int *splits, int *stages,
                    int64_t *smem, int *wt, int *pair) {
  // The plan of a call with a TMA-aligned output (2-SM tiles allowed).
  const GemmPlan p = plan_gemm(bits, m, npad, kpad, sms, 232448, true);
  *pair = p.pair;
  *wt = p.wt;
  *bn = p.bn;
  *mtiles = p.mtiles;
  *splits = p.splits;
  *stages = p.stages;
  *smem = int64_t(p.smem);
  return p.smem == 0 ? fail(PIR2B_EINVAL, "no GEMM tile plan") : PIR2B_OK;
}

} // extern "C"
