// Small-query attention for the DiT action head, writing the rows the
// quantized output projection packs.
//
// piR2 runs the DiT attention through torch SDPA (coexecution/
// groot_pointwise.py:58-92) and then transposes its output back to
// [B, T, H*D] before the integer pack of to_out.  Here one kernel reads q, k
// and v straight from the projection outputs (row-major [rows, ld], head h at
// columns h*D..h*D+D-1), and writes the attention output as [B*T, H*D]
// rows: no transpose copy.
//
// The problem is tiny (17 queries, 17 or 544 keys, 32 heads of 48), far below
// one 128-row tcgen05 tile, and latency-bound, so the products run on
// warp-level bf16 MMAs (m16n8k16, fp32 accumulate) held in registers,
// flash-attention style:
//
// Grid (H, C, B) with a cluster of C CTAs along y when C > 1: CTA c owns keys
// [c*chunk, (c+1)*chunk) of head h and stages them (K and V, bf16, zero-
// padded to a multiple of 16 keys) plus a tile of up to 64 queries in shared
// memory with 16-byte asynchronous copies.  Each of the four warps takes 16
// queries: for every block of up to 64 keys it forms S = q.k (fp32),
// scales it, keeps a running row maximum m and sum l (online softmax),
// rounds P = exp(S - m) to bf16 and accumulates O += P.V.  With C = 1 the
// warp writes O / l.  With C > 1 the (m, l, O) partials stay in shared
// memory and, after a cluster barrier, rank r combines every C-th output
// element through distributed shared memory:
// out = sum_c e^(m_c - M) O_c / sum_c e^(m_c - M) l_c, M = max_c m_c.
// No mask (the DiT's context has no padding).  head_dim in {32, 48, 64, 96,
// 128}.
#pragma once
#include "args.cuh"
#include "ptx.cuh"

namespace pir2b {

struct AttnArgs {
  const __nv_bfloat16 *q;
  int64_t ldq;
  const __nv_bfloat16 *k;
  int64_t ldk;
  const __nv_bfloat16 *v;
  int64_t ldv;
  __nv_bfloat16 *out;
  int64_t ldo;
  int T, S, H, D;
  int chunk;          // keys per CTA
  float scale;
};

constexpr int kAttnThreads = 128;
constexpr int kAttnQTile = 64;   // queries per pass (16 per warp)
constexpr int kAttnKBlock = 64;  // keys per online-softmax step

// Shared-memory row pitch (elements) of staged q/K/V rows: an odd number of
// 16-byte units, so the eight row addresses of an ldmatrix phase fall on
// distinct bank groups.
__host__ __device__ constexpr int attn_pitch(int D) {
  return ((D / 8) & 1) ? D : D + 8;
}

__host__ __device__ inline int attn_chunk_pad(int chunk) { return (chunk + 15) / 16 * 16; }

__host__ __device__ inline size_t attention_smem(int chunk, int D, int clusters) {
  const size_t P = size_t(attn_pitch(D));
  const size_t kv = size_t(attn_chunk_pad(chunk)) * P * 2 * 2;
  const size_t qs = size_t(kAttnQTile) * P * 2;
  const size_t part = clusters > 1 ? size_t(kAttnQTile) * (size_t(D) + 2) * 4 : 0;
  return kv + qs + part;
}

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1,
                                        uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t &r0, uint32_t &r1,
                                              uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}

// D[16x8] += A[16x16] . B[16x8], bf16 inputs, fp32 accumulators.
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4],
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&v);
}

template <int D>
__global__ void __launch_bounds__(kAttnThreads) attention_rows_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  constexpr int P = attn_pitch(D);
  constexpr int KS = D / 16;           // k16 steps over the head dimension
  constexpr int DN = D / 8;            // n8 blocks over the head dimension
  constexpr int NB = kAttnKBlock / 8;  // n8 blocks per key block
  const int h = blockIdx.x;
  const int b = blockIdx.z;
  const int C = gridDim.y;
  const int c = blockIdx.y;            // == cluster rank (the cluster spans y)
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q4 = lane & 3;
  const int j0 = c * a.chunk;
  const int keys = max(0, min(a.chunk, a.S - j0));
  const int kpad = (keys + 15) / 16 * 16;
  const int cpad = attn_chunk_pad(a.chunk);
  __nv_bfloat16 *ks = reinterpret_cast<__nv_bfloat16 *>(smem_raw);
  __nv_bfloat16 *vs = ks + cpad * P;
  __nv_bfloat16 *qs = vs + cpad * P;                                  // [QTile][P]
  float *part = reinterpret_cast<float *>(qs + kAttnQTile * P);     // [QTile][D + 2]

  pdl_wait();
  pdl_launch_dependents();
  constexpr int vecs = D / 8;
  for (int i = tid; i < kpad * vecs; i += kAttnThreads) {
    const int j = i / vecs, d0 = (i % vecs) * 8;
    if (j < keys) {
      const int64_t row = int64_t(b) * a.S + j0 + j;
      cp_async_16(ks + j * P + d0, a.k + row * a.ldk + h * D + d0);
      cp_async_16(vs + j * P + d0, a.v + row * a.ldv + h * D + d0);
    } else {   // padding keys: zero (their probabilities are exactly 0)
      *reinterpret_cast<uint4 *>(ks + j * P + d0) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4 *>(vs + j * P + d0) = make_uint4(0, 0, 0, 0);
    }
  }
  const uint32_t ks_addr = smem_u32(ks), vs_addr = smem_u32(vs), qs_addr = smem_u32(qs);

  for (int t0 = 0; t0 < a.T; t0 += kAttnQTile) {
    const int tn = min(kAttnQTile, a.T - t0);
    const int64_t qbase = int64_t(b) * a.T + t0;
    for (int i = tid; i < kAttnQTile * vecs; i += kAttnThreads) {
      const int t = i / vecs, d0 = (i % vecs) * 8;
      if (t < tn)
        cp_async_16(qs + t * P + d0, a.q + (qbase + t) * a.ldq + h * D + d0);
      else
        *reinterpret_cast<uint4 *>(qs + t * P + d0) = make_uint4(0, 0, 0, 0);
    }
    cp_async_wait_all();
    __syncthreads();

    const int r0 = warp * 16;          // this warp's first query of the tile
    if (r0 < tn) {
      float o[DN][4];
#pragma unroll
      for (int n = 0; n < DN; ++n)
        o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
      float m_lo = -INFINITY, m_hi = -INFINITY;   // rows g and g + 8
      float l_lo = 0.f, l_hi = 0.f;               // this thread's partial row sums
      // q fragments for every k16 step of the head dimension.
      uint32_t qa[KS][4];
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        const int row = r0 + (lane & 15);
        const int col = s * 16 + (lane >> 4) * 8;
        ldsm_x4(qs_addr + uint32_t((row * P + col) * 2), qa[s][0], qa[s][1], qa[s][2], qa[s][3]);
      }
      for (int kb = 0; kb < kpad; kb += kAttnKBlock) {
        const int nbk = min(kAttnKBlock, kpad - kb) / 8;   // n8 key blocks (even)
        float s_acc[NB][4];
#pragma unroll
        for (int n = 0; n < NB; ++n) {
          s_acc[n][0] = s_acc[n][1] = s_acc[n][2] = s_acc[n][3] = 0.f;
          if (n < nbk) {
#pragma unroll
            for (int s = 0; s < KS; s += 2) {
              // K rows kb+n*8 .. +7, dims s*16 .. s*16+31: B fragments of
              // the k16 steps s and s + 1.
              uint32_t b0, b1, b2, b3;
              const int row = kb + n * 8 + (lane & 7);
              if (s + 1 < KS) {
                const int col = s * 16 + (lane >> 3) * 8;
                ldsm_x4(ks_addr + uint32_t((row * P + col) * 2), b0, b1, b2, b3);
                mma_bf16_16816(s_acc[n], qa[s], b0, b1);
                mma_bf16_16816(s_acc[n], qa[s + 1], b2, b3);
              } else {
                // Odd step count (D = 48): the last step alone.
                const int col = s * 16 + ((lane >> 3) & 1) * 8;
                ldsm_x4(ks_addr + uint32_t((row * P + col) * 2), b0, b1, b2, b3);
                mma_bf16_16816(s_acc[n], qa[s], b0, b1);
              }
            }
          }
        }
        // Scale, mask padding keys, running maxima of rows g and g + 8.
        float bm_lo = -INFINITY, bm_hi = -INFINITY;
#pragma unroll
        for (int n = 0; n < NB; ++n) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = kb + n * 8 + 2 * q4 + (e & 1);
            float v = s_acc[n][e] * a.scale;
            if (n >= nbk || key >= keys)
              v = -INFINITY;
            s_acc[n][e] = v;
          }
          bm_lo = fmaxf(bm_lo, fmaxf(s_acc[n][0], s_acc[n][1]));
          bm_hi = fmaxf(bm_hi, fmaxf(s_acc[n][2], s_acc[n][3]));
        }
        bm_lo = fmaxf(bm_lo, __shfl_xor_sync(0xffffffffu, bm_lo, 1));
        bm_lo = fmaxf(bm_lo, __shfl_xor_sync(0xffffffffu, bm_lo, 2));
        bm_hi = fmaxf(bm_hi, __shfl_xor_sync(0xffffffffu, bm_hi, 1));
        bm_hi = fmaxf(bm_hi, __shfl_xor_sync(0xffffffffu, bm_hi, 2));
        const float mn_lo = fmaxf(m_lo, bm_lo), mn_hi = fmaxf(m_hi, bm_hi);
        const float al_lo = m_lo == -INFINITY ? 0.f : expf(m_lo - mn_lo);
        const float al_hi = m_hi == -INFINITY ? 0.f : expf(m_hi - mn_hi);
        m_lo = mn_lo;
        m_hi = mn_hi;
        l_lo *= al_lo;
        l_hi *= al_hi;
#pragma unroll
        for (int n = 0; n < DN; ++n) {
          o[n][0] *= al_lo;
          o[n][1] *= al_lo;
          o[n][2] *= al_hi;
          o[n][3] *= al_hi;
        }
        // P = exp(S - m) as bf16 A fragments (two n8 key blocks per k16).
        uint32_t pa[NB / 2][4];
#pragma unroll
        for (int n = 0; n < NB; ++n) {
          const float p0 = expf(s_acc[n][0] - m_lo), p1 = expf(s_acc[n][1] - m_lo);
          const float p2 = expf(s_acc[n][2] - m_hi), p3 = expf(s_acc[n][3] - m_hi);
          l_lo += p0 + p1;
          l_hi += p2 + p3;
          pa[n / 2][(n & 1) * 2 + 0] = pack_bf16x2(p0, p1);
          pa[n / 2][(n & 1) * 2 + 1] = pack_bf16x2(p2, p3);
        }
        // O += P . V over the block's keys.
#pragma unroll
        for (int kk = 0; kk < NB / 2; ++kk) {
          if (2 * kk < nbk) {
            const int row = kb + kk * 16 + (lane & 15);
#pragma unroll
            for (int n = 0; n < DN; n += 2) {
              // V rows kk*16 .. +15 of the block, dims n*8 .. n*8+15.
              uint32_t b0, b1, b2, b3;
              if (n + 1 < DN) {
                const int col = n * 8 + (lane >> 4) * 8;
                ldsm_x4_trans(vs_addr + uint32_t((row * P + col) * 2), b0, b1, b2, b3);
                mma_bf16_16816(o[n], pa[kk], b0, b1);
                mma_bf16_16816(o[n + 1], pa[kk], b2, b3);
              } else {
                ldsm_x4_trans(vs_addr + uint32_t((row * P + n * 8) * 2), b0, b1, b2, b3);
                mma_bf16_16816(o[n], pa[kk], b0, b1);
              }
            }
          }
        }
      }
      l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
      l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
      l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
      l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
      const int t_lo = r0 + g, t_hi = r0 + g + 8;
      if (C > 1) {
#pragma unroll
        for (int n = 0; n < DN; ++n) {
          const int d = n * 8 + 2 * q4;
          part[t_lo * (D + 2) + 2 + d] = o[n][0];
          part[t_lo * (D + 2) + 3 + d] = o[n][1];
          part[t_hi * (D + 2) + 2 + d] = o[n][2];
          part[t_hi * (D + 2) + 3 + d] = o[n][3];
        }
        if (q4 == 0) {
          part[t_lo * (D + 2)] = m_lo;
          part[t_lo * (D + 2) + 1] = l_lo;
          part[t_hi * (D + 2)] = m_hi;
          part[t_hi * (D + 2) + 1] = l_hi;
        }
      } else {
        const float i_lo = 1.0f / l_lo, i_hi = 1.0f / l_hi;
#pragma unroll
        for (int n = 0; n < DN; ++n) {
          const int d = h * D + n * 8 + 2 * q4;
          if (t_lo < tn) {
            __nv_bfloat16 *dst = a.out + (qbase + t_lo) * a.ldo + d;
            dst[0] = __float2bfloat16_rn(o[n][0] * i_lo);
            dst[1] = __float2bfloat16_rn(o[n][1] * i_lo);
          }
          if (t_hi < tn) {
            __nv_bfloat16 *dst = a.out + (qbase + t_hi) * a.ldo + d;
            dst[0] = __float2bfloat16_rn(o[n][2] * i_hi);
            dst[1] = __float2bfloat16_rn(o[n][3] * i_hi);
          }
        }
      }
    }

    if (C > 1) {
      // Partials of this tile are complete in every CTA of the cluster.
      cluster_sync();
      const uint32_t part_base = smem_u32(part);
      for (int i = c * kAttnThreads + tid; i < tn * D; i += C * kAttnThreads) {
        const int t = i / D, d = i % D;
        const uint32_t row = part_base + uint32_t(t * (D + 2) * 4);
        float mc[8], lc[8], oc[8];
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          if (r < C) {
            const uint32_t peer = map_peer(row, uint32_t(r));
            mc[r] = ld_cluster_f32(peer);
            lc[r] = ld_cluster_f32(peer + 4);
            oc[r] = ld_cluster_f32(peer + uint32_t((2 + d) * 4));
          } else {
            mc[r] = -INFINITY;
            lc[r] = 0.f;
            oc[r] = 0.f;
          }
          M = fmaxf(M, mc[r]);
        }
        float L = 0.f, acc = 0.f;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const float w = mc[r] == -INFINITY ? 0.f : expf(mc[r] - M);   // empty chunk: weight 0
          L = fmaf(w, lc[r], L);
          acc = fmaf(w, oc[r], acc);
        }
        a.out[(qbase + t) * a.ldo + h * D + d] = __float2bfloat16_rn(acc / L);
      }
      // Peers are done reading this tile's partials before they are reused
      // (and before any CTA of the cluster exits).
      cluster_sync();
    } else {
      __syncthreads();
    }
  }
}

// ------------------------------------------------------------------
// Causal attention of the VLM text layers (head_dim 128, grouped-query):
// q [B, HQ, T, 128], k and v [B, HK, T, 128] (the layout of
// qk_norm_rope_kernel), output rows out[b*T + t, h*128 + d] for the o_proj
// pack, replacing torch SDPA (is_causal, enable_gqa) and its transpose copy.
// Grid (HQ, ceil(T / 64), B), eight warps per CTA: warp w takes queries
// 16*(w & 3) .. +16 of the CTA's 64 and the key blocks of parity w >> 2, so
// the two warp groups walk the causal key range side by side (half the
// serial path of the last query tile).  Pairs of 64-key blocks stream
// through a two-stage cp.async ring (the next pair in flight while the
// current one is used); each warp keeps the register-resident bf16 MMA +
// online softmax state of the row kernel, keys after the query masked, and
// the groups' states (m, l, O) are merged through shared memory at the end.
struct CausalArgs {
  const __nv_bfloat16 *q;
  const __nv_bfloat16 *k;
  const __nv_bfloat16 *v;
  __nv_bfloat16 *out;
  int64_t ldo;
  int T, hq, hk;
  float scale;
};

constexpr int kCausalD = 128;
constexpr int kCausalP = kCausalD + 8;           // odd number of 16-byte units
constexpr int kCausalThreads = 256;
constexpr int kCausalPair = 2 * kAttnKBlock;     // keys per ring stage

__host__ __device__ inline size_t attention_causal_smem() {
  // q tile + two stages of K and V for a pair of key blocks.
  return size_t(kAttnQTile) * kCausalP * 2 + size_t(2) * 2 * kCausalPair * kCausalP * 2;
}

__global__ void __launch_bounds__(kCausalThreads) attention_causal_kernel(const CausalArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  constexpr int D = kCausalD, P = kCausalP, KS = D / 16, DN = D / 8, NB = kAttnKBlock / 8;
  const int h = blockIdx.x, b = blockIdx.z;
  const int t0 = blockIdx.y * kAttnQTile;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q4 = lane & 3;
  const int qg = warp & 3, kg = warp >> 2;
  const int kvh = h / (a.hq / a.hk);
  __nv_bfloat16 *qs = reinterpret_cast<__nv_bfloat16 *>(smem_raw);   // [64][P]
  __nv_bfloat16 *kv = qs + kAttnQTile * P;                            // [2][K|V][128][P]
  const __nv_bfloat16 *qg_ptr = a.q + ((int64_t(b) * a.hq + h) * a.T) * D;
  const __nv_bfloat16 *kg_ptr = a.k + ((int64_t(b) * a.hk + kvh) * a.T) * D;
  const __nv_bfloat16 *vg_ptr = a.v + ((int64_t(b) * a.hk + kvh) * a.T) * D;
  constexpr int vecs = D / 8;
  const int tn = min(kAttnQTile, a.T - t0);
  const int nblocks = (min(a.T, t0 + kAttnQTile) + kAttnKBlock - 1) / kAttnKBlock;
  const int npairs = (nblocks + 1) / 2;

  pdl_wait();
  pdl_launch_dependents();
  for (int i = tid; i < kAttnQTile * vecs; i += kCausalThreads) {
    const int t = i / vecs, d0 = (i % vecs) * 8;
    if (t < tn)
      cp_async_16(qs + t * P + d0, qg_ptr + int64_t(t0 + t) * D + d0);
    else
      *reinterpret_cast<uint4 *>(qs + t * P + d0) = make_uint4(0, 0, 0, 0);
  }
  auto load_pair = [&](int pair, int stage) {
    __nv_bfloat16 *ks = kv + stage * 2 * kCausalPair * P;
    __nv_bfloat16 *vs = ks + kCausalPair * P;
    const int kend = min(a.T, nblocks * kAttnKBlock);   // keys any query here can see
    for (int i = tid; i < kCausalPair * vecs; i += kCausalThreads) {
      const int j = i / vecs, d0 = (i % vecs) * 8;
      const int key = pair * kCausalPair + j;
      if (key < kend) {
        cp_async_16(ks + j * P + d0, kg_ptr + int64_t(key) * D + d0);
        cp_async_16(vs + j * P + d0, vg_ptr + int64_t(key) * D + d0);
      } else {
        *reinterpret_cast<uint4 *>(ks + j * P + d0) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4 *>(vs + j * P + d0) = make_uint4(0, 0, 0, 0);
      }
    }
  };
  load_pair(0, 0);
  cp_async_commit();                               // group: q tile + pair 0

  const int r0 = qg * 16;
  const bool active = r0 < tn;
  float o[DN][4];
#pragma unroll
  for (int n = 0; n < DN; ++n)
    o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float m_lo = -INFINITY, m_hi = -INFINITY, l_lo = 0.f, l_hi = 0.f;
  uint32_t qa[KS][4];
  const int t_lo = t0 + r0 + g, t_hi = t_lo + 8;    // this thread's query rows
  for (int pr = 0; pr < npairs; ++pr) {
    if (pr + 1 < npairs) {
      load_pair(pr + 1, (pr + 1) & 1);
      cp_async_commit();
      cp_async_wait_group<1>();
    } else {
      cp_async_wait_group<0>();
    }
    __syncthreads();
    if (pr == 0 && active) {
#pragma unroll
      for (int s = 0; s < KS; ++s) {
        const int row = r0 + (lane & 15);
        const int col = s * 16 + (lane >> 4) * 8;
        ldsm_x4(smem_u32(qs) + uint32_t((row * P + col) * 2), qa[s][0], qa[s][1], qa[s][2], qa[s][3]);
      }
    }
    const int kb = 2 * pr + kg;
    // A block past the tile or after the warp's last query adds nothing.
    if (active && kb < nblocks && kb * kAttnKBlock <= t0 + r0 + 15) {
      const uint32_t ks_addr =
          smem_u32(kv + (pr & 1) * 2 * kCausalPair * P + kg * kAttnKBlock * P);
      const uint32_t vs_addr = ks_addr + uint32_t(kCausalPair * P * 2);
      float s_acc[NB][4];
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        s_acc[n][0] = s_acc[n][1] = s_acc[n][2] = s_acc[n][3] = 0.f;
#pragma unroll
        for (int s = 0; s < KS; s += 2) {
          uint32_t b0, b1, b2, b3;
          const int row = n * 8 + (lane & 7);
          const int col = s * 16 + (lane >> 3) * 8;
          ldsm_x4(ks_addr + uint32_t((row * P + col) * 2), b0, b1, b2, b3);
          mma_bf16_16816(s_acc[n], qa[s], b0, b1);
          mma_bf16_16816(s_acc[n], qa[s + 1], b2, b3);
        }
      }
      float bm_lo = -INFINITY, bm_hi = -INFINITY;
#pragma unroll
      for (int n = 0; n < NB; ++n) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int key = kb * kAttnKBlock + n * 8 + 2 * q4 + (e & 1);
          const int tq = e < 2 ? t_lo : t_hi;
          float v = s_acc[n][e] * a.scale;
          if (key > tq || key >= a.T)
            v = -INFINITY;
          s_acc[n][e] = v;
        }
        bm_lo = fmaxf(bm_lo, fmaxf(s_acc[n][0], s_acc[n][1]));
        bm_hi = fmaxf(bm_hi, fmaxf(s_acc[n][2], s_acc[n][3]));
      }
      bm_lo = fmaxf(bm_lo, __shfl_xor_sync(0xffffffffu, bm_lo, 1));
      bm_lo = fmaxf(bm_lo, __shfl_xor_sync(0xffffffffu, bm_lo, 2));
      bm_hi = fmaxf(bm_hi, __shfl_xor_sync(0xffffffffu, bm_hi, 1));
      bm_hi = fmaxf(bm_hi, __shfl_xor_sync(0xffffffffu, bm_hi, 2));
      const float mn_lo = fmaxf(m_lo, bm_lo), mn_hi = fmaxf(m_hi, bm_hi);
      // A row with every key so far masked keeps m = -inf and adds nothing;
      // the guards keep exp(-inf - -inf) out.
      const float al_lo = (m_lo == -INFINITY) ? 0.f : expf(m_lo - mn_lo);
      const float al_hi = (m_hi == -INFINITY) ? 0.f : expf(m_hi - mn_hi);
      m_lo = mn_lo;
      m_hi = mn_hi;
      l_lo *= al_lo;
      l_hi *= al_hi;
#pragma unroll
      for (int n = 0; n < DN; ++n) {
        o[n][0] *= al_lo;
        o[n][1] *= al_lo;
        o[n][2] *= al_hi;
        o[n][3] *= al_hi;
      }
      uint32_t pa[NB / 2][4];
#pragma unroll
      for (int n = 0; n < NB; ++n) {
        const float p0 = m_lo == -INFINITY ? 0.f : expf(s_acc[n][0] - m_lo);
        const float p1 = m_lo == -INFINITY ? 0.f : expf(s_acc[n][1] - m_lo);
        const float p2 = m_hi == -INFINITY ? 0.f : expf(s_acc[n][2] - m_hi);
        const float p3 = m_hi == -INFINITY ? 0.f : expf(s_acc[n][3] - m_hi);
        l_lo += p0 + p1;
        l_hi += p2 + p3;
        pa[n / 2][(n & 1) * 2 + 0] = pack_bf16x2(p0, p1);
        pa[n / 2][(n & 1) * 2 + 1] = pack_bf16x2(p2, p3);
      }
#pragma unroll
      for (int kk = 0; kk < NB / 2; ++kk) {
        const int row = kk * 16 + (lane & 15);
#pragma unroll
        for (int n = 0; n < DN; n += 2) {
          uint32_t b0, b1, b2, b3;
          const int col = n * 8 + (lane >> 4) * 8;
          ldsm_x4_trans(vs_addr + uint32_t((row * P + col) * 2), b0, b1, b2, b3);
          mma_bf16_16816(o[n], pa[kk], b0, b1);
          mma_bf16_16816(o[n + 1], pa[kk], b2, b3);
        }
      }
    }
    __syncthreads();   // this stage is refilled by the next iteration's prefetch
  }
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  // Merge: the odd-block warps leave (m, l, O) in the (now idle) K/V ring,
  // the even-block warps of the same queries fold them in and store.  Key 0
  // lies in block 0, so the even group's m is finite for every query.
  float *xo = reinterpret_cast<float *>(kv);                // [4][DN][4][32]
  float *xs = xo + 4 * DN * 4 * 32;                         // [4][4][32]: m_lo m_hi l_lo l_hi
  if (kg == 1 && active) {
#pragma unroll
    for (int n = 0; n < DN; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        xo[((qg * DN + n) * 4 + e) * 32 + lane] = o[n][e];
    xs[(qg * 4 + 0) * 32 + lane] = m_lo;
    xs[(qg * 4 + 1) * 32 + lane] = m_hi;
    xs[(qg * 4 + 2) * 32 + lane] = l_lo;
    xs[(qg * 4 + 3) * 32 + lane] = l_hi;
  }
  __syncthreads();
  if (kg == 1 || !active)
    return;
  const float m1_lo = xs[(qg * 4 + 0) * 32 + lane], m1_hi = xs[(qg * 4 + 1) * 32 + lane];
  const float l1_lo = xs[(qg * 4 + 2) * 32 + lane], l1_hi = xs[(qg * 4 + 3) * 32 + lane];
  const float mm_lo = fmaxf(m_lo, m1_lo), mm_hi = fmaxf(m_hi, m1_hi);
  const float a0_lo = expf(m_lo - mm_lo), a0_hi = expf(m_hi - mm_hi);
  const float a1_lo = m1_lo == -INFINITY ? 0.f : expf(m1_lo - mm_lo);
  const float a1_hi = m1_hi == -INFINITY ? 0.f : expf(m1_hi - mm_hi);
  const float i_lo = 1.0f / (l_lo * a0_lo + l1_lo * a1_lo);
  const float i_hi = 1.0f / (l_hi * a0_hi + l1_hi * a1_hi);
#pragma unroll
  for (int n = 0; n < DN; ++n) {
    const float *x = xo + ((qg * DN + n) * 4) * 32 + lane;
    const float v0 = (o[n][0] * a0_lo + x[0] * a1_lo) * i_lo;
    const float v1 = (o[n][1] * a0_lo + x[32] * a1_lo) * i_lo;
    const float v2 = (o[n][2] * a0_hi + x[64] * a1_hi) * i_hi;
    const float v3 = (o[n][3] * a0_hi + x[96] * a1_hi) * i_hi;
    const int d = h * D + n * 8 + 2 * q4;
    if (t_lo < a.T)
      *reinterpret_cast<uint32_t *>(a.out + (int64_t(b) * a.T + t_lo) * a.ldo + d) = pack_bf16x2(v0, v1);
    if (t_hi < a.T)
      *reinterpret_cast<uint32_t *>(a.out + (int64_t(b) * a.T + t_hi) * a.ldo + d) = pack_bf16x2(v2, v3);
  }
}

cudaError_t run_attention_causal(const CausalArgs &a, int B, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(a.hq), unsigned((a.T + kAttnQTile - 1) / kAttnQTile), unsigned(B));
  cfg.blockDim = dim3(kCausalThreads, 1, 1);
  cfg.dynamicSmemBytes = attention_causal_smem();
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attention_causal_kernel, a);
}

// Chunks per head: a power of two up to 8 keeping at least 64 keys per CTA,
// so every chunk is non-empty.
static int attention_chunks(int S) {
  int c = 1;
  while (c < 8 && S >= 64 * (2 * c))
    c *= 2;
  return c;
}

static bool attention_head_dim_supported(int D) {
  return D == 32 || D == 48 || D == 64 || D == 96 || D == 128;
}

template <int D>
static cudaError_t attention_set_smem(int bytes) {
  return cudaFuncSetAttribute(attention_rows_kernel<D>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

static cudaError_t attention_set_smem_all(int bytes) {
  cudaError_t e = cudaFuncSetAttribute(attention_causal_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) e = attention_set_smem<32>(bytes);
  if (e == cudaSuccess) e = attention_set_smem<48>(bytes);
  if (e == cudaSuccess) e = attention_set_smem<64>(bytes);
  if (e == cudaSuccess) e = attention_set_smem<96>(bytes);
  if (e == cudaSuccess) e = attention_set_smem<128>(bytes);
  return e;
}

cudaError_t run_attention_rows(AttnArgs a, int B, cudaStream_t st) {
  const int C = attention_chunks(a.S);
  a.chunk = (a.S + C - 1) / C;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(a.H), unsigned(C), unsigned(B));
  cfg.blockDim = dim3(kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = attention_smem(a.chunk, a.D, C);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 1;
  attr[1].val.clusterDim.y = unsigned(C);
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = C > 1 ? 2 : 1;      // no cluster launch for a single chunk
  switch (a.D) {
  case 32: return cudaLaunchKernelEx(&cfg, attention_rows_kernel<32>, a);
  case 48: return cudaLaunchKernelEx(&cfg, attention_rows_kernel<48>, a);
  case 64: return cudaLaunchKernelEx(&cfg, attention_rows_kernel<64>, a);
  case 96: return cudaLaunchKernelEx(&cfg, attention_rows_kernel<96>, a);
  default: return cudaLaunchKernelEx(&cfg, attention_rows_kernel<128>, a);
  }
}

} // namespace pir2b
