// Small-sequence attention for the DiT action head, writing the rows the
// quantized output projection packs.
//
// piR2 runs the DiT attention through torch SDPA (coexecution/
// groot_pointwise.py:58-92) and then transposes its output back to
// [B, T, H*D] before the integer pack of to_out.  Here one kernel reads q, k
// and v straight from the projection outputs (row-major [rows, ld], head h at
// columns h*D..h*D+D-1), and writes the attention output as [B*T, H*D]
// rows: no transpose copy, and the DiT block stays a chain of this library's
// kernels (programmatic dependent launch between them).
//
// Grid (H, C, B) with a cluster of C CTAs along y: CTA c of the cluster owns
// keys [c*chunk, (c+1)*chunk) of head h.  It copies its K and V rows into
// shared memory with 16-byte asynchronous copies (all in flight at once),
// then for each tile of up to 32 queries computes fp32 scores
// s_j = scale * q.k over the chunk, p_j = exp(s_j - m) with the chunk
// maximum m, l = sum p_j and o[d] = sum p_j v_j[d].  With C = 1 the CTA
// writes o / l.  With C > 1 the (m, l, o) partials stay in shared memory
// and, after a cluster barrier, rank r combines every C-th output element
// of the tile through distributed shared memory:
// out = sum_c e^(m_c - M) o_c / sum_c e^(m_c - M) l_c, M = max_c m_c.
// No mask (the DiT's context has no padding); D % 8 == 0, D <= 128.
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

constexpr int kAttnThreads = 256;
constexpr int kAttnQTile = 32;   // queries held in shared memory at a time

// Shared-memory row pitch (elements) of staged K/V rows: D rounded so the
// pitch is an odd number of 16-byte units, which keeps the 16-byte loads of
// eight consecutive keys (one per thread) on distinct bank groups.
__host__ __device__ inline int attn_pitch(int D) {
  return ((D / 8) & 1) ? D : D + 8;
}

// Score rows are padded to an odd number of words.
__host__ __device__ inline int attn_spitch(int chunk) { return chunk | 1; }

__host__ __device__ inline size_t attention_smem(int chunk, int D, int clusters) {
  const size_t kv = size_t(chunk) * attn_pitch(D) * 2 * 2;
  const size_t qs = size_t(kAttnQTile) * D * 4;
  const size_t sc = size_t(kAttnQTile) * attn_spitch(chunk) * 4;
  const size_t ml = size_t(kAttnQTile) * 2 * 4;
  const size_t part = clusters > 1 ? size_t(kAttnQTile) * D * 4 : 0;
  return kv + qs + sc + ml + part;
}

__device__ __forceinline__ void cp_async_16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}

__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Work is spread over all 256 threads in three phases per tile of up to 32
// queries, each with independent accumulators for instruction-level
// parallelism: scores (a thread owns one key and four queries), row
// softmax (a warp per query), and P.V (a thread owns one query and a pair
// of head dimensions).
__global__ void __launch_bounds__(kAttnThreads) attention_rows_kernel(const AttnArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int h = blockIdx.x;
  const int b = blockIdx.z;
  const int C = gridDim.y;
  const int c = blockIdx.y;                      // == cluster rank (cluster spans y)
  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int D = a.D, P = attn_pitch(D), SP = attn_spitch(a.chunk);
  const int j0 = c * a.chunk;
  const int keys = max(0, min(a.chunk, a.S - j0));
  __nv_bfloat16 *ks = reinterpret_cast<__nv_bfloat16 *>(smem_raw);
  __nv_bfloat16 *vs = ks + a.chunk * P;
  float *qs = reinterpret_cast<float *>(vs + a.chunk * P);   // [QTile][D]
  float *sc = qs + kAttnQTile * D;                           // [QTile][SP]
  float *ml = sc + kAttnQTile * SP;                          // [QTile][2]
  float *part = ml + kAttnQTile * 2;                         // [QTile][D]

  pdl_wait();
  pdl_launch_dependents();
  // K and V rows of this chunk: every 16-byte copy in flight before the wait.
  const int vecs = D / 8;
  for (int i = tid; i < keys * vecs; i += kAttnThreads) {
    const int j = i / vecs, d0 = (i % vecs) * 8;
    const int64_t row = int64_t(b) * a.S + j0 + j;
    cp_async_16(ks + j * P + d0, a.k + row * a.ldk + h * D + d0);
    cp_async_16(vs + j * P + d0, a.v + row * a.ldv + h * D + d0);
  }

  for (int t0 = 0; t0 < a.T; t0 += kAttnQTile) {
    const int tn = min(kAttnQTile, a.T - t0);
    const int64_t qbase = int64_t(b) * a.T + t0;
    for (int i = tid; i < tn * D; i += kAttnThreads) {
      const int t = i / D, d = i % D;
      qs[i] = __bfloat162float(a.q[(qbase + t) * a.ldq + h * D + d]) * a.scale;
    }
    cp_async_wait_all();
    __syncthreads();

    // Scores: item = (key j, group of four queries).
    const int groups = (tn + 3) / 4;
    for (int i = tid; i < keys * groups; i += kAttnThreads) {
      const int j = i % keys, t = (i / keys) * 4;
      const __nv_bfloat16 *kr = ks + j * P;
      const float *q0 = qs + t * D;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int d = 0; d < D; d += 8) {
        const uint4 raw = *reinterpret_cast<const uint4 *>(kr + d);
        const __nv_bfloat162 *k2 = reinterpret_cast<const __nv_bfloat162 *>(&raw);
        float kf[8];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(k2[e]);
          kf[2 * e] = f.x;
          kf[2 * e + 1] = f.y;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if (t + u < tn) {
            const float4 qa = *reinterpret_cast<const float4 *>(q0 + u * D + d);
            const float4 qb = *reinterpret_cast<const float4 *>(q0 + u * D + d + 4);
            acc[u] = fmaf(qa.x, kf[0], acc[u]);
            acc[u] = fmaf(qa.y, kf[1], acc[u]);
            acc[u] = fmaf(qa.z, kf[2], acc[u]);
            acc[u] = fmaf(qa.w, kf[3], acc[u]);
            acc[u] = fmaf(qb.x, kf[4], acc[u]);
            acc[u] = fmaf(qb.y, kf[5], acc[u]);
            acc[u] = fmaf(qb.z, kf[6], acc[u]);
            acc[u] = fmaf(qb.w, kf[7], acc[u]);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (t + u < tn)
          sc[(t + u) * SP + j] = acc[u];
    }
    __syncthreads();

    // Row softmax over this chunk's keys: a warp per query.
    for (int t = warp; t < tn; t += kAttnThreads / 32) {
      float *row = sc + t * SP;
      float m = -INFINITY;
      for (int j = lane; j < keys; j += 32)
        m = fmaxf(m, row[j]);
      for (int o = 16; o; o >>= 1)
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      float l = 0.f;
      for (int j = lane; j < keys; j += 32) {
        const float e = expf(row[j] - m);
        row[j] = e;
        l += e;
      }
      for (int o = 16; o; o >>= 1)
        l += __shfl_xor_sync(0xffffffffu, l, o);
      if (lane == 0) {
        ml[2 * t] = m;
        ml[2 * t + 1] = l;
      }
    }
    __syncthreads();

    // P.V: item = (query t, pair of head dimensions).
    const int pairs = D / 2;
    for (int i = tid; i < tn * pairs; i += kAttnThreads) {
      const int t = i / pairs, d = (i % pairs) * 2;
      const float *prow = sc + t * SP;
      float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
      int j = 0;
      for (; j + 1 < keys; j += 2) {
        const float2 va = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(vs + j * P + d));
        const float2 vb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(vs + (j + 1) * P + d));
        o0 = fmaf(prow[j], va.x, o0);
        o1 = fmaf(prow[j], va.y, o1);
        o2 = fmaf(prow[j + 1], vb.x, o2);
        o3 = fmaf(prow[j + 1], vb.y, o3);
      }
      if (j < keys) {
        const float2 va = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(vs + j * P + d));
        o0 = fmaf(prow[j], va.x, o0);
        o1 = fmaf(prow[j], va.y, o1);
      }
      o0 += o2;
      o1 += o3;
      if (C > 1) {
        part[t * D + d] = o0;
        part[t * D + d + 1] = o1;
      } else {
        const float inv = 1.0f / ml[2 * t + 1];
        __nv_bfloat16 *dst = a.out + (qbase + t) * a.ldo + h * D + d;
        dst[0] = __float2bfloat16_rn(o0 * inv);
        dst[1] = __float2bfloat16_rn(o1 * inv);
      }
    }

    if (C > 1) {
      // Partials of this tile are complete in every CTA of the cluster.
      cluster_sync();
      const uint32_t ml_base = smem_u32(ml), part_base = smem_u32(part);
      for (int i = c * kAttnThreads + tid; i < tn * D; i += C * kAttnThreads) {
        const int t = i / D;
        float mc[8], lc[8], oc[8];
        float M = -INFINITY;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          if (r < C) {
            mc[r] = ld_cluster_f32(map_peer(ml_base + uint32_t(8 * t), uint32_t(r)));
            lc[r] = ld_cluster_f32(map_peer(ml_base + uint32_t(8 * t + 4), uint32_t(r)));
            oc[r] = ld_cluster_f32(map_peer(part_base + uint32_t(4 * i), uint32_t(r)));
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
        a.out[(qbase + t) * a.ldo + h * D + (i % D)] = __float2bfloat16_rn(acc / L);
      }
      // Peers are done reading this tile's partials before they are reused
      // (and before any CTA of the cluster exits).
      cluster_sync();
    } else {
      __syncthreads();
    }
  }
}

// Chunks per head: a power of two up to 8 keeping at least 64 keys per CTA,
// so every chunk is non-empty.
static int attention_chunks(int S) {
  int c = 1;
  while (c < 8 && S >= 64 * (2 * c))
    c *= 2;
  return c;
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
  return cudaLaunchKernelEx(&cfg, attention_rows_kernel, a);
}

} // namespace pir2b
