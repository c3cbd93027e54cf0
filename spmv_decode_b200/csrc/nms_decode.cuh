// Decode-step kernels around the sparse GEMV: token embedding gather and
// single-token attention over a static KV cache.
//
// Attention semantics follow the reference decode step:
//   gpt-fast (model.py:215-245, apply_rotary_emb :310-322): RoPE on pairs
//     (2i, 2i+1) computed in fp32 from an fp16 cos/sin table, result cast to
//     fp16; KVCache.update (:114-123) writes k, v at input_pos; causal
//     attention with scale 1/sqrt(head_dim) and GQA.
//   HF Qwen3 (the reference's Qwen3 benchmarks): per-head RMSNorm on q and k
//     (q_norm / k_norm) before RoPE, RoPE on pairs (i, i + D/2)
//     ("rotate_half") computed with fp16 rounding after every elementwise op.
// One kernel does, for one KV head and one slice of the context: q/k norm,
// RoPE, the KV-cache append of the new token (last slice only), scores,
// an online softmax and P*V; the slices of a KV head form one thread-block
// cluster and are combined through distributed shared memory.
#pragma once

#include "nms_common.cuh"

namespace nms {

constexpr int kAttnThreads = 512;  // one (head, position) score and one (head, dim) output per thread at GQA 8
constexpr int kAttnD = 128;       // head_dim supported by this kernel
constexpr int kAttnMaxGroup = 8;  // q heads per KV head (one warp each)
constexpr int kAttnTile = 64;     // positions per tile (two per lane in the softmax)

enum RopeStyle : int32_t { kRopeInterleaved = 0, kRopeHalf = 1 };

struct AttnParams {
  const __half* qkv;    // [Hq*D | Hkv*D | Hkv*D]
  __half* k_cache;      // [Hkv][S_max][D]
  __half* v_cache;      // [Hkv][S_max][D]
  const __half* rope;   // [S_max][D/2][2] = (cos, sin)
  const __half* q_norm; // [D] or nullptr
  const __half* k_norm; // [D] or nullptr
  const int64_t* pos;   // device scalar: position of the new token
  __half* y;            // [Hq*D]
  float norm_eps;
  float scale;
  int32_t Hq, Hkv, S_max;
  int32_t rope_style;
  int32_t splits;       // CTAs per KV head (cluster size)
  const char* next_pf[2];  // weights of the next launch (see prefetch_shares_l2)
  uint32_t next_pf_bytes[2];
  uint32_t next_pf_head;
};

// RMSNorm over one head held as 4 values per lane of a warp (fp32 math,
// result rounded to fp16, then multiplied by the fp16 weight with fp16
// rounding -- the reference RMSNorm's order of roundings).
__device__ __forceinline__ void head_rmsnorm(float (&v)[4], const __half* wgt, int lane, float eps) {
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) ss = fmaf(v[e], v[e], ss);
  ss = warp_reduce_sum(ss);
  const float rstd = 1.0f / sqrtf(ss / (float)kAttnD + eps);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float nv = h2f(f2h(v[e] * rstd));
    v[e] = h2f(f2h(nv * h2f(wgt[lane * 4 + e])));
  }
}

// RoPE for one head held as 4 values per lane (dims 4*lane .. 4*lane+3).
__device__ __forceinline__ void head_rope(float (&v)[4], const __half* rope_row, int lane, int style) {
  if (style == kRopeInterleaved) {
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int i = (lane * 4 + e) >> 1;
      const float c = h2f(rope_row[2 * i]), s = h2f(rope_row[2 * i + 1]);
      const float x0 = v[e], x1 = v[e + 1];
      const float o0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
      const float o1 = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s));
      v[e] = h2f(f2h(o0));
      v[e + 1] = h2f(f2h(o1));
    }
  } else {
    // Partner dims are 64 apart: lane ^ 16 holds them.
    float other[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) other[e] = __shfl_xor_sync(0xffffffffu, v[e], 16);
    const bool lo = lane < 16;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = lane * 4 + e;
      const int i = lo ? d : d - kAttnD / 2;
      const float c = h2f(rope_row[2 * i]), s = h2f(rope_row[2 * i + 1]);
      const float t1 = h2f(f2h(v[e] * c));
      const float rot = lo ? -other[e] : other[e];
      const float t2 = h2f(f2h(rot * s));
      v[e] = h2f(f2h(t1 + t2));
    }
  }
}

__global__ void __launch_bounds__(kAttnThreads) attention_decode_kernel(const __grid_constant__ AttnParams p) {
  constexpr int D = kAttnD, PT = kAttnTile, KS = D + 8, GM = kAttnMaxGroup;
  constexpr int NT = kAttnThreads;
  __shared__ float sq[GM][D];                 // q heads (values exactly fp16), pre-scaled
  __shared__ __align__(16) __half sk[PT][KS];  // K tile (padded rows: conflict-free row reads)
  __shared__ __align__(16) __half sv[PT][D];   // V tile
  __shared__ float sp[GM][PT];                 // scores, then probabilities
  __shared__ __align__(16) __half knew[D];
  __shared__ __align__(16) __half vnew[D];
  __shared__ float sm[GM], sl[GM], scorr[GM];  // running max / sum / rescale per head
  __shared__ float so[GM][D];                  // running (unnormalised) output
  __shared__ float cm[16][GM], cl[16][GM];     // cluster combine: every rank's (m, l)

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x, kvh = blockIdx.y;
  const int G = p.Hq / p.Hkv;

  if (tid == 0) {
    const unsigned b = blockIdx.y * gridDim.x + blockIdx.x;
    prefetch_shares_l2(p.next_pf, p.next_pf_bytes, p.next_pf_head, b, gridDim.x * gridDim.y);
  }
  grid_dep_wait();
  const int64_t pos64 = *p.pos;
  if (pos64 < 0 || pos64 >= p.S_max) {  // uniform across the grid: every CTA reads the same value
    if (tid == 0) set_device_error(kDevBadPosition);
    return;
  }
  const int pos = (int)pos64;
  const int P = pos + 1;
  const int pb = (int)(((int64_t)split * P) / p.splits);
  const int pe = (int)(((int64_t)(split + 1) * P) / p.splits);
  const bool has_new = (split == p.splits - 1);
  const __half* rope_row = p.rope + (size_t)pos * D;

  // q heads of this KV group: norm + RoPE; the softmax scale is folded in.
  if (warp < G) {
    const __half* qsrc = p.qkv + (size_t)(kvh * G + warp) * D;
    float v[4];
    const uint2 qv = *reinterpret_cast<const uint2*>(qsrc + lane * 4);
    const float2 q0 = __half22float2(*reinterpret_cast<const __half2*>(&qv.x));
    const float2 q1 = __half22float2(*reinterpret_cast<const __half2*>(&qv.y));
    v[0] = q0.x; v[1] = q0.y; v[2] = q1.x; v[3] = q1.y;
    if (p.q_norm) head_rmsnorm(v, p.q_norm, lane, p.norm_eps);
    head_rope(v, rope_row, lane, p.rope_style);
#pragma unroll
    for (int e = 0; e < 4; ++e) sq[warp][lane * 4 + e] = v[e];
  }
  if (has_new && warp == GM - 2) {  // new k: norm + RoPE, append to the cache
    const __half* ksrc = p.qkv + (size_t)p.Hq * D + (size_t)kvh * D;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = h2f(ksrc[lane * 4 + e]);
    if (p.k_norm) head_rmsnorm(v, p.k_norm, lane, p.norm_eps);
    head_rope(v, rope_row, lane, p.rope_style);
    __half* kdst = p.k_cache + ((size_t)kvh * p.S_max + pos) * D;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      knew[lane * 4 + e] = f2h(v[e]);
      kdst[lane * 4 + e] = f2h(v[e]);
    }
  }
  if (has_new && warp == GM - 1) {  // new v: append to the cache
    const __half* vsrc = p.qkv + (size_t)(p.Hq + p.Hkv) * D + (size_t)kvh * D;
    __half* vdst = p.v_cache + ((size_t)kvh * p.S_max + pos) * D;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      vnew[lane * 4 + e] = vsrc[lane * 4 + e];
      vdst[lane * 4 + e] = vsrc[lane * 4 + e];
    }
  }
  for (int i = tid; i < GM * D; i += NT) (&so[0][0])[i] = 0.f;
  if (tid < GM) {
    sm[tid] = -INFINITY;
    sl[tid] = 0.f;
  }
  __syncthreads();
  grid_dep_launch_dependents();

  const __half* kbase = p.k_cache + (size_t)kvh * p.S_max * D;
  const __half* vbase = p.v_cache + (size_t)kvh * p.S_max * D;
  for (int t0 = pb; t0 < pe; t0 += PT) {
    const int nt = min(PT, pe - t0);
    // (a) K and V tiles in one batch of independent 16-byte loads.
    constexpr int PIECES = 2 * PT * (D / 8);
#pragma unroll
    for (int it = 0; it < PIECES / NT; ++it) {
      const int c = tid + it * NT;
      const int which = c / (PT * (D / 8));
      const int rem = c - which * PT * (D / 8);
      const int r = rem / (D / 8), q8 = rem % (D / 8);
      uint4 val = make_uint4(0u, 0u, 0u, 0u);
      if (r < nt) {
        const int tpos = t0 + r;
        if (tpos == pos) {
          val = *reinterpret_cast<const uint4*>((which ? vnew : knew) + q8 * 8);
        } else {
          val = __ldg(reinterpret_cast<const uint4*>((which ? vbase : kbase) + (size_t)tpos * D + q8 * 8));
        }
      }
      if (which == 0)
        *reinterpret_cast<uint4*>(&sk[r][q8 * 8]) = val;
      else
        *reinterpret_cast<uint4*>(&sv[r][q8 * 8]) = val;
    }
    __syncthreads();
    // (b) scores: one (head, position) pair per thread.
    for (int i = tid; i < G * PT; i += NT) {
      const int g = i / PT, r = i % PT;
      float s = -INFINITY;
      if (r < nt) {
        float d0 = 0.f, d1 = 0.f;
#pragma unroll
        for (int q8 = 0; q8 < D / 8; ++q8) {
          const uint4 kk = *reinterpret_cast<const uint4*>(&sk[r][q8 * 8]);
          const float4 qa = *reinterpret_cast<const float4*>(&sq[g][q8 * 8]);
          const float4 qb = *reinterpret_cast<const float4*>(&sq[g][q8 * 8 + 4]);
          const float2 k0 = __half22float2(*reinterpret_cast<const __half2*>(&kk.x));
          const float2 k1 = __half22float2(*reinterpret_cast<const __half2*>(&kk.y));
          const float2 k2 = __half22float2(*reinterpret_cast<const __half2*>(&kk.z));
          const float2 k3 = __half22float2(*reinterpret_cast<const __half2*>(&kk.w));
          d0 = fmaf(qa.x, k0.x, d0);
          d1 = fmaf(qa.y, k0.y, d1);
          d0 = fmaf(qa.z, k1.x, d0);
          d1 = fmaf(qa.w, k1.y, d1);
          d0 = fmaf(qb.x, k2.x, d0);
          d1 = fmaf(qb.y, k2.y, d1);
          d0 = fmaf(qb.z, k3.x, d0);
          d1 = fmaf(qb.w, k3.y, d1);
        }
        s = (d0 + d1) * p.scale;
      }
      sp[g][r] = s;
    }
    __syncthreads();
    // (c) online softmax statistics: one warp per head.
    if (warp < G) {
      static_assert(PT == 64, "two positions per lane");
      const float s0 = sp[warp][lane], s1 = sp[warp][lane + 32];
      float mt = fmaxf(s0, s1);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float m_old = sm[warp];
      const float m_new = fmaxf(m_old, mt);
      const float p0 = (lane < nt) ? expf(s0 - m_new) : 0.f;
      const float p1 = (lane + 32 < nt) ? expf(s1 - m_new) : 0.f;
      const float tot = warp_reduce_sum(p0 + p1);
      sp[warp][lane] = p0;
      sp[warp][lane + 32] = p1;
      if (lane == 0) {
        const float corr = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
        scorr[warp] = corr;
        sl[warp] = sl[warp] * corr + tot;
        sm[warp] = m_new;
      }
    }
    __syncthreads();
    // (d) P*V: (head, dim) pairs spread over the CTA; four independent FMA
    //     chains over the tile's positions (a single chain made this loop,
    //     not the loads, grow the kernel with the context).
    for (int i = tid; i < G * D; i += NT) {
      const int g = i / D, d = i - g * D;
      float a0 = so[g][d] * scorr[g], a1 = 0.f, a2 = 0.f, a3 = 0.f;
      int r = 0;
      for (; r + 3 < nt; r += 4) {
        a0 = fmaf(sp[g][r], h2f(sv[r][d]), a0);
        a1 = fmaf(sp[g][r + 1], h2f(sv[r + 1][d]), a1);
        a2 = fmaf(sp[g][r + 2], h2f(sv[r + 2][d]), a2);
        a3 = fmaf(sp[g][r + 3], h2f(sv[r + 3][d]), a3);
      }
      for (; r < nt; ++r) a0 = fmaf(sp[g][r], h2f(sv[r][d]), a0);
      so[g][d] = (a0 + a1) + (a2 + a3);
    }
    __syncthreads();
  }

  // Cluster combine, distributed: rank r finalises dims [r*D/splits, ...).
  if (p.splits > 1) {
    cluster_sync_all();
    for (int i = tid; i < p.splits * G; i += NT) {
      const int r = i / G, g = i - r * G;
      cm[r][g] = (r == split) ? sm[g] : ld_dsmem_f32(&sm[g], (uint32_t)r);
      cl[r][g] = (r == split) ? sl[g] : ld_dsmem_f32(&sl[g], (uint32_t)r);
    }
    __syncthreads();
    const int dpr = (D + p.splits - 1) / p.splits;
    const int d0 = split * dpr, d1 = min(D, d0 + dpr);
    const int nd = max(0, d1 - d0);
    for (int i = tid; i < G * nd; i += NT) {
      const int g = i / nd, d = d0 + (i - g * nd);
      float M = -INFINITY;
      for (int r = 0; r < p.splits; ++r) M = fmaxf(M, cm[r][g]);
      float Lsum = 0.f, O = 0.f;
      for (int r = 0; r < p.splits; ++r) {
        if (cm[r][g] == -INFINITY) continue;
        const float f = expf(cm[r][g] - M);
        const float orr = (r == split) ? so[g][d] : ld_dsmem_f32(&so[g][d], (uint32_t)r);
        Lsum = fmaf(cl[r][g], f, Lsum);
        O = fmaf(orr, f, O);
      }
      p.y[(size_t)(kvh * G + g) * D + d] = f2h(O / Lsum);
    }
    cluster_sync_all();  // keep every rank's shared memory alive until all reads are done
  } else {
    for (int i = tid; i < G * D; i += NT) {
      const int g = i / D, d = i - g * D;
      p.y[(size_t)(kvh * G + g) * D + d] = f2h(so[g][d] / sl[g]);
    }
  }
}

// x[i] = table[token * K + i]; the token id is read on the device.
__global__ void embedding_kernel(const __half* __restrict__ table, const int64_t* __restrict__ token,
                                 __half* __restrict__ x, int K, int64_t vocab) {
  grid_dep_wait();
  int64_t t = *token;
  if (t < 0 || t >= vocab) t = 0;  // out-of-range ids read row 0 (host validates ids it supplies)
  const __half* row = table + (size_t)t * K;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < K; i += gridDim.x * blockDim.x) x[i] = row[i];
  grid_dep_launch_dependents();
}

}  // namespace nms
