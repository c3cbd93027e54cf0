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

constexpr int kAttnThreads = 256;
constexpr int kAttnD = 128;       // head_dim supported by this kernel
constexpr int kAttnMaxGroup = 8;  // q heads per KV head (one warp each)
constexpr int kAttnTile = 32;     // positions per tile

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
  constexpr int D = kAttnD, PT = kAttnTile, KS = D + 8;
  __shared__ float sq[kAttnMaxGroup][D];
  __shared__ __align__(16) __half sk[PT][KS];
  __shared__ __align__(16) __half sv[PT][D];
  __shared__ __align__(16) __half knew[D];
  __shared__ __align__(16) __half vnew[D];
  __shared__ float sm[kAttnMaxGroup], sl[kAttnMaxGroup];
  __shared__ float so[kAttnMaxGroup][D];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x, kvh = blockIdx.y;
  const int G = p.Hq / p.Hkv;

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

  // q heads of this KV group: norm + RoPE, kept as fp32 copies of fp16 values.
  if (warp < G) {
    const __half* qsrc = p.qkv + (size_t)(kvh * G + warp) * D;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = h2f(qsrc[lane * 4 + e]);
    if (p.q_norm) head_rmsnorm(v, p.q_norm, lane, p.norm_eps);
    head_rope(v, rope_row, lane, p.rope_style);
#pragma unroll
    for (int e = 0; e < 4; ++e) sq[warp][lane * 4 + e] = v[e];
  }
  if (has_new && warp == kAttnMaxGroup - 2) {  // new k
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
  if (has_new && warp == kAttnMaxGroup - 1) {  // new v
    const __half* vsrc = p.qkv + (size_t)(p.Hq + p.Hkv) * D + (size_t)kvh * D;
    __half* vdst = p.v_cache + ((size_t)kvh * p.S_max + pos) * D;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      vnew[lane * 4 + e] = vsrc[lane * 4 + e];
      vdst[lane * 4 + e] = vsrc[lane * 4 + e];
    }
  }
  __syncthreads();
  grid_dep_launch_dependents();

  float m_run = -INFINITY, l_run = 0.f;
  float o[4] = {0.f, 0.f, 0.f, 0.f};
  const __half* kbase = p.k_cache + (size_t)kvh * p.S_max * D;
  const __half* vbase = p.v_cache + (size_t)kvh * p.S_max * D;

  for (int t0 = pb; t0 < pe; t0 += PT) {
    const int nt = min(PT, pe - t0);
    // Load the K and V tiles (16-byte pieces; the new token comes from smem).
    for (int c = tid; c < 2 * PT * (D / 8); c += kAttnThreads) {
      const int which = c / (PT * (D / 8));
      const int rem = c - which * PT * (D / 8);
      const int r = rem / (D / 8), q8 = rem % (D / 8);
      uint4 val = make_uint4(0u, 0u, 0u, 0u);
      if (r < nt) {
        const int tpos = t0 + r;
        if (tpos == pos) {
          val = *reinterpret_cast<const uint4*>((which ? vnew : knew) + q8 * 8);
        } else {
          const __half* src = (which ? vbase : kbase) + (size_t)tpos * D + q8 * 8;
          val = __ldg(reinterpret_cast<const uint4*>(src));
        }
      }
      if (which == 0)
        *reinterpret_cast<uint4*>(&sk[r][q8 * 8]) = val;
      else
        *reinterpret_cast<uint4*>(&sv[r][q8 * 8]) = val;
    }
    __syncthreads();
    if (warp < G) {
      float s = -INFINITY;
      if (lane < nt) {
        float d0 = 0.f, d1 = 0.f;
#pragma unroll 4
        for (int q8 = 0; q8 < D / 8; ++q8) {
          const uint4 kk = *reinterpret_cast<const uint4*>(&sk[lane][q8 * 8]);
          const float4 qa = *reinterpret_cast<const float4*>(&sq[warp][q8 * 8]);
          const float4 qb = *reinterpret_cast<const float4*>(&sq[warp][q8 * 8 + 4]);
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
      float mt = s;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float m_new = fmaxf(m_run, mt);
      const float corr = (m_run == -INFINITY) ? 0.f : expf(m_run - m_new);
      const float pe_ = (lane < nt) ? expf(s - m_new) : 0.f;
      l_run = l_run * corr + warp_reduce_sum(pe_);
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] *= corr;
      for (int j = 0; j < nt; ++j) {
        const float pj = __shfl_sync(0xffffffffu, pe_, j);
        const uint2 vv = *reinterpret_cast<const uint2*>(&sv[j][lane * 4]);
        const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(&vv.x));
        const float2 v1 = __half22float2(*reinterpret_cast<const __half2*>(&vv.y));
        o[0] = fmaf(pj, v0.x, o[0]);
        o[1] = fmaf(pj, v0.y, o[1]);
        o[2] = fmaf(pj, v1.x, o[2]);
        o[3] = fmaf(pj, v1.y, o[3]);
      }
      m_run = m_new;
    }
    __syncthreads();
  }

  if (warp < G) {
    if (lane == 0) {
      sm[warp] = m_run;
      sl[warp] = l_run;
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) so[warp][lane * 4 + e] = o[e];
  }

  if (p.splits > 1) {
    cluster_sync_all();
    if (split == 0) {
      for (int c = tid; c < G * D; c += kAttnThreads) {
        const int g = c / D, d = c - g * D;
        float M = -INFINITY;
        for (int r = 0; r < p.splits; ++r) M = fmaxf(M, r == 0 ? sm[g] : ld_dsmem_f32(&sm[g], (uint32_t)r));
        float Lsum = 0.f, O = 0.f;
        for (int r = 0; r < p.splits; ++r) {
          const float mr = r == 0 ? sm[g] : ld_dsmem_f32(&sm[g], (uint32_t)r);
          if (mr == -INFINITY) continue;
          const float lr = r == 0 ? sl[g] : ld_dsmem_f32(&sl[g], (uint32_t)r);
          const float orr = r == 0 ? so[g][d] : ld_dsmem_f32(&so[g][d], (uint32_t)r);
          const float f = expf(mr - M);
          Lsum = fmaf(lr, f, Lsum);
          O = fmaf(orr, f, O);
        }
        p.y[(size_t)(kvh * G + g) * D + d] = f2h(O / Lsum);
      }
    }
    cluster_sync_all();
  } else {
    __syncthreads();
    for (int c = tid; c < G * D; c += kAttnThreads) {
      const int g = c / D, d = c - g * D;
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
