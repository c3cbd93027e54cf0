// Persistent decode step: every stage of one decode step (per layer: q/k/v
// GEMV, attention, o-projection, gate/up + SwiGLU, down-projection; then the
// output head with greedy argmax) runs inside ONE cooperative launch of one
// 1024-thread CTA per SM.
//
// Why: a batch-1 decode step is ~160 small HBM-bound launches.  Each launch
// pays a fixed cost (CTA start-up, the first loads' latency, the prologue,
// the tail) of several microseconds during which HBM idles.  Inside one
// persistent kernel the stages are separated by grid barriers instead, and
// before a CTA waits at a barrier it already issues the next GEMV stage's
// first weight loads (weights never depend on activations) and stages that
// stage's mask offsets, so the memory system keeps streaming through the
// barrier.
//
// Grid barrier: arrival counter + generation word in global memory (reset
// by the last arriver, generation monotonic across launches); waits are
// bounded by %globaltimer and record kDevBarrierTimeout instead of hanging.
// Attention: one (KV head, context split) unit per CTA; the last unit of a
// head to finish (per-head arrival counter) combines the splits' partial
// softmax states from L2.
#pragma once

#include "nms_common.cuh"
#include "nms_decode.cuh"
#include "nms_gemv.cuh"

namespace nms {

constexpr int kStepThreads = 1024;
constexpr int kStepWarps = kStepThreads / kWarp;
constexpr int kStepU = 4;  // register ring depth (32-byte loads per lane)
constexpr uint64_t kBarrierLimitNs = 200ull * 1000 * 1000;
constexpr int kMaxSplits = 16;  // attention splits per KV head (cluster-size bound of the standalone kernel)

enum StageKind : int32_t { kStageGemv = 0, kStageAttn = 1 };

struct StepStage {
  int32_t kind;
  int32_t units;  // attention: KV heads x splits
  int32_t lanes;  // GEMV: lanes per packed row (32, 16, 8 or 4)
  int32_t pad_;
  GemvParams g;
  AttnParams a;
};

struct StepParams {
  const StepStage* stages;  // device array
  int32_t nstages;
  unsigned* bar_count;      // grid barrier arrivals (grows within a launch, reset at exit)
  unsigned* bar_exit;       // CTAs that have left the kernel (reset at exit)
  float* attn_part;         // [units][kAttnMaxGroup][kAttnD + 2] partial softmax states
  unsigned* attn_count;     // [Hkv] per-head arrival counters (return to 0)
  // Optional timeline (%globaltimer ns): trace[0] = kernel start (CTA 0);
  // trace[1 + s*(ncta+1) + c] = time CTA c finished stage s's work;
  // trace[1 + s*(ncta+1) + ncta] = time CTA 0 left the barrier after stage s.
  unsigned long long* trace;
};

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_add_u32(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid barrier number `k` (0, 1, 2, ... within one launch), split in an
// arrive and a wait so a CTA can issue the next stage's weight loads in
// between (they may stall on a full memory system; the arrival does not wait
// for them).  The arrival counter only grows during a launch, so barrier k
// completes when it reaches ncta*(k+1): arriving is one fire-and-forget
// release reduction, waiting is acquire polling.  The counter is reset to
// zero by the last CTA to leave the kernel (step_exit).
__device__ __forceinline__ void grid_arrive(unsigned* count) {
  __syncthreads();
  if (threadIdx.x == 0) red_release_add_u32(count, 1u);
}

// Returns false (uniformly per CTA) when the wait ran past its limit
// (kDevBarrierTimeout recorded).
__device__ __forceinline__ bool grid_wait(const unsigned* count, unsigned ncta, unsigned k) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned target = ncta * (k + 1);
    if (ld_acquire_u32(count) < target) {
      const uint64_t t0 = global_timer_ns();
      while (ld_acquire_u32(count) < target) {
        if (global_timer_ns() - t0 > kBarrierLimitNs) {
          set_device_error(kDevBarrierTimeout);
          ok = 0;
          break;
        }
      }
    }
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

// Called once by every CTA as it leaves: the last one resets the barrier
// counter (no CTA of this launch reads it any more).
__device__ __forceinline__ void step_exit(unsigned* count, unsigned* exit_count, unsigned ncta) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(exit_count, 1u);
    if (prev == ncta - 1) {
      atomicExch(count, 0u);
      atomicExch(exit_count, 0u);
    }
  }
}

__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit_wait_all() {
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory");
}

// ---------------------------------------------------------------------------
// GEMV stage, split in the part that may run before the barrier (weights and
// masks only) and the part after it.
// ---------------------------------------------------------------------------
struct StepGemvSmem {
  __half* xs;
  uint8_t* sidx;
  __half* xc;
  float* acc;
  float* red;
};

__device__ __forceinline__ StepGemvSmem step_gemv_smem(const GemvParams& p, unsigned char* base, int max_vrows,
                                                       int nsegx) {
  StepGemvSmem s;
  size_t off = 0;
  s.xs = reinterpret_cast<__half*>(base + off);
  off += align_up_sz((size_t)p.K * 2, 16);
  s.sidx = base + off;
  off += align_up_sz((size_t)p.w, 16) * nsegx;
  s.xc = reinterpret_cast<__half*>(base + off);
  off += align_up_sz((size_t)p.w_pad * 2 * nsegx, 16);
  s.acc = reinterpret_cast<float*>(base + off);
  off += align_up_sz((size_t)max_vrows * 4, 16);
  s.red = reinterpret_cast<float*>(base + off);
  return s;
}

struct GemvGeom {
  int g0, ng, vgroups, cpr, t0, t1, max_vrows, nsegx;
  bool paired, dense;
};

template <int L>
__device__ __forceinline__ GemvGeom gemv_geom(const GemvParams& p, unsigned cta, unsigned ncta) {
  constexpr int RG = kWarp / L;
  GemvGeom q;
  q.paired = (p.mode == kModePaired);
  q.nsegx = q.paired ? 2 : p.nseg;
  q.dense = (p.seg[0].idx == nullptr);
  q.g0 = (int)(((int64_t)cta * p.row_groups) / ncta);
  const int g1 = (int)(((int64_t)(cta + 1) * p.row_groups) / ncta);
  q.ng = g1 - q.g0;
  q.vgroups = q.paired ? 2 * q.ng : q.ng;
  q.max_vrows = (q.paired ? 2 : 1) * ((p.row_groups + ncta - 1) / ncta) * RG;
  q.cpr = p.w_pad / (16 * L);
  const int T = q.vgroups * q.cpr;
  const int warp = threadIdx.x >> 5;
  q.t0 = (int)(((int64_t)warp * T) / kStepWarps);
  q.t1 = (int)(((int64_t)(warp + 1) * T) / kStepWarps);
  return q;
}

// This CTA's rows of a GEMV stage (every segment) into L2, in bulk prefetches
// issued by one thread -- used while the grid runs a latency-bound stage.
template <int L>
__device__ __forceinline__ void gemv_l2_prefetch_own(const GemvParams& p, const GemvGeom& q) {
  constexpr int RG = kWarp / L;
  if (threadIdx.x != 0 || q.ng <= 0) return;
  const int r0 = q.g0 * RG;
  const int r1 = min((q.g0 + q.ng) * RG, p.rows_total);
  for (int sx = 0; sx < p.nseg; ++sx) {
    int a = r0, b = r1;
    if (!q.paired) {
      a = max(r0, p.seg[sx].row_start) - p.seg[sx].row_start;
      b = min(r1, p.seg[sx].row_start + p.seg[sx].rows) - p.seg[sx].row_start;
    }
    if (a >= b) continue;
    const char* base = reinterpret_cast<const char*>(p.seg[sx].w + (size_t)a * p.w_pad);
    const size_t bytes = (size_t)(b - a) * p.w_pad * 2;
    for (size_t o = 0; o < bytes; o += 65536) {
      const size_t n = bytes - o < 65536 ? bytes - o : 65536;
      bulk_prefetch_l2(base + o, (uint32_t)n);
    }
  }
}

// Pre-barrier: the first kStepU loads of this warp into the register ring and
// the mask offsets into shared memory (plain 16-byte loads).
template <int L>
__device__ __forceinline__ void gemv_pre(const GemvParams& p, const GemvGeom& q, unsigned char* smem_base,
                                         U32x8 (&buf)[kStepU]) {
  constexpr int RG = kWarp / L, CH = 16 * L;
  const int lane = threadIdx.x & 31, sub = lane / L, li = lane % L;
  int vg = q.t0 / q.cpr, c = q.t0 - vg * q.cpr;
  LaneRow r = lane_row(p, q.paired, q.g0, q.ng, vg, RG, sub);
#pragma unroll
  for (int u = 0; u < kStepU; ++u) {
    // Every slot is written (zeros past the range) so the ring carries no
    // value across stages that do not refill it.
    if (q.t0 + u < q.t1 && r.valid) {
      buf[u] = ld_stream_256(p.seg[r.segi].w + (size_t)r.lrow * p.w_pad + li * 16 + (size_t)c * CH);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) buf[u].v[e] = 0u;
    }
    if (q.t0 + u < q.t1) {
      if (++c == q.cpr) {
        c = 0;
        ++vg;
        r = lane_row(p, q.paired, q.g0, q.ng, vg, RG, sub);
      }
    }
  }
  if (!q.dense) {
    StepGemvSmem s = step_gemv_smem(p, smem_base, q.max_vrows, q.nsegx);
    const int w_al = (int)align_up_sz((size_t)p.w, 16);
    const bool vec = (p.w & 15) == 0;
    for (int sx = 0; sx < q.nsegx; ++sx) {
      const uint8_t* src = p.seg[sx].idx;
      uint8_t* dst = s.sidx + (size_t)sx * w_al;
      if (vec && ((reinterpret_cast<uintptr_t>(src) & 15u) == 0)) {
        // Asynchronous copies: nothing here waits for them; gemv_post does.
        for (int i = threadIdx.x; i < p.w / 16; i += kStepThreads)
          cp_async_16(reinterpret_cast<uint4*>(dst) + i, reinterpret_cast<const uint4*>(src) + i);
      } else {
        for (int i = threadIdx.x; i < p.w; i += kStepThreads) dst[i] = src[i];
      }
    }
  }
}

// Post-barrier: input prologue, gather, streaming, epilogue.
template <int L>
__device__ __forceinline__ void gemv_post(const GemvParams& p, const GemvGeom& q, unsigned char* smem_base,
                                          U32x8 (&buf)[kStepU], unsigned cta, unsigned ncta) {
  constexpr int RG = kWarp / L, CH = 16 * L, U = kStepU, NT = kStepThreads;
  const int tid = threadIdx.x, lane = tid & 31;
  const int sub = lane / L, li = lane % L;
  StepGemvSmem s = step_gemv_smem(p, smem_base, q.max_vrows, q.nsegx);
  const int w_al = (int)align_up_sz((size_t)p.w, 16);

  // Mask offsets staged by gemv_pre's asynchronous copies (no-op if none).
  cp_async_commit_wait_all();
  // Input vector (+ residual) into shared memory, with the RMSNorm statistic.
  const __half* xsrc = input_row(p);
  const bool resid = (p.prologue == kProResidNorm);
  const bool add = resid && (p.x2 != nullptr);
  float ss = 0.f;
  if ((p.K & 7) == 0 && (reinterpret_cast<uintptr_t>(xsrc) & 15u) == 0 &&
      (!add || (reinterpret_cast<uintptr_t>(p.x2) & 15u) == 0)) {
    for (int i8 = tid; i8 < p.K / 8; i8 += NT) {
      const uint4 a = *reinterpret_cast<const uint4*>(xsrc + (size_t)i8 * 8);
      uint4 b = make_uint4(0u, 0u, 0u, 0u);
      if (add) b = *reinterpret_cast<const uint4*>(p.x2 + (size_t)i8 * 8);
      const __half* ah = reinterpret_cast<const __half*>(&a);
      const __half* bh = reinterpret_cast<const __half*>(&b);
      uint4 o;
      __half* oh = reinterpret_cast<__half*>(&o);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const __half hv = add ? f2h(h2f(ah[e]) + h2f(bh[e])) : ah[e];
        oh[e] = hv;
        ss = fmaf(h2f(hv), h2f(hv), ss);
      }
      *reinterpret_cast<uint4*>(s.xs + (size_t)i8 * 8) = o;
    }
  } else {
    for (int i = tid; i < p.K; i += NT) {
      float v = h2f(xsrc[i]);
      if (add) v = h2f(f2h(v + h2f(p.x2[i])));
      s.xs[i] = f2h(v);
      ss = fmaf(v, v, ss);
    }
  }
  for (int v = tid; v < q.vgroups * RG; v += NT) s.acc[v] = 0.f;
  float rstd = 1.f;
  if (resid) {
    const float tot = block_reduce_sum(ss, s.red);
    rstd = 1.0f / sqrtf(tot / (float)p.K + p.eps);
  }
  __syncthreads();
  if (resid && p.resid_out != nullptr && cta == 0)
    for (int i = tid; i < p.K; i += NT) p.resid_out[i] = s.xs[i];

  // Gather the compressed vectors (permuted for conflict-free reads).
  for (int sx = 0; sx < q.nsegx; ++sx) {
    const uint8_t* idx = s.sidx + (size_t)sx * w_al;
    __half* xc = s.xc + (size_t)sx * p.w_pad;
    for (int j = tid; j < p.w_pad; j += NT) {
      __half val = __ushort_as_half((unsigned short)0);
      if (j < p.w) {
        const int col = q.dense ? j : (j / p.n) * p.m + (int)idx[j];
        if (col < p.K) {
          val = s.xs[col];
          if (resid) val = f2h(h2f(f2h(h2f(val) * rstd)) * h2f(p.norm_w[col]));
        }
      }
      xc[xc_perm<L>(j)] = val;
    }
  }
  __syncthreads();

  // Stream: the ring holds items t0 .. t0+U-1; the load cursor starts at t0+U.
  int l_vg, l_c;
  {
    const int ls = min(q.t1, q.t0 + U);
    l_vg = ls / q.cpr;
    l_c = ls - l_vg * q.cpr;
  }
  LaneRow lr = lane_row(p, q.paired, q.g0, q.ng, l_vg, RG, sub);
  const __half* l_ptr = p.seg[lr.segi].w + (size_t)lr.lrow * p.w_pad + li * 16;
  bool l_valid = lr.valid;
  int c_vg = q.t0 / q.cpr, c_c = q.t0 - c_vg * q.cpr;
  LaneRow cr = lane_row(p, q.paired, q.g0, q.ng, c_vg, RG, sub);
  bool c_valid = cr.valid;
  const __half* xcs = s.xc + (size_t)cr.segi * p.w_pad + li * 8;
  float a0 = 0.f, a1 = 0.f;
  for (int base = q.t0; base < q.t1; base += U) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int t = base + u;
      if (t < q.t1) {
        const uint4 xa = *reinterpret_cast<const uint4*>(xcs + c_c * CH);
        const uint4 xb = *reinterpret_cast<const uint4*>(xcs + c_c * CH + 8 * L);
        fma2_f32_f16(a0, a1, buf[u].v[0], xa.x);
        fma2_f32_f16(a0, a1, buf[u].v[1], xa.y);
        fma2_f32_f16(a0, a1, buf[u].v[2], xa.z);
        fma2_f32_f16(a0, a1, buf[u].v[3], xa.w);
        fma2_f32_f16(a0, a1, buf[u].v[4], xb.x);
        fma2_f32_f16(a0, a1, buf[u].v[5], xb.y);
        fma2_f32_f16(a0, a1, buf[u].v[6], xb.z);
        fma2_f32_f16(a0, a1, buf[u].v[7], xb.w);
        if (t + U < q.t1) {
          if (l_valid) {
            buf[u] = ld_stream_256(l_ptr + (size_t)l_c * CH);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e) buf[u].v[e] = 0u;
          }
          if (++l_c == q.cpr) {
            l_c = 0;
            ++l_vg;
            lr = lane_row(p, q.paired, q.g0, q.ng, l_vg, RG, sub);
            l_valid = lr.valid;
            l_ptr = p.seg[lr.segi].w + (size_t)lr.lrow * p.w_pad + li * 16;
          }
        }
        const bool row_end = (++c_c == q.cpr);
        if (row_end || t + 1 == q.t1) {
          const float tot = group_reduce_sum<L>(a0 + a1);
          if (li == 0 && c_valid) atomicAdd(&s.acc[c_vg * RG + sub], tot);
          a0 = a1 = 0.f;
          if (row_end) {
            c_c = 0;
            ++c_vg;
            if (c_vg < q.vgroups) {
              cr = lane_row(p, q.paired, q.g0, q.ng, c_vg, RG, sub);
              c_valid = cr.valid;
              xcs = s.xc + (size_t)cr.segi * p.w_pad + li * 8;
            }
          }
        }
      }
    }
  }
  __syncthreads();
  gemv_epilogue<NT>(p, s.acc, q.g0, q.ng, RG, cta, ncta);
  __syncthreads();
}

// ---------------------------------------------------------------------------
// Attention unit (one KV head, one context split) with the whole CTA, and the
// last-unit-per-head combine.
// ---------------------------------------------------------------------------
struct StepAttnSmem {
  float sq[kAttnMaxGroup][kAttnD];
  __half sk[kAttnTile][kAttnD + 8];
  __half sv[kAttnTile][kAttnD];
  float sp[kAttnMaxGroup][kAttnTile];
  __half knew[kAttnD];
  __half vnew[kAttnD];
  float sm[kAttnMaxGroup], sl[kAttnMaxGroup], scorr[kAttnMaxGroup];
  float so[kAttnMaxGroup][kAttnD];
  int last;
};

__device__ __forceinline__ void attention_unit(const AttnParams& p, int split, int kvh, StepAttnSmem& S,
                                               float* part, unsigned* head_count) {
  constexpr int D = kAttnD, PT = kAttnTile, GM = kAttnMaxGroup, NT = kStepThreads;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = p.Hq / p.Hkv;
  const int64_t pos64 = *p.pos;
  if (pos64 < 0 || pos64 >= p.S_max) {  // uniform: every CTA reads the same value
    if (tid == 0 && split == 0 && kvh == 0) set_device_error(kDevBadPosition);
    return;
  }
  const int pos = (int)pos64;
  const int P = pos + 1;
  const int pb = (int)(((int64_t)split * P) / p.splits);
  const int pe = (int)(((int64_t)(split + 1) * P) / p.splits);
  const bool has_new = (split == p.splits - 1);
  const __half* rope_row = p.rope + (size_t)pos * D;
  const __half* kbase = p.k_cache + (size_t)kvh * p.S_max * D;
  const __half* vbase = p.v_cache + (size_t)kvh * p.S_max * D;
  // K and V rows of a tile: cached rows by asynchronous copies, rows past the
  // range zero; the new token's row is filled from shared memory later.
  auto issue_tile = [&](int t0) {
    const int nt = min(PT, pe - t0);
    constexpr int PIECES = 2 * PT * (D / 8);
#pragma unroll
    for (int c0 = 0; c0 < PIECES; c0 += NT) {
      const int c = c0 + tid;
      if (c >= PIECES) break;
      const int which = c / (PT * (D / 8));
      const int rem = c - which * PT * (D / 8);
      const int r = rem / (D / 8), q8 = rem % (D / 8);
      __half* dst = which ? &S.sv[r][q8 * 8] : &S.sk[r][q8 * 8];
      const int tpos = t0 + r;
      if (r < nt && tpos != pos)
        cp_async_16(dst, (which ? vbase : kbase) + (size_t)tpos * D + q8 * 8);
      else if (r >= nt)
        *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
    }
  };
  if (pb < pe) issue_tile(pb);  // in flight during the q / k / v work below

  if (warp < G) {
    const __half* qsrc = p.qkv + (size_t)(kvh * G + warp) * D;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = h2f(qsrc[lane * 4 + e]);
    if (p.q_norm) head_rmsnorm(v, p.q_norm, lane, p.norm_eps);
    head_rope(v, rope_row, lane, p.rope_style);
#pragma unroll
    for (int e = 0; e < 4; ++e) S.sq[warp][lane * 4 + e] = v[e];
  }
  if (has_new && warp == GM) {  // new k
    const __half* ksrc = p.qkv + (size_t)p.Hq * D + (size_t)kvh * D;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) v[e] = h2f(ksrc[lane * 4 + e]);
    if (p.k_norm) head_rmsnorm(v, p.k_norm, lane, p.norm_eps);
    head_rope(v, rope_row, lane, p.rope_style);
    __half* kdst = p.k_cache + ((size_t)kvh * p.S_max + pos) * D;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      S.knew[lane * 4 + e] = f2h(v[e]);
      kdst[lane * 4 + e] = f2h(v[e]);
    }
  }
  if (has_new && warp == GM + 1) {  // new v
    const __half* vsrc = p.qkv + (size_t)(p.Hq + p.Hkv) * D + (size_t)kvh * D;
    __half* vdst = p.v_cache + ((size_t)kvh * p.S_max + pos) * D;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      S.vnew[lane * 4 + e] = vsrc[lane * 4 + e];
      vdst[lane * 4 + e] = vsrc[lane * 4 + e];
    }
  }
  for (int i = tid; i < GM * D; i += NT) (&S.so[0][0])[i] = 0.f;
  if (tid < GM) {
    S.sm[tid] = -INFINITY;
    S.sl[tid] = 0.f;
  }
  __syncthreads();  // state initialised (an empty split publishes it unchanged)

  for (int t0 = pb; t0 < pe; t0 += PT) {
    const int nt = min(PT, pe - t0);
    if (t0 != pb) issue_tile(t0);
    __syncthreads();  // knew / vnew (written above) visible
    if (pos >= t0 && pos < t0 + nt) {
      const int r = pos - t0;
      for (int i = tid; i < 2 * (D / 8); i += NT) {
        const int which = i / (D / 8), q8 = i % (D / 8);
        *reinterpret_cast<uint4*>(which ? &S.sv[r][q8 * 8] : &S.sk[r][q8 * 8]) =
            *reinterpret_cast<const uint4*>((which ? S.vnew : S.knew) + q8 * 8);
      }
    }
    cp_async_commit_wait_all();
    __syncthreads();
    for (int i = tid; i < G * PT; i += NT) {
      const int g = i / PT, r = i % PT;
      float sc = -INFINITY;
      if (r < nt) {
        float d0 = 0.f, d1 = 0.f;
#pragma unroll
        for (int q8 = 0; q8 < D / 8; ++q8) {
          const uint4 kk = *reinterpret_cast<const uint4*>(&S.sk[r][q8 * 8]);
          const float4 qa = *reinterpret_cast<const float4*>(&S.sq[g][q8 * 8]);
          const float4 qb = *reinterpret_cast<const float4*>(&S.sq[g][q8 * 8 + 4]);
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
        sc = (d0 + d1) * p.scale;
      }
      S.sp[g][r] = sc;
    }
    __syncthreads();
    if (warp < G) {
      const float s0 = S.sp[warp][lane], s1 = S.sp[warp][lane + 32];
      float mt = fmaxf(s0, s1);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
      const float m_old = S.sm[warp];
      const float m_new = fmaxf(m_old, mt);
      const float p0 = (lane < nt) ? expf(s0 - m_new) : 0.f;
      const float p1 = (lane + 32 < nt) ? expf(s1 - m_new) : 0.f;
      const float tot = warp_reduce_sum(p0 + p1);
      S.sp[warp][lane] = p0;
      S.sp[warp][lane + 32] = p1;
      if (lane == 0) {
        const float corr = (m_old == -INFINITY) ? 0.f : expf(m_old - m_new);
        S.scorr[warp] = corr;
        S.sl[warp] = S.sl[warp] * corr + tot;
        S.sm[warp] = m_new;
      }
    }
    __syncthreads();
    for (int i = tid; i < G * D; i += NT) {
      const int g = i / D, d = i - g * D;
      float acc = S.so[g][d] * S.scorr[g];
      for (int r = 0; r < nt; ++r) acc = fmaf(S.sp[g][r], h2f(S.sv[r][d]), acc);
      S.so[g][d] = acc;
    }
    __syncthreads();
  }

  // Publish this split's state [g][m, l, o[D]] and count arrivals per head.
  constexpr int STRIDE = D + 2;
  float* my = part + ((size_t)kvh * p.splits + split) * GM * STRIDE;
  for (int i = tid; i < G * STRIDE; i += NT) {
    const int g = i / STRIDE, k = i - g * STRIDE;
    my[g * STRIDE + k] = (k == 0) ? S.sm[g] : (k == 1) ? S.sl[g] : S.so[g][k - 2];
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned prev = atomicAdd(&head_count[kvh], 1u);
    S.last = (prev == (unsigned)p.splits - 1) ? 1 : 0;
    if (S.last) {
      __threadfence();
      head_count[kvh] = 0u;
    }
  }
  __syncthreads();
  if (!S.last) return;
  // Last split of this head: combine every split's state (read through L2,
  // all loads of a thread independent so they overlap).
  const float* hp = part + (size_t)kvh * p.splits * GM * STRIDE;
  float* fw = &S.so[0][0];                 // reuse: per (split, head) weight exp(m_r - M) / L
  float* mlr = &S.sq[0][0];                // reuse: per (split, head) (m, l)
  for (int i = tid; i < p.splits * G; i += NT) {
    const int r = i / G, g = i - r * G;
    mlr[2 * (r * GM + g)] = __ldcg(hp + ((size_t)r * GM + g) * STRIDE);
    mlr[2 * (r * GM + g) + 1] = __ldcg(hp + ((size_t)r * GM + g) * STRIDE + 1);
  }
  __syncthreads();
  if (tid < G) {
    const int g = tid;
    float M = -INFINITY;
    for (int r = 0; r < p.splits; ++r) M = fmaxf(M, mlr[2 * (r * GM + g)]);
    float Lsum = 0.f;
    for (int r = 0; r < p.splits; ++r) {
      const float mr = mlr[2 * (r * GM + g)];
      const float f = (mr == -INFINITY) ? 0.f : expf(mr - M);
      fw[r * GM + g] = f;
      Lsum = fmaf(mlr[2 * (r * GM + g) + 1], f, Lsum);
    }
    const float inv = 1.0f / Lsum;
    for (int r = 0; r < p.splits; ++r) fw[r * GM + g] *= inv;
  }
  __syncthreads();
  for (int i = tid; i < G * D; i += NT) {
    const int g = i / D, d = i - g * D;
    float O = 0.f;
#pragma unroll
    for (int r = 0; r < kMaxSplits; ++r)
      if (r < p.splits) O = fmaf(__ldcg(hp + ((size_t)r * GM + g) * STRIDE + 2 + d), fw[r * GM + g], O);
    p.y[(size_t)(kvh * G + g) * D + d] = f2h(O);
  }
}

// ---------------------------------------------------------------------------
// The persistent kernel.  The lanes-per-row variant of each GEMV stage is
// chosen per stage, so stages of different packed widths share one launch.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void step_gemv_pre(const StepStage& st, unsigned cta, unsigned ncta, unsigned char* smem,
                                              U32x8 (&buf)[kStepU]) {
  switch (st.lanes) {
    case 32: gemv_pre<32>(st.g, gemv_geom<32>(st.g, cta, ncta), smem, buf); break;
    case 16: gemv_pre<16>(st.g, gemv_geom<16>(st.g, cta, ncta), smem, buf); break;
    case 8: gemv_pre<8>(st.g, gemv_geom<8>(st.g, cta, ncta), smem, buf); break;
    default: gemv_pre<4>(st.g, gemv_geom<4>(st.g, cta, ncta), smem, buf); break;
  }
}

__device__ __forceinline__ void step_gemv_l2_prefetch(const StepStage& st, unsigned cta, unsigned ncta) {
  switch (st.lanes) {
    case 32: gemv_l2_prefetch_own<32>(st.g, gemv_geom<32>(st.g, cta, ncta)); break;
    case 16: gemv_l2_prefetch_own<16>(st.g, gemv_geom<16>(st.g, cta, ncta)); break;
    case 8: gemv_l2_prefetch_own<8>(st.g, gemv_geom<8>(st.g, cta, ncta)); break;
    default: gemv_l2_prefetch_own<4>(st.g, gemv_geom<4>(st.g, cta, ncta)); break;
  }
}

__device__ __forceinline__ void step_gemv_post(const StepStage& st, unsigned cta, unsigned ncta, unsigned char* smem,
                                               U32x8 (&buf)[kStepU]) {
  switch (st.lanes) {
    case 32: gemv_post<32>(st.g, gemv_geom<32>(st.g, cta, ncta), smem, buf, cta, ncta); break;
    case 16: gemv_post<16>(st.g, gemv_geom<16>(st.g, cta, ncta), smem, buf, cta, ncta); break;
    case 8: gemv_post<8>(st.g, gemv_geom<8>(st.g, cta, ncta), smem, buf, cta, ncta); break;
    default: gemv_post<4>(st.g, gemv_geom<4>(st.g, cta, ncta), smem, buf, cta, ncta); break;
  }
}

__global__ void __launch_bounds__(kStepThreads, 1) decode_step_kernel(const __grid_constant__ StepParams sp) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ StepStage s_stage[2];  // current and next stage parameters
  const unsigned cta = blockIdx.x, ncta = gridDim.x;
  const int tid = threadIdx.x;

  auto load_stage = [&](int s, int slot) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(sp.stages + s);
    uint32_t* dst = reinterpret_cast<uint32_t*>(&s_stage[slot]);
    for (int i = tid; i < (int)(sizeof(StepStage) / 4); i += kStepThreads) dst[i] = src[i];
  };

  grid_dep_wait();
  if (sp.trace != nullptr && cta == 0 && tid == 0) sp.trace[0] = global_timer_ns();
  U32x8 buf[kStepU];
  load_stage(0, 0);
  __syncthreads();
  if (s_stage[0].kind == kStageGemv) {
    step_gemv_pre(s_stage[0], cta, ncta, smem_raw, buf);
    __syncthreads();
  }
  for (int s = 0; s < sp.nstages; ++s) {
    const int cur = s & 1, nxt = cur ^ 1;
    const StepStage& st = s_stage[cur];
    if (s + 1 < sp.nstages) load_stage(s + 1, nxt);  // read by the pre-barrier work below
    if (st.kind == kStageGemv) {
      step_gemv_post(st, cta, ncta, smem_raw, buf);
    } else {
      // Latency-bound stage: meanwhile pull this CTA's rows of the following
      // GEMV into L2 (HBM is otherwise idle).
      __syncthreads();
      if (s + 1 < sp.nstages && s_stage[nxt].kind == kStageGemv) step_gemv_l2_prefetch(s_stage[nxt], cta, ncta);
      StepAttnSmem& S = *reinterpret_cast<StepAttnSmem*>(smem_raw);
      for (int u = cta; u < st.units; u += ncta) {
        attention_unit(st.a, u % st.a.splits, u / st.a.splits, S, sp.attn_part, sp.attn_count);
        __syncthreads();
      }
    }
    unsigned long long* tr = sp.trace ? sp.trace + 1 + (size_t)s * (ncta + 1) : nullptr;
    if (tr != nullptr && tid == 0) tr[cta] = global_timer_ns();
    if (s + 1 < sp.nstages) {
      grid_arrive(sp.bar_count);
      if (s_stage[nxt].kind == kStageGemv) step_gemv_pre(s_stage[nxt], cta, ncta, smem_raw, buf);
      if (!grid_wait(sp.bar_count, ncta, (unsigned)s)) return;
      if (tr != nullptr && cta == 0 && tid == 0) tr[ncta] = global_timer_ns();
    }
  }
  step_exit(sp.bar_count, sp.bar_exit, ncta);
  grid_dep_launch_dependents();
}

}  // namespace nms
