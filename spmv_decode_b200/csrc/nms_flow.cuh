// Dataflow persistent decode step: the same stages as decode_step_kernel
// (q/k/v GEMV, attention, o, gate/up + SwiGLU, down per layer; the head with
// greedy argmax), one cooperative launch of one CTA per SM, the same
// per-warp weight rings -- but no grid barriers.
//
// Why: while the weight rings keep HBM saturated, every global-memory round
// trip (an L2 hit included) takes 1-1.4 us on this B200 instead of 0.15 us
// idle, because L2 and the on-chip network are queued up with streaming
// requests.  A grid barrier plus the next stage's input load plus its mask
// staging chains three or four such round trips at every stage boundary.
// Here a stage's output travels as tagged words -- {fp16 value, 16-bit tag}
// in 32 bits, or {fp32 value, 32-bit tag} in 64 bits -- stored with single
// relaxed stores; a consumer polls exactly the words it needs, and a word
// whose tag names the current step IS the value of this step (a 32- or
// 64-bit aligned access is single-copy atomic), so the data are their own
// arrival signal: one round trip per boundary, no fence, no counter.
//
// Every handoff buffer belongs to one stage and is written once per step,
// so a tag only has to tell this step from earlier ones: tag16 =
// epoch % 65535 + 1, tag32 = epoch + 1 (a zeroed buffer never matches).
//
// The consumer's work moves to the producer where it can:
//   * residual add: the o- and down-projection epilogues own their output
//     rows of the residual stream and write resid_new = resid_old + out
//     (fp16 rounding as the reference's residual add) as tagged words, plus
//     their share of sum(resid_new^2) as one tagged fp32 partial per CTA;
//   * gather: a producer scatters each output row straight to the positions
//     the consumer's N:M masks keep (static inverse tables built on the host
//     from mat_index), so the consumer's compressed input arrives ready;
//   * RMSNorm: the consumer adds the ncta partials in CTA order (the same
//     sum in every CTA, so results stay deterministic) and scales its
//     compressed input by rstd and the mask-gathered norm weights.
// Attention: each (KV head, context split) unit publishes its partial
// softmax state as tagged fp32 words; the unit holding the new token (the
// last split) polls the others', combines them and scatters the head's
// output into the o-projection's input.
// The first stage (q/k/v of layer 0) reads the embedding row and gathers by
// mask itself, as the barrier kernel does, and publishes the row as the
// first residual.
#pragma once

#include "nms_step.cuh"

namespace nms {

// ---------------------------------------------------------------------------
// Tagged words.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t ld_rlx_b32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Four words; each 32-bit element is its own single-copy-atomic access.
__device__ __forceinline__ uint4 ld_rlx_v4(const uint32_t* p) {
  uint4 v;
  asm volatile("ld.relaxed.gpu.global.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_rlx_b64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_rlx_b32(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_rlx_b64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint32_t h16_word(__half v, uint32_t tag16) {
  return (tag16 << 16) | (uint32_t)__half_as_ushort(v);
}
__device__ __forceinline__ __half h16_value(uint32_t w) { return __ushort_as_half((unsigned short)(w & 0xffffu)); }
__device__ __forceinline__ unsigned long long f32_word(float v, uint32_t tag32) {
  return ((unsigned long long)tag32 << 32) | (unsigned long long)__float_as_uint(v);
}

constexpr uint64_t kPollLimitNs = 200ull * 1000 * 1000;

// Wait until the word at p carries `tag16` (w holds the last value read).
// Bounded: gives up (false) after the limit (kDevBarrierTimeout recorded) or
// as soon as the device error word is set.
__device__ __noinline__ bool poll_h16(const uint32_t* p, uint32_t tag16, uint32_t& w) {
  const uint64_t t0 = global_timer_ns();
  while ((w >> 16) != tag16) {
    if (*reinterpret_cast<volatile int*>(&g_device_error) != 0) return false;
    if (global_timer_ns() - t0 > kPollLimitNs) {
      set_device_error(kDevBarrierTimeout);
      return false;
    }
    __nanosleep(32);
    w = ld_rlx_b32(p);
  }
  return true;
}

__device__ __noinline__ bool poll_f32t(const unsigned long long* p, uint32_t tag32, unsigned long long& w) {
  const uint64_t t0 = global_timer_ns();
  while ((uint32_t)(w >> 32) != tag32) {
    if (*reinterpret_cast<volatile int*>(&g_device_error) != 0) return false;
    if (global_timer_ns() - t0 > kPollLimitNs) {
      set_device_error(kDevBarrierTimeout);
      return false;
    }
    __nanosleep(32);
    w = ld_rlx_b64(p);
  }
  return true;
}

// Stage completion hints.  A producer CTA bumps its stage's counter with a
// fire-and-forget relaxed add after its stores; one thread of a consumer CTA
// waits (bounded) for the count of this step before the CTA reads its words,
// so a CTA that is early does not have all its threads spinning on L2.  The
// counter is only a hint: the tags stay the proof that a word is of this
// step (a word seen early is polled by itself).  Counters are zeroed by the
// last CTA to leave the kernel.
__device__ __forceinline__ void red_rlx_add_u32(unsigned* p, unsigned v) {
  asm volatile("red.relaxed.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_rlx_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Whole CTA: returns false (uniformly) if the wait gave up.
__device__ __forceinline__ bool flow_wait_done(const unsigned* cnt, unsigned need, int* s_fail) {
  if (cnt != nullptr && threadIdx.x == 0 && ld_rlx_u32(cnt) < need) {
    const uint64_t t0 = global_timer_ns();
    while (ld_rlx_u32(cnt) < need) {
      if (*reinterpret_cast<volatile int*>(&g_device_error) != 0) {
        atomicExch(s_fail, 1);
        break;
      }
      if (global_timer_ns() - t0 > kPollLimitNs) {
        set_device_error(kDevBarrierTimeout);
        atomicExch(s_fail, 1);
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  return *reinterpret_cast<volatile int*>(s_fail) == 0;
}

// Read a tagged fp32 word, polling until it carries tag32.
__device__ __forceinline__ float get_f32t(const unsigned long long* p, uint32_t tag32, bool& ok) {
  unsigned long long w = ld_rlx_b64(p);
  if ((uint32_t)(w >> 32) != tag32 && !poll_f32t(p, tag32, w)) ok = false;
  return __uint_as_float((uint32_t)w);
}

// ---------------------------------------------------------------------------
// Stage tables.
// ---------------------------------------------------------------------------
enum FlowIn : int32_t {
  kFlowInGather = 0,  // stage x (+ x2) from a plain fp16 vector, gather by mask (the first stage)
  kFlowInTagged = 1,  // poll the producer's words, already in compressed order
};
enum FlowOut : int32_t {
  kFlowOutWords = 0,   // rows as tagged words in natural order (q/k/v)
  kFlowOutResid = 1,   // residual update + sum-of-squares partial + scatter (o, down)
  kFlowOutAct = 2,     // SwiGLU rows, scatter (gate/up)
  kFlowOutArgmax = 3,  // logits (plain fp16) + greedy token (the head)
};
constexpr int kFlowMaxScat = 4;

struct FlowGemv {
  StepGemv sg;
  int32_t in_mode, out_mode, nscat;
  uint32_t done_need;                 // increments of done_in per step
  const unsigned* done_in;            // the input producer's completion counter (nullptr: none)
  unsigned* done_out;                 // this stage's completion counter
  // kFlowInTagged: gathered vector sx is the word array xc_in[sx] (position
  // j < w; positions >= w are zero), norm stages also take the producer's
  // per-CTA sum-of-squares partials and the norm weights gathered by mask.
  const uint32_t* xc_in[kMaxSegs];
  const __half* nwc;                  // [nsegx][w_pad] (staged into shared memory)
  const unsigned long long* ssq_in;   // [ncta]
  // kFlowInGather: the staged input row as the first residual, written by CTA 0.
  uint32_t* gather_resid;             // [K] words or nullptr
  // Output.
  uint32_t* out_words;                // natural-order words [rows] (resid_new / act / rows) or nullptr
  const uint32_t* resid_old;          // kFlowOutResid: [rows] words
  unsigned long long* ssq_out;        // kFlowOutResid: [ncta]
  uint32_t* scat_dst[kFlowMaxScat];   // consumer's compressed word arrays
  const int32_t* scat_inv[kFlowMaxScat];  // [rows] position in that array, -1 if the mask drops the row
};

struct FlowAttn {
  AttnParams a;
  uint32_t done_need, pad_;
  const unsigned* done_in;      // the q/k/v stage's completion counter
  unsigned* done_out;           // bumped by each combining unit
  const uint32_t* qkv_in;       // [(Hq + 2 Hkv) * D] words of the q/k/v stage
  unsigned long long* part;     // [units][G][D + 2] partial softmax states (m, l, o)
  uint32_t* y_words;            // natural-order y words [Hq * D] (dense o-projection) or nullptr
  uint32_t* y_dst;              // the o-projection's compressed word array, or nullptr
  const int32_t* y_inv;         // [Hq * D]
};

struct FlowParams {
  const int32_t* kind;     // [nstages] StageKind
  const FlowGemv* gemv;    // [ngemv]
  const ProdDesc* desc;    // [ngemv]
  const FlowAttn* attn;    // [nattn]
  int32_t nstages, ngemv, nattn;
  int32_t ring_bytes, act_bytes;
  unsigned* exit_count;           // CTAs that have left (reset by the last)
  unsigned* counters;             // [ncounters] stage completion hints (zeroed by the last CTA to leave)
  int32_t ncounters, pad_;
  unsigned* spare;                // zeroed word (step_exit's barrier-counter slot)
  unsigned long long* epoch;      // completed steps (tags)
  unsigned long long* trace;      // as StepParams::trace (no barrier release times: 0)
  unsigned long long* trace_detail;
  const int64_t* pos;
};

// Shared-memory working set of a flow GEMV stage (after the rings):
// [xs K halves (gather) | sidx nsegx*w_al (gather) | xc nsegx*w_pad halves |
//  nw (gather: K halves; tagged norm: nsegx*w_pad halves) | acc max_vrows |
//  red 32 | inv kFlowMaxScat*NT | res NT].
__host__ __device__ inline size_t flow_gemv_layout(int K, int w, int w_pad, int nsegx, int max_vrows, bool norm,
                                                   bool gather, size_t* o_sidx, size_t* o_xc, size_t* o_nw,
                                                   size_t* o_acc, size_t* o_red, size_t* o_inv, size_t* o_res) {
  size_t off = gather ? align_up_sz((size_t)K * 2, 16) : 0;
  *o_sidx = off;
  if (gather) off += align_up_sz((size_t)w, 16) * nsegx;
  *o_xc = off;
  off += align_up_sz((size_t)w_pad * 2 * nsegx, 16);
  *o_nw = off;
  if (norm) off += gather ? align_up_sz((size_t)K * 2, 16) : align_up_sz((size_t)w_pad * 2 * nsegx, 16);
  *o_acc = off;
  off += align_up_sz((size_t)max_vrows * 4, 16);
  *o_red = off;
  off += 32 * 4;
  *o_inv = off;
  off += (size_t)kFlowMaxScat * kStepThreads * 4;
  *o_res = off;
  off += (size_t)kStepThreads * 4;
  return off;
}

struct FlowSmem {
  __half* xs;
  uint8_t* sidx;
  __half* xc;
  __half* nw;
  float* acc;
  float* red;
  int32_t* inv;   // [kFlowMaxScat][NT]
  uint32_t* res;  // [NT]
};

__device__ __forceinline__ FlowSmem flow_smem(const FlowGemv& fg, unsigned char* base, int nsegx, int max_vrows) {
  const GemvParams& p = fg.sg.g;
  size_t a, b, c, d, e, f, g;
  flow_gemv_layout(p.K, p.w, p.w_pad, nsegx, max_vrows, p.prologue == kProResidNorm, fg.in_mode == kFlowInGather,
                   &a, &b, &c, &d, &e, &f, &g);
  FlowSmem s;
  s.xs = reinterpret_cast<__half*>(base);
  s.sidx = base + a;
  s.xc = reinterpret_cast<__half*>(base + b);
  s.nw = reinterpret_cast<__half*>(base + c);
  s.acc = reinterpret_cast<float*>(base + d);
  s.red = reinterpret_cast<float*>(base + e);
  s.inv = reinterpret_cast<int32_t*>(base + f);
  s.res = reinterpret_cast<uint32_t*>(base + g);
  return s;
}

// Static operands of a GEMV stage, staged while the previous stage ends (one
// thread issues bulk copies; completion on the stage mbarrier): mask offsets
// and norm weights for the gather stage, the mask-gathered norm weights for a
// tagged norm stage.
__device__ __forceinline__ bool flow_pre_bulk(const FlowGemv& fg) {
  const GemvParams& p = fg.sg.g;
  if (fg.in_mode == kFlowInGather) return pre_bulk(p);
  return p.prologue == kProResidNorm && (reinterpret_cast<uintptr_t>(fg.nwc) & 15u) == 0;
}

__device__ __forceinline__ void flow_pre_smem(const FlowGemv& fg, unsigned ncta, unsigned char* act, uint64_t* bar,
                                              unsigned& uses) {
  const GemvParams& p = fg.sg.g;
  const int nsegx = stage_nsegx(p);
  const bool norm = p.prologue == kProResidNorm;
  FlowSmem s = flow_smem(fg, act, nsegx, stage_max_vrows(p, kWarp / fg.sg.lanes, ncta));
  if (fg.in_mode == kFlowInGather) {
    const int w_al = (int)align_up_sz((size_t)p.w, 16);
    const bool has_idx = p.seg[0].idx != nullptr;
    if (pre_bulk(p)) {
      if (threadIdx.x == 0) {
        const uint32_t bytes = (has_idx ? (uint32_t)(nsegx * p.w) : 0u) + (norm ? (uint32_t)p.K * 2u : 0u);
        if (bytes > 0) {
          fence_proxy_async_smem();
          mbar_arrive_expect_tx(bar, bytes);
          if (has_idx)
            for (int sx = 0; sx < nsegx; ++sx) bulk_copy_g2s(s.sidx + (size_t)sx * w_al, p.seg[sx].idx, p.w, bar);
          if (norm) bulk_copy_g2s(s.nw, p.norm_w, (uint32_t)p.K * 2u, bar);
        } else {
          asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
        }
      }
      ++uses;
      return;
    }
    if (has_idx)
      for (int sx = 0; sx < nsegx; ++sx)
        for (int i = threadIdx.x; i < p.w; i += kStepThreads) s.sidx[(size_t)sx * w_al + i] = p.seg[sx].idx[i];
    if (norm)
      for (int i = threadIdx.x; i < p.K; i += kStepThreads) s.nw[i] = p.norm_w[i];
    return;
  }
  if (!norm) return;
  if (flow_pre_bulk(fg)) {
    if (threadIdx.x == 0) {
      fence_proxy_async_smem();
      const uint32_t bytes = (uint32_t)(nsegx * p.w_pad * 2);
      mbar_arrive_expect_tx(bar, bytes);
      bulk_copy_g2s(s.nw, fg.nwc, bytes, bar);
    }
    ++uses;
    return;
  }
  for (int i = threadIdx.x; i < nsegx * p.w_pad; i += kStepThreads) s.nw[i] = fg.nwc[i];
}

// ---------------------------------------------------------------------------
// GEMV stage.
// ---------------------------------------------------------------------------
template <int L, int D>
__device__ __forceinline__ bool flow_gemv_stage(const FlowGemv& fg, const ProdDesc* descs, int ngemv, unsigned cta,
                                                unsigned ncta, unsigned char* act, Ring& R, uint64_t* pre_bar,
                                                unsigned pre_uses, uint32_t tag16, uint32_t tag32,
                                                unsigned long long* td, int* s_fail) {
  constexpr int RG = kWarp / L, NT = kStepThreads, CB = 32 * L;
  const GemvParams& p = fg.sg.g;
  const int tid = threadIdx.x, lane = tid & 31;
  const int sub = lane / L, li = lane % L;
  const bool paired = (p.mode == kModePaired);
  const WarpGeom q = warp_geom(p.row_groups, paired, p.w_pad, L, cta, ncta, tid >> 5);
  const int nsegx = stage_nsegx(p);
  const int max_vrows = stage_max_vrows(p, RG, ncta);
  const bool norm = (p.prologue == kProResidNorm);
  FlowSmem s = flow_smem(fg, act, nsegx, max_vrows);
  const int row_lo = q.g0 * RG;
  const int nrows = min(q.ng * RG, max(0, p.rows_total - row_lo));
  const int out_mode = fg.out_mode;

  // Epilogue operands for this thread's output row (row_lo + tid): loads
  // issued now, kept in registers through the prologue, then parked in
  // shared memory.  The residual words were written stages ago.
  int32_t inv_r[kFlowMaxScat];
  uint32_t res_r = 0u;
  const bool mine = tid < nrows && (out_mode == kFlowOutResid || out_mode == kFlowOutAct);
  if (mine) {
#pragma unroll
    for (int t = 0; t < kFlowMaxScat; ++t) inv_r[t] = t < fg.nscat ? __ldg(fg.scat_inv[t] + row_lo + tid) : -1;
    if (out_mode == kFlowOutResid) res_r = ld_rlx_b32(fg.resid_old + row_lo + tid);
  }

  for (int v = tid; v < max_vrows; v += NT) s.acc[v] = 0.f;
  bool ok = true;
  if (fg.in_mode == kFlowInGather) {
    // -------- first stage: the embedding row, gathered by mask ----------
    const __half* xsrc = input_row(p);
    const bool add = norm && (p.x2 != nullptr);
    float ss = 0.f;
    if ((p.K & 7) == 0 && (reinterpret_cast<uintptr_t>(xsrc) & 15u) == 0 &&
        (!add || (reinterpret_cast<uintptr_t>(p.x2) & 15u) == 0)) {
      ss = add ? stage_input<2, true>(xsrc, p.x2, p.K, s.xs) : stage_input<4, false>(xsrc, nullptr, p.K, s.xs);
    } else {
      for (int i = tid; i < p.K; i += NT) {
        float v = h2f(xsrc[i]);
        if (add) v = h2f(f2h(v + h2f(p.x2[i])));
        s.xs[i] = f2h(v);
        ss = fmaf(v, v, ss);
      }
    }
    trace_at(td, 1);
    float rstd = 1.f;
    if (norm) {
      const float tot = block_reduce_sum(ss, s.red);
      rstd = 1.0f / sqrtf(tot / (float)p.K + p.eps);
    } else {
      __syncthreads();
    }
    trace_at(td, 2);
    if (fg.gather_resid != nullptr && cta == 0)
      for (int i = tid; i < p.K; i += NT) st_rlx_b32(fg.gather_resid + i, h16_word(s.xs[i], tag16));
    if (flow_pre_bulk(fg)) mbar_wait_bounded(pre_bar, (pre_uses - 1u) & 1u, kPreWaitLimitNs);
    trace_at(td, 3);
    const bool dense = (p.seg[0].idx == nullptr);
    const int w_al = (int)align_up_sz((size_t)p.w, 16);
    const int n_shift = ((p.n & (p.n - 1)) == 0) ? __ffs(p.n) - 1 : -1;
    const int wq = p.w_pad >> 2;
    for (int sx = 0; sx < nsegx; ++sx) {
      const uint8_t* idx = s.sidx + (size_t)sx * w_al;
      __half* xc = s.xc + (size_t)sx * p.w_pad;
      for (int t = tid; t < wq; t += NT) {
        const int j0 = t << 2;
        const uint32_t ib = (!dense && j0 < p.w) ? *reinterpret_cast<const uint32_t*>(idx + j0) : 0u;
        __align__(8) __half v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int j = j0 + e;
          __half val = __ushort_as_half((unsigned short)0);
          if (j < p.w) {
            const int grp = n_shift >= 0 ? (j >> n_shift) : j / p.n;
            const int col = dense ? j : grp * p.m + (int)((ib >> (8 * e)) & 0xffu);
            if (col < p.K) {
              val = s.xs[col];
              if (norm) val = f2h(h2f(f2h(h2f(val) * rstd)) * h2f(s.nw[col]));
            }
          }
          v[e] = val;
        }
        *reinterpret_cast<uint2*>(xc + j0) = *reinterpret_cast<const uint2*>(v);
      }
    }
  } else {
    // -------- tagged input: poll the compressed words (and partials) -----
    if (!flow_wait_done(fg.done_in, fg.done_need, s_fail)) return false;
    const int wq = p.w_pad >> 2;
    for (int t = tid; t < nsegx * wq; t += NT) {
      const int sx = t / wq, j0 = (t - sx * wq) << 2;
      const uint32_t* src = fg.xc_in[sx] + j0;
      uint4 wv = make_uint4(0u, 0u, 0u, 0u);
      if (j0 < p.w) wv = ld_rlx_v4(src);
      uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
      __align__(8) __half v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        v[e] = __ushort_as_half((unsigned short)0);
        if (j0 + e < p.w) {
          if ((wd[e] >> 16) != tag16 && !poll_h16(src + e, tag16, wd[e])) ok = false;
          v[e] = h16_value(wd[e]);
        }
      }
      *reinterpret_cast<uint2*>(s.xc + (size_t)sx * p.w_pad + j0) = *reinterpret_cast<const uint2*>(v);
    }
    if (norm && tid < kWarp) {
      // The producer's ncta partial sums, added in CTA order (every CTA
      // forms the same sum): lane l takes CTAs l, l + 32, ...; the lane
      // sums are then added in lane order.
      float part = 0.f;
      for (int c = lane; c < (int)ncta; c += kWarp) part += get_f32t(fg.ssq_in + c, tag32, ok);
      float tot = 0.f;
      for (int l2 = 0; l2 < kWarp; ++l2) tot += __shfl_sync(0xffffffffu, part, l2);
      if (lane == 0) s.red[0] = 1.0f / sqrtf(tot / (float)p.K + p.eps);
    }
    trace_at(td, 1);
    if (!ok) atomicExch(s_fail, 1);
    __syncthreads();
    trace_at(td, 2);
    if (norm) {
      if (flow_pre_bulk(fg)) mbar_wait_bounded(pre_bar, (pre_uses - 1u) & 1u, kPreWaitLimitNs);
      trace_at(td, 3);
      const float rstd = s.red[0];
      const int n8 = (nsegx * p.w_pad) >> 3;
      for (int i = tid; i < n8; i += NT) {
        uint4 xv = *reinterpret_cast<const uint4*>(s.xc + (size_t)i * 8);
        const uint4 nv = *reinterpret_cast<const uint4*>(s.nw + (size_t)i * 8);
        __half* xh = reinterpret_cast<__half*>(&xv);
        const __half* nh = reinterpret_cast<const __half*>(&nv);
#pragma unroll
        for (int e = 0; e < 8; ++e) xh[e] = f2h(h2f(f2h(h2f(xh[e]) * rstd)) * h2f(nh[e]));
        *reinterpret_cast<uint4*>(s.xc + (size_t)i * 8) = xv;
      }
    }
  }
  if (mine) {
#pragma unroll
    for (int t = 0; t < kFlowMaxScat; ++t) s.inv[t * NT + tid] = inv_r[t];
    s.res[tid] = res_r;
  }
  __syncthreads();
  trace_at(td, 4);
  if (*reinterpret_cast<volatile int*>(s_fail) != 0) return false;

  // -------- main loop: this warp's weight items (as decode_step_kernel) -----
  if (q.t0 < q.t1) {
    int vg = q.t0 / q.cpr, c = q.t0 - vg * q.cpr;
    LaneRow r = lane_row(p, paired, q.g0, q.ng, vg, RG, sub);
    const unsigned char* xcs = reinterpret_cast<const unsigned char*>(s.xc + (size_t)r.segi * p.w_pad) + li * 16;
    float a0 = 0.f, a1 = 0.f;
    for (int t = q.t0; t < q.t1; ++t) {
      cp_async_wait<D - 1>();
      const unsigned char* slot = R.wring + R.cslot * kRingItemBytes + lane * 16;
      const uint4 wa = *reinterpret_cast<const uint4*>(slot);
      const uint4 wb = *reinterpret_cast<const uint4*>(slot + 512);
      const uint4 xa = *reinterpret_cast<const uint4*>(xcs + c * CB);
      const uint4 xb = *reinterpret_cast<const uint4*>(xcs + c * CB + CB / 2);
      fma2_f32_f16(a0, a1, wa.x, xa.x);
      fma2_f32_f16(a0, a1, wa.y, xa.y);
      fma2_f32_f16(a0, a1, wa.z, xa.z);
      fma2_f32_f16(a0, a1, wa.w, xa.w);
      fma2_f32_f16(a0, a1, wb.x, xb.x);
      fma2_f32_f16(a0, a1, wb.y, xb.y);
      fma2_f32_f16(a0, a1, wb.z, xb.z);
      fma2_f32_f16(a0, a1, wb.w, xb.w);
      R.cslot = (R.cslot + 1 == D) ? 0 : R.cslot + 1;
      prod_next<D>(R.P, descs, ngemv, R.wring, cta, ncta);
      if (++c == q.cpr || t + 1 == q.t1) {
        const float tot = group_reduce_sum<L>(a0 + a1);
        if (li == 0 && r.valid) atomicAdd(&s.acc[vg * RG + sub], tot);
        a0 = a1 = 0.f;
        if (c == q.cpr && t + 1 < q.t1) {
          c = 0;
          ++vg;
          r = lane_row(p, paired, q.g0, q.ng, vg, RG, sub);
          xcs = reinterpret_cast<const unsigned char*>(s.xc + (size_t)r.segi * p.w_pad) + li * 16;
        }
      }
    }
  }
  __syncthreads();
  trace_at(td, 5);

  // -------- epilogue ----------------------------------------------------------
  if (out_mode == kFlowOutWords) {
    for (int v = tid; v < nrows; v += NT) st_rlx_b32(fg.out_words + row_lo + v, h16_word(f2h(s.acc[v]), tag16));
  } else if (out_mode == kFlowOutResid) {
    float sq = 0.f;
    if (tid < nrows) {
      uint32_t old = s.res[tid];
      if ((old >> 16) != tag16 && !poll_h16(fg.resid_old + row_lo + tid, tag16, old)) atomicExch(s_fail, 1);
      const __half o16 = f2h(s.acc[tid]);
      const __half n16 = f2h(h2f(h16_value(old)) + h2f(o16));
      const uint32_t word = h16_word(n16, tag16);
      if (fg.out_words != nullptr) st_rlx_b32(fg.out_words + row_lo + tid, word);
      for (int t = 0; t < fg.nscat; ++t) {
        const int j = s.inv[t * NT + tid];
        if (j >= 0) st_rlx_b32(fg.scat_dst[t] + j, word);
      }
      sq = h2f(n16) * h2f(n16);
    }
    const float tot = block_reduce_sum(sq, s.red);
    if (tid == 0) st_rlx_b64(fg.ssq_out + cta, f32_word(tot, tag32));
  } else if (out_mode == kFlowOutAct) {
    if (tid < nrows) {
      const float g = h2f(f2h(s.acc[tid]));
      const float u = h2f(f2h(s.acc[q.ng * RG + tid]));
      const float sg = h2f(f2h(g / (1.0f + expf(-g))));
      const uint32_t word = h16_word(f2h(sg * u), tag16);
      if (fg.out_words != nullptr) st_rlx_b32(fg.out_words + row_lo + tid, word);
      for (int t = 0; t < fg.nscat; ++t) {
        const int j = s.inv[t * NT + tid];
        if (j >= 0) st_rlx_b32(fg.scat_dst[t] + j, word);
      }
    }
  } else {
    gemv_epilogue<NT>(p, s.acc, q.g0, q.ng, RG, cta, ncta);
  }
  __syncthreads();
  if (tid == 0 && fg.done_out != nullptr) red_rlx_add_u32(fg.done_out, 1u);
  return *reinterpret_cast<volatile int*>(s_fail) == 0;
}

template <int D>
__device__ __forceinline__ bool run_flow_gemv(const FlowGemv& fg, const ProdDesc* descs, int ngemv, unsigned cta,
                                              unsigned ncta, unsigned char* act, Ring& R, uint64_t* pre_bar,
                                              unsigned pre_uses, uint32_t tag16, uint32_t tag32,
                                              unsigned long long* td, int* s_fail) {
  switch (fg.sg.lanes) {
    case 32: return flow_gemv_stage<32, D>(fg, descs, ngemv, cta, ncta, act, R, pre_bar, pre_uses, tag16, tag32, td, s_fail);
    case 16: return flow_gemv_stage<16, D>(fg, descs, ngemv, cta, ncta, act, R, pre_bar, pre_uses, tag16, tag32, td, s_fail);
    case 8: return flow_gemv_stage<8, D>(fg, descs, ngemv, cta, ncta, act, R, pre_bar, pre_uses, tag16, tag32, td, s_fail);
    default: return flow_gemv_stage<4, D>(fg, descs, ngemv, cta, ncta, act, R, pre_bar, pre_uses, tag16, tag32, td, s_fail);
  }
}

// ---------------------------------------------------------------------------
// Attention unit (one KV head, one context split).  As attention_unit, with
// q/k/v polled from the q/k/v stage's words and the partial state published
// as tagged words; the last split (it holds the new token) combines.
// ---------------------------------------------------------------------------
__device__ __noinline__ bool flow_attention_unit(const FlowAttn& fa, int pos_in, int split, int kvh,
                                                 StepAttnSmem& S, uint32_t tag16, uint32_t tag32,
                                                 unsigned long long* td, int* s_fail) {
  constexpr int D = kAttnD, PT = kAttnTile, GM = kAttnMaxGroup, NT = kStepThreads;
  const AttnParams& p = fa.a;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = p.Hq / p.Hkv;
  if (pos_in < 0 || pos_in >= p.S_max) {
    if (tid == 0 && split == 0 && kvh == 0) set_device_error(kDevBadPosition);
    return false;
  }
  const int pos = pos_in;
  const int P = pos + 1;
  const int pb = (int)(((int64_t)split * P) / p.splits);
  const int pe = (int)(((int64_t)(split + 1) * P) / p.splits);
  const bool has_new = (split == p.splits - 1);
  const __half* rope_row = p.rope + (size_t)pos * D;
  const __half* kbase = p.k_cache + (size_t)kvh * p.S_max * D;
  const __half* vbase = p.v_cache + (size_t)kvh * p.S_max * D;
  constexpr int PIECES = 2 * PT * (D / 8);
  constexpr int PPT = (PIECES + NT - 1) / NT;
  uint4 kv[PPT];
  auto load_tile = [&](int t0) {
    const int nt = min(PT, pe - t0);
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int c = k * NT + tid;
      kv[k] = make_uint4(0u, 0u, 0u, 0u);
      if (c < PIECES) {
        const int which = c / (PT * (D / 8));
        const int rem = c - which * PT * (D / 8);
        const int r = rem / (D / 8), q8 = rem % (D / 8);
        const int tpos = t0 + r;
        if (r < nt && tpos != pos)
          kv[k] = __ldg(reinterpret_cast<const uint4*>((which ? vbase : kbase) + (size_t)tpos * D + q8 * 8));
      }
    }
  };
  auto store_tile = [&](int t0) {
    const int nt = min(PT, pe - t0);
#pragma unroll
    for (int k = 0; k < PPT; ++k) {
      const int c = k * NT + tid;
      if (c < PIECES) {
        const int which = c / (PT * (D / 8));
        const int rem = c - which * PT * (D / 8);
        const int r = rem / (D / 8), q8 = rem % (D / 8);
        if (r >= nt || t0 + r != pos)
          *reinterpret_cast<uint4*>(which ? &S.sv[r][q8 * 8] : &S.sk[r][q8 * 8]) = kv[k];
      }
    }
  };
  // Cached K/V do not depend on this step's q/k/v: their loads go out
  // before the q/k/v words are polled.
  if (pb < pe) load_tile(pb);

  if (!flow_wait_done(fa.done_in, fa.done_need, s_fail)) return false;
  bool ok = true;
  // Four consecutive dims per lane: one 16-byte read of the words.
  auto head_words = [&](int row0, float (&v)[4]) {
    const uint32_t* src = fa.qkv_in + (size_t)row0 + lane * 4;
    const uint4 wv = ld_rlx_v4(src);
    uint32_t wd[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if ((wd[e] >> 16) != tag16 && !poll_h16(src + e, tag16, wd[e])) ok = false;
      v[e] = h2f(h16_value(wd[e]));
    }
  };
  if (warp < G) {
    float v[4];
    head_words((kvh * G + warp) * D, v);
    if (p.q_norm) head_rmsnorm(v, p.q_norm, lane, p.norm_eps);
    head_rope(v, rope_row, lane, p.rope_style);
#pragma unroll
    for (int e = 0; e < 4; ++e) S.sq[warp][lane * 4 + e] = v[e];
  }
  if (has_new && warp == GM) {  // new k
    float v[4];
    head_words(p.Hq * D + kvh * D, v);
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
    float v[4];
    head_words((p.Hq + p.Hkv) * D + kvh * D, v);
    __half* vdst = p.v_cache + ((size_t)kvh * p.S_max + pos) * D;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      S.vnew[lane * 4 + e] = f2h(v[e]);
      vdst[lane * 4 + e] = f2h(v[e]);
    }
  }
  for (int i = tid; i < GM * D; i += NT) (&S.so[0][0])[i] = 0.f;
  if (tid < GM) {
    S.sm[tid] = -INFINITY;
    S.sl[tid] = 0.f;
  }
  if (!ok) atomicExch(s_fail, 1);
  __syncthreads();
  trace_at(td, 4);
  if (*reinterpret_cast<volatile int*>(s_fail) != 0) return false;

  for (int t0 = pb; t0 < pe; t0 += PT) {
    const int nt = min(PT, pe - t0);
    if (t0 != pb) load_tile(t0);
    store_tile(t0);
    __syncthreads();
    if (pos >= t0 && pos < t0 + nt) {
      const int r = pos - t0;
      for (int i = tid; i < 2 * (D / 8); i += NT) {
        const int which = i / (D / 8), q8 = i % (D / 8);
        *reinterpret_cast<uint4*>(which ? &S.sv[r][q8 * 8] : &S.sk[r][q8 * 8]) =
            *reinterpret_cast<const uint4*>((which ? S.vnew : S.knew) + q8 * 8);
      }
    }
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

  // Publish this split's state [g][m, l, o[D]] as tagged fp32 words.
  constexpr int STRIDE = D + 2;
  unsigned long long* my = fa.part + ((size_t)kvh * p.splits + split) * G * STRIDE;
  for (int i = tid; i < G * STRIDE; i += NT) {
    const int g = i / STRIDE, k = i - g * STRIDE;
    const float val = (k == 0) ? S.sm[g] : (k == 1) ? S.sl[g] : S.so[g][k - 2];
    st_rlx_b64(my + i, f32_word(val, tag32));
  }
  trace_at(td, 5);
  if (!has_new) return true;

  // The last split combines every split's state of this KV head: the
  // partial outputs a thread weights are read together with the (m, l)
  // pairs (one round trip); the split weights of a query head are computed
  // by one lane per split with shuffles.
  const unsigned long long* hp = fa.part + (size_t)kvh * p.splits * G * STRIDE;
  float* fw = &S.so[0][0];
  constexpr int IPT = (kAttnMaxGroup * D + NT - 1) / NT;
  float ov[IPT][kMaxSplits];
  {
    // All loads first (one round trip), then the tags: a word that has not
    // arrived yet is polled by address.
    unsigned long long wv[IPT][kMaxSplits];
#pragma unroll
    for (int k = 0; k < IPT; ++k) {
      const int i = tid + k * NT;
      const int g = i / D, d = i - g * D;
#pragma unroll
      for (int r = 0; r < kMaxSplits; ++r)
        wv[k][r] = (i < G * D && r < p.splits) ? ld_rlx_b64(hp + ((size_t)r * G + g) * STRIDE + 2 + d)
                                               : ((unsigned long long)tag32 << 32);
    }
#pragma unroll
    for (int k = 0; k < IPT; ++k)
#pragma unroll
      for (int r = 0; r < kMaxSplits; ++r) ov[k][r] = __uint_as_float((uint32_t)wv[k][r]);
    unsigned miss = 0u;  // bit k * kMaxSplits + r: word not yet arrived
#pragma unroll
    for (int k = 0; k < IPT; ++k)
#pragma unroll
      for (int r = 0; r < kMaxSplits; ++r)
        if ((uint32_t)(wv[k][r] >> 32) != tag32) miss |= 1u << (k * kMaxSplits + r);
    static_assert(IPT * kMaxSplits <= 32, "one miss bit per word");
    while (miss != 0u) {
      const int b = __ffs(miss) - 1;
      miss &= miss - 1u;
      const int k = b / kMaxSplits, r = b - k * kMaxSplits;
      const int i = tid + k * NT;
      const int g = i / D, d = i - g * D;
      const float v = get_f32t(hp + ((size_t)r * G + g) * STRIDE + 2 + d, tag32, ok);
#pragma unroll
      for (int k2 = 0; k2 < IPT; ++k2)
#pragma unroll
        for (int r2 = 0; r2 < kMaxSplits; ++r2)
          if (k2 == k && r2 == r) ov[k2][r2] = v;
    }
  }
  __syncthreads();  // every thread is done with S.so (it becomes the weights)
  const bool fast = (p.splits & (p.splits - 1)) == 0 && p.splits <= kWarp && G * p.splits <= NT;
  if (fast) {
    const int i = tid, g = i / p.splits, r = i - g * p.splits;
    const bool on = i < G * p.splits;
    float mr = -INFINITY, lr = 0.f;
    if (on) {
      const unsigned long long* a = hp + ((size_t)r * G + g) * STRIDE;
      mr = get_f32t(a, tag32, ok);
      lr = get_f32t(a + 1, tag32, ok);
    }
    float M = mr;
    for (int o = p.splits >> 1; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const float f = (mr == -INFINITY) ? 0.f : expf(mr - M);
    float Ls = lr * f;
    for (int o = p.splits >> 1; o > 0; o >>= 1) Ls += __shfl_xor_sync(0xffffffffu, Ls, o);
    if (on) fw[r * GM + g] = f / Ls;
  } else {
    float* mlr = &S.sq[0][0];
    for (int i = tid; i < p.splits * G; i += NT) {
      const int r = i / G, g = i - r * G;
      const unsigned long long* a = hp + ((size_t)r * G + g) * STRIDE;
      mlr[2 * (r * GM + g)] = get_f32t(a, tag32, ok);
      mlr[2 * (r * GM + g) + 1] = get_f32t(a + 1, tag32, ok);
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
  }
  if (!ok) atomicExch(s_fail, 1);
  __syncthreads();
#pragma unroll
  for (int k = 0; k < IPT; ++k) {
    const int i = tid + k * NT;
    if (i < G * D) {
      const int g = i / D, d = i - g * D;
      float O = 0.f;
#pragma unroll
      for (int r = 0; r < kMaxSplits; ++r)
        if (r < p.splits) O = fmaf(ov[k][r], fw[r * GM + g], O);
      const int col = (kvh * G + g) * D + d;
      const uint32_t word = h16_word(f2h(O), tag16);
      if (fa.y_words != nullptr) st_rlx_b32(fa.y_words + col, word);
      if (fa.y_dst != nullptr) {
        const int j = __ldg(fa.y_inv + col);
        if (j >= 0) st_rlx_b32(fa.y_dst + j, word);
      }
    }
  }
  __syncthreads();
  if (tid == 0 && fa.done_out != nullptr) red_rlx_add_u32(fa.done_out, 1u);
  return *reinterpret_cast<volatile int*>(s_fail) == 0;
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
constexpr int kFlowGemvWords = (int)(sizeof(FlowGemv) / 4);
constexpr int kFlowAttnWords = (int)(sizeof(FlowAttn) / 4);
static_assert(sizeof(FlowGemv) % 4 == 0 && sizeof(FlowAttn) % 4 == 0, "parameter blocks are copied as words");
static_assert(kFlowGemvWords <= kStepThreads && kFlowAttnWords <= kStepThreads, "one parameter word per thread");

template <int D>
__global__ void __launch_bounds__(kStepThreads, 1) decode_flow_kernel(const __grid_constant__ FlowParams fp) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ FlowGemv s_g[2];
  __shared__ FlowAttn s_attn[2];
  __shared__ int s_pos;
  __shared__ int s_fail;
  __shared__ uint64_t s_pre_bar;
  const unsigned cta = blockIdx.x, ncta = gridDim.x;
  const int tid = threadIdx.x;
  unsigned char* act = smem_raw + fp.ring_bytes;
  ProdDesc* s_desc = reinterpret_cast<ProdDesc*>(act + fp.act_bytes);
  int* s_kind = reinterpret_cast<int*>(s_desc + fp.ngemv);

  for (int s = tid; s < fp.nstages; s += kStepThreads) s_kind[s] = fp.kind[s];
  for (int i = tid; i < fp.ngemv * (int)(sizeof(ProdDesc) / 16); i += kStepThreads)
    reinterpret_cast<uint4*>(s_desc)[i] = __ldg(reinterpret_cast<const uint4*>(fp.desc) + i);
  if (tid < kFlowGemvWords && fp.ngemv > 0)
    reinterpret_cast<uint32_t*>(&s_g[0])[tid] = reinterpret_cast<const uint32_t*>(fp.gemv)[tid];
  if (tid < kFlowAttnWords && fp.nattn > 0)
    reinterpret_cast<uint32_t*>(&s_attn[0])[tid] = reinterpret_cast<const uint32_t*>(fp.attn)[tid];
  if (tid == 0) {
    mbar_init(&s_pre_bar, 1);
    s_fail = 0;
  }
  unsigned pre_uses = 0;
  __syncthreads();
  Ring R;
  R.wring = smem_raw + (size_t)(tid >> 5) * D * kRingItemBytes;
  R.cslot = 0;
  R.P.n = -1;
  R.P.t = R.P.t1 = 0;
  R.P.slot = 0;
  for (int i = 0; i < D; ++i) prod_next<D>(R.P, s_desc, fp.ngemv, R.wring, cta, ncta);

  grid_dep_wait();
  if (fp.trace != nullptr && cta == 0 && tid == 0) fp.trace[0] = global_timer_ns();
  const unsigned long long epoch = *reinterpret_cast<volatile unsigned long long*>(fp.epoch);
  const uint32_t tag16 = (uint32_t)(epoch % 65535ull) + 1u;
  const uint32_t tag32 = (uint32_t)(epoch + 1ull);
  if (tid == 0) s_pos = (fp.pos != nullptr) ? (int)min((int64_t)0x7fffffff, max((int64_t)-1, *fp.pos)) : 0;
  if (fp.nstages > 0 && s_kind[0] == kStageGemv) flow_pre_smem(s_g[0], ncta, act, &s_pre_bar, pre_uses);
  __syncthreads();
  int gn = 0, an = 0;
  bool aborted = false;
  for (int s = 0; s < fp.nstages; ++s) {
    unsigned long long* td = fp.trace_detail ? fp.trace_detail + ((size_t)s * ncta + cta) * kTraceMarks : nullptr;
    trace_at(td, 0);
    bool ok = true;
    if (s_kind[s] == kStageGemv) {
      const bool more = gn + 1 < fp.ngemv;
      uint32_t stash = 0u;
      if (more && tid < kFlowGemvWords) stash = __ldg(reinterpret_cast<const uint32_t*>(fp.gemv + gn + 1) + tid);
      ok = run_flow_gemv<D>(s_g[gn & 1], s_desc, fp.ngemv, cta, ncta, act, R, &s_pre_bar, pre_uses, tag16, tag32, td,
                            &s_fail);
      if (more && tid < kFlowGemvWords) reinterpret_cast<uint32_t*>(&s_g[(gn + 1) & 1])[tid] = stash;
      ++gn;
    } else {
      const bool more = an + 1 < fp.nattn;
      uint32_t stash = 0u;
      if (more && tid < kFlowAttnWords) stash = __ldg(reinterpret_cast<const uint32_t*>(fp.attn + an + 1) + tid);
      const FlowAttn& a = s_attn[an & 1];
      const int units = a.a.Hkv * a.a.splits;
      StepAttnSmem& A = *reinterpret_cast<StepAttnSmem*>(act);
      if ((int)cta < units) ok = flow_attention_unit(a, s_pos, (int)cta % a.a.splits, (int)cta / a.a.splits, A, tag16,
                                                     tag32, td, &s_fail);
      if (more && tid < kFlowAttnWords) reinterpret_cast<uint32_t*>(&s_attn[(an + 1) & 1])[tid] = stash;
      ++an;
    }
    __syncthreads();  // the next stage's parameters are stored; this stage is done with its shared memory
    if (fp.trace != nullptr && tid == 0) fp.trace[1 + (size_t)s * (ncta + 1) + cta] = global_timer_ns();
    trace_at(td, 6);
    if (!ok || s_fail != 0) {
      aborted = true;
      break;
    }
    if (s + 1 < fp.nstages && s_kind[s + 1] == kStageGemv) flow_pre_smem(s_g[gn & 1], ncta, act, &s_pre_bar, pre_uses);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  if (aborted && tid == 0 && pre_uses > 0u) mbar_wait_bounded(&s_pre_bar, (pre_uses - 1u) & 1u, kPreWaitLimitNs);
  __syncthreads();
  // Leave: the last CTA zeroes the completion counters (no CTA of this
  // launch reads them any more), then counts the step.
  __shared__ int s_last;
  if (tid == 0) {
    __threadfence();
    s_last = (atomicAdd(fp.exit_count, 1u) == ncta - 1) ? 1 : 0;
  }
  __syncthreads();
  if (s_last) {
    for (int i = tid; i < fp.ncounters; i += kStepThreads) fp.counters[i] = 0u;
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      atomicExch(fp.exit_count, 0u);
      atomicAdd(fp.epoch, 1ull);
    }
  }
  grid_dep_launch_dependents();
}

}  // namespace nms
